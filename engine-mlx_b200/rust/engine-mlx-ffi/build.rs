//! Links libemx.so.  EMX_LIB_DIR names the directory holding it (default:
//! engine-mlx_b200/lib of this checkout, where `python
//! engine-mlx_b200/build.py` puts it); the rpath lets binaries find it at
//! run time without LD_LIBRARY_PATH.
use std::path::PathBuf;

fn main() {
    let dir = std::env::var("EMX_LIB_DIR").map(PathBuf::from).unwrap_or_else(|_| {
        PathBuf::from(env!("CARGO_MANIFEST_DIR")).join("..").join("..").join("lib")
    });
    let dir = dir.canonicalize().unwrap_or(dir);
    println!("cargo:rerun-if-env-changed=EMX_LIB_DIR");
    println!("cargo:rerun-if-changed=src/sys.rs");
    println!("cargo:rustc-link-search=native={}", dir.display());
    println!("cargo:rustc-link-lib=dylib=emx");
    println!("cargo:rustc-link-arg=-Wl,-rpath,{}", dir.display());
}
