"""Builds libemx.so (the sm_100a kernels + C ABI) in-tree.

    python engine-mlx_b200/build.py [--force] [-j N]

Every translation unit under csrc/ is compiled by nvcc for sm_100a only
(-gencode arch=compute_100a,code=sm_100a) and linked into lib/libemx.so next
to this file.  Objects are rebuilt when their source or any header changed.
"""
import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
INCLUDE = os.path.join(os.path.dirname(HERE), "include")
OBJ = os.path.join(HERE, "lib", "obj")
LIB = os.path.join(HERE, "lib", "libemx.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-std=c++17", "-O3", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
              "--expt-relaxed-constexpr", "-I" + INCLUDE]


def nvcc():
    cand = os.environ.get("NVCC") or shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand) and not shutil.which(cand):
        raise RuntimeError("nvcc not found")
    return cand


def sources():
    return sorted(f for f in os.listdir(CSRC) if f.endswith(".cu"))


def newest_header():
    hs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    hs.append(os.path.join(INCLUDE, "emx.h"))
    return max(os.path.getmtime(h) for h in hs if os.path.exists(h))


def compile_one(src, force, hdr_time):
    s = os.path.join(CSRC, src)
    o = os.path.join(OBJ, src[:-3] + ".o")
    if not force and os.path.exists(o) and os.path.getmtime(o) >= max(os.path.getmtime(s), hdr_time):
        return o, None
    cmd = [nvcc()] + ARCH + NVCC_FLAGS + ["-c", s, "-o", o]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        return o, r.stdout + r.stderr
    return o, None


def build(force=False, jobs=None, verbose=False):
    os.makedirs(OBJ, exist_ok=True)
    hdr = newest_header()
    srcs = sources()
    jobs = jobs or min(len(srcs), os.cpu_count() or 4)
    objs, errors = [], []
    with cf.ThreadPoolExecutor(max_workers=jobs) as ex:
        for o, err in ex.map(lambda f: compile_one(f, force, hdr), srcs):
            objs.append(o)
            if err:
                errors.append(err)
    if errors:
        raise RuntimeError("nvcc failed:\n" + "\n".join(errors))
    if force or not os.path.exists(LIB) or os.path.getmtime(LIB) < max(os.path.getmtime(o) for o in objs):
        # visibility: only the extern "C" entry points (marked default below) are exported
        cmd = [nvcc()] + ARCH + ["-shared", "-o", LIB] + objs + ["-ldl", "-Xcompiler", "-fPIC"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError("link failed:\n" + r.stdout + r.stderr)
    if verbose:
        print(LIB)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-j", type=int, default=None)
    a = ap.parse_args()
    try:
        build(a.force, a.j, verbose=True)
    except RuntimeError as e:
        print(e, file=sys.stderr)
        sys.exit(1)
