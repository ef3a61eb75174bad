"""The Rust crate that replaces crates/mlx-ffi
(engine-mlx_b200/rust/engine-mlx-ffi) declares exactly the C ABI of
include/emx.h: its generated src/sys.rs is what gen_sys.py derives from the
header today, and it declares every function the header declares (no Rust
toolchain exists here, so the crate itself is not compiled by the tests)."""
import os
import re
import subprocess
import sys

import emx

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
RUST = os.path.join(ROOT, "engine-mlx_b200", "rust")


def test_sys_rs_matches_header():
    r = subprocess.run([sys.executable, os.path.join(RUST, "gen_sys.py"), "--check"], capture_output=True, text=True)
    assert r.returncode == 0, r.stdout + r.stderr


def test_crate_declares_every_header_symbol():
    src = open(os.path.join(RUST, "engine-mlx-ffi", "src", "sys.rs")).read()
    declared = set(re.findall(r"pub fn (emx_\w+)\(", src))
    assert declared == set(emx.declared_symbols())


def test_safe_layer_calls_only_declared_symbols():
    lib = open(os.path.join(RUST, "engine-mlx-ffi", "src", "lib.rs")).read()
    used = set(re.findall(r"sys::(emx_\w+)\(", lib))
    assert used and used <= set(emx.declared_symbols())
    # the engine adapter covers the serve path: load, prefill, decode, stream, sampling
    for f in ("emx_qwen3_load_safetensors", "emx_qwen3_prefill", "emx_qwen3_decode_step", "emx_qwen3_decode",
              "emx_qwen3_decode_stream", "emx_qwen3_set_sampling", "emx_qwen3_prefill_chunked"):
        assert f in used, f
