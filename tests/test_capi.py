"""The C-ABI library without a GPU: it loads, exports exactly what
include/emx.h declares, and refuses work loudly (no host fallback)."""
import ctypes as C
import os
import re

import pytest

import emx

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "emx.h")


def header_symbols():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(emx_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    lib = emx.lib()
    declared = header_symbols()
    assert len(declared) >= 50
    missing = [s for s in declared if not hasattr(lib, s)]
    assert not missing, f"declared but not exported: {missing}"
    # the Python binding covers the whole header
    assert sorted(emx.declared_symbols()) == declared


def test_nothing_else_is_exported():
    import subprocess

    out = subprocess.run(["nm", "-D", "--defined-only", emx.LIB_PATH], capture_output=True, text=True).stdout
    exported = sorted({line.split()[-1] for line in out.splitlines() if " T " in line})
    assert exported == header_symbols()


def test_version_string():
    assert b"sm_100a" in emx.lib().emx_version()


def _has_gpu():
    try:
        import torch

        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.mark.skipif(_has_gpu(), reason="checks the no-GPU failure path")
def test_ctx_create_fails_loudly_without_gpu():
    with pytest.raises(emx.EmxError) as ei:
        emx.Ctx(0)
    assert ei.value.code == emx.ERR_CUDA
    assert "CUDA" in ei.value.msg or "device" in ei.value.msg


def test_null_arguments_rejected_before_any_device_work():
    lib = emx.lib()
    assert lib.emx_quantized_matmul(None, None, None, None, None, None, 1, 16, 64, 1, 64, 4) == emx.ERR_INVALID
    assert "null" in lib.emx_last_error().decode()
    assert lib.emx_qwen3_create(None, None, None, None) == emx.ERR_INVALID
    assert lib.emx_comm_init(None, None, 2, 0, None) == emx.ERR_INVALID


def test_error_handler_receives_messages():
    lib = emx.lib()
    got = []
    CB = C.CFUNCTYPE(None, C.c_char_p, C.c_void_p)
    cb = CB(lambda msg, data: got.append(msg.decode()))
    lib.emx_set_error_handler(C.cast(cb, C.c_void_p), None)
    try:
        lib.emx_synchronize(None)
    finally:
        lib.emx_set_error_handler(None, None)
    assert got and "null" in got[0]
