"""emx — Python host binding of libemx (the sm_100a Qwen3 path).

A thin ctypes layer over include/emx.h, shaped like the reference's MlxCtx
(crates/mlx-ffi/src/ops/real/*.rs) and Qwen3Engine (crates/serve/src/engine*.rs,
forward_qwen3.rs): every method is one C call, a non-zero status raises
EmxError carrying emx_last_error() (MlxCtx::check, mod.rs:35-40).

Host arrays are numpy; bf16 tensors are uint16 bit patterns (see bf16()).
The library must already be built (engine-mlx_b200/build.py); importing this
module without it, or calling it without an sm_100 GPU, raises — there is no
host fallback.
"""
from __future__ import annotations

import ctypes as C
import dataclasses
import os
from typing import Dict, Optional

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(os.path.dirname(_HERE), "lib", "libemx.so")

OK, ERR_INVALID, ERR_CUDA, ERR_OOM, ERR_DEVICE, ERR_NCCL, ERR_STATE = range(7)
BF16, F32, U32, I32 = range(4)


class EmxError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"emx error {code}: {msg}")
        self.code = code
        self.msg = msg


class QwenConfig(C.Structure):
    _fields_ = [(n, C.c_int) for n in ("hidden", "layers", "n_q", "n_kv", "head_dim", "inter", "vocab")] + [
        ("eps", C.c_float), ("rope_theta", C.c_float)] + [(n, C.c_int) for n in (
            "tied", "norm_groups", "attn_bits", "attn_group", "mlp_bits", "mlp_group", "embed_bits", "embed_group",
            "lm_bits", "lm_group", "n_experts", "top_k", "moe_inter", "norm_topk", "router_bits", "router_group",
            "expert_bits", "expert_group", "kv_cap", "max_prefill")]


_SIGS = {
    "emx_last_error": (C.c_char_p, []),
    "emx_version": (C.c_char_p, []),
    "emx_set_error_handler": (None, [C.c_void_p, C.c_void_p]),
    "emx_ctx_create": (C.c_int, [C.c_int, C.POINTER(C.c_void_p)]),
    "emx_ctx_destroy": (C.c_int, [C.c_void_p]),
    "emx_ctx_stream": (C.c_int, [C.c_void_p, C.POINTER(C.c_void_p)]),
    "emx_ctx_num_sms": (C.c_int, [C.c_void_p, C.POINTER(C.c_int)]),
    "emx_synchronize": (C.c_int, [C.c_void_p]),
    "emx_device_status": (C.c_int, [C.c_void_p, C.POINTER(C.c_int), C.c_int]),
    "emx_malloc": (C.c_int, [C.c_void_p, C.c_size_t, C.POINTER(C.c_void_p)]),
    "emx_free": (C.c_int, [C.c_void_p, C.c_void_p]),
    "emx_memcpy_h2d": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_size_t]),
    "emx_memcpy_d2h": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_size_t]),
    "emx_memset": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.c_size_t]),
    "emx_get_active_memory": (C.c_int, [C.c_void_p, C.POINTER(C.c_size_t)]),
    "emx_get_peak_memory": (C.c_int, [C.c_void_p, C.POINTER(C.c_size_t)]),
    "emx_set_memory_limit": (C.c_int, [C.c_void_p, C.c_size_t, C.POINTER(C.c_size_t)]),
    "emx_quantized_matmul": (C.c_int, [C.c_void_p] + [C.c_void_p] * 5 + [C.c_int] * 6),
    "emx_dequantize": (C.c_int, [C.c_void_p] + [C.c_void_p] * 4 + [C.c_int] * 4),
    "emx_quantize": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int] + [C.c_void_p] * 3 + [C.c_int] * 4),
    "emx_rms_norm": (C.c_int, [C.c_void_p] + [C.c_void_p] * 3 + [C.c_int, C.c_int, C.c_float]),
    "emx_grouped_rms_norm": (C.c_int, [C.c_void_p] + [C.c_void_p] * 3 + [C.c_int, C.c_int, C.c_float, C.c_int]),
    "emx_rope": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_float, C.c_int,
                           C.c_void_p]),
    "emx_sdpa_causal": (C.c_int, [C.c_void_p] + [C.c_void_p] * 4 + [C.c_int] * 4 + [C.c_float, C.c_int]),
    "emx_qpack_bytes": (C.c_int, [C.c_int] * 4 + [C.POINTER(C.c_size_t)]),
    "emx_qpack": (C.c_int, [C.c_void_p] * 5 + [C.c_int] * 4),
    "emx_quantized_matvec_packed": (C.c_int, [C.c_void_p] * 4 + [C.c_int] * 4),
    "emx_quantized_matmul_packed": (C.c_int, [C.c_void_p] * 4 + [C.c_int] * 5),
    "emx_sdpa_decode": (C.c_int, [C.c_void_p] + [C.c_void_p] * 4 + [C.c_int] * 5 + [C.c_float]),
    "emx_sdpa_decode_noalloc": (C.c_int, [C.c_void_p] + [C.c_void_p] * 4 + [C.c_int] * 5 + [C.c_float]),
    "emx_silu": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_size_t]),
    "emx_multiply": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_size_t]),
    "emx_add": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_size_t]),
    "emx_argmax": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_void_p]),
    "emx_softmax": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_int]),
    "emx_embed_quantized": (C.c_int, [C.c_void_p] + [C.c_void_p] * 4 + [C.c_int] * 5 + [C.c_void_p]),
    "emx_slice_update": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p] + [C.c_int] * 5),
    "emx_scatter_single": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p] + [C.c_int] * 3),
    "emx_moe_route": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_void_p]),
    "emx_gather_qmm": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int] + [C.c_void_p] * 4 + [C.c_int, C.c_void_p] +
                       [C.c_int] * 5),
    "emx_comm_unique_id": (C.c_int, [C.c_void_p]),
    "emx_comm_init": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.POINTER(C.c_void_p)]),
    "emx_comm_destroy": (C.c_int, [C.c_void_p]),
    "emx_all_reduce_sum": (C.c_int, [C.c_void_p, C.c_void_p, C.c_size_t, C.c_int]),
    "emx_qwen3_create": (C.c_int, [C.c_void_p, C.POINTER(QwenConfig), C.c_void_p, C.POINTER(C.c_void_p)]),
    "emx_qwen3_destroy": (C.c_int, [C.c_void_p]),
    "emx_qwen3_load_tensor": (C.c_int, [C.c_void_p, C.c_char_p, C.c_void_p, C.c_size_t]),
    "emx_qwen3_read_tensor": (C.c_int, [C.c_void_p, C.c_char_p, C.c_void_p, C.c_size_t]),
    "emx_qwen3_load_safetensors": (C.c_int, [C.c_void_p, C.c_char_p, C.POINTER(C.c_int)]),
    "emx_qwen3_tensor_names": (C.c_int, [C.c_void_p, C.c_void_p, C.c_size_t, C.POINTER(C.c_size_t)]),
    "emx_qwen3_tensor_shape": (C.c_int, [C.c_void_p, C.c_char_p, C.POINTER(C.c_int64), C.POINTER(C.c_int),
                                         C.POINTER(C.c_int)]),
    "emx_safetensors_index": (C.c_int, [C.c_char_p, C.c_void_p, C.c_int, C.POINTER(C.c_int)]),
    "emx_qwen3_config_from_dir": (C.c_int, [C.c_char_p, C.c_int, C.c_int, C.POINTER(QwenConfig)]),
    "emx_qwen3_prefill_chunked": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.POINTER(C.c_int32),
                                            C.c_void_p]),
    "emx_qwen3_set_sampling": (C.c_int, [C.c_void_p, C.c_float, C.c_float, C.c_int, C.c_uint64]),
    "emx_sample_token": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.c_float, C.c_float, C.c_int, C.c_void_p,
                                   C.c_void_p]),
    "emx_qwen3_read_kv": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_size_t]),
    "emx_qwen3_set_compiled": (C.c_int, [C.c_void_p, C.c_int]),
    "emx_qwen3_shard": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.c_char_p, C.POINTER(C.c_int32)]),
    "emx_qwen3_is_compiled": (C.c_int, [C.c_void_p, C.POINTER(C.c_int)]),
    "emx_qwen3_set_fused": (C.c_int, [C.c_void_p, C.c_int]),
    "emx_qwen3_is_fused": (C.c_int, [C.c_void_p, C.POINTER(C.c_int)]),
    "emx_qwen3_init_random": (C.c_int, [C.c_void_p, C.c_uint64]),
    "emx_qwen3_reset": (C.c_int, [C.c_void_p]),
    "emx_qwen3_offset": (C.c_int, [C.c_void_p, C.POINTER(C.c_int)]),
    "emx_qwen3_prefill": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.POINTER(C.c_int32), C.c_void_p]),
    "emx_qwen3_decode_step": (C.c_int, [C.c_void_p, C.c_int32, C.POINTER(C.c_int32), C.c_void_p]),
    "emx_qwen3_decode": (C.c_int, [C.c_void_p, C.c_int32, C.c_int, C.c_void_p]),
    "emx_qwen3_prefill_device": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int]),
    "emx_qwen3_decode_device": (C.c_int, [C.c_void_p, C.c_int]),
    "emx_qwen3_decode_stream": (C.c_int, [C.c_void_p, C.c_int32, C.c_int, C.c_void_p, C.c_void_p,
                                          C.POINTER(C.c_int)]),
    "emx_qwen3_step_launches": (C.c_int, [C.c_void_p, C.POINTER(C.c_int)]),
}

_lib: Optional[C.CDLL] = None

# emx_token_cb: int (*)(int32_t token, int index, void* user)
TOKEN_CB = C.CFUNCTYPE(C.c_int, C.c_int32, C.c_int, C.c_void_p)


def lib() -> C.CDLL:
    """Loads libemx.so (raises if it has not been built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"libemx.so not built: run python engine-mlx_b200/build.py ({LIB_PATH} missing)")
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in _SIGS.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def declared_symbols():
    return sorted(_SIGS)


def _check(rc: int):
    if rc != 0:
        raise EmxError(rc, lib().emx_last_error().decode(errors="replace"))


# ------------------------------------------------------------------ bf16 helpers
def bf16(x) -> np.ndarray:
    """float array -> bf16 bit patterns (round-to-nearest-even)."""
    a = np.ascontiguousarray(np.asarray(x, dtype=np.float32))
    u = a.view(np.uint32).astype(np.uint64)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    r[nan] = ((u[nan] >> 16) | 0x40).astype(np.uint16)
    return r


def f32(b: np.ndarray) -> np.ndarray:
    """bf16 bit patterns -> float32."""
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


# ---------------------------------------------------------------------- context
class Buffer:
    """A device allocation owned by a Ctx."""

    def __init__(self, ctx: "Ctx", nbytes: int):
        self.ctx = ctx
        self.nbytes = int(nbytes)
        p = C.c_void_p()
        _check(lib().emx_malloc(ctx.h, self.nbytes, C.byref(p)))
        self.ptr = p.value

    def free(self):
        if self.ptr:
            _check(lib().emx_free(self.ctx.h, self.ptr))
            self.ptr = None

    def write(self, arr: np.ndarray, offset: int = 0):
        a = np.ascontiguousarray(arr)
        if a.nbytes + offset > self.nbytes:
            raise ValueError("write past the end of the buffer")
        _check(lib().emx_memcpy_h2d(self.ctx.h, self.ptr + offset, a.ctypes.data, a.nbytes))
        return self

    def read(self, dtype, shape) -> np.ndarray:
        out = np.empty(shape, dtype=dtype)
        _check(lib().emx_memcpy_d2h(self.ctx.h, out.ctypes.data, self.ptr, out.nbytes))
        return out


class Ctx:
    """MlxCtx equivalent: one device and one stream (crates/mlx-ffi/src/ops/real/mod.rs:4-41)."""

    def __init__(self, device: int = 0):
        h = C.c_void_p()
        _check(lib().emx_ctx_create(int(device), C.byref(h)))
        self.h = h.value
        self.device = device

    def close(self):
        if self.h:
            lib().emx_ctx_destroy(self.h)
            self.h = None

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    @property
    def num_sms(self) -> int:
        n = C.c_int()
        _check(lib().emx_ctx_num_sms(self.h, C.byref(n)))
        return n.value

    def synchronize(self):
        _check(lib().emx_synchronize(self.h))

    def device_status(self, clear: bool = True) -> int:
        s = C.c_int()
        _check(lib().emx_device_status(self.h, C.byref(s), int(clear)))
        return s.value

    def alloc(self, nbytes: int) -> Buffer:
        return Buffer(self, nbytes)

    def put(self, arr: np.ndarray) -> Buffer:
        a = np.ascontiguousarray(arr)
        return Buffer(self, max(a.nbytes, 1)).write(a)

    def active_memory(self) -> int:
        v = C.c_size_t()
        _check(lib().emx_get_active_memory(self.h, C.byref(v)))
        return v.value

    def peak_memory(self) -> int:
        v = C.c_size_t()
        _check(lib().emx_get_peak_memory(self.h, C.byref(v)))
        return v.value

    def set_memory_limit(self, limit: int) -> int:
        prev = C.c_size_t()
        _check(lib().emx_set_memory_limit(self.h, int(limit), C.byref(prev)))
        return prev.value

    # --- ops (MlxCtx method names); arguments are Buffers, results Buffers
    def quantized_matmul(self, x, w, s, b, M, N, K, group_size, bits, out=None, transpose=True):
        out = out or self.alloc(M * N * 2)
        _check(lib().emx_quantized_matmul(self.h, x.ptr, w.ptr, s.ptr, b.ptr, out.ptr, M, N, K, int(transpose),
                                          group_size, bits))
        return out

    def qpack(self, w, s, b, N, K, group_size, bits):
        """Packed (decode-GEMV) layout of an affine tensor, in a new buffer."""
        n = C.c_size_t()
        _check(lib().emx_qpack_bytes(N, K, group_size, bits, C.byref(n)))
        out = self.alloc(n.value)
        _check(lib().emx_qpack(self.h, w.ptr, s.ptr, b.ptr, out.ptr, N, K, group_size, bits))
        return out

    def quantized_matvec_packed(self, x, packed, N, K, group_size, bits):
        y = self.alloc(N * 2)
        _check(lib().emx_quantized_matvec_packed(self.h, x.ptr, packed.ptr, y.ptr, N, K, group_size, bits))
        return y

    def quantized_matmul_packed(self, x, packed, M, N, K, group_size, bits, out=None):
        """y[M, N] = x[M, K] . dequant(w)^T over the packed layout (qpack)."""
        out = out or self.alloc(M * N * 2)
        _check(lib().emx_quantized_matmul_packed(self.h, x.ptr, packed.ptr, out.ptr, M, N, K, group_size, bits))
        return out

    def dequantize(self, w, s, b, N, K, group_size, bits):
        out = self.alloc(N * K * 2)
        _check(lib().emx_dequantize(self.h, w.ptr, s.ptr, b.ptr, out.ptr, N, K, group_size, bits))
        return out

    def quantize(self, src, src_dtype, N, K, group_size, bits):
        w = self.alloc(N * K * bits // 8)
        s = self.alloc(N * (K // group_size) * 2)
        b = self.alloc(N * (K // group_size) * 2)
        _check(lib().emx_quantize(self.h, src.ptr, src_dtype, w.ptr, s.ptr, b.ptr, N, K, group_size, bits))
        return w, s, b

    def rms_norm(self, x, w, rows, dims, eps):
        out = self.alloc(rows * dims * 2)
        _check(lib().emx_rms_norm(self.h, x.ptr, w.ptr, out.ptr, rows, dims, eps))
        return out

    def grouped_rms_norm(self, x, w, rows, dims, eps, groups):
        out = self.alloc(rows * dims * 2)
        _check(lib().emx_grouped_rms_norm(self.h, x.ptr, w.ptr, out.ptr, rows, dims, eps, groups))
        return out

    def rope(self, x, heads, T, dims, theta, offset=0, offset_dev=None):
        out = self.alloc(heads * T * dims * 2)
        _check(lib().emx_rope(self.h, x.ptr, out.ptr, heads, T, dims, theta, offset,
                              offset_dev.ptr if offset_dev else None))
        return out

    def sdpa_causal(self, q, k, v, nq, nkv, T, hd, scale, out_tnd=False):
        out = self.alloc(nq * T * hd * 2)
        _check(lib().emx_sdpa_causal(self.h, q.ptr, k.ptr, v.ptr, out.ptr, nq, nkv, T, hd, scale, int(out_tnd)))
        return out

    def sdpa_decode(self, q, kc, vc, nq, nkv, cap, hd, length, scale):
        out = self.alloc(nq * hd * 2)
        _check(lib().emx_sdpa_decode(self.h, q.ptr, kc.ptr, vc.ptr, out.ptr, nq, nkv, cap, hd, length, scale))
        return out

    def sdpa_decode_noalloc(self, q, kc, vc, out, nq, nkv, cap, hd, length, scale):
        """emx_sdpa_decode into a caller-provided `out`, with no device allocation."""
        _check(lib().emx_sdpa_decode_noalloc(self.h, q.ptr, kc.ptr, vc.ptr, out.ptr, nq, nkv, cap, hd, length, scale))
        return out

    def silu(self, x, n):
        out = self.alloc(n * 2)
        _check(lib().emx_silu(self.h, x.ptr, out.ptr, n))
        return out

    def multiply(self, a, b, n):
        out = self.alloc(n * 2)
        _check(lib().emx_multiply(self.h, a.ptr, b.ptr, out.ptr, n))
        return out

    def add(self, a, b, n):
        out = self.alloc(n * 2)
        _check(lib().emx_add(self.h, a.ptr, b.ptr, out.ptr, n))
        return out

    def argmax(self, x, rows, n):
        out = self.alloc(rows * 4)
        _check(lib().emx_argmax(self.h, x.ptr, rows, n, out.ptr))
        return out

    def sample_token(self, logits, n, temperature, top_p, top_k, rng):
        """sampler.rs sample_token on device bf16 logits; `rng` is a device
        buffer holding the uint64 generator state (advanced in place).
        Returns a device int32 buffer with the token."""
        out = self.alloc(4)
        _check(lib().emx_sample_token(self.h, logits.ptr, n, temperature, top_p, int(top_k), rng.ptr, out.ptr))
        return out

    def softmax(self, x, rows, n):
        out = self.alloc(rows * n * 2)
        _check(lib().emx_softmax(self.h, x.ptr, out.ptr, rows, n))
        return out

    def embed_quantized(self, w, s, b, ids, T, hidden, vocab, group_size, bits):
        out = self.alloc(T * hidden * 2)
        _check(lib().emx_embed_quantized(self.h, w.ptr, s.ptr, b.ptr, ids.ptr, T, hidden, vocab, group_size, bits,
                                         out.ptr))
        return out

    def slice_update(self, cache, upd, nkv, cap, hd, offset, T):
        _check(lib().emx_slice_update(self.h, cache.ptr, upd.ptr, nkv, cap, hd, offset, T))

    def scatter_single(self, cache, offset_dev, upd, nkv, cap, hd):
        _check(lib().emx_scatter_single(self.h, cache.ptr, offset_dev.ptr, upd.ptr, nkv, cap, hd))

    def moe_route(self, logits, n_experts, top_k, normalize=True):
        idx = self.alloc(top_k * 4)
        w = self.alloc(top_k * 4)
        _check(lib().emx_moe_route(self.h, logits.ptr, n_experts, top_k, int(normalize), idx.ptr, w.ptr))
        return idx, w

    def gather_qmm(self, x, x_per_slot, w, s, b, idx, n_slots, n_experts, N, K, group_size, bits):
        out = self.alloc(n_slots * N * 2)
        _check(lib().emx_gather_qmm(self.h, x.ptr, int(x_per_slot), w.ptr, s.ptr, b.ptr, idx.ptr, n_slots, out.ptr,
                                    n_experts, N, K, group_size, bits))
        return out


# --------------------------------------------------------------------- comm
class Comm:
    """NCCL communicator for the tensor- / expert-parallel configs."""

    @staticmethod
    def unique_id() -> bytes:
        buf = C.create_string_buffer(128)
        _check(lib().emx_comm_unique_id(buf))
        return buf.raw

    def __init__(self, ctx: Ctx, uid: bytes, nranks: int, rank: int):
        h = C.c_void_p()
        buf = C.create_string_buffer(bytes(uid), 128)
        _check(lib().emx_comm_init(ctx.h, buf, nranks, rank, C.byref(h)))
        self.h = h.value
        self.ctx = ctx
        self.nranks, self.rank = nranks, rank

    def all_reduce_sum(self, buf: Buffer, count: int, dtype: int):
        _check(lib().emx_all_reduce_sum(self.h, buf.ptr, count, dtype))

    def close(self):
        if self.h:
            lib().emx_comm_destroy(self.h)
            self.h = None


# -------------------------------------------------------------------- Qwen3
@dataclasses.dataclass
class Qwen3Config:
    hidden: int
    layers: int
    n_q: int
    n_kv: int
    inter: int
    vocab: int
    head_dim: int = 128
    eps: float = 1e-6
    rope_theta: float = 1e6
    tied: bool = True
    norm_groups: int = 1
    attn_bits: int = 4
    attn_group: int = 64
    mlp_bits: int = 4
    mlp_group: int = 64
    embed_bits: int = 4
    embed_group: int = 64
    lm_bits: int = 4
    lm_group: int = 64
    n_experts: int = 0
    top_k: int = 0
    moe_inter: int = 0
    norm_topk: bool = True
    router_bits: int = 4
    router_group: int = 64
    expert_bits: int = 4
    expert_group: int = 64
    kv_cap: int = 4096
    max_prefill: int = 512

    def c_struct(self) -> QwenConfig:
        c = QwenConfig()
        for f in QwenConfig._fields_:
            v = getattr(self, f[0])
            setattr(c, f[0], float(v) if f[1] is C.c_float else int(v))
        return c

    @staticmethod
    def from_dir(model_dir: str, kv_cap: int = 4096, max_prefill: int = 512) -> "Qwen3Config":
        """Qwen3Config::from_dir: the shape and quantization of an MLX model
        directory's config.json (host only)."""
        c = QwenConfig()
        _check(lib().emx_qwen3_config_from_dir(model_dir.encode(), kv_cap, max_prefill, C.byref(c)))
        kw = {f[0]: getattr(c, f[0]) for f in QwenConfig._fields_}
        for b in ("tied", "norm_topk"):
            kw[b] = bool(kw[b])
        return Qwen3Config(**kw)


# The BASELINE configurations (random-init shapes of the named models).
CONFIGS: Dict[str, Qwen3Config] = {
    # Qwen3-0.6B: all linears int4 gs64, tied embeddings, KV 4096
    "c2": Qwen3Config(hidden=1024, layers=28, n_q=16, n_kv=8, inter=3072, vocab=151936, kv_cap=4096,
                      max_prefill=512),
    # Qwen3-1.7B: attention int8 gs64, MLP int4 gs64, tied, KV 16384
    "c3": Qwen3Config(hidden=2048, layers=28, n_q=16, n_kv=8, inter=6144, vocab=151936, attn_bits=8,
                      kv_cap=16384, max_prefill=8192),
    # Qwen3-30B-A3B: 48 layers, 32q/4kv, 128 experts top-8, moe_inter 768, untied
    "c4": Qwen3Config(hidden=2048, layers=48, n_q=32, n_kv=4, inter=6144, vocab=151936, tied=False,
                      n_experts=128, top_k=8, moe_inter=768, kv_cap=2048, max_prefill=1024),
    # Qwen3-32B: 64 layers, 64q/8kv, intermediate 25600, untied, KV 32768
    "c5": Qwen3Config(hidden=5120, layers=64, n_q=64, n_kv=8, inter=25600, vocab=151936, tied=False,
                      kv_cap=32768, max_prefill=4096),
}


class StTensor(C.Structure):
    """emx_st_tensor: one tensor of a .safetensors file."""
    _fields_ = [("name", C.c_char * 256), ("dtype", C.c_char * 12), ("ndim", C.c_int), ("shape", C.c_int64 * 8),
                ("offset", C.c_uint64), ("bytes", C.c_uint64)]


def safetensors_index(path: str):
    """[{name, dtype, shape, offset, bytes}] of a .safetensors file, validated
    by the library (host only; no device needed)."""
    n = C.c_int(0)
    _check(lib().emx_safetensors_index(path.encode(), None, 0, C.byref(n)))
    arr = (StTensor * max(1, n.value))()
    _check(lib().emx_safetensors_index(path.encode(), arr, n.value, C.byref(n)))
    return [{"name": t.name.decode(), "dtype": t.dtype.decode(), "shape": tuple(t.shape[:t.ndim]),
             "offset": int(t.offset), "bytes": int(t.bytes)} for t in arr[:n.value]]


_ST_DTYPES = {np.dtype(np.uint32): "U32", np.dtype(np.uint16): "BF16", np.dtype(np.float32): "F32",
              np.dtype(np.int32): "I32", np.dtype(np.uint8): "U8", np.dtype(np.float16): "F16"}


def write_safetensors(path: str, tensors, metadata=None):
    """Writes a .safetensors file: `tensors` maps name -> array (uint16 arrays
    are written as BF16 bit patterns) or (dtype name, array)."""
    import json
    import struct

    header, blobs, off = {}, [], 0
    for name, v in tensors.items():
        dt, a = v if isinstance(v, tuple) else (_ST_DTYPES[np.asarray(v).dtype], v)
        a = np.ascontiguousarray(a)
        b = a.tobytes()
        header[name] = {"dtype": dt, "shape": list(a.shape), "data_offsets": [off, off + len(b)]}
        blobs.append(b)
        off += len(b)
    if metadata:
        header["__metadata__"] = dict(metadata)
    h = json.dumps(header, separators=(",", ":")).encode()
    h += b" " * ((8 - len(h) % 8) % 8)  # the format pads the header to 8 bytes
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)


def shard(cfg: "Qwen3Config", world: int, rank: int, name: str):
    """(row0, n_rows, col0, n_cols, block0, blocks) of tensor `name` kept by rank (host only)."""
    out = (C.c_int32 * 6)()
    c = cfg.c_struct()
    _check(lib().emx_qwen3_shard(C.byref(c), world, rank, name.encode(), out))
    return tuple(out)


def quant_shapes(N: int, K: int, bits: int, gs: int, blocks: int = 0):
    lead = (blocks,) if blocks else ()
    return {"weight": (lead + (N, K * bits // 32), np.uint32), "scales": (lead + (N, K // gs), np.uint16),
            "biases": (lead + (N, K // gs), np.uint16)}


def checkpoint_tensors(cfg: Qwen3Config):
    """name -> (shape, dtype, kind, bits, gs) of every tensor of an MLX Qwen3 checkpoint."""
    out = {}
    H, hd = cfg.hidden, cfg.head_dim

    def q(base, N, K, bits, gs, blocks=0):
        for part, (shape, dt) in quant_shapes(N, K, bits, gs, blocks).items():
            out[f"{base}.{part}"] = (shape, dt, "quant", bits, gs, base, N, K, blocks)

    def norm(name, n):
        out[name] = ((n,), np.uint16, "norm", 0, 0, name, n, 0, 0)

    q("model.embed_tokens", cfg.vocab, H, cfg.embed_bits, cfg.embed_group)
    if not cfg.tied:
        q("lm_head", cfg.vocab, H, cfg.lm_bits, cfg.lm_group)
    norm("model.norm.weight", H)
    for l in range(cfg.layers):
        p = f"model.layers.{l}."
        norm(p + "input_layernorm.weight", H)
        norm(p + "post_attention_layernorm.weight", H)
        norm(p + "self_attn.q_norm.weight", hd)
        norm(p + "self_attn.k_norm.weight", hd)
        q(p + "self_attn.q_proj", cfg.n_q * hd, H, cfg.attn_bits, cfg.attn_group)
        q(p + "self_attn.k_proj", cfg.n_kv * hd, H, cfg.attn_bits, cfg.attn_group)
        q(p + "self_attn.v_proj", cfg.n_kv * hd, H, cfg.attn_bits, cfg.attn_group)
        q(p + "self_attn.o_proj", H, cfg.n_q * hd, cfg.attn_bits, cfg.attn_group)
        if cfg.n_experts:
            q(p + "mlp.gate", cfg.n_experts, H, cfg.router_bits, cfg.router_group)
            q(p + "mlp.switch_mlp.gate_proj", cfg.moe_inter, H, cfg.expert_bits, cfg.expert_group, cfg.n_experts)
            q(p + "mlp.switch_mlp.up_proj", cfg.moe_inter, H, cfg.expert_bits, cfg.expert_group, cfg.n_experts)
            q(p + "mlp.switch_mlp.down_proj", H, cfg.moe_inter, cfg.expert_bits, cfg.expert_group, cfg.n_experts)
        else:
            q(p + "mlp.gate_proj", cfg.inter, H, cfg.mlp_bits, cfg.mlp_group)
            q(p + "mlp.up_proj", cfg.inter, H, cfg.mlp_bits, cfg.mlp_group)
            q(p + "mlp.down_proj", H, cfg.inter, cfg.mlp_bits, cfg.mlp_group)
    return out


class Qwen3:
    """Qwen3Engine equivalent over the C ABI (crates/serve/src/engine.rs, forward_qwen3.rs)."""

    def __init__(self, ctx: Ctx, cfg: Qwen3Config, comm: Optional[Comm] = None):
        self.ctx, self.cfg, self.comm = ctx, cfg, comm
        self._c = cfg.c_struct()
        h = C.c_void_p()
        _check(lib().emx_qwen3_create(ctx.h, C.byref(self._c), comm.h if comm else None, C.byref(h)))
        self.h = h.value

    @classmethod
    def from_dir(cls, ctx: Ctx, model_dir: str, kv_cap: int = 4096, max_prefill: int = 512,
                 comm: Optional[Comm] = None) -> "Qwen3":
        """Qwen3Engine::load: config.json, then the checkpoint files of an MLX
        model directory (this rank's shard under TP / EP)."""
        m = cls(ctx, Qwen3Config.from_dir(model_dir, kv_cap, max_prefill), comm)
        try:
            m.load_safetensors(model_dir)
        except Exception:
            m.close()
            raise
        return m

    def close(self):
        if self.h:
            lib().emx_qwen3_destroy(self.h)
            self.h = None

    def load_tensor(self, name: str, arr: np.ndarray):
        a = np.ascontiguousarray(arr)
        _check(lib().emx_qwen3_load_tensor(self.h, name.encode(), a.ctypes.data, a.nbytes))

    def set_sampling(self, temperature: float = 0.0, top_p: float = 1.0, top_k: int = 0, seed: int = 42):
        """Qwen3Engine::set_sampling: temperature < 1e-6 is greedy; otherwise
        prefill and decode sample on the device."""
        _check(lib().emx_qwen3_set_sampling(self.h, temperature, top_p, int(top_k), C.c_uint64(seed)))

    def load_safetensors(self, path: str) -> int:
        """Loads an MLX checkpoint directory or .safetensors file; returns the
        number of checkpoint tensors used."""
        n = C.c_int(0)
        _check(lib().emx_qwen3_load_safetensors(self.h, path.encode(), C.byref(n)))
        return n.value

    def tensor_names(self):
        need = C.c_size_t(0)
        _check(lib().emx_qwen3_tensor_names(self.h, None, 0, C.byref(need)))
        buf = C.create_string_buffer(need.value)
        _check(lib().emx_qwen3_tensor_names(self.h, buf, need.value, C.byref(need)))
        return [x for x in buf.value.decode().split("\n") if x]

    def tensor_shape(self, name: str):
        """(full MLX shape, numpy dtype) of a tensor the model takes."""
        shp = (C.c_int64 * 3)()
        nd, dt = C.c_int(0), C.c_int(0)
        _check(lib().emx_qwen3_tensor_shape(self.h, name.encode(), shp, C.byref(nd), C.byref(dt)))
        return tuple(shp[:nd.value]), (np.uint32 if dt.value == 2 else np.uint16)

    def read_tensor(self, name: str, nbytes: int) -> bytes:
        buf = np.empty(nbytes, dtype=np.uint8)
        _check(lib().emx_qwen3_read_tensor(self.h, name.encode(), buf.ctypes.data, nbytes))
        return buf.tobytes()

    def read_kv(self, layer: int, which: int) -> np.ndarray:
        """This rank's K (which=0) or V (which=1) cache of one layer, bf16 bits [n_kv_local, kv_cap, head_dim]."""
        c = self.cfg
        nkv = c.n_kv // (self.comm.nranks if self.comm is not None and c.n_experts == 0 else 1)
        out = np.empty((nkv, c.kv_cap, c.head_dim), dtype=np.uint16)
        _check(lib().emx_qwen3_read_kv(self.h, layer, which, out.ctypes.data, out.nbytes))
        return out

    @property
    def compiled(self) -> bool:
        """Decode through the captured CUDA graph (True) or eagerly (False)."""
        v = C.c_int()
        _check(lib().emx_qwen3_is_compiled(self.h, C.byref(v)))
        return bool(v.value)

    @compiled.setter
    def compiled(self, on: bool):
        _check(lib().emx_qwen3_set_compiled(self.h, int(bool(on))))

    @property
    def fused(self) -> bool:
        """Decode through the persistent step kernel (True) or one kernel per op."""
        v = C.c_int()
        _check(lib().emx_qwen3_is_fused(self.h, C.byref(v)))
        return bool(v.value)

    @fused.setter
    def fused(self, on: bool):
        _check(lib().emx_qwen3_set_fused(self.h, int(bool(on))))

    def init_random(self, seed: int):
        _check(lib().emx_qwen3_init_random(self.h, C.c_uint64(seed)))

    def reset(self):
        _check(lib().emx_qwen3_reset(self.h))

    @property
    def offset(self) -> int:
        v = C.c_int()
        _check(lib().emx_qwen3_offset(self.h, C.byref(v)))
        return v.value

    def prefill(self, tokens, want_logits=False):
        ids = np.ascontiguousarray(np.asarray(tokens, dtype=np.int32))
        nxt = C.c_int32()
        logits = np.empty(self.cfg.vocab, dtype=np.uint16) if want_logits else None
        _check(lib().emx_qwen3_prefill(self.h, ids.ctypes.data, len(ids), C.byref(nxt),
                                       logits.ctypes.data if want_logits else None))
        return (nxt.value, logits) if want_logits else nxt.value

    def prefill_chunked(self, tokens, chunk: int, want_logits=False):
        """Prefill in chunks of `chunk` tokens, each attending the cache before it."""
        ids = np.ascontiguousarray(np.asarray(tokens, dtype=np.int32))
        nxt = C.c_int32()
        logits = np.empty(self.cfg.vocab, dtype=np.uint16) if want_logits else None
        _check(lib().emx_qwen3_prefill_chunked(self.h, ids.ctypes.data, len(ids), int(chunk), C.byref(nxt),
                                               logits.ctypes.data if want_logits else None))
        return (nxt.value, logits) if want_logits else nxt.value

    def decode_step(self, token: int, want_logits=False):
        nxt = C.c_int32()
        logits = np.empty(self.cfg.vocab, dtype=np.uint16) if want_logits else None
        _check(lib().emx_qwen3_decode_step(self.h, int(token), C.byref(nxt),
                                           logits.ctypes.data if want_logits else None))
        return (nxt.value, logits) if want_logits else nxt.value

    def decode(self, token: int, n: int) -> np.ndarray:
        out = np.empty(n, dtype=np.int32)
        _check(lib().emx_qwen3_decode(self.h, int(token), n, out.ctypes.data))
        return out

    def decode_stream(self, token: int, n: int, on_token) -> int:
        """Per-token streaming (emx_qwen3_decode_stream): on_token(token, index)
        is called as each token is produced; a true return value stops after
        that token.  Returns the number of tokens delivered."""
        err = []

        def cb(tok, idx, _user):
            try:
                return 1 if on_token(int(tok), int(idx)) else 0
            except BaseException as e:  # an exception stops the stream and is raised after it
                err.append(e)
                return 1

        fn = TOKEN_CB(cb)
        done = C.c_int()
        rc = lib().emx_qwen3_decode_stream(self.h, int(token), n, C.cast(fn, C.c_void_p), None, C.byref(done))
        if err:
            raise err[0]
        _check(rc)
        return done.value

    def prefill_device(self, ids: Buffer, T: int):
        _check(lib().emx_qwen3_prefill_device(self.h, ids.ptr, T))

    def decode_device(self, n: int):
        _check(lib().emx_qwen3_decode_device(self.h, n))

    def step_launches(self) -> int:
        v = C.c_int()
        _check(lib().emx_qwen3_step_launches(self.h, C.byref(v)))
        return v.value
