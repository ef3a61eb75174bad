"""ctypes wrapper of oracle/lib/liboracle.so — TEST INFRASTRUCTURE ONLY.

The CPU restatement of engine-mlx's quantized Qwen3 path (see emx_oracle.h
for what it restates and what is pinned).  Only tests/, __graft_entry__.smoke()
and bench.py's cpu_baseline / --impl reference legs import this module; the
product (engine-mlx_b200/) never does.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "lib", "liboracle.so")

_P = C.c_void_p
_SIGS = {
    "orc_f32_to_bf16": (C.c_uint16, [C.c_float]),
    "orc_f64_to_bf16": (C.c_uint16, [C.c_double]),
    "orc_num_threads": (C.c_int, []),
    "orc_set_num_threads": (None, [C.c_int]),
    "orc_set_sum_order": (None, [C.c_int]),
    "orc_name_stream": (C.c_uint64, [C.c_char_p]),
    "orc_fill_normal": (None, [C.c_uint64, C.c_uint64, C.c_size_t, C.c_float, C.c_float, _P]),
    "orc_quantize": (None, [_P, C.c_int, C.c_int, C.c_int, C.c_int, _P, _P, _P]),
    "orc_dequantize": (None, [_P, _P, _P, C.c_int, C.c_int, C.c_int, C.c_int, _P]),
    "orc_qmatmul": (None, [_P, _P, _P, _P, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, _P]),
    "orc_rms_norm": (None, [_P, _P, C.c_int, C.c_int, C.c_float, _P]),
    "orc_grouped_rms_norm": (None, [_P, _P, C.c_int, C.c_int, C.c_float, C.c_int, _P]),
    "orc_grouped_rms_norm_f32": (None, [_P, _P, C.c_int, C.c_int, C.c_float, C.c_int, _P]),
    "orc_rope": (None, [_P, C.c_int, C.c_int, C.c_int, C.c_float, C.c_int, _P]),
    "orc_rope_inv_freq": (None, [C.c_int, C.c_float, _P]),
    "orc_silu": (None, [_P, C.c_size_t, _P]),
    "orc_multiply": (None, [_P, _P, C.c_size_t, _P]),
    "orc_add": (None, [_P, _P, C.c_size_t, _P]),
    "orc_argmax": (C.c_int, [_P, C.c_int]),
    "orc_rng_seed": (C.c_uint64, [C.c_uint64]),
    "orc_rng_next_f32": (C.c_float, [_P]),
    "orc_sample_token": (C.c_int, [_P, C.c_int, C.c_float, C.c_float, C.c_int, _P]),
    "orc_sdpa": (None, [_P, _P, _P] + [C.c_int] * 6 + [C.c_float, C.c_int, _P]),
    "orc_slice_update": (None, [_P, _P] + [C.c_int] * 5),
    "orc_softmax_bf16": (None, [_P, C.c_int, _P]),
    "orc_topk": (None, [_P, C.c_int, C.c_int, C.c_int, _P, _P]),
    "orc_qwen3_create": (_P, [_P]),
    "orc_qwen3_destroy": (None, [_P]),
    "orc_qwen3_set_tensor": (C.c_int, [_P, C.c_char_p, _P]),
    "orc_qwen3_reset": (C.c_int, [_P]),
    "orc_qwen3_prefill": (C.c_int, [_P, _P, C.c_int, _P]),
    "orc_qwen3_decode": (C.c_int, [_P, C.c_int32, _P]),
    "orc_qwen3_offset": (C.c_int, [_P]),
    "orc_qwen3_kv": (_P, [_P, C.c_int, C.c_int]),
}

_lib = None


def build():
    subprocess.run(["make", "-s", "-C", HERE], check=True)


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB):
            build()
        L = C.CDLL(LIB)
        for n, (r, a) in _SIGS.items():
            f = getattr(L, n)
            f.restype = r
            f.argtypes = a
        _lib = L
    return _lib


def _p(a):
    return a.ctypes.data


def _c(a, dt):
    return np.ascontiguousarray(a, dtype=dt)


def name_stream(name: str) -> int:
    return lib().orc_name_stream(name.encode())


def fill_normal(seed: int, stream: int, n: int, mean: float, std: float) -> np.ndarray:
    out = np.empty(n, dtype=np.float32)
    lib().orc_fill_normal(C.c_uint64(seed), C.c_uint64(stream), n, mean, std, _p(out))
    return out


def quantize(w: np.ndarray, gs: int, bits: int):
    w = _c(w, np.float32)
    N, K = w.shape
    wq = np.empty((N, K * bits // 32), dtype=np.uint32)
    s = np.empty((N, K // gs), dtype=np.uint16)
    b = np.empty((N, K // gs), dtype=np.uint16)
    lib().orc_quantize(_p(w), N, K, gs, bits, _p(wq), _p(s), _p(b))
    return wq, s, b


def dequantize(wq, s, b, gs, bits):
    N = wq.shape[0]
    K = wq.shape[1] * 32 // bits
    out = np.empty((N, K), dtype=np.uint16)
    lib().orc_dequantize(_p(_c(wq, np.uint32)), _p(_c(s, np.uint16)), _p(_c(b, np.uint16)), N, K, gs, bits, _p(out))
    return out


def qmatmul(x, wq, s, b, gs, bits):
    x = _c(x, np.uint16)
    M, K = x.shape
    N = wq.shape[0]
    y = np.empty((M, N), dtype=np.uint16)
    lib().orc_qmatmul(_p(x), _p(_c(wq, np.uint32)), _p(_c(s, np.uint16)), _p(_c(b, np.uint16)), M, N, K, gs, bits,
                      _p(y))
    return y


def rms_norm(x, w, eps):
    x = _c(x, np.uint16)
    rows, dims = x.shape
    out = np.empty_like(x)
    lib().orc_rms_norm(_p(x), _p(_c(w, np.uint16)), rows, dims, eps, _p(out))
    return out


def grouped_rms_norm(x, w, eps, groups):
    x = _c(x, np.uint16)
    rows, dims = x.shape
    out = np.empty_like(x)
    lib().orc_grouped_rms_norm(_p(x), _p(_c(w, np.uint16)), rows, dims, eps, groups, _p(out))
    return out


def grouped_rms_norm_f32(x, w, eps, groups):
    x = _c(x, np.float32)
    if x.ndim == 1:
        x = x[None]
    rows, dims = x.shape
    out = np.empty_like(x)
    lib().orc_grouped_rms_norm_f32(_p(x), _p(_c(w, np.float32)), rows, dims, eps, groups, _p(out))
    return out


def rope(x, theta, offset):
    x = _c(x, np.uint16)
    heads, T, dims = x.shape
    out = np.empty_like(x)
    lib().orc_rope(_p(x), heads, T, dims, theta, offset, _p(out))
    return out


def silu(x):
    x = _c(x, np.uint16)
    out = np.empty_like(x)
    lib().orc_silu(_p(x), x.size, _p(out))
    return out


def multiply(a, b):
    a, b = _c(a, np.uint16), _c(b, np.uint16)
    out = np.empty_like(a)
    lib().orc_multiply(_p(a), _p(b), a.size, _p(out))
    return out


def add(a, b):
    a, b = _c(a, np.uint16), _c(b, np.uint16)
    out = np.empty_like(a)
    lib().orc_add(_p(a), _p(b), a.size, _p(out))
    return out


def argmax(x):
    x = _c(x, np.uint16)
    return lib().orc_argmax(_p(x), x.size)


def rng_seed(seed: int) -> int:
    return int(lib().orc_rng_seed(C.c_uint64(seed)))


def sample_token(logits_f32, temperature, top_p, top_k, state: int):
    """sampler.rs sample_token on f32 logits; returns (token, new rng state)."""
    x = _c(logits_f32, np.float32)
    st = C.c_uint64(state)
    tok = lib().orc_sample_token(_p(x), x.size, temperature, top_p, int(top_k), C.cast(C.byref(st), C.c_void_p))
    return tok, st.value


def sdpa(q, k, v, nkv, Tk, kv_stride, scale, causal):
    q = _c(q, np.uint16)
    nq, Tq, D = q.shape
    out = np.empty_like(q)
    lib().orc_sdpa(_p(q), _p(_c(k, np.uint16)), _p(_c(v, np.uint16)), nq, nkv, Tq, Tk, kv_stride, D, scale,
                   int(causal), _p(out))
    return out


def softmax_bf16(x):
    x = _c(x, np.uint16)
    out = np.empty_like(x)
    lib().orc_softmax_bf16(_p(x), x.size, _p(out))
    return out


def topk(scores, k, normalize):
    s = _c(scores, np.float32)
    idx = np.empty(k, dtype=np.int32)
    w = np.empty(k, dtype=np.float32)
    lib().orc_topk(_p(s), s.size, k, int(normalize), _p(idx), _p(w))
    return idx, w


# ------------------------------------------------------------- checkpoints
def gen_tensor(seed: int, base: str, N: int, K: int, bits: int, gs: int, blocks: int = 0):
    """The synthetic quantized tensor `base` (weight/scales/biases), bit-identical
    to what emx_qwen3_init_random puts on the device."""
    rows = N * (blocks or 1)
    w = fill_normal(seed, name_stream(base), rows * K, 0.0, 0.02).reshape(rows, K)
    wq, s, b = quantize(w, gs, bits)
    if blocks:
        wq, s, b = (a.reshape(blocks, N, -1) for a in (wq, s, b))
    return {"weight": wq, "scales": s, "biases": b}


def to_bf16(x) -> np.ndarray:
    """float32 -> bf16 bit patterns, round-to-nearest-even (orc_f32_to_bf16)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def gen_norm(seed: int, name: str, n: int):
    return to_bf16(fill_normal(seed, name_stream(name), n, 1.0, 0.05))


def make_checkpoint(cfg, seed: int):
    """name -> host array for every tensor of the config (emx.checkpoint_tensors layout)."""
    import emx  # the tensor list lives with the host binding

    out = {}
    done = set()
    for name, (shape, dt, kind, bits, gs, base, N, K, blocks) in emx.checkpoint_tensors(cfg).items():
        if kind == "norm":
            out[name] = gen_norm(seed, name, N)
        elif base not in done:
            done.add(base)
            for part, arr in gen_tensor(seed, base, N, K, bits, gs, blocks).items():
                out[f"{base}.{part}"] = arr
    return out


class Model:
    """orc_qwen3_* — the CPU restatement of Qwen3Engine prefill/decode."""

    def __init__(self, cfg, tensors):
        # packed in the field order of orc_qwen3_config (emx_oracle.h)
        fields = [cfg.hidden, cfg.layers, cfg.n_q, cfg.n_kv, cfg.head_dim, cfg.inter, cfg.vocab]
        arr = (C.c_int * 7)(*fields)
        raw = bytearray(bytes(arr))
        raw += bytes((C.c_float * 2)(cfg.eps, cfg.rope_theta))
        ints = [int(cfg.tied), cfg.norm_groups, cfg.attn_bits, cfg.attn_group, cfg.mlp_bits, cfg.mlp_group,
                cfg.embed_bits, cfg.embed_group, cfg.lm_bits, cfg.lm_group, cfg.n_experts, cfg.top_k, cfg.moe_inter,
                int(cfg.norm_topk), cfg.router_bits, cfg.router_group, cfg.expert_bits, cfg.expert_group,
                cfg.kv_cap]
        raw += bytes((C.c_int * len(ints))(*ints))
        self._cfgbuf = C.create_string_buffer(bytes(raw), len(raw))
        self.h = lib().orc_qwen3_create(self._cfgbuf)
        self.cfg = cfg
        self._keep = []
        for name, a in tensors.items():
            a = np.ascontiguousarray(a)
            self._keep.append(a)
            if lib().orc_qwen3_set_tensor(self.h, name.encode(), _p(a)) != 0:
                raise KeyError(name)

    def close(self):
        if self.h:
            lib().orc_qwen3_destroy(self.h)
            self.h = None

    def reset(self):
        lib().orc_qwen3_reset(self.h)

    @property
    def offset(self):
        return lib().orc_qwen3_offset(self.h)

    def prefill(self, tokens, want_logits=False):
        ids = np.ascontiguousarray(np.asarray(tokens, dtype=np.int32))
        logits = np.empty(self.cfg.vocab, dtype=np.uint16)
        t = lib().orc_qwen3_prefill(self.h, _p(ids), len(ids), _p(logits))
        if t < 0:
            raise RuntimeError(f"oracle prefill failed ({t})")
        return (t, logits) if want_logits else t

    def decode(self, token, want_logits=False):
        logits = np.empty(self.cfg.vocab, dtype=np.uint16)
        t = lib().orc_qwen3_decode(self.h, int(token), _p(logits))
        if t < 0:
            raise RuntimeError(f"oracle decode failed ({t})")
        return (t, logits) if want_logits else t

    def kv(self, layer, which):
        per = self.cfg.n_kv * self.cfg.kv_cap * self.cfg.head_dim
        p = lib().orc_qwen3_kv(self.h, layer, which)
        return np.ctypeslib.as_array(C.cast(p, C.POINTER(C.c_uint16)), shape=(per,)).reshape(
            self.cfg.n_kv, self.cfg.kv_cap, self.cfg.head_dim)
