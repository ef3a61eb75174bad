"""Regenerates tests/golden/*.npz from the CPU oracle.

    python tests/golden/make_golden.py

Two kinds of fixture:
  kats.npz  — the known-answer vectors of the reference's own tests, with the
              expected values computed by the reference's own formulas:
              crates/mlx-ffi/tests/grouped_rms_norm.rs:82-200 (reference_groups*),
              crates/serve/tests/forward_grouped_norm.rs:43-83,
              crates/serve/tests/forward_separate.rs:58-62 (pattern() inputs) and
              crates/serve/tests/profile_decode.rs:224-260 (scatter vs slice_update).
  ops.npz   — seeded inputs and oracle outputs for every op on the path, small
              enough for the CPU suite; the GPU tests compare libemx to them.
  tiny_model.npz — a 2-layer random-init Qwen3 (dense int4 + mixed int8/int4)
              prompt, oracle greedy tokens and last logits.
The oracle is test infrastructure; nothing in the product reads these files.
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path[:0] = [os.path.join(ROOT, "oracle"), os.path.join(ROOT, "engine-mlx_b200")]

import emx  # noqa: E402  (host config / tensor list only; no GPU)
import oracle  # noqa: E402


def pattern(n, offset):
    """crates/serve/tests/forward_separate.rs:58-62: ((i*0.013 + offset) % 1.0) - 0.5 in f32."""
    i = np.arange(n, dtype=np.float32)
    return (np.fmod(i * np.float32(0.013) + np.float32(offset), np.float32(1.0)) - np.float32(0.5)).astype(np.float32)


def ref_groups(x, w, eps, groups):
    """reference_groups / reference_groups2 of the reference tests, in f32."""
    x = np.asarray(x, np.float32)
    w = np.asarray(w, np.float32)
    dims = x.shape[-1]
    gd = dims // groups
    out = np.zeros_like(x)
    flat = x.reshape(-1, dims)
    o = out.reshape(-1, dims)
    for r in range(flat.shape[0]):
        for g in range(groups):
            sl = slice(g * gd, (g + 1) * gd)
            ms = np.float32(np.sum(flat[r, sl] * flat[r, sl], dtype=np.float32)) / np.float32(gd)
            rms = np.sqrt(ms + np.float32(eps), dtype=np.float32)
            o[r, sl] = w[sl] * (flat[r, sl] / rms)
    return out


def kats():
    d = {}
    eps = np.float32(1e-5)
    # grouped_rms_norm_groups1_matches_plain / forward_groups1_unchanged
    d["g1_x"] = np.array([1, 2, 3, 4], np.float32)
    d["g1_w"] = np.ones(4, np.float32)
    d["g1_expected"] = ref_groups(d["g1_x"], d["g1_w"], eps, 1)
    # grouped_rms_norm_groups2_matches_reference
    d["g2_x"] = np.array([4, 4, 4, 4], np.float32)
    d["g2_w"] = np.array([1, 2, 3, 4], np.float32)
    d["g2_expected"] = ref_groups(d["g2_x"], d["g2_w"], eps, 2)
    # grouped_rms_norm_groups4
    d["g4_x"] = np.full(8, 4, np.float32)
    d["g4_w"] = np.arange(1, 9, dtype=np.float32)
    d["g4_expected"] = ref_groups(d["g4_x"], d["g4_w"], eps, 4)
    # grouped_rms_norm_multidim: [2,3,4], groups 2
    d["md_x"] = np.full((2, 3, 4), 4, np.float32)
    d["md_w"] = np.array([1, 2, 3, 4], np.float32)
    d["md_expected"] = ref_groups(d["md_x"], d["md_w"], eps, 2)
    # forward_grouped_norm_groups2_matches_reference (bf16 weight, tol 2e-2)
    d["fg_x"] = np.array([1.0, 2.0, 5.0, 8.0], np.float32)
    d["fg_w"] = np.array([1.1, 2.7, 0.5, 3.3], np.float32)
    d["fg_expected"] = ref_groups(d["fg_x"], d["fg_w"], eps, 2)
    # forward_separate.rs: pattern() pieces (qkv 16x64 each at gs 64 int4; gate/up 8x64 at gs 32 int4)
    d["sep_q"] = pattern(16 * 64, 0.00).reshape(16, 64)
    d["sep_k"] = pattern(16 * 64, 0.17).reshape(16, 64)
    d["sep_v"] = pattern(16 * 64, 0.31).reshape(16, 64)
    d["sep_x"] = pattern(2 * 64, 0.07).reshape(2, 64)
    d["sep_gate"] = pattern(8 * 64, 0.11).reshape(8, 64)
    d["sep_up"] = pattern(8 * 64, 0.43).reshape(8, 64)
    d["sep_xg"] = pattern(2 * 64, 0.23).reshape(2, 64)
    # profile_decode.rs scatter_equals_slice_update: cache i*0.5+1 (bf16), update 999 at offset 7
    nkv, cap, hd = 8, 32, 128
    d["sc_cache"] = oracle.to_bf16(np.arange(nkv * cap * hd, dtype=np.float32) * np.float32(0.5) + np.float32(1.0))
    d["sc_update"] = oracle.to_bf16(np.full(nkv * hd, 999.0, np.float32))
    d["sc_dims"] = np.array([nkv, cap, hd, 7], np.int32)
    return d


def ops(seed=1234):
    rng = np.random.default_rng(seed)
    d = {}
    # quantized matmul: every bits x group_size combination at a small shape
    for bits in (4, 8):
        for gs in (32, 64, 128):
            N, K = 64, 1024
            w = oracle.fill_normal(seed, oracle.name_stream(f"qmm{bits}_{gs}"), N * K, 0.0, 0.02).reshape(N, K)
            wq, s, b = oracle.quantize(w, gs, bits)
            x1 = oracle.to_bf16(rng.standard_normal((1, K)).astype(np.float32))
            xm = oracle.to_bf16(rng.standard_normal((32, K)).astype(np.float32))
            tag = f"q{bits}_{gs}"
            d[tag + "_w"], d[tag + "_s"], d[tag + "_b"] = wq, s, b
            d[tag + "_x1"], d[tag + "_xm"] = x1, xm
            d[tag + "_y1"] = oracle.qmatmul(x1, wq, s, b, gs, bits)
            d[tag + "_ym"] = oracle.qmatmul(xm, wq, s, b, gs, bits)
            d[tag + "_deq"] = oracle.dequantize(wq, s, b, gs, bits)
    # norms
    x = oracle.to_bf16(rng.standard_normal((8, 256)).astype(np.float32) * 3)
    wn = oracle.to_bf16(1 + 0.05 * rng.standard_normal(256).astype(np.float32))
    d["norm_x"], d["norm_w"] = x, wn
    d["norm_y"] = oracle.rms_norm(x, wn, 1e-6)
    d["gnorm_y"] = oracle.grouped_rms_norm(x, wn, 1e-6, 4)
    # rope over [heads, T, 128] at offset 37
    xr = oracle.to_bf16(rng.standard_normal((4, 9, 128)).astype(np.float32))
    d["rope_x"] = xr
    d["rope_y"] = oracle.rope(xr, 1e6, 37)
    # elementwise
    a = oracle.to_bf16(rng.standard_normal(4096).astype(np.float32) * 4)
    bb = oracle.to_bf16(rng.standard_normal(4096).astype(np.float32))
    d["ew_a"], d["ew_b"] = a, bb
    d["silu_y"] = oracle.silu(a)
    d["mul_y"] = oracle.multiply(a, bb)
    d["add_y"] = oracle.add(a, bb)
    # attention: causal prefill (GQA 4:2, T=70) and decode over a cache
    T, nq, nkv = 70, 4, 2
    q = oracle.to_bf16(rng.standard_normal((nq, T, 128)).astype(np.float32))
    k = oracle.to_bf16(rng.standard_normal((nkv, T, 128)).astype(np.float32))
    v = oracle.to_bf16(rng.standard_normal((nkv, T, 128)).astype(np.float32))
    sc = np.float32(1 / np.sqrt(128))
    d["att_q"], d["att_k"], d["att_v"] = q, k, v
    d["att_y"] = oracle.sdpa(q, k, v, nkv, T, T, sc, True)
    cap, L = 300, 213
    kc = oracle.to_bf16(rng.standard_normal((nkv, cap, 128)).astype(np.float32))
    vc = oracle.to_bf16(rng.standard_normal((nkv, cap, 128)).astype(np.float32))
    qd = oracle.to_bf16(rng.standard_normal((nq, 1, 128)).astype(np.float32))
    d["dec_q"], d["dec_k"], d["dec_v"], d["dec_len"] = qd, kc, vc, np.array([L], np.int32)
    d["dec_y"] = oracle.sdpa(qd, kc, vc, nkv, L, cap, sc, False)
    # argmax with ties (first index wins) and softmax / top-k routing
    lg = oracle.to_bf16(rng.standard_normal(1000).astype(np.float32))
    lg[[17, 400, 999]] = oracle.to_bf16(np.array([9.0, 9.0, 9.0], np.float32))
    d["am_x"] = lg
    d["am_y"] = np.array([oracle.argmax(lg)], np.int32)
    rl = oracle.to_bf16(rng.standard_normal(128).astype(np.float32))
    d["route_x"] = rl
    probs = oracle.softmax_bf16(rl)
    d["route_p"] = probs
    idx, wt = oracle.topk(oracle_f32(probs), 8, True)
    d["route_idx"], d["route_w"] = idx, wt
    return d


def oracle_f32(b):
    return (np.asarray(b, np.uint16).astype(np.uint32) << 16).view(np.float32)


TINY = {
    "dense_int4": emx.Qwen3Config(hidden=256, layers=2, n_q=4, n_kv=2, inter=512, vocab=1024, kv_cap=256,
                                  max_prefill=64),
    "mixed_int8": emx.Qwen3Config(hidden=256, layers=2, n_q=4, n_kv=2, inter=512, vocab=1024, attn_bits=8,
                                  kv_cap=256, max_prefill=64),
}


def tiny_model(seed=99):
    d = {}
    rng = np.random.default_rng(seed)
    for tag, cfg in TINY.items():
        ck = oracle.make_checkpoint(cfg, seed)
        m = oracle.Model(cfg, ck)
        prompt = rng.integers(0, cfg.vocab, 24).astype(np.int32)
        forced = rng.integers(0, cfg.vocab, 8).astype(np.int32)
        tok, lg = m.prefill(prompt, want_logits=True)
        toks, logits = [tok], [lg]
        for t in forced:  # teacher-forced steps: random inputs, oracle outputs
            nt, lg = m.decode(int(t), want_logits=True)
            toks.append(nt)
            logits.append(lg)
        d[tag + "_prompt"] = prompt
        d[tag + "_forced"] = forced
        d[tag + "_tokens"] = np.array(toks, np.int32)
        d[tag + "_logits"] = np.stack(logits)
        m.close()
    return d


if __name__ == "__main__":
    np.savez_compressed(os.path.join(HERE, "kats.npz"), **kats())
    np.savez_compressed(os.path.join(HERE, "ops.npz"), **ops())
    np.savez_compressed(os.path.join(HERE, "tiny_model.npz"), **tiny_model())
    for f in ("kats.npz", "ops.npz", "tiny_model.npz"):
        print(f, os.path.getsize(os.path.join(HERE, f)))
