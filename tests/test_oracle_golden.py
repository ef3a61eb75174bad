"""Pins the CPU oracle (test infrastructure) before it is trusted as the checker.

1. The reference's own known-answer tests, re-run against the oracle with the
   reference's tolerances (tests/golden/kats.npz, see make_golden.py).
2. Properties the reference asserts (fused == separate projections,
   scatter_single == slice_update bit-identical).
3. Independent float64 numpy restatements of each op on small inputs.
4. The committed oracle fixtures (ops.npz, tiny_model.npz) still reproduce
   bit-for-bit, so a silent oracle change cannot move the GPU checks.
"""
import os

import numpy as np
import pytest

import emx
import oracle

G = os.path.join(os.path.dirname(__file__), "golden")
KATS = np.load(os.path.join(G, "kats.npz"))
OPS = np.load(os.path.join(G, "ops.npz"))
TINY = np.load(os.path.join(G, "tiny_model.npz"))


def f32(b):
    return emx.f32(b)


def approx_eq(a, b, tol):
    """approx_eq of crates/mlx-ffi/tests/grouped_rms_norm.rs: |a-b| <= tol*(1+|b|)."""
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return a.shape == b.shape and bool(np.all(np.abs(a - b) <= tol * (1 + np.abs(b))))


# ---------------------------------------------------------------- reference KATs
@pytest.mark.parametrize("tag,groups", [("g1", 1), ("g2", 2), ("g4", 4)])
def test_grouped_rms_norm_kats_f32(tag, groups):
    got = oracle.grouped_rms_norm_f32(KATS[tag + "_x"], KATS[tag + "_w"], 1e-5, groups)[0]
    assert approx_eq(got, KATS[tag + "_expected"], 1e-5)


def test_grouped_rms_norm_multidim_kat():
    x = KATS["md_x"].reshape(-1, 4)
    got = oracle.grouped_rms_norm_f32(x, KATS["md_w"], 1e-5, 2)
    assert approx_eq(got.reshape(2, 3, 4), KATS["md_expected"], 1e-5)


def test_grouped_rms_norm_bf16_weight_kats():
    # grouped_rms_norm_bf16_weight_matches_reference + forward_grouped_norm_groups2 (tol 2e-2)
    for tag in ("g2", "fg"):
        x = oracle.to_bf16(KATS[tag + "_x"])[None]
        w = oracle.to_bf16(KATS[tag + "_w"])
        got = f32(oracle.grouped_rms_norm(x, w, 1e-5, 2))[0]
        assert approx_eq(got, KATS[tag + "_expected"], 2e-2)


def test_groups1_equals_plain_rms_norm():
    x = oracle.to_bf16(KATS["g1_x"])[None]
    w = oracle.to_bf16(KATS["g1_w"])
    assert np.array_equal(oracle.grouped_rms_norm(x, w, 1e-5, 1), oracle.rms_norm(x, w, 1e-5))
    assert approx_eq(f32(oracle.rms_norm(x, w, 1e-5))[0], KATS["g1_expected"], 1e-2)


def _fused_vs_separate(pieces, x, gs):
    parts = [oracle.quantize(p, gs, 4) for p in pieces]
    fused = [np.concatenate([p[i] for p in parts], axis=0) for i in range(3)]
    xb = oracle.to_bf16(x)
    y_f = oracle.qmatmul(xb, *fused, gs, 4)
    y_s = np.concatenate([oracle.qmatmul(xb, *p, gs, 4) for p in parts], axis=1)
    return y_f, y_s


def test_qkv_separate_matches_fused():
    # crates/serve/tests/forward_separate.rs:96-131 (16x64 pieces, gs 64, int4, x [2,64]); tol 1e-3
    y_f, y_s = _fused_vs_separate([KATS["sep_q"], KATS["sep_k"], KATS["sep_v"]], KATS["sep_x"], 64)
    assert y_f.shape == (2, 48)
    assert np.max(np.abs(f32(y_f) - f32(y_s))) < 1e-3


def test_gate_up_separate_matches_fused():
    # crates/serve/tests/forward_separate.rs:133-162 (8x64 pieces, gs 32); tol 1e-3
    y_f, y_s = _fused_vs_separate([KATS["sep_gate"], KATS["sep_up"]], KATS["sep_xg"], 32)
    assert y_f.shape == (2, 16)
    assert np.max(np.abs(f32(y_f) - f32(y_s))) < 1e-3


def test_scatter_single_equals_slice_update():
    # crates/serve/tests/profile_decode.rs:224-260: bit-identical writes
    nkv, cap, hd, off = (int(v) for v in KATS["sc_dims"])
    base = KATS["sc_cache"].reshape(nkv, cap, hd)
    upd = KATS["sc_update"].reshape(nkv, 1, hd)
    via_slice = base.copy()
    via_slice[:, off:off + 1, :] = upd
    via_oracle = base.copy()
    oracle.lib().orc_slice_update(via_oracle.ctypes.data, np.ascontiguousarray(upd).ctypes.data, nkv, cap, hd, off, 1)
    assert np.array_equal(via_slice, via_oracle)


# ------------------------------------------------------ independent restatements
def test_quantize_formula_and_roundtrip():
    rng = np.random.default_rng(0)
    for bits in (4, 8):
        for gs in (32, 64, 128):
            w = (rng.standard_normal((16, 512)) * 0.02).astype(np.float32)
            wq, s, b = oracle.quantize(w, gs, bits)
            g = w.reshape(16, -1, gs)
            mn, mx = g.min(-1), g.max(-1)
            assert np.array_equal(s, oracle.to_bf16((mx - mn) / np.float32(2 ** bits - 1)))
            assert np.array_equal(b, oracle.to_bf16(mn))
            deq = f32(oracle.dequantize(wq, s, b, gs, bits)).reshape(16, -1, gs)
            sf = f32(s)[..., None]
            assert np.all(np.abs(deq - g) <= 0.5 * sf + 0.01 * np.abs(g) + 1e-6)


def test_dequantize_is_exactly_rounded():
    """Each element is the bf16 nearest to s*q+b (float64 is exact here)."""
    wq, s, b = OPS["q4_64_w"], OPS["q4_64_s"], OPS["q4_64_b"]
    q = np.stack([(wq >> (4 * i)) & 0xF for i in range(8)], axis=-1).reshape(wq.shape[0], -1).astype(np.float64)
    sf = np.repeat(f32(s).astype(np.float64), 64, axis=1)
    bf = np.repeat(f32(b).astype(np.float64), 64, axis=1)
    exact = sf * q + bf
    deq = f32(OPS["q4_64_deq"]).astype(np.float64)
    up = f32(oracle.to_bf16(exact.astype(np.float32))).astype(np.float64)
    # the stored value is one of the two bf16 neighbours and the nearer one
    err = np.abs(deq - exact)
    assert np.all(err <= np.abs(up - exact) + 1e-30)


@pytest.mark.parametrize("bits,gs", [(4, 32), (4, 64), (4, 128), (8, 32), (8, 64), (8, 128)])
def test_qmatmul_vs_float64(bits, gs):
    tag = f"q{bits}_{gs}"
    deq = f32(OPS[tag + "_deq"]).astype(np.float64)
    for xs, ys in (("_x1", "_y1"), ("_xm", "_ym")):
        x = f32(OPS[tag + xs]).astype(np.float64)
        ref = x @ deq.T
        got = f32(OPS[tag + ys]).astype(np.float64)
        assert np.max(np.abs(got - ref)) <= 1e-2 * np.max(np.abs(ref))


def test_rms_norm_vs_float64():
    x = f32(OPS["norm_x"]).astype(np.float64)
    w = f32(OPS["norm_w"]).astype(np.float64)
    ref = x / np.sqrt((x * x).mean(-1, keepdims=True) + 1e-6) * w
    assert np.allclose(f32(OPS["norm_y"]), ref, rtol=1e-2, atol=1e-2)


def test_rope_vs_float64():
    x = f32(OPS["rope_x"]).astype(np.float64)
    H, T, D = x.shape
    half = D // 2
    inv = 1e6 ** (-np.arange(half) * 2.0 / D)
    pos = 37 + np.arange(T)
    th = pos[:, None] * inv[None]
    c, s = np.cos(th), np.sin(th)
    x1, x2 = x[..., :half], x[..., half:]
    ref = np.concatenate([x1 * c - x2 * s, x1 * s + x2 * c], -1)
    assert np.allclose(f32(OPS["rope_y"]), ref, rtol=1e-2, atol=2e-2)


def test_sdpa_vs_float64():
    q, k, v = (f32(OPS["att_" + n]).astype(np.float64) for n in "qkv")
    nq, T, D = q.shape
    rep = nq // k.shape[0]
    ref = np.zeros_like(q)
    for h in range(nq):
        s = q[h] @ k[h // rep].T / np.sqrt(D)
        s = np.where(np.tril(np.ones((T, T))) > 0, s, -np.inf)
        p = np.exp(s - s.max(-1, keepdims=True))
        ref[h] = (p / p.sum(-1, keepdims=True)) @ v[h // rep]
    assert np.allclose(f32(OPS["att_y"]), ref, rtol=1e-2, atol=1e-2)


def test_argmax_first_index_on_ties():
    assert int(OPS["am_y"][0]) == 17


def test_topk_stable_and_renormalised():
    p = f32(OPS["route_p"])
    idx, w = OPS["route_idx"], OPS["route_w"]
    order = sorted(range(len(p)), key=lambda i: (-p[i], i))[:8]
    assert list(idx) == order
    assert abs(float(w.sum()) - 1.0) < 1e-6


# -------------------------------------------------------- fixture reproduction
def test_fixtures_reproduce():
    import importlib.util

    spec = importlib.util.spec_from_file_location("make_golden", os.path.join(G, "make_golden.py"))
    mg = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mg)
    for name, fresh in (("ops", mg.ops()), ("tiny", mg.tiny_model())):
        ref = OPS if name == "ops" else TINY
        for k, v in fresh.items():
            assert np.array_equal(ref[k], v), f"{name}:{k} no longer reproduces"


def test_generator_statistics():
    z = oracle.fill_normal(5, oracle.name_stream("stats"), 200000, 0.0, 1.0)
    assert abs(float(z.mean())) < 0.01 and abs(float(z.std()) - 1.0) < 0.01
    z2 = oracle.fill_normal(5, oracle.name_stream("stats"), 1000, 0.0, 1.0)
    assert np.array_equal(z[:1000], z2)


def test_sum_order_switch_changes_only_rounding():
    """The descending-order reductions (used to measure the noise floor) give a
    different but equally valid fp32 evaluation, and the switch resets."""
    rng = np.random.default_rng(5)
    x = oracle.to_bf16(rng.standard_normal((8, 2048)).astype(np.float32))
    wq, s, b = oracle.quantize(oracle.to_bf16(rng.standard_normal((1024, 2048)).astype(np.float32) * 0.02), 64, 4)
    fwd = oracle.qmatmul(x, wq, s, b, 64, 4)
    oracle.lib().orc_set_sum_order(1)
    try:
        rev = oracle.qmatmul(x, wq, s, b, 64, 4)
    finally:
        oracle.lib().orc_set_sum_order(0)
    again = oracle.qmatmul(x, wq, s, b, 64, 4)
    assert np.array_equal(fwd, again)
    ulps = np.abs(fwd.astype(np.int32) - rev.astype(np.int32))
    assert ulps.max() <= 1 and 0 < np.count_nonzero(ulps) < ulps.size // 100
