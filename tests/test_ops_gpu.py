"""libemx ops vs the CPU oracle, through the C ABI, on an sm_100 GPU.

Bars: dequantized weights, quantized codes, KV writes,
argmax / top-k indices and the elementwise add/multiply are bit-exact; every
other bf16 op output agrees with the oracle to a relative error of 1e-2,
measured per element as |got - ref| <= 1e-2 * (|ref| + rms(ref)).
"""
import os

import numpy as np
import pytest

import emx
import oracle

pytestmark = pytest.mark.gpu

G = os.path.join(os.path.dirname(__file__), "golden")
OPS = np.load(os.path.join(G, "ops.npz"))
KATS = np.load(os.path.join(G, "kats.npz"))
RTOL = 1e-2


@pytest.fixture(scope="module")
def ctx():
    c = emx.Ctx(0)
    yield c
    c.close()


def f32(b):
    return emx.f32(b).astype(np.float64)


def assert_close(got, ref, rtol=RTOL, what=""):
    g, r = f32(got), f32(ref)
    assert g.shape == r.shape, what
    scale = np.sqrt(np.mean(r * r)) + 1e-30
    err = np.abs(g - r)
    bad = err > rtol * (np.abs(r) + scale)
    assert not bad.any(), f"{what}: {int(bad.sum())}/{bad.size} outside rtol={rtol}, max err {err.max():.3g}"


def bf16_ulps(a, b):
    """Distance in bf16 units of last place (same-sign finite values)."""
    ia = np.asarray(a, np.uint16).astype(np.int32)
    ib = np.asarray(b, np.uint16).astype(np.int32)
    sa = np.where(ia & 0x8000, -(ia & 0x7FFF), ia)
    sb = np.where(ib & 0x8000, -(ib & 0x7FFF), ib)
    return np.abs(sa - sb)


# ---------------------------------------------------------- quantized matmul
QCASES = [(4, 32), (4, 64), (4, 128), (8, 32), (8, 64), (8, 128)]


@pytest.mark.parametrize("bits,gs", QCASES)
def test_qmatmul_gemv_matches_oracle(ctx, bits, gs):
    t = f"q{bits}_{gs}"
    w, s, b = (ctx.put(OPS[t + p]) for p in ("_w", "_s", "_b"))
    y = ctx.quantized_matmul(ctx.put(OPS[t + "_x1"]), w, s, b, 1, 64, 1024, gs, bits)
    assert_close(y.read(np.uint16, (1, 64)), OPS[t + "_y1"], what=t)


@pytest.mark.parametrize("bits,gs", QCASES)
def test_qmatmul_gemm_matches_oracle(ctx, bits, gs):
    t = f"q{bits}_{gs}"
    w, s, b = (ctx.put(OPS[t + p]) for p in ("_w", "_s", "_b"))
    y = ctx.quantized_matmul(ctx.put(OPS[t + "_xm"]), w, s, b, 32, 64, 1024, gs, bits)
    assert_close(y.read(np.uint16, (32, 64)), OPS[t + "_ym"], what=t)


@pytest.mark.parametrize("bits,gs", QCASES)
def test_dequantize_bit_exact(ctx, bits, gs):
    t = f"q{bits}_{gs}"
    w, s, b = (ctx.put(OPS[t + p]) for p in ("_w", "_s", "_b"))
    out = ctx.dequantize(w, s, b, 64, 1024, gs, bits).read(np.uint16, (64, 1024))
    assert np.array_equal(out, OPS[t + "_deq"])


@pytest.mark.parametrize("bits,gs", QCASES)
def test_quantize_bit_exact(ctx, bits, gs):
    src = oracle.fill_normal(1234, oracle.name_stream(f"qmm{bits}_{gs}"), 64 * 1024, 0.0, 0.02)
    w, s, b = ctx.quantize(ctx.put(src), emx.F32, 64, 1024, gs, bits)
    t = f"q{bits}_{gs}"
    assert np.array_equal(w.read(np.uint32, OPS[t + "_w"].shape), OPS[t + "_w"])
    assert np.array_equal(s.read(np.uint16, OPS[t + "_s"].shape), OPS[t + "_s"])
    assert np.array_equal(b.read(np.uint16, OPS[t + "_b"].shape), OPS[t + "_b"])


def _linear(seed, name, N, K, gs, bits):
    return oracle.gen_tensor(seed, name, N, K, bits, gs)


# Prefill shapes of the in-kernel-dequant GEMM (K split across a cluster):
# the C3 gate|up, down (int4) and q|k|v, o (int8) projections at up to 128
# rows, ragged row counts included.
PREFILL_LINEARS = [(128, 6144, 2048, 4), (100, 2048, 6144, 4), (77, 4096, 2048, 8), (128, 2048, 2048, 8),
                   (16, 12288, 2048, 4), (3, 512, 1024, 8)]


# the MLX-layout entry dequantises inside the kernel up to 256 rows (two row
# tiles), beyond that through bf16 scratch
@pytest.mark.parametrize("M,N,K,bits", PREFILL_LINEARS + [(200, 2048, 6144, 4), (256, 4096, 2048, 8)])
def test_prefill_linear_shapes(ctx, M, N, K, bits):
    q = _linear(11, f"prefill.{N}x{K}.{bits}", N, K, 64, bits)
    rng = np.random.default_rng(M + N)
    x = oracle.to_bf16(rng.standard_normal((M, K)).astype(np.float32))
    ref = oracle.qmatmul(x, q["weight"], q["scales"], q["biases"], 64, bits)
    y = ctx.quantized_matmul(ctx.put(x), ctx.put(q["weight"]), ctx.put(q["scales"]), ctx.put(q["biases"]), M, N, K,
                             64, bits)
    assert_close(y.read(np.uint16, (M, N)), ref, what=f"prefill linear {M}x{N}x{K} int{bits}")


@pytest.mark.parametrize("M,N,K,bits", PREFILL_LINEARS + [(200, 1024, 2048, 4), (1, 2048, 2048, 8),
                                                      (600, 2048, 2048, 4), (1100, 1024, 2048, 8)])
def test_prefill_linear_packed(ctx, M, N, K, bits):
    """The prefill GEMM over the packed decode layout (emx_qpack) against the
    oracle's MLX-layout matmul of the same tensor; the model takes it up to
    2048 rows (256-token row tiles above 128, ragged ones included)."""
    q = _linear(11, f"prefill.{N}x{K}.{bits}", N, K, 64, bits)
    rng = np.random.default_rng(M + N)
    x = oracle.to_bf16(rng.standard_normal((M, K)).astype(np.float32))
    ref = oracle.qmatmul(x, q["weight"], q["scales"], q["biases"], 64, bits)
    pk = ctx.qpack(ctx.put(q["weight"]), ctx.put(q["scales"]), ctx.put(q["biases"]), N, K, 64, bits)
    y = ctx.quantized_matmul_packed(ctx.put(x), pk, M, N, K, 64, bits)
    assert_close(y.read(np.uint16, (M, N)), ref, what=f"packed prefill linear {M}x{N}x{K} int{bits}")


@pytest.mark.parametrize("M", [1, 128, 512])
def test_config1_single_linear(ctx, M):
    """x bf16 [M, 2048] ~N(0,1); W [6144, 2048] ~N(0, 0.02^2) int4 gs64."""
    N, K = 6144, 2048
    q = _linear(7, "config1.linear", N, K, 64, 4)
    rng = np.random.default_rng(7)
    x = oracle.to_bf16(rng.standard_normal((M, K)).astype(np.float32))
    ref = oracle.qmatmul(x, q["weight"], q["scales"], q["biases"], 64, 4)
    y = ctx.quantized_matmul(ctx.put(x), ctx.put(q["weight"]), ctx.put(q["scales"]), ctx.put(q["biases"]), M, N, K,
                             64, 4)
    assert_close(y.read(np.uint16, (M, N)), ref, what=f"config1 M={M}")


@pytest.mark.parametrize("N,K,bits", [(151936, 2048, 4), (256, 25600, 4), (4096, 2048, 8), (2048, 6144, 4),
                                      (1024, 768, 4), (128, 2048, 4)])
def test_gemv_model_shapes(ctx, N, K, bits):
    """Decode shapes of the configs: lm_head, 32B down (k-split rounds), 1.7B qkv int8,
    1.7B down, MoE expert down (K=768, partial span), router."""
    q = _linear(11, f"shape.{N}.{K}", N, K, 64, bits)
    x = oracle.to_bf16(np.random.default_rng(N + K).standard_normal((1, K)).astype(np.float32))
    ref = oracle.qmatmul(x, q["weight"], q["scales"], q["biases"], 64, bits)
    y = ctx.quantized_matmul(ctx.put(x), ctx.put(q["weight"]), ctx.put(q["scales"]), ctx.put(q["biases"]), 1, N, K,
                             64, bits)
    assert_close(y.read(np.uint16, (1, N)), ref, what=f"N={N} K={K}")


@pytest.mark.parametrize("bits,gs", QCASES)
def test_packed_gemv_matches_oracle(ctx, bits, gs):
    """The engine's decode GEMV (load-time packed layout) on the committed fixtures."""
    t = f"q{bits}_{gs}"
    w, s, b = (ctx.put(OPS[t + p]) for p in ("_w", "_s", "_b"))
    pk = ctx.qpack(w, s, b, 64, 1024, gs, bits)
    y = ctx.quantized_matvec_packed(ctx.put(OPS[t + "_x1"]), pk, 64, 1024, gs, bits)
    got = y.read(np.uint16, (1, 64))
    assert_close(got, OPS[t + "_y1"], what=t)


@pytest.mark.parametrize("N,K,bits", [(151936, 2048, 4), (256, 25600, 4), (4096, 2048, 8), (2048, 6144, 4),
                                      (12288, 2048, 4), (2048, 2048, 8), (1024, 768, 4), (128, 2048, 4),
                                      (2048, 3072, 4), (1536, 2048, 4)])
def test_packed_gemv_model_shapes(ctx, N, K, bits):
    """Decode shapes of the configs through the packed GEMV: lm_head, 32B down,
    1.7B qkv / o int8, 1.7B gate_up / down, MoE expert down (K=768: a half-empty
    last span), router, 0.6B down, MoE expert gate_up."""
    q = _linear(11, f"shape.{N}.{K}", N, K, 64, bits)
    x = oracle.to_bf16(np.random.default_rng(N + K).standard_normal((1, K)).astype(np.float32))
    ref = oracle.qmatmul(x, q["weight"], q["scales"], q["biases"], 64, bits)
    pk = ctx.qpack(ctx.put(q["weight"]), ctx.put(q["scales"]), ctx.put(q["biases"]), N, K, 64, bits)
    got = ctx.quantized_matvec_packed(ctx.put(x), pk, N, K, 64, bits).read(np.uint16, (1, N))
    assert_close(got, ref, what=f"N={N} K={K}")
    # fp32 sums in another order flip the bf16 rounding of a few outputs
    assert np.mean(got != ref) <= 0.03, f"bit-equal fraction {np.mean(got == ref):.4f}"
    assert ctx.device_status() == 0


def test_packed_gemv_rejects_bad_shapes(ctx):
    b = ctx.alloc(1 << 16)
    with pytest.raises(emx.EmxError):
        ctx.quantized_matvec_packed(b, b, 72, 1024, 64, 4)  # N not a multiple of 16
    with pytest.raises(emx.EmxError):
        ctx.quantized_matvec_packed(b, b, 64, 1000, 64, 4)  # K not a multiple of the group
    with pytest.raises(emx.EmxError):
        ctx.qpack(b, b, b, 64, 1024, 64, 3)


def test_qmatmul_rejects_bad_shapes(ctx):
    x = ctx.alloc(4096)
    with pytest.raises(emx.EmxError) as ei:
        ctx.quantized_matmul(x, x, x, x, 1, 16, 100, 64, 4)
    assert ei.value.code == emx.ERR_INVALID
    with pytest.raises(emx.EmxError):
        ctx.quantized_matmul(x, x, x, x, 1, 16, 128, 64, 3)


# ---------------------------------------------------------------- norms etc.
def test_rms_norm(ctx):
    x = OPS["norm_x"]
    out = ctx.rms_norm(ctx.put(x), ctx.put(OPS["norm_w"]), 8, 256, 1e-6).read(np.uint16, x.shape)
    assert_close(out, OPS["norm_y"], what="rms_norm")
    assert bf16_ulps(out, OPS["norm_y"]).max() <= 1


def test_grouped_rms_norm(ctx):
    x = OPS["norm_x"]
    out = ctx.grouped_rms_norm(ctx.put(x), ctx.put(OPS["norm_w"]), 8, 256, 1e-6, 4).read(np.uint16, x.shape)
    assert_close(out, OPS["gnorm_y"], what="grouped_rms_norm")


def test_grouped_rms_norm_reference_kats(ctx):
    """crates/mlx-ffi/tests/grouped_rms_norm.rs + forward_grouped_norm.rs vectors (bf16 weight: tol 2e-2)."""
    for tag, groups in (("g2", 2), ("fg", 2), ("g4", 4), ("g1", 1)):
        x = oracle.to_bf16(KATS[tag + "_x"])[None]
        w = oracle.to_bf16(KATS[tag + "_w"])
        n = x.shape[1]
        out = ctx.grouped_rms_norm(ctx.put(x), ctx.put(w), 1, n, 1e-5, groups).read(np.uint16, (1, n))
        exp = KATS[tag + "_expected"].astype(np.float64)
        assert np.all(np.abs(f32(out)[0] - exp) <= 2e-2 * (1 + np.abs(exp))), tag


def test_grouped_rms_norm_rejects_indivisible(ctx):
    x = ctx.put(oracle.to_bf16(np.array([1, 2, 3, 4], np.float32)))
    with pytest.raises(emx.EmxError) as ei:
        ctx.grouped_rms_norm(x, x, 1, 4, 1e-5, 3)
    assert "divisible" in ei.value.msg


def test_rope(ctx):
    x = OPS["rope_x"]
    out = ctx.rope(ctx.put(x), 4, 9, 128, 1e6, 37).read(np.uint16, x.shape)
    assert_close(out, OPS["rope_y"], what="rope")
    off = ctx.put(np.array([30], np.int32))
    out2 = ctx.rope(ctx.put(x), 4, 9, 128, 1e6, 7, off).read(np.uint16, x.shape)
    assert np.array_equal(out, out2)


def test_elementwise(ctx):
    a, b = ctx.put(OPS["ew_a"]), ctx.put(OPS["ew_b"])
    n = OPS["ew_a"].size
    assert np.array_equal(ctx.multiply(a, b, n).read(np.uint16, (n,)), OPS["mul_y"])
    assert np.array_equal(ctx.add(a, b, n).read(np.uint16, (n,)), OPS["add_y"])
    silu = ctx.silu(a, n).read(np.uint16, (n,))
    assert bf16_ulps(silu, OPS["silu_y"]).max() <= 1


def test_argmax_first_index_on_ties(ctx):
    x = OPS["am_x"]
    got = ctx.argmax(ctx.put(x), 1, x.size).read(np.int32, (1,))
    assert int(got[0]) == int(OPS["am_y"][0]) == 17


def test_softmax_and_route(ctx):
    x = OPS["route_x"]
    p = ctx.softmax(ctx.put(x), 1, x.size).read(np.uint16, (x.size,))
    assert bf16_ulps(p, OPS["route_p"]).max() <= 1
    idx, w = ctx.moe_route(ctx.put(x), 128, 8, True)
    assert np.array_equal(idx.read(np.int32, (8,)), OPS["route_idx"])
    assert np.allclose(w.read(np.float32, (8,)), OPS["route_w"], rtol=1e-5, atol=1e-7)


@pytest.mark.parametrize("E", [128, 256, 300])
def test_route_ties_take_the_lowest_index(ctx, E):
    """Experts with equal router probabilities are taken lowest index first
    (the oracle's stable top-k), for the one-warp routing (up to 256
    experts) and the block one (more)."""
    x = np.full(E, oracle.to_bf16(np.array([-10.0], np.float32))[0], np.uint16)
    hi = oracle.to_bf16(np.array([3.0], np.float32))[0]
    mid = oracle.to_bf16(np.array([2.0], np.float32))[0]
    for i in (3, 7, 40, 64, 100):
        x[i] = hi
    for i in (1, 90, E - 1):
        x[i] = mid
    p = oracle.softmax_bf16(x)
    want_idx, want_w = oracle.topk((p.astype(np.uint32) << 16).view(np.float32), 8, True)
    idx, w = ctx.moe_route(ctx.put(x), E, 8, True)
    got_idx = idx.read(np.int32, (8,))
    assert np.array_equal(got_idx, want_idx), (got_idx, want_idx)
    assert list(got_idx) == [3, 7, 40, 64, 100, 1, 90, E - 1]
    assert np.allclose(w.read(np.float32, (8,)), want_w, rtol=1e-5, atol=1e-7)


# ----------------------------------------------------------------- attention
@pytest.mark.parametrize("tnd", [False, True])
def test_sdpa_causal(ctx, tnd):
    q, k, v = (OPS["att_" + n] for n in "qkv")
    nq, T, D = q.shape
    out = ctx.sdpa_causal(ctx.put(q), ctx.put(k), ctx.put(v), nq, 2, T, D, 1 / np.sqrt(D), out_tnd=tnd)
    got = out.read(np.uint16, (T, nq, D) if tnd else (nq, T, D))
    if tnd:
        got = got.transpose(1, 0, 2)
    assert_close(got, OPS["att_y"], what="sdpa causal")


@pytest.mark.parametrize("T,nq,nkv", [(128, 2, 1), (300, 4, 2), (1000, 4, 1)])
def test_sdpa_causal_tiles(ctx, T, nq, nkv):
    """Several 128-row query and key tiles (diagonal, full and ragged) against the oracle."""
    rng = np.random.default_rng(T)
    q = oracle.to_bf16(rng.standard_normal((nq, T, 128)).astype(np.float32))
    k = oracle.to_bf16(rng.standard_normal((nkv, T, 128)).astype(np.float32))
    v = oracle.to_bf16(rng.standard_normal((nkv, T, 128)).astype(np.float32))
    sc = np.float32(1 / np.sqrt(128))
    ref = oracle.sdpa(q, k, v, nkv, T, T, sc, True)
    got = ctx.sdpa_causal(ctx.put(q), ctx.put(k), ctx.put(v), nq, nkv, T, 128, float(sc)).read(np.uint16, (nq, T, 128))
    assert_close(got, ref, what=f"sdpa causal T={T}")


def test_sdpa_decode(ctx):
    q, kc, vc = OPS["dec_q"], OPS["dec_k"], OPS["dec_v"]
    L = int(OPS["dec_len"][0])
    out = ctx.sdpa_decode(ctx.put(q), ctx.put(kc), ctx.put(vc), 4, 2, 300, 128, L, 1 / np.sqrt(128))
    assert_close(out.read(np.uint16, (4, 1, 128)), OPS["dec_y"], what="sdpa decode")


# --------------------------------------------------------- cache and embed
def test_scatter_single_equals_slice_update(ctx):
    """crates/serve/tests/profile_decode.rs:224-260 — bit-identical writes at offset 7."""
    nkv, cap, hd, off = (int(v) for v in KATS["sc_dims"])
    base = KATS["sc_cache"]
    upd = KATS["sc_update"]
    a = ctx.put(base)
    ctx.slice_update(a, ctx.put(upd), nkv, cap, hd, off, 1)
    b = ctx.put(base)
    ctx.scatter_single(b, ctx.put(np.array([off], np.int32)), ctx.put(upd), nkv, cap, hd)
    ra, rb = a.read(np.uint16, base.shape), b.read(np.uint16, base.shape)
    assert np.array_equal(ra, rb)
    exp = base.reshape(nkv, cap, hd).copy()
    exp[:, off, :] = upd.reshape(nkv, hd)
    assert np.array_equal(ra, exp.reshape(-1))


def test_slice_update_bounds_checked(ctx):
    buf = ctx.alloc(2 * 8 * 16 * 128)
    with pytest.raises(emx.EmxError):
        ctx.slice_update(buf, buf, 2, 8, 128, 6, 4)


def test_embed_quantized_bit_exact(ctx):
    q = _linear(3, "embed.test", 1000, 512, 64, 4)
    ids = np.array([0, 999, 17, 17, 500], np.int32)
    out = ctx.embed_quantized(ctx.put(q["weight"]), ctx.put(q["scales"]), ctx.put(q["biases"]), ctx.put(ids), 5,
                              512, 1000, 64, 4).read(np.uint16, (5, 512))
    full = oracle.dequantize(q["weight"], q["scales"], q["biases"], 64, 4)
    assert np.array_equal(out, full[ids])


def test_embed_bad_token_reported(ctx):
    q = _linear(3, "embed.test", 1000, 512, 64, 4)
    ctx.device_status(clear=True)
    ids = np.array([1000], np.int32)
    ctx.embed_quantized(ctx.put(q["weight"]), ctx.put(q["scales"]), ctx.put(q["biases"]), ctx.put(ids), 1, 512,
                        1000, 64, 4)
    assert ctx.device_status(clear=True) == 3  # EMX_DEV_BAD_TOKEN


# ------------------------------------------------------------- gather qmm
@pytest.mark.parametrize("per_slot", [False, True])
def test_gather_qmm(ctx, per_slot):
    E, N, K, S = 16, 128, 768, 4
    q = oracle.gen_tensor(5, "experts.test", N, K, 4, 64, blocks=E)
    idx = np.array([9, 2, 15, 2], np.int32)
    rng = np.random.default_rng(1)
    x = oracle.to_bf16(rng.standard_normal((S if per_slot else 1, K)).astype(np.float32))
    out = ctx.gather_qmm(ctx.put(x), per_slot, ctx.put(q["weight"]), ctx.put(q["scales"]), ctx.put(q["biases"]),
                         ctx.put(idx), S, E, N, K, 64, 4).read(np.uint16, (S, N))
    for s_, e in enumerate(idx):
        xs = x[s_:s_ + 1] if per_slot else x
        ref = oracle.qmatmul(xs, q["weight"][e], q["scales"][e], q["biases"][e], 64, 4)
        assert_close(out[s_:s_ + 1], ref, what=f"slot {s_}")


def test_memory_accounting(ctx):
    before = ctx.active_memory()
    b = ctx.alloc(1 << 20)
    assert ctx.active_memory() == before + (1 << 20)
    assert ctx.peak_memory() >= before + (1 << 20)
    b.free()
    assert ctx.active_memory() == before
    prev = ctx.set_memory_limit(before + 1024)
    try:
        with pytest.raises(emx.EmxError) as ei:
            ctx.alloc(1 << 20)
        assert ei.value.code == emx.ERR_OOM
    finally:
        ctx.set_memory_limit(prev)
