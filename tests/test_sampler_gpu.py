"""Device sampling (emx_sample_token, emx_qwen3_set_sampling) against the CPU
oracle's restatement of the host sampler (crates/serve/src/sampler.rs:101-202).

The generator stream is bit-exact, so both sides draw the same r.  The host
sums sequentially in fp32 and the device per slice; a token may differ only
when r lies within the accumulated rounding of a CDF boundary, and then the
two tokens are neighbours in the kept distribution.  Such draws are checked
against a float64 CDF and must be rare.
"""
import numpy as np
import pytest

import emx
import oracle

pytestmark = pytest.mark.gpu

F32 = np.float32


@pytest.fixture(scope="module")
def ctx():
    c = emx.Ctx(0)
    yield c
    c.close()


def cdf64(x, temperature, top_p, top_k):
    """The kept, renormalised distribution in float64 (index order CDF)."""
    f = x.astype(np.float64) / max(temperature, 1e-6)
    n = f.size
    if 0 < top_k < n:
        kth = np.sort(f)[::-1][top_k - 1]
        f = np.where(f < kth, -np.inf, f)
    e = np.exp(f - f[np.isfinite(f)].max())
    p = e / e.sum()
    order = np.argsort(-p, kind="stable")
    keep = np.zeros(n, bool)
    c = 0.0
    for i in order:
        c += p[i]
        keep[i] = True
        if top_p < 1.0 and c >= top_p:
            break
    q = np.where(keep, p, 0.0)
    return np.cumsum(q / q.sum())


def check_draws(ctx, x, temperature, top_p, top_k, seed, draws):
    n = x.size
    lg = ctx.put(emx.bf16(x))
    xs = emx.f32(emx.bf16(x))  # the bf16 logits the device reads
    st = oracle.rng_seed(seed)
    rng = ctx.put(np.array([st], dtype=np.uint64))
    cdf = cdf64(xs, temperature, top_p, top_k)
    tol = max(2e-4, 4e-6 * np.sqrt(n))  # fp32 running sums over n entries
    mism = 0
    for _ in range(draws):
        g = int(ctx.sample_token(lg, n, temperature, top_p, top_k, rng).read(np.int32, 1)[0])
        prev = st
        o, st = oracle.sample_token(xs, temperature, top_p, top_k, st)
        dev_state = int(rng.read(np.uint64, 1)[0])
        assert dev_state == st  # one xorshift64* step per draw, bit-exact
        if g != o:
            mism += 1
            import ctypes as C

            c = C.c_uint64(prev)
            r = float(oracle.lib().orc_rng_next_f32(C.cast(C.byref(c), C.c_void_p)))
            lo, hi = min(g, o), max(g, o)
            # neighbours: no kept mass strictly between them, r at their boundary
            assert cdf[hi - 1] - cdf[lo] < tol, (g, o)
            assert abs(r - cdf[lo]) < tol, (g, o, r, cdf[lo])
    return mism


@pytest.mark.parametrize("n", [2048, 151936])
@pytest.mark.parametrize("temperature,top_p,top_k", [(1.0, 1.0, 0), (0.7, 0.9, 0), (0.8, 0.9, 40), (1.3, 0.5, 5),
                                                     (0.6, 0.95, 2000)])
def test_device_sampler_matches_the_oracle(ctx, n, temperature, top_p, top_k):
    rng = np.random.default_rng(n + top_k)
    x = (rng.normal(size=n) * 4).astype(F32)
    draws = 40 if n > 10000 else 120
    mism = check_draws(ctx, x, temperature, top_p, top_k, seed=int(rng.integers(0, 2**63)), draws=draws)
    assert mism <= max(3, draws // 10)


def test_ties_and_peaked_distributions(ctx):
    n = 4096
    x = np.full(n, -20.0, F32)  # a tail of negligible mass
    x[[5, 77, 1000, 3001]] = 6.0  # four tied leaders
    x[[9, 10]] = 5.5
    for tp, tk in ((0.5, 0), (0.0, 0), (1.0, 3), (0.9, 5)):
        assert check_draws(ctx, x, 1.0, tp, tk, seed=7, draws=60) == 0


def test_engine_sampling_equals_the_op_on_its_logits(ctx):
    cfg = emx.Qwen3Config(hidden=512, layers=2, n_q=8, n_kv=2, inter=1024, vocab=2048, kv_cap=128, max_prefill=32)
    m = emx.Qwen3(ctx, cfg)
    m.init_random(5)
    prompt = np.array([3, 14, 15, 92, 65, 35], np.int32)
    T, P, K, S = 0.8, 0.9, 40, 123
    m.set_sampling(T, P, K, S)
    st = ctx.put(np.array([S], dtype=np.uint64))
    tok, logits = m.prefill(prompt, want_logits=True)
    want = int(ctx.sample_token(ctx.put(logits), cfg.vocab, T, P, K, st).read(np.int32, 1)[0])
    assert tok == want
    toks = [tok]
    for _ in range(6):
        tok, logits = m.decode_step(tok, want_logits=True)
        want = int(ctx.sample_token(ctx.put(logits), cfg.vocab, T, P, K, st).read(np.int32, 1)[0])
        assert tok == want
        toks.append(tok)
    # n steps with one host synchronisation draw the same stream
    m.reset()
    m.set_sampling(T, P, K, S)
    first = m.prefill(prompt)
    rest = [int(t) for t in m.decode(first, 6)]
    assert [first] + rest == toks
    # greedy again: the in-graph argmax
    m.reset()
    m.set_sampling(0.0)
    g = m.prefill(prompt, want_logits=True)
    assert g[0] == oracle.argmax(g[1])
    m.close()
