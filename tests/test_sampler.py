"""The host sampler's restatement in the CPU oracle (crates/serve/src/sampler.rs).

Pinned by the reference's own sampler tests (crates/serve/tests/sampler.rs),
by an independent NumPy restatement of sample_token in float32 with the same
sequential sums and stable sorts, and by the SimpleRng stream (xorshift64*)
restated in Python integers.
"""
import numpy as np
import pytest

import oracle

F32 = np.float32


def py_rng(seed):
    """SimpleRng (sampler.rs:50-78) in Python integers."""
    s = seed if seed else 0x9E3779B97F4A7C15
    mask = (1 << 64) - 1
    while True:
        s ^= s >> 12
        s ^= (s << 25) & mask
        s ^= s >> 27
        out = (s * 0x2545F4914F6CDD1D) & mask
        yield s, F32((out >> 11) / float(1 << 53))


def py_sample(logits, temperature, top_p, top_k, r):
    """sample_token (sampler.rs:101-202) in float32, sequential sums, stable sorts."""
    x = np.asarray(logits, dtype=F32)
    n = x.size
    if temperature < 1e-6:
        return int(n - 1 - np.argmax(x[::-1]))
    t = F32(max(temperature, 1e-6))
    f = (x / t).astype(F32)
    if 0 < top_k < n:
        order = sorted(range(n), key=lambda i: -f[i])  # stable
        kth = f[order[top_k - 1]]
        f = np.where(f < kth, F32(-np.inf), f).astype(F32)
    fin = np.isfinite(f)
    mx = F32(np.max(f[fin]))
    e = np.where(fin, np.exp((f - mx).astype(F32)), F32(0)).astype(F32)
    s = F32(0)
    for v in e:
        s = F32(s + v)
    p = (e / s).astype(F32)
    order = sorted(range(n), key=lambda i: -p[i])
    keep = np.zeros(n, bool)
    cum = F32(0)
    for i in order:
        cum = F32(cum + p[i])
        keep[i] = True
        if cum >= F32(top_p):
            break
    fs = F32(0)
    for i in range(n):
        if keep[i]:
            fs = F32(fs + p[i])
    q = np.where(keep, (p / fs).astype(F32), F32(0)).astype(F32)
    cs = F32(0)
    for i in range(n):
        cs = F32(cs + q[i])
        if r < cs:
            return i
    return int(np.nonzero(keep)[0][-1])


# crates/serve/tests/sampler.rs:8-13
def test_greedy_picks_max():
    tok, _ = oracle.sample_token(np.array([1.0, 5.0, 2.0, 3.0], F32), 0.0, 1.0, 0, oracle.rng_seed(42))
    assert tok == 1


# crates/serve/tests/sampler.rs:15-25
def test_temperature_diversifies():
    tok, _ = oracle.sample_token(np.array([1.0, 5.0, 2.0, 3.0, 4.0], F32), 1.0, 1.0, 0, oracle.rng_seed(1))
    assert 0 <= tok < 5


# crates/serve/tests/sampler.rs:27-39
def test_top_k_filters():
    st = oracle.rng_seed(0)
    for _ in range(20):
        tok, st = oracle.sample_token(np.array([10.0, 9.0, 1.0, 1.0, 1.0], F32), 1.0, 1.0, 2, st)
        assert tok in (0, 1)


def test_rng_stream_matches_the_restatement():
    import ctypes as C

    for seed in (0, 1, 42, 123, 2**63 + 5):
        st = oracle.rng_seed(seed)
        gen = py_rng(seed)
        for _ in range(50):
            state, want = next(gen)
            c = C.c_uint64(st)
            got = oracle.lib().orc_rng_next_f32(C.cast(C.byref(c), C.c_void_p))
            st = c.value
            assert st == state
            assert F32(got) == want


@pytest.mark.parametrize("temperature,top_p,top_k", [(1.0, 1.0, 0), (0.7, 0.9, 0), (0.8, 0.9, 40), (1.3, 0.5, 5),
                                                     (0.5, 0.0, 0), (2.0, 1.0, 100)])
def test_sample_token_matches_the_numpy_restatement(temperature, top_p, top_k):
    rng = np.random.default_rng(int(temperature * 100) + top_k)
    for trial in range(12):
        n = int(rng.integers(2, 300))
        x = (rng.normal(size=n) * 3).astype(F32)
        if trial % 3 == 0:
            x[rng.integers(0, n, size=max(1, n // 4))] = x[0]  # ties
        seed = int(rng.integers(0, 2**63))
        st = oracle.rng_seed(seed)
        gen = py_rng(seed)
        for _ in range(3):
            tok, st = oracle.sample_token(x, temperature, top_p, top_k, st)
            _, r = next(gen)
            assert tok == py_sample(x, temperature, top_p, top_k, r)
