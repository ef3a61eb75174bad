"""A plain C program (engine-mlx_b200/capi/greedy.c, built by gcc against
include/emx.h with engine-mlx_b200/capi/Makefile) drives the library the way a
non-Python host does: context, model, seeded weights, prefill, greedy decode,
and the per-token stream.  Its tokens must be the ones the Python binding gets
from the same calls, the streamed ones the decoded ones, and the greedy chain
must pass the oracle's bar (each token the oracle's argmax, or within twice
its noise floor)."""
import os
import subprocess

import numpy as np
import pytest

import emx
from test_model_gpu import check_steps, noise_floor, oracle_run

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CAPI = os.path.join(ROOT, "engine-mlx_b200", "capi")


@pytest.fixture(scope="module")
def greedy_bin():
    subprocess.run(["make", "-s", "-C", CAPI], check=True)
    return os.path.join(CAPI, "greedy")


@pytest.mark.parametrize("shape", [(256, 2, 4, 2, 512, 1024, 8), (512, 3, 8, 2, 1024, 2048, 4)],
                         ids=["mixed_int8", "dense_int4"])
def test_c_caller_matches_python_and_oracle(greedy_bin, shape):
    hidden, layers, n_q, n_kv, inter, vocab, attn_bits = shape
    seed, T, n = 17, 20, 24
    out = subprocess.run([greedy_bin, *map(str, shape), str(seed), str(T), str(n)], capture_output=True, text=True,
                         timeout=300)
    assert out.returncode == 0, out.stderr
    lines = {ln.split()[0]: [int(v) for v in ln.split()[1:]] for ln in out.stdout.strip().splitlines()}
    c_dec, c_str = lines["decode"], lines["stream"]
    assert len(c_dec) == n + 1 and c_str == c_dec

    cfg = emx.Qwen3Config(hidden=hidden, layers=layers, n_q=n_q, n_kv=n_kv, inter=inter, vocab=vocab,
                          attn_bits=attn_bits, kv_cap=T + n + 8, max_prefill=T)
    prompt = ((np.arange(T) * 37 + 5) % vocab).astype(np.int32)
    with emx.Ctx(0) as ctx:
        m = emx.Qwen3(ctx, cfg)
        m.init_random(seed)
        first = m.prefill(prompt)
        py = [first] + [int(t) for t in m.decode(first, n)]
        m.close()
    assert c_dec == py
    ref = oracle_run(cfg, seed, prompt, c_dec[:-1])
    noise = noise_floor(ref, oracle_run(cfg, seed, prompt, c_dec[:-1], reverse=True))
    check_steps([(t, r[1]) for t, r in zip(c_dec, ref)], ref, noise, "C caller")
