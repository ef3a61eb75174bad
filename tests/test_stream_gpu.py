"""Per-token streaming (emx_qwen3_decode_stream) on an sm_100 GPU.

The server's SSE path (crates/serve/src/server.rs:131-181) needs each token as
it is produced.  The streamed tokens must be the ones emx_qwen3_decode
returns for the same state, through the persistent step and the per-kernel
chain, greedy and sampled; a stop requested by the callback must leave the
engine exactly where an uninterrupted decode of that many tokens would have
(offset, device token, history), although greedy decoding ran further steps
ahead on the device.
"""
import numpy as np
import pytest

import emx

pytestmark = pytest.mark.gpu

CFG = emx.Qwen3Config(hidden=256, layers=2, n_q=4, n_kv=2, inter=512, vocab=1024, attn_bits=8, kv_cap=256,
                      max_prefill=64)
PROMPT = (np.arange(24, dtype=np.int32) * 37 + 5) % CFG.vocab
N = 40


@pytest.fixture(scope="module")
def ctx():
    c = emx.Ctx(0)
    yield c
    c.close()


def _model(ctx, fused):
    m = emx.Qwen3(ctx, CFG)
    m.init_random(11)
    m.fused = fused
    return m


@pytest.mark.parametrize("fused", [True, False], ids=["persistent", "per_op"])
def test_stream_equals_decode(ctx, fused):
    m = _model(ctx, fused)
    tok = m.prefill(PROMPT)
    ref = m.decode(tok, N)
    m.reset()
    assert m.prefill(PROMPT) == tok
    got, idx = [], []
    n = m.decode_stream(tok, N, lambda t, i: got.append(t) or idx.append(i) or False)
    assert n == N and idx == list(range(N))
    np.testing.assert_array_equal(np.array(got, np.int32), ref)
    assert m.offset == len(PROMPT) + N
    m.close()


@pytest.mark.parametrize("fused", [True, False], ids=["persistent", "per_op"])
@pytest.mark.parametrize("stop_at", [0, 9, N - 1])
def test_stream_stop_rolls_back(ctx, fused, stop_at):
    m = _model(ctx, fused)
    tok = m.prefill(PROMPT)
    ref = m.decode(tok, N)
    m.reset()
    m.prefill(PROMPT)
    got = []
    n = m.decode_stream(tok, N, lambda t, i: got.append(t) or i == stop_at)
    assert n == stop_at + 1
    np.testing.assert_array_equal(np.array(got, np.int32), ref[: stop_at + 1])
    # the engine stands just after the stop: offset, and the continuation
    # equals the uninterrupted run
    assert m.offset == len(PROMPT) + stop_at + 1
    rest = N - stop_at - 1
    if rest:
        np.testing.assert_array_equal(m.decode(int(ref[stop_at]), rest), ref[stop_at + 1:])
    m.close()


def test_stream_sampled_equals_decode(ctx):
    m = _model(ctx, False)
    m.set_sampling(0.8, 0.9, 40, 1234)
    tok = m.prefill(PROMPT)
    ref = m.decode(tok, 16)
    m.set_sampling(0.8, 0.9, 40, 1234)
    m.reset()
    assert m.prefill(PROMPT) == tok
    got = []
    assert m.decode_stream(tok, 16, lambda t, i: got.append(t) or False) == 16
    np.testing.assert_array_equal(np.array(got, np.int32), ref)
    m.close()


def test_stream_callback_exception_stops(ctx):
    m = _model(ctx, True)
    tok = m.prefill(PROMPT)

    def cb(t, i):
        if i == 3:
            raise ValueError("client went away")
        return False

    with pytest.raises(ValueError):
        m.decode_stream(tok, N, cb)
    assert m.offset == len(PROMPT) + 4
    m.close()
