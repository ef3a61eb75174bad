"""emx_sdpa_decode_noalloc against emx_sdpa_decode, on an sm_100 GPU.

The variant keeps its partials in a static device array instead of the
context's scratch; its output must be bit-identical to the allocating entry
point's, call after call, and the context's device memory must not change
while it runs.  Named to be collected last: it must also pass after every
other test has used the same process and device.
"""
import numpy as np
import pytest

import emx
import oracle

pytestmark = pytest.mark.gpu


def _case(rng, nq, nkv, cap):
    q = oracle.to_bf16(rng.standard_normal((nq, 128)).astype(np.float32))
    kc = oracle.to_bf16(rng.standard_normal((nkv, cap, 128)).astype(np.float32))
    vc = oracle.to_bf16(rng.standard_normal((nkv, cap, 128)).astype(np.float32))
    return q, kc, vc


def test_noalloc_decode_matches_allocating_entry_point():
    ctx = emx.Ctx(0)
    try:
        rng = np.random.default_rng(17)
        # two calls in a row per shape: a different length each time, so the
        # second call reuses tickets and partials the first one left behind
        for nq, nkv, cap, lengths in ((16, 8, 700, (137, 700)), (32, 4, 2100, (2100, 5)), (4, 2, 300, (64, 65))):
            q, kc, vc = _case(rng, nq, nkv, cap)
            bq, bk, bv = ctx.put(q), ctx.put(kc), ctx.put(vc)
            out = ctx.alloc(nq * 128 * 2)
            scale = 1 / np.sqrt(128)
            for length in lengths:
                ref = ctx.sdpa_decode(bq, bk, bv, nq, nkv, cap, 128, length, scale).read(np.uint16, (nq, 128))
                before = ctx.active_memory()
                ctx.sdpa_decode_noalloc(bq, bk, bv, out, nq, nkv, cap, 128, length, scale)
                ctx.synchronize()
                assert ctx.active_memory() == before
                got = out.read(np.uint16, (nq, 128))
                assert np.array_equal(got, ref), f"nq={nq} nkv={nkv} length={length}"
                want = oracle.sdpa(q[:, None], kc, vc, nkv, length, cap, scale, False)[:, 0]
                g, r = emx.f32(got).astype(np.float64), emx.f32(want).astype(np.float64)
                assert np.linalg.norm(g - r) <= 1e-2 * np.linalg.norm(r)
            assert ctx.device_status() == 0
    finally:
        ctx.close()


def test_noalloc_decode_rejects_shapes_beyond_its_scratch():
    ctx = emx.Ctx(0)
    try:
        b = ctx.alloc(1 << 16)
        # 128 kv heads: more tickets than the static scratch holds
        with pytest.raises(emx.EmxError) as ei:
            ctx.sdpa_decode_noalloc(b, b, b, b, 128, 128, 16, 128, 4, 0.1)
        assert ei.value.code == emx.ERR_INVALID and "tickets" in ei.value.msg
        with pytest.raises(emx.EmxError) as ei:
            ctx.sdpa_decode_noalloc(b, b, b, b, 65, 65, 16, 128, 4, 0.1)
        assert ei.value.code == emx.ERR_INVALID and "65" in ei.value.msg
        with pytest.raises(emx.EmxError) as ei:
            ctx.sdpa_decode_noalloc(b, b, b, b, 8, 4, 16, 64, 4, 0.1)
        assert ei.value.code == emx.ERR_INVALID and "head_dim" in ei.value.msg
        before = ctx.active_memory()
        with pytest.raises(emx.EmxError):
            ctx.sdpa_decode_noalloc(b, b, b, b, 8, 4, 16, 128, 17, 0.1)  # length > cap
        assert ctx.active_memory() == before
    finally:
        ctx.close()
