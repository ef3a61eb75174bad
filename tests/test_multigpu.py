"""Tensor- and expert-parallel decode on two GPUs against the unsharded oracle.

The dense model is split by tensor parallelism (q/k/v and gate/up rows by
heads / intermediate, o/down columns); the fp32 partials after o and down
are summed through NVLink peer memory inside the GEMVs (each rank stores its
rows into every rank's exchange region and the consuming prologue adds the
ranks' slots in rank order), with an NCCL all-reduce only as the fallback
when the regions cannot be mapped.  The MoE model is split by expert
parallelism (experts across ranks), its weighted expert sums exchanged the
same way.  Each rank is its own
process with its own context on its own GPU; both generate their shard of the
same seeded weights.  Rank 0's logits must meet the single-GPU bars against
the oracle of the whole model, and both ranks must produce the same greedy
tokens.  Skipped unless two GPUs are visible.
"""
import multiprocessing as mp
import os
import queue

import numpy as np
import pytest

from test_model_gpu import check_steps, noise_floor, oracle_run

pytestmark = pytest.mark.gpu

WORLD = 2
DENSE = dict(hidden=512, layers=2, n_q=8, n_kv=2, inter=1024, vocab=2048, kv_cap=128, max_prefill=32)
MOE = dict(hidden=512, layers=2, n_q=8, n_kv=2, inter=1024, vocab=2048, tied=False, n_experts=16, top_k=4,
           moe_inter=256, kv_cap=128, max_prefill=32)


def _gpus():
    try:
        import torch
        return torch.cuda.device_count()
    except Exception:
        return 0


def _worker(rank, uid_q, out_q, cfg_kw, seed, prompt, forced, n_greedy):
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    try:
        import emx
        ctx = emx.Ctx(rank)
        if rank == 0:
            uid = emx.Comm.unique_id()
            for _ in range(WORLD - 1):
                uid_q.put(uid)
        else:
            uid = uid_q.get(timeout=120)
        comm = emx.Comm(ctx, uid, WORLD, rank)
        m = emx.Qwen3(ctx, emx.Qwen3Config(**cfg_kw), comm)
        m.init_random(seed)
        res = [m.prefill(prompt, want_logits=True)]
        for t in forced:
            res.append(m.decode_step(int(t), want_logits=True))
        m.reset()
        first = m.prefill(prompt)
        greedy = [first] + [int(t) for t in m.decode(first, n_greedy)]
        m.close()
        comm.close()
        ctx.close()
        out_q.put((rank, "ok", res, greedy))
    except Exception as e:  # reported to the parent
        out_q.put((rank, repr(e), None, None))


def _run(cfg_kw, seed, prompt, forced, n_greedy=8):
    ctx = mp.get_context("spawn")
    uid_q, out_q = ctx.Queue(), ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, uid_q, out_q, cfg_kw, seed, prompt, forced, n_greedy))
             for r in range(WORLD)]
    for p in procs:
        p.start()
    got = {}
    try:
        for _ in range(WORLD):
            r, status, res, greedy = out_q.get(timeout=600)
            got[r] = (status, res, greedy)
    except queue.Empty:
        pass
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    assert sorted(got) == list(range(WORLD)), f"ranks that reported: {sorted(got)}"
    for r, (status, _, _) in got.items():
        assert status == "ok", f"rank {r}: {status}"
    return got


@pytest.mark.skipif(_gpus() < WORLD, reason="needs two GPUs")
@pytest.mark.parametrize("kind", ["tensor_parallel_dense", "expert_parallel_moe"])
def test_two_gpu_decode_matches_oracle(kind):
    import emx
    cfg_kw = DENSE if kind.startswith("tensor") else MOE
    cfg = emx.Qwen3Config(**cfg_kw)
    rng = np.random.default_rng(11)
    prompt = rng.integers(0, cfg.vocab, 20).astype(np.int32)
    forced = rng.integers(0, cfg.vocab, 6)
    got = _run(cfg_kw, 31, prompt, forced)
    ref = oracle_run(cfg, 31, prompt, forced)
    noise = noise_floor(ref, oracle_run(cfg, 31, prompt, forced, reverse=True))
    for r in range(WORLD):
        check_steps(got[r][1], ref, noise, f"{kind} rank {r}")
    # every rank computes the same replicated logits, hence the same tokens
    assert got[0][2] == got[1][2]
    for a, b in zip(got[0][1], got[1][1]):
        assert a[0] == b[0]
