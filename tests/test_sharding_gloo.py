"""Multi-rank partitioning on the CPU: two `gloo` ranks.

The engine splits a dense model by tensor parallelism (q/k/v and gate/up rows
by heads / intermediate, o/down columns, fp32 partials summed by an
all-reduce) and an MoE model by expert parallelism (expert blocks, partial
expert sums all-reduced).  emx_qwen3_shard states which slice of each
checkpoint tensor a rank keeps; the engine checks its own layout against the
same rule at creation.  Here each rank takes its slices of the oracle
checkpoint, computes its part of a layer's linears in float64, and the gloo
all-reduce / all-gather must reproduce the unsharded result — the
decomposition a multi-GPU run relies on, tested without a GPU.
"""
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import emx
import oracle

WORLD = 2
DENSE = emx.Qwen3Config(hidden=256, layers=1, n_q=4, n_kv=2, inter=512, vocab=1024, kv_cap=64, max_prefill=16)
MOE = emx.Qwen3Config(hidden=256, layers=1, n_q=4, n_kv=2, inter=512, vocab=1024, tied=False, n_experts=4, top_k=2,
                      moe_inter=128, kv_cap=64, max_prefill=16)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _deq(ck, stem, bits, gs):
    """Dequantized weight as float64 [rows (experts stacked), cols]."""
    w, s, b = (ck[stem + p] for p in (".weight", ".scales", ".biases"))
    w, s, b = (a.reshape(-1, a.shape[-1]) for a in (w, s, b))
    return emx.f32(oracle.dequantize(w, s, b, gs, bits)).astype(np.float64)


def _worker(rank, port, out_q):
    try:
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=WORLD)
        x = emx.f32(oracle.to_bf16(np.random.default_rng(3).standard_normal(256).astype(np.float32)))
        x = x.astype(np.float64)
        p = "model.layers.0."
        # ---- dense, tensor parallel
        ck = oracle.make_checkpoint(DENSE, 5)
        for stem, bits, kind in ((p + "self_attn.q_proj", 4, "rows"), (p + "self_attn.k_proj", 4, "rows"),
                                 (p + "self_attn.v_proj", 4, "rows"), (p + "mlp.gate_proj", 4, "rows"),
                                 (p + "mlp.up_proj", 4, "rows"), (p + "self_attn.o_proj", 4, "cols"),
                                 (p + "mlp.down_proj", 4, "cols")):
            W = _deq(ck, stem, bits, 64)
            r0, nr, c0, nc, _, _ = emx.shard(DENSE, WORLD, rank, stem + ".weight")
            xin = x if W.shape[1] == x.size else np.random.default_rng(7).standard_normal(W.shape[1])
            full = W @ xin
            if kind == "rows":
                part = torch.from_numpy(W[r0:r0 + nr] @ xin)
                parts = [torch.zeros_like(part) for _ in range(WORLD)]
                dist.all_gather(parts, part)
                got = torch.cat(parts).numpy()
                assert np.array_equal(got, full), stem  # row slices: the same sums
            else:
                part = torch.from_numpy(W[:, c0:c0 + nc] @ xin[c0:c0 + nc])
                dist.all_reduce(part)
                assert np.allclose(part.numpy(), full, rtol=1e-12, atol=1e-12), stem
        # ---- MoE, expert parallel: each rank sums its experts among the top-k
        ck = oracle.make_checkpoint(MOE, 6)
        logits = _deq(ck, p + "mlp.gate", 4, 64) @ x
        probs = np.exp(logits - logits.max())
        probs /= probs.sum()
        top = np.argsort(-probs, kind="stable")[:MOE.top_k]
        wts = probs[top] / probs[top].sum()
        Wg, Wu, Wd = (_deq(ck, p + "mlp.switch_mlp." + n, 4, 64) for n in ("gate_proj", "up_proj", "down_proj"))
        Im = MOE.moe_inter

        def expert(e):
            g = Wg[e * Im:(e + 1) * Im] @ x
            u = Wu[e * Im:(e + 1) * Im] @ x
            return Wd[e * 256:(e + 1) * 256] @ (g / (1 + np.exp(-g)) * u)

        full = sum(w * expert(e) for e, w in zip(top, wts))
        _, _, _, _, b0, nb = emx.shard(MOE, WORLD, rank, p + "mlp.switch_mlp.gate_proj.weight")
        mine = [(e, w) for e, w in zip(top, wts) if b0 <= e < b0 + nb]
        part = torch.from_numpy(sum((w * expert(e) for e, w in mine), np.zeros(256)))
        dist.all_reduce(part)
        assert np.allclose(part.numpy(), full, rtol=1e-12, atol=1e-12), "experts"
        dist.barrier()
        out_q.put((rank, "ok"))
    except Exception as e:  # reported to the parent
        out_q.put((rank, repr(e)))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def test_two_rank_partitioning_reproduces_the_full_layer():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, port, q)) for r in range(WORLD)]
    for pr in procs:
        pr.start()
    results = dict(q.get(timeout=240) for _ in range(WORLD))
    for pr in procs:
        pr.join(timeout=60)
    assert results == {0: "ok", 1: "ok"}, results


@pytest.mark.parametrize("cfg,world", [(DENSE, 2), (MOE, 2), (MOE, 4)])
def test_shards_tile_every_tensor_exactly_once(cfg, world):
    """Over all ranks the slices of every checkpoint tensor cover it once."""
    for name, arr in oracle.make_checkpoint(cfg, 1).items():
        sl = [emx.shard(cfg, world, r, name) for r in range(world)]
        full = emx.shard(cfg, 1, 0, name)
        cells = set()
        for r0, nr, c0, nc, b0, nb in sl:
            for b in range(b0, b0 + nb):
                for rr in range(r0, r0 + nr, 16):
                    for cc in range(c0, c0 + nc, 64):
                        key = (b, rr, cc)
                        # replicated tensors repeat the full slice on every rank
                        if (r0, nr, c0, nc, b0, nb) == full:
                            continue
                        assert key not in cells, name
                        cells.add(key)
        if any(s != full for s in sl):
            r0, nr, c0, nc, b0, nb = full
            assert len(cells) == nb * ((nr + 15) // 16) * ((nc + 63) // 64), name


def test_shard_rejects_indivisible_and_unknown():
    with pytest.raises(emx.EmxError):
        emx.shard(DENSE, 3, 0, "model.layers.0.self_attn.q_proj.weight")
    with pytest.raises(emx.EmxError):
        emx.shard(DENSE, 2, 0, "model.layers.0.nope.weight")
    with pytest.raises(emx.EmxError):
        emx.shard(DENSE, 2, 2, "model.norm.weight")
