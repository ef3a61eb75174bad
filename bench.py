"""Benchmark: batch-1 greedy decode (and prefill) of the Qwen3-1.7B-shape
random-init model (attention int8 gs64, MLP int4 gs64, tied int4 embeddings)
on B200, through libemx.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config c3] [--prompt 128]
    python bench.py --impl reference ...   # the CPU oracle (reference restatement) arm

One step = one greedy decode token (the whole 28-layer forward + lm_head +
argmax: one persistent kernel launch, replayed from a CUDA graph).  The timed
region holds exactly K steps, bracketed by a barrier and a device synchronise,
timed with CUDA events on the engine's stream; with N GPUs (torchrun) every
rank runs its own replica (the 1.7B model is not sharded: "replicas only") and
`value` is the sum of all ranks' tokens over the slowest rank's time.  Weights
(1.1 GB) are larger than L2 (126 MB), so every step streams them from HBM.

Besides the headline the line carries: prefill tok/s at 128 / 2048 / 8192
tokens, decode after 2048- and 8192-token prompts, the single quantized linear
of BASELINE configs[0] (M = 1 and 512), the packed GEMV alone, end-to-end
rates through the public API (per-step and streamed), `sharded`: the
32B-shape model tensor-parallel over the job's GPUs (every N of a scaling run),
so the 1 -> 8 curve holds the collective's scaling, not only replicas, and
`moe`: the 30B-A3B-shape model expert-parallel over the job's GPUs, a
1024-token prefill (grouped expert GEMMs) and decode after it.
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path[:0] = [os.path.join(ROOT, "engine-mlx_b200"), os.path.join(ROOT, "oracle")]

METRIC = "bs1 decode tok/s + prefill tok/s, Qwen3-1.7B-shape int4; % HBM roofline"
UNIT = "tok/s"


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d.get("hbm_gbs", 6650.0), d.get("bf16_tflops", 1590.0), "measured"
    return 6650.0, 1590.0, "fallback"


# ------------------------------------------------------------- roofline bytes
def qbytes(N, K, bits, gs):
    return N * K * bits // 8 + 2 * N * (K // gs) * 2


def decode_bytes(cfg, ctx_len):
    """Algorithmic HBM bytes of one decode token at `ctx_len` valid KV rows:
    packed weights + bf16 scales/biases of every linear, norm weights, the
    embedding row, the KV rows read and the new K/V row written."""
    H, hd, L = cfg.hidden, cfg.head_dim, cfg.layers
    per_layer = qbytes((cfg.n_q + 2 * cfg.n_kv) * hd, H, cfg.attn_bits, cfg.attn_group)
    per_layer += qbytes(H, cfg.n_q * hd, cfg.attn_bits, cfg.attn_group)
    if cfg.n_experts:
        per_layer += qbytes(cfg.n_experts, H, cfg.router_bits, cfg.router_group)
        per_layer += cfg.top_k * (qbytes(2 * cfg.moe_inter, H, cfg.expert_bits, cfg.expert_group) +
                                  qbytes(H, cfg.moe_inter, cfg.expert_bits, cfg.expert_group))
    else:
        per_layer += qbytes(2 * cfg.inter, H, cfg.mlp_bits, cfg.mlp_group)
        per_layer += qbytes(H, cfg.inter, cfg.mlp_bits, cfg.mlp_group)
    per_layer += 2 * H * 2 + 2 * hd * 2                       # norm weights
    per_layer += 2 * cfg.n_kv * ctx_len * hd * 2               # K and V rows read
    per_layer += 2 * cfg.n_kv * hd * 2                         # new K/V row written
    lm = qbytes(cfg.vocab, H, cfg.lm_bits if not cfg.tied else cfg.embed_bits,
                cfg.lm_group if not cfg.tied else cfg.embed_group)
    embed_row = H * cfg.embed_bits // 8 + 2 * (H // cfg.embed_group) * 2
    return L * per_layer + lm + H * 2 + embed_row


# ---------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi samples (SM clock, throttle reasons) during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device):
        self.device = device
        self.lines = []
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "100", "-i", str(self.device)], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None
        time.sleep(0.3)
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *a):
        time.sleep(0.2)
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() in ("active", "1"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# ------------------------------------------------------------------ arms
def cpu_model():
    """The host CPU's model name (for the CPU baseline's record)."""
    try:
        with open("/proc/cpuinfo") as f:
            for ln in f:
                if ln.startswith("model name"):
                    return ln.split(":", 1)[1].strip()
    except OSError:
        pass
    import platform

    return platform.processor() or "unknown"


def cpu_baseline(cfg, seed, prompt_len, steps, warmup=0, threads=None):
    """The CPU oracle (restatement of the reference path, OpenMP) on this host:
    a prefill of `prompt_len` random ids (seeded as the GPU arm's prompt), then
    `warmup` untimed and `steps` timed greedy decode steps.  Returns decode
    tok/s, the threads used and the prefill seconds."""
    import numpy as np
    import oracle

    if threads:
        oracle.lib().orc_set_num_threads(threads)
    ck = oracle.make_checkpoint(cfg, seed)
    m = oracle.Model(cfg, ck)
    prompt = np.random.default_rng(seed).integers(0, cfg.vocab, prompt_len).astype(np.int32)
    t0 = time.perf_counter()
    t = m.prefill(prompt)
    prefill_s = time.perf_counter() - t0
    for _ in range(warmup):
        t = m.decode(t)
    t0 = time.perf_counter()
    for _ in range(steps):
        t = m.decode(t)
    dt = time.perf_counter() - t0
    m.close()
    return steps / dt, oracle.lib().orc_num_threads(), prefill_s


def run_reference(args, cfg, rank):
    """The reference arm: the CPU restatement of the reference's algorithm (MLX
    and mlx-c cannot be built here) on the GPU arm's workload -- the same
    prompt length, then the same warm-up and timed decode steps (at most 64) --
    with every host thread."""
    if rank != 0:
        return
    steps = max(1, min(args.steps, 64))
    warm = max(0, min(args.warmup, 5))
    v, cores, pre_s = cpu_baseline(cfg, args.seed, args.prompt, steps, warmup=warm)
    cfg_w = workload(args, cfg)
    cfg_w["decode_tokens"] = steps
    sample = (f"{args.config}: {args.prompt}-token prompt ({pre_s:.1f} s), {warm} untimed then {steps} timed greedy "
              f"decode steps on {cpu_model()} (CPU oracle restatement of the reference path; MLX itself is not "
              "buildable here)")
    line = {"metric": METRIC, "value": v, "unit": UNIT, "impl": "reference", "n_gpus": args.gpus, "steps": steps,
            "warmup": warm, "ms_per_step": 1000.0 / v, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16 activations, int4/int8 affine weights", "data": "synthetic",
            "config": cfg_w,
            "cpu_baseline": {"value": v, "unit": UNIT, "cores": cores, "kind": "port", "cpu_model": cpu_model(),
                             "prefill_s": pre_s, "sample": sample},
            "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def workload(args, cfg):
    """The config block both arms print (the driver compares them)."""
    return {"workload": f"{args.config} (Qwen3-1.7B shape)" if args.config == "c3" else args.config,
            "model": f"random-init {args.config}", "hidden": cfg.hidden, "layers": cfg.layers,
            "attn_bits": cfg.attn_bits, "mlp_bits": cfg.mlp_bits, "group_size": cfg.mlp_group,
            "global_batch": 1, "prompt": args.prompt, "decode_tokens": args.steps, "seq_len": args.prompt,
            "parallelism": (f"{'expert' if cfg.n_experts else 'tensor'} parallel x{args.gpus}" if args.shard
                            else f"replicas x{args.gpus}"),
            "l2": "inputs larger than L2 (1.1 GB of weights streamed per token)"}


def profiled_traffic(kernel_tag):
    """Per-launch DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) of
    the kernel from its committed ncu summary (profiles/<kernel_tag>.md, line
    'dram bytes per launch: N'), or None."""
    p = os.path.join(ROOT, "profiles", kernel_tag + ".md")
    try:
        with open(p) as f:
            for ln in f:
                if ln.lower().startswith("dram bytes per launch:"):
                    return float(ln.split(":", 1)[1].split()[0].replace(",", ""))
    except (OSError, ValueError):
        pass
    return None


def timed_decode(m, ctx, st, torch, n, barrier=None):
    """Device time (ms) of n decode steps from the model's current state,
    CUDA events on the engine's stream, synchronised on both sides."""
    ctx.synchronize()
    if barrier:
        barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    m.decode_device(n)
    e1.record(st)
    e1.synchronize()
    return e0.elapsed_time(e1)


def decode_at_context(ctx, st, torch, cfg, m, hbm, seed, ctx_len, steps=32):
    """Decode tok/s and the step roofline after a ctx_len-token prompt (the
    BASELINE C3 prompt lengths 2048 / 8192)."""
    import numpy as np

    if ctx_len > cfg.max_prefill or ctx_len + steps + 8 > cfg.kv_cap:
        return None
    ids = ctx.put(np.random.default_rng(seed + ctx_len).integers(0, cfg.vocab, ctx_len).astype(np.int32))
    m.reset()
    m.prefill_device(ids, ctx_len)
    m.decode_device(3)
    ms = timed_decode(m, ctx, st, torch, steps)
    ids.free()
    mean_ctx = ctx_len + 3 + (steps - 1) / 2.0
    ach = decode_bytes(cfg, mean_ctx) / (ms / steps / 1000.0) / 1e9
    return {"tok_s": steps / (ms / 1000.0), "ms_per_step": ms / steps,
            "decode_context": [ctx_len + 3, ctx_len + 3 + steps],
            "step_roofline": {"bound": "hbm", "achieved": ach, "peak": hbm, "unit": "GB/s", "frac": ach / hbm}}


def c1_linear(ctx, st, torch, hbm, tflops):
    """one quantized linear, N=6144, K=2048, int4 gs64,
    through emx_quantized_matmul: M=1 (GB/s over 24 weight copies, > L2) and
    M=512 (TFLOP/s)."""
    import numpy as np

    import emx

    N, K, gs, bits = 6144, 2048, 64, 4
    copies = 24
    wsz, ssz = N * K * bits // 8, N * (K // gs) * 2
    rng = np.random.default_rng(7)
    res = {}
    ws = []
    for _ in range(copies):
        w, s, b = ctx.alloc(wsz), ctx.alloc(ssz), ctx.alloc(ssz)
        emx.lib().emx_memset(ctx.h, w.ptr, int(rng.integers(1, 255)), wsz)
        emx.lib().emx_memset(ctx.h, s.ptr, 0x3C, ssz)
        emx.lib().emx_memset(ctx.h, b.ptr, 0x00, ssz)
        ws.append((w, s, b))
    for M in (1, 512):
        x, y = ctx.alloc(M * K * 2), ctx.alloc(M * N * 2)
        emx.lib().emx_memset(ctx.h, x.ptr, 0x3C, M * K * 2)
        for i in range(4):
            w, s, b = ws[i % copies]
            ctx.quantized_matmul(x, w, s, b, M, N, K, gs, bits, out=y)
        ctx.synchronize()
        n = 96 if M == 1 else 24
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        for i in range(n):
            w, s, b = ws[i % copies]
            ctx.quantized_matmul(x, w, s, b, M, N, K, gs, bits, out=y)
        e1.record(st)
        e1.synchronize()
        us = e0.elapsed_time(e1) * 1000.0 / n
        if M == 1:
            per = qbytes(N, K, bits, gs) + K * 2 + N * 2
            ach = per / (us * 1e-6) / 1e9
            res["m1"] = {"us_per_call": us, "bytes_per_call": per, "achieved": ach, "unit": "GB/s", "peak": hbm,
                         "frac": ach / hbm, "bound": "hbm"}
        else:
            ach = 2.0 * M * N * K / (us * 1e-6) / 1e12
            res["m512"] = {"us_per_call": us, "achieved": ach, "unit": "TFLOP/s", "peak": tflops,
                           "frac": ach / tflops, "bound": "tensor"}
        x.free()
        y.free()
    for w, s, b in ws:
        w.free()
        s.free()
        b.free()
    res["shape"] = {"N": N, "K": K, "bits": bits, "group_size": gs, "api": "emx_quantized_matmul"}
    return res


def sharded_c5(args, rank, world, dist, torch, hbm, steps=32, prompt=128):
    """The 32B-shape dense model split tensor-parallel
    across the job's GPUs (one GPU: the whole model), decode after a prompt:
    tok/s from CUDA events, max over ranks, and the per-GPU step roofline.
    Every rank takes part."""
    import dataclasses

    import numpy as np

    import emx

    cfg = dataclasses.replace(emx.CONFIGS["c5"], kv_cap=prompt + steps + 64, max_prefill=prompt)
    dev = int(os.environ.get("LOCAL_RANK", "0"))
    ctx = emx.Ctx(dev)
    sp = emx.C.c_void_p()
    emx.lib().emx_ctx_stream(ctx.h, emx.C.byref(sp))
    st = torch.cuda.ExternalStream(sp.value, device=dev)
    comm = None
    if world > 1:
        obj = [emx.Comm.unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        comm = emx.Comm(ctx, obj[0], world, rank)
    m = emx.Qwen3(ctx, cfg, comm)
    m.init_random(args.seed)
    ids = ctx.put(np.random.default_rng(args.seed).integers(0, cfg.vocab, prompt).astype(np.int32))
    m.prefill_device(ids, prompt)
    m.decode_device(3)
    barrier = dist.barrier if dist is not None else None
    ms = timed_decode(m, ctx, st, torch, steps, barrier)
    if dist is not None:
        t = torch.tensor([ms], device=f"cuda:{dev}")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    launches = m.step_launches()
    ids.free()
    m.close()
    if comm is not None:
        comm.close()
    ctx.close()
    mean_ctx = prompt + 3 + (steps - 1) / 2.0
    per_gpu = decode_bytes(cfg, mean_ctx) / world
    ach = per_gpu / (ms / steps / 1000.0) / 1e9
    return {"model": "c5 (Qwen3-32B shape, int4 gs64, random-init)", "parallelism": f"tensor parallel x{world}",
            "tok_s": steps / (ms / 1000.0), "ms_per_step": ms / steps, "steps": steps, "prompt": prompt,
            "launches_per_step": launches,
            "step_roofline": {"bound": "hbm", "achieved": ach, "peak": hbm, "unit": "GB/s", "frac": ach / hbm,
                              "scope": "per GPU: 1/world of the weights + this rank's KV heads",
                              "bytes_per_step": per_gpu}}


def moe_c4(args, rank, world, dist, torch, hbm, steps=32, prompt=1024):
    """The 30B-A3B-shape MoE model split expert-parallel
    across the job's GPUs (one GPU: the whole model): a 1024-token prefill
    (the grouped expert GEMMs) and decode after it, CUDA events, max over
    ranks; the decode step roofline counts the active experts' bytes."""
    import dataclasses

    import numpy as np

    import emx

    cfg = dataclasses.replace(emx.CONFIGS["c4"], kv_cap=prompt + steps + 64, max_prefill=prompt)
    dev = int(os.environ.get("LOCAL_RANK", "0"))
    ctx = emx.Ctx(dev)
    sp = emx.C.c_void_p()
    emx.lib().emx_ctx_stream(ctx.h, emx.C.byref(sp))
    st = torch.cuda.ExternalStream(sp.value, device=dev)
    comm = None
    if world > 1:
        obj = [emx.Comm.unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        comm = emx.Comm(ctx, obj[0], world, rank)
    m = emx.Qwen3(ctx, cfg, comm)
    m.init_random(args.seed)
    ids = ctx.put(np.random.default_rng(args.seed).integers(0, cfg.vocab, prompt).astype(np.int32))
    m.prefill_device(ids, prompt)  # warm
    times = []
    for _ in range(2):
        m.reset()
        ctx.synchronize()
        if dist is not None:
            dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        m.prefill_device(ids, prompt)
        e1.record(st)
        e1.synchronize()
        times.append(e0.elapsed_time(e1))
    pre_ms = min(times)
    m.decode_device(3)
    barrier = dist.barrier if dist is not None else None
    ms = timed_decode(m, ctx, st, torch, steps, barrier)
    if dist is not None:
        t = torch.tensor([ms, pre_ms], device=f"cuda:{dev}")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, pre_ms = float(t[0].item()), float(t[1].item())
    path = "persistent step (one launch per token)" if m.fused else "kernel chain"
    ids.free()
    m.close()
    if comm is not None:
        comm.close()
    ctx.close()
    mean_ctx = prompt + 3 + (steps - 1) / 2.0
    per_gpu = decode_bytes(cfg, mean_ctx) / world
    ach = per_gpu / (ms / steps / 1000.0) / 1e9
    return {"model": "c4 (Qwen3-30B-A3B shape, 128 experts top-8, int4 gs64, random-init)",
            "parallelism": f"expert parallel x{world}", "prefill_tokens": prompt,
            "prefill_tok_s": prompt / (pre_ms / 1000.0), "prefill_ms": pre_ms,
            "decode_tok_s": steps / (ms / 1000.0), "ms_per_step": ms / steps, "steps": steps, "decode_path": path,
            "step_roofline": {"bound": "hbm", "achieved": ach, "peak": hbm, "unit": "GB/s", "frac": ach / hbm,
                              "scope": "per GPU: attention + router + the top-8 experts' weights, 1/world",
                              "bytes_per_step": per_gpu}}


def run_engine(args, cfg, rank, world, dist):
    import numpy as np

    import emx

    dev = int(os.environ.get("LOCAL_RANK", "0"))
    import torch

    torch.cuda.set_device(dev)
    ctx = emx.Ctx(dev)
    stream_ptr = emx.C.c_void_p()
    emx.lib().emx_ctx_stream(ctx.h, emx.C.byref(stream_ptr))
    st = torch.cuda.ExternalStream(stream_ptr.value, device=dev)
    if args.kernel_only == "prefill":
        # one warm prefill, then one timed: the launch list of a whole prefill
        # (the KV cache sized to the prompt)
        import dataclasses

        cfg = dataclasses.replace(cfg, kv_cap=args.prompt + 64, max_prefill=max(args.prompt, 128))
        m = emx.Qwen3(ctx, cfg)
        m.init_random(args.seed)
        ids = ctx.put(np.random.default_rng(args.seed).integers(0, cfg.vocab, args.prompt).astype(np.int32))
        m.prefill_device(ids, args.prompt)
        m.reset()
        ctx.synchronize()
        if args.profile_range:
            torch.cuda.profiler.start()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        m.prefill_device(ids, args.prompt)
        e1.record(st)
        e1.synchronize()
        if args.profile_range:
            torch.cuda.profiler.stop()
        ms = e0.elapsed_time(e1)
        if rank == 0:
            print(json.dumps({"prefill_tokens": args.prompt, "ms": ms, "tok_s": args.prompt / (ms / 1000.0)}),
                  flush=True)
        m.close()
        ctx.close()
        return
    if args.kernel_only == "step":
        # the decode step kernel alone: prefill --prompt tokens, --warmup
        # steps, then --steps timed steps (a short command for the profiler;
        # the KV cache sized to the run, so the device holds little besides
        # the weights)
        import dataclasses

        cfg = dataclasses.replace(cfg, kv_cap=args.prompt + args.steps + max(args.warmup, 3) + 64,
                                  max_prefill=max(args.prompt, 128))
        m = emx.Qwen3(ctx, cfg)
        m.init_random(args.seed)
        if args.per_op and m.fused:
            m.fused = False
        if args.eager:
            m.compiled = False
        ids = ctx.put(np.random.default_rng(args.seed).integers(0, cfg.vocab, args.prompt).astype(np.int32))
        m.prefill_device(ids, args.prompt)
        m.decode_device(max(args.warmup, 3))
        if args.profile_range:
            torch.cuda.profiler.start()
        ms = timed_decode(m, ctx, st, torch, args.steps)
        if args.profile_range:
            torch.cuda.profiler.stop()
        if rank == 0:
            print(json.dumps({"decode_steps": args.steps, "ms_per_step": ms / args.steps,
                              "tok_s": args.steps / (ms / 1000.0), "launches_per_step": m.step_launches()}),
                  flush=True)
        m.close()
        ctx.close()
        return
    if args.kernel_only:
        hbm, tf, kind = peaks()
        if rank == 0:
            if args.kernel_only == "gemm":
                r = gemm_kernel_roofline(ctx, st, cfg, torch, tf)
            elif args.kernel_only == "attn":
                r = attn_kernel_roofline(ctx, st, cfg, torch, hbm)
            elif args.kernel_only == "c1":
                r = c1_linear(ctx, st, torch, hbm, tf)
            else:
                r = gemv_kernel_roofline(ctx, st, cfg, torch, hbm)
            print(json.dumps(dict(r, peak_kind=kind)), flush=True)
        ctx.close()
        return
    comm = None
    if args.shard and world > 1:
        # one model split across the ranks (tensor parallel for dense, expert
        # parallel for MoE): the NCCL id travels over the bench's own group
        obj = [emx.Comm.unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        comm = emx.Comm(ctx, obj[0], world, rank)
    m = emx.Qwen3(ctx, cfg, comm)
    m.init_random(args.seed)
    m.compiled = not args.eager
    if args.per_op:
        m.fused = False

    def barrier():
        if dist is not None:
            dist.barrier()

    sharded = comm is not None
    streams = 1 if sharded else world  # decode streams: one sharded model, or one replica per rank
    rng = np.random.default_rng(args.seed + (0 if sharded else rank))
    prompt = rng.integers(0, cfg.vocab, args.prompt).astype(np.int32)
    ids = ctx.put(prompt)
    # ---- prefill tok/s (device-resident ids), a few repetitions
    pre = {}
    for T in sorted({args.prompt, *args.prefill_lengths}):
        if T > cfg.max_prefill or T + 8 > cfg.kv_cap:
            continue
        idsT = ctx.put(rng.integers(0, cfg.vocab, T).astype(np.int32))
        reps = 3 if T <= 2048 else 1
        times = []
        for r in range(reps + 1):
            m.reset()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            ctx.synchronize()
            e0.record(st)
            m.prefill_device(idsT, T)
            e1.record(st)
            e1.synchronize()
            if r:
                times.append(e0.elapsed_time(e1))
        pre[str(T)] = T / (statistics.median(times) / 1000.0)
        idsT.free()
    # ---- decode: warm-up W steps, then K timed steps
    m.reset()
    m.prefill_device(ids, args.prompt)
    m.decode_device(max(args.warmup, 3))
    ctx.synchronize()
    launches = m.step_launches()
    barrier()
    with ClockSampler(dev) as clk:
        ms = timed_decode(m, ctx, st, torch, args.steps, barrier)
        barrier()
    start_ctx = args.prompt + max(args.warmup, 3)
    ms_max = ms
    if dist is not None:
        t = torch.tensor([ms], device=f"cuda:{dev}")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms_max = float(t.item())
    value = streams * args.steps / (ms_max / 1000.0)
    # ---- end to end through the public API: host token in, host token out
    m.reset()
    tok = m.prefill(prompt)
    for _ in range(3):
        tok = m.decode_step(tok)
    n_e2e = min(args.steps, 256)
    barrier()
    t0 = time.perf_counter()
    for _ in range(n_e2e):
        tok = m.decode_step(tok)
    e2e_s = time.perf_counter() - t0
    # the same through the per-token streaming entry point (steps in flight)
    m.reset()
    tok = m.prefill(prompt)
    barrier()
    t0 = time.perf_counter()
    n_str = m.decode_stream(tok, n_e2e, lambda t, i: False)
    str_s = time.perf_counter() - t0
    e2e = n_e2e / e2e_s
    e2e_str = n_str / str_s
    if dist is not None:
        t = torch.tensor([e2e_s, str_s], device=f"cuda:{dev}")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e = streams * n_e2e / float(t[0].item())
        e2e_str = streams * n_str / float(t[1].item())
    # ---- roofline of the decode step (all GEMVs + attention + lm_head)
    hbm, tf, kind = peaks()
    mean_ctx = start_ctx + (args.steps - 1) / 2.0
    step_bytes = decode_bytes(cfg, mean_ctx) / (world if sharded else 1)  # per GPU
    achieved = step_bytes / (ms_max / args.steps / 1000.0) / 1e9
    fused = m.fused
    extras = {}
    if rank == 0 and not sharded:
        for L in (2048, 8192):
            r = decode_at_context(ctx, st, torch, cfg, m, hbm, args.seed, L)
            if r:
                extras[str(L)] = r
    m.close()
    if comm is not None:
        comm.close()
    kern = c1 = None
    if rank == 0:
        kern = gemv_kernel_roofline(ctx, st, cfg, torch, hbm)
        c1 = c1_linear(ctx, st, torch, hbm, tf)
    ctx.close()
    barrier()
    sh = mo = None
    if not args.shard and not args.no_sharded:
        sh = sharded_c5(args, rank, world, dist, torch, hbm)
    if not args.shard and not args.no_moe:
        mo = moe_c4(args, rank, world, dist, torch, hbm)
    if rank != 0:
        return
    if fused:
        tag = f"step_kernel_{args.config}"
        kname = "step_kernel (the whole decode step: one persistent launch per token)"
    else:
        tag = f"decode_chain_{args.config}"
        kname = "decode kernel chain (one CUDA graph per token)"
    traffic = profiled_traffic(tag)
    line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": max(args.warmup, 3), "ms_per_step": ms_max / args.steps, "higher_is_better": True,
            "scaling": "strong" if sharded else "weak", "vs_baseline": None,
            "dtype": "bf16 activations, int4/int8 affine weights",
            "data": "synthetic (seeded random-init weights and token ids)", "config": workload(args, cfg),
            "decode_path": ("one persistent kernel per decode step" if fused
                            else "one kernel per operation, CUDA graph"),
            "prefill_tok_s": pre, "decode_context": [start_ctx, start_ctx + args.steps],
            "roofline": {"kernel": kname, "bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s",
                         "frac": achieved / hbm, "traffic": traffic, "peak_kind": kind,
                         "bytes_per_launch": step_bytes,
                         "traffic_source": f"profiles/{tag}.md" if traffic else None,
                         "scope": "algorithmic bytes of one decode step (weights + scales/biases + KV rows read + "
                                  "norms) / its CUDA-event time"},
            "step_roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s",
                              "frac": achieved / hbm, "traffic": traffic, "peak_kind": kind,
                              "scope": "whole decode step (weights + scales/biases + KV read per token)",
                              "bytes_per_step": step_bytes},
            "decode_long_context": extras,
            "gemv_kernel": dict(kern, peak_kind=kind) if kern else None,
            "c1_single_linear": c1,
            "e2e": {"value": e2e, "unit": UNIT, "h2d_bytes_per_step": 4, "d2h_bytes_per_step": 4,
                    "api": "emx_qwen3_decode_step", "steps": n_e2e},
            "e2e_stream": {"value": e2e_str, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 8,
                           "api": "emx_qwen3_decode_stream (per-token callback, steps in flight)",
                           "steps": n_str},
            "gpu_launches": launches * args.steps, "launches_per_step": launches,
            "clocks": clk.summary()}
    if sh:
        line["sharded"] = sh
    if mo:
        line["moe"] = mo
    if sharded:
        line["step_roofline"]["scope"] += ", per GPU (1/world of the weights)"
    if world == 1 and not args.no_cpu_baseline:
        v, cores, pre_s = cpu_baseline(cfg, args.seed, args.prompt, args.cpu_steps)
        line["cpu_baseline"] = {"value": v, "unit": UNIT, "cores": cores, "kind": "port", "cpu_model": cpu_model(),
                                "prefill_s": pre_s,
                                "sample": f"{args.config}: {args.prompt}-token prompt then {args.cpu_steps} greedy "
                                          f"decode steps on the CPU oracle (OpenMP, {cores} threads, {cpu_model()})"}
    print(json.dumps(line), flush=True)


def gemv_kernel_roofline(ctx, st, cfg, torch, hbm):
    """The packed batch-1 GEMV (pgemv_kernel, the per-kernel decode chain's
    GEMV; the persistent step runs the same inner loop) alone on the step's
    most expensive shape, the fused gate|up projection [2*inter, hidden]: 16
    packed copies (> L2) rotated over 160 launches, CUDA events on the
    context's stream.  Algorithmic bytes per launch: packed codes + bf16
    scales and biases + x in + y out."""
    import numpy as np

    import emx

    N, K = 2 * cfg.inter, cfg.hidden
    bits, gs = cfg.mlp_bits, cfg.mlp_group
    copies = 16
    wsz, ssz = N * K * bits // 8, N * (K // gs) * 2
    w, s, b = ctx.alloc(wsz), ctx.alloc(ssz), ctx.alloc(ssz)
    emx.lib().emx_memset(ctx.h, w.ptr, 0x5A, wsz)
    emx.lib().emx_memset(ctx.h, s.ptr, 0x3C, ssz)
    emx.lib().emx_memset(ctx.h, b.ptr, 0x00, ssz)
    pk = [ctx.qpack(w, s, b, N, K, gs, bits) for _ in range(copies)]
    x = ctx.put(np.full(K, 0x3F80, np.uint16))
    y = ctx.alloc(N * 2)
    L = emx.lib()
    for i in range(8):
        L.emx_quantized_matvec_packed(ctx.h, x.ptr, pk[i % copies].ptr, y.ptr, N, K, gs, bits)
    ctx.synchronize()
    n = 160
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for i in range(n):
        L.emx_quantized_matvec_packed(ctx.h, x.ptr, pk[i % copies].ptr, y.ptr, N, K, gs, bits)
    e1.record(st)
    e1.synchronize()
    us = e0.elapsed_time(e1) * 1000.0 / n
    per = qbytes(N, K, bits, gs) + K * 2 + N * 2
    for a in pk + [w, s, b, x, y]:
        a.free()
    ach = per / (us * 1e-6) / 1e9
    return {"kernel": f"pgemv_kernel<{bits},{gs}> (gate|up shape, standalone: no PDL overlap with a neighbour)",
            "shape": [N, K], "bound": "hbm", "achieved": ach, "peak": hbm, "unit": "GB/s", "frac": ach / hbm,
            "us_per_launch": us, "bytes_per_launch": per, "traffic": profiled_traffic("pgemv_gate_up_c3"),
            "traffic_source": "profiles/pgemv_gate_up_c3.md"}


def gemm_kernel_roofline(ctx, st, cfg, torch, tflops, M=2048):
    """The prefill GEMM alone: emx_quantized_matmul on the gate|up shape
    [2*inter, hidden] with M = 2048 rows of x (dequantize the weights into
    scratch, then tc_gemm_kernel: TMA-fed tcgen05 MMAs into a TMEM
    accumulator).  Algorithmic work: 2*M*N*K FLOP per call; the time is the
    whole call (dequant + GEMM), CUDA events over 20 calls."""
    import emx

    N, K = 2 * cfg.inter, cfg.hidden
    bits, gs = cfg.mlp_bits, cfg.mlp_group
    wsz, ssz = N * K * bits // 8, N * (K // gs) * 2
    w, s, b = ctx.alloc(wsz), ctx.alloc(ssz), ctx.alloc(ssz)
    x, y = ctx.alloc(M * K * 2), ctx.alloc(M * N * 2)
    L = emx.lib()
    L.emx_memset(ctx.h, w.ptr, 0x5A, wsz)
    L.emx_memset(ctx.h, s.ptr, 0x3C, ssz)
    L.emx_memset(ctx.h, b.ptr, 0x00, ssz)
    L.emx_memset(ctx.h, x.ptr, 0x3C, M * K * 2)
    for _ in range(3):
        ctx.quantized_matmul(x, w, s, b, M, N, K, gs, bits, out=y)
    ctx.synchronize()
    n = 20
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for _ in range(n):
        ctx.quantized_matmul(x, w, s, b, M, N, K, gs, bits, out=y)
    e1.record(st)
    e1.synchronize()
    us = e0.elapsed_time(e1) * 1000.0 / n
    for a in (w, s, b, x, y):
        a.free()
    ach = 2.0 * M * N * K / (us * 1e-6) / 1e12
    return {"kernel": "emx_quantized_matmul = dequantize + tc_gemm_kernel (tcgen05, TMEM accumulator)",
            "shape": [M, N, K], "bound": "tensor", "achieved": ach, "peak": tflops, "unit": "TFLOP/s",
            "frac": ach / tflops, "us_per_call": us, "traffic": None}


def attn_kernel_roofline(ctx, st, cfg, torch, hbm, L=8192):
    """Decode attention alone (split-KV flash-decode, emx_sdpa_decode_noalloc)
    at L valid rows of the static cache: 8 K/V cache copies (> L2) rotated
    over 64 calls.  Algorithmic bytes per call: the L K and V rows of every
    KV head + q in + the output."""
    import numpy as np

    import emx

    nq, nkv, hd = cfg.n_q, cfg.n_kv, cfg.head_dim
    cap = L
    copies = 8
    kv = [(ctx.alloc(nkv * cap * hd * 2), ctx.alloc(nkv * cap * hd * 2)) for _ in range(copies)]
    for k, v in kv:
        emx.lib().emx_memset(ctx.h, k.ptr, 0x3C, nkv * cap * hd * 2)
        emx.lib().emx_memset(ctx.h, v.ptr, 0x3C, nkv * cap * hd * 2)
    q = ctx.put(np.full(nq * hd, 0x3F80, np.uint16))
    out = ctx.alloc(nq * hd * 2)
    scale = 1.0 / float(np.sqrt(hd))
    for i in range(4):
        ctx.sdpa_decode_noalloc(q, kv[i][0], kv[i][1], out, nq, nkv, cap, hd, L, scale)
    ctx.synchronize()
    n = 64
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for i in range(n):
        k, v = kv[i % copies]
        ctx.sdpa_decode_noalloc(q, k, v, out, nq, nkv, cap, hd, L, scale)
    e1.record(st)
    e1.synchronize()
    us = e0.elapsed_time(e1) * 1000.0 / n
    for k, v in kv:
        k.free()
        v.free()
    q.free()
    out.free()
    per = 2 * nkv * L * hd * 2 + 2 * nq * hd * 2
    ach = per / (us * 1e-6) / 1e9
    return {"kernel": "attn_decode_kernel (split-KV flash-decode)", "shape": {"n_q": nq, "n_kv": nkv, "rows": L},
            "bound": "hbm", "achieved": ach, "peak": hbm, "unit": "GB/s", "frac": ach / hbm, "us_per_call": us,
            "bytes_per_call": per, "traffic": None}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1024)
    ap.add_argument("--warmup", type=int, default=16)
    ap.add_argument("--config", default="c3")
    ap.add_argument("--prompt", type=int, default=128)
    ap.add_argument("--prefill-lengths", type=int, nargs="*", default=[128, 2048, 8192])
    ap.add_argument("--impl", default="emx", choices=["emx", "reference"])
    ap.add_argument("--seed", type=int, default=1234)
    ap.add_argument("--cpu-steps", type=int, default=4)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--eager", action="store_true",
                    help="decode without the CUDA graph (kernels in plain stream order): for profilers")
    ap.add_argument("--shard", action="store_true",
                    help="with N > 1: one model split across the N GPUs (tensor parallel for dense, expert "
                         "parallel for MoE; NCCL all-reduce) instead of N replicas")
    ap.add_argument("--per-op", action="store_true",
                    help="decode with one kernel per operation instead of the persistent step kernel")
    ap.add_argument("--no-sharded", action="store_true",
                    help="skip the tensor-parallel 32B-shape measurement added to every line")
    ap.add_argument("--no-moe", action="store_true",
                    help="skip the expert-parallel 30B-A3B-shape prefill + decode measurement added to every line")
    ap.add_argument("--profile-range", action="store_true",
                    help="with --kernel-only step / prefill: bracket the timed region with cudaProfilerStart / "
                         "Stop (for ncu --profile-from-start off)")
    ap.add_argument("--kernel-only", nargs="?", const="gemv", default=None,
                    choices=["gemv", "gemm", "attn", "prefill", "c1", "step"],
                    help="time one kernel alone and print its roofline: the packed decode GEMV (gate|up shape, "
                         "default), the prefill GEMM (gate|up shape, 2048 rows), decode attention (8192 rows), "
                         "one whole prefill of --prompt tokens, or --steps decode steps (step)")
    args = ap.parse_args()

    import emx

    cfg = emx.CONFIGS[args.config]
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if args.impl == "reference":
        run_reference(args, cfg, rank)
        return
    import dataclasses

    cfg = dataclasses.replace(cfg, kv_cap=max(cfg.kv_cap, args.prompt + args.steps + max(args.warmup, 3) + 8))
    dist = None
    if world > 1:
        import datetime

        import torch
        import torch.distributed as td

        torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
        td.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
        dist = td
    try:
        run_engine(args, cfg, rank, world, dist)
    finally:
        if dist is not None:
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
