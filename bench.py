#!/usr/bin/env python
"""Decode-attention benchmark for the B200 attention operator.

A step is one decode step of the whole layer stack's attention op: for every layer, the fused
append (QK-norm + RoPE + fp16 store of the new K/V) and decode attention over the resident
fp16 KV cache, for B independent sequences, one new token each.  Default workload: the
Qwen3-4B shape of BASELINE config 2 (36 layers, 32 q / 8 kv heads, head_dim 128, KV length
4096, batch 64).  Inputs are seeded synthetic N(0,1) tensors (there is no dataset).

value   = KV bytes read per step (fp16, all layers, all sequences, all ranks) / step time, GB/s,
          with inputs resident in HBM; CUDA events on the launching stream, max over ranks.
e2e     = the same metric through the public host API with the step's q/k/v inputs copied from
          pinned host memory and the attention outputs copied back inside the timed region; the
          copies of layer l run on copy streams, overlapped with the attention of other layers.
N > 1   = strong scaling (default): the global batch (64 for the default workload) is split
          over the N ranks, B/N independent sequences per GPU, no communication on the path;
          --weak gives every rank the full batch instead.  value and tokens/s are whole-job
          figures (all ranks' KV bytes or tokens over the max-over-ranks step time).
prefill = at N = 1 the default run also measures BASELINE config 3 (Qwen3-4B chunked prefill on
          the tensor-core kernel) and reports it, with its own roofline and CPU baseline, under
          the line's "prefill" key (--no-prefill skips it).

--impl reference times the reference's CPU attention (the C restatement of attentionCpu in
oracle/, the reference itself being TypeScript with no JavaScript runtime on the box) on the
host cores, on a bounded sample of the same workload.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

CONFIGS = {
    # the reference's CPU-runnable case (Qwen2.5-0.5B, one layer, one sequence).
    "qwen2.5-0.5b": dict(layers=1, Hq=14, Hkv=2, D=64, L=1025, base=1e6, qk_norm=False, batch=1, scale=None,
                         softcap=0.0, window_even=0, ff=None, d_model=896),
    # BASELINE config 2 at batch 64 (the north-star target shape).
    "qwen3-4b": dict(layers=36, Hq=32, Hkv=8, D=128, L=4096, base=1e6, qk_norm=True, batch=64, scale=None,
                     softcap=0.0, window_even=0, ff=None, d_model=2560),
    # BASELINE config 4.
    "gemma2-2b": dict(layers=26, Hq=8, Hkv=4, D=256, L=8192, base=1e4, qk_norm=False, batch=32, scale=1 / 16,
                      softcap=50.0, window_even=4096, ff=None, d_model=2304),
    # 2048-token prompt in 512-token chunks on the tensor-core prefill kernel.
    "qwen3-4b-prefill": dict(layers=36, Hq=32, Hkv=8, D=128, L=2048, chunk=512, base=1e6, qk_norm=True, batch=4,
                             scale=None, softcap=0.0, window_even=0, ff=None, prefill=True),
    # BASELINE config 5 on one GPU (the long-context shape; sequence sharding is the multi-GPU form).
    "llama3.2-1b-long": dict(layers=16, Hq=32, Hkv=8, D=64, L=131072, base=5e5, qk_norm=False, batch=8, scale=None,
                             softcap=0.0, window_even=0, ff=(32.0, 1.0, 4.0, 8192), d_model=2048),
}


def kv_bytes_per_step(c, batch):
    """Algorithmic KV bytes one step reads: per layer and sequence, K and V rows of the attended
    range (the window on windowed layers), Hkv x D fp16 each -- or, for the int8 cache, Hkv x D
    one-byte codes plus one f32 scale per (row, kv head)."""
    row_bytes = c["D"] + 4 if c.get("kv") == "q8" else c["D"] * 2
    total = 0
    for layer in range(c["layers"]):
        keys = c["L"]
        if c["window_even"] and layer % 2 == 0:
            keys = min(keys, c["window_even"])
        total += batch * keys * c["Hkv"] * row_bytes * 2
    return total


def weight_bytes_per_step(c):
    """fp16 q/k/v and output projection weights of every layer (read once per decode step)."""
    d, qd, kvd = c["d_model"], c["Hq"] * c["D"], c["Hkv"] * c["D"]
    return c["layers"] * (qd + 2 * kvd + qd) * d * 2


def prefill_flops(c, batch):
    """Causal-exact FLOPs of one prefill launch per chunk: QK^T and PV, 2 FLOPs per MAC, over the
    keys each query attends (pastLen + t + 1)."""
    out = []
    T = c["chunk"]
    for c0 in range(0, c["L"], T):
        keys = sum(c0 + t + 1 for t in range(min(T, c["L"] - c0)))
        out.append(4 * c["D"] * keys * c["Hq"] * batch)
    return out


class CopyPipeline:
    """The e2e legs' host <-> device traffic, overlapped with the attention as a serving host
    would do it: unit i's inputs are copied from pinned host memory on one stream ahead of unit
    i's attention; its output is copied back on another stream as soon as it is done.  Every copy
    of the step stays inside the timed region (the compute stream waits for the last one)."""

    def __init__(self, dev, n):
        import torch
        self.torch = torch
        self.cin = torch.cuda.Stream(device=dev)
        self.cout = torch.cuda.Stream(device=dev)
        self.ev_in = [torch.cuda.Event() for _ in range(n)]
        self.ev_done = [torch.cuda.Event() for _ in range(n)]

    def run(self, stream, n, h2d, compute, d2h):
        torch = self.torch
        self.cin.wait_stream(stream)  # the previous step is done with the device buffers
        with torch.cuda.stream(self.cin):
            for i in range(n):
                h2d(i)
                self.ev_in[i].record(self.cin)
        for i in range(n):
            stream.wait_event(self.ev_in[i])
            compute(i)
            self.ev_done[i].record(stream)
            self.cout.wait_event(self.ev_done[i])
            with torch.cuda.stream(self.cout):
                d2h(i)
        stream.wait_stream(self.cout)


def load_tflops_peak():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as fh:
            js = json.load(fh)
            return float(js["bf16_tflops_sustained"]), float(js["bf16_tflops"]), "measured"
    except Exception:
        return 1400.0, 1590.0, "fallback"


def cpu_prefill_sample(c, target_s, seed=13):
    """Time the CPU attention (oracle restatement of attentionCpu) on a bounded sample of the
    prefill workload: the last chunk of one sequence of one layer (its queries attend the whole
    prompt so far), repeated for about target_s seconds.  Returns (TFLOP/s, threads, desc) with the
    FLOPs counted causal-exact like the GPU line."""
    import numpy as np

    from oracle import oracle as O

    rng = np.random.default_rng(seed)
    P, T, Hq, Hkv, D = c["L"], c["chunk"], c["Hq"], c["Hkv"], c["D"]
    past = P - T
    k = rng.standard_normal(P * Hkv * D, dtype=np.float32)
    v = rng.standard_normal(P * Hkv * D, dtype=np.float32)
    q = rng.standard_normal(T * Hq * D, dtype=np.float32)
    flops = 4 * D * sum(past + t + 1 for t in range(T)) * Hq
    t0 = time.perf_counter()
    _, used = O.attention_batch(q, k, v, 1, P * Hkv * D, T, Hq, Hkv, D, [past], c["scale"], c["softcap"], 0, 0)
    reps = max(1, int(target_s / max(time.perf_counter() - t0, 1e-3)))
    t0 = time.perf_counter()
    for _ in range(reps):
        O.attention_batch(q, k, v, 1, P * Hkv * D, T, Hq, Hkv, D, [past], c["scale"], c["softcap"], 0, 0)
    dt = time.perf_counter() - t0
    desc = (f"{reps} x the last {T}-token chunk of one sequence and layer (past {past}, {Hq}q/{Hkv}kv, D {D}), "
            f"JS-faithful double arithmetic over f32 q/K/V, {used} threads, {dt:.1f} s; FLOPs counted "
            f"causal-exact as on the GPU")
    return reps * flops / dt / 1e12, used, desc


def run_prefill(args, c, workload, eng=None, emit=True):
    """Prefill bench: a step is the whole prompt through every layer, chunk by chunk: append
    (QK-norm + RoPE + fp16 store) then the tensor-core prefill kernel over the cache so far.
    With `eng` (the default decode run at N = 1) it reuses that engine and returns its line
    instead of printing it."""
    import torch
    import torch.distributed as dist

    from brimkern_b200.engine import AttentionEngine, AttnConfig, KvCache, RopeTable

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    own_engine = eng is None
    if world > 1 and own_engine:
        import datetime
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    B, P, CH, layers = args.batch, c["L"], c["chunk"], c["layers"]
    Hq, Hkv, D = c["Hq"], c["Hkv"], c["D"]
    nch = (P + CH - 1) // CH
    if own_engine:
        eng = AttentionEngine(local)
    rope = RopeTable(eng.ctx, D, c["base"], None, P)
    gen = torch.Generator(device=dev)
    gen.manual_seed(2000 + rank)
    qn = (1 + 0.02 * torch.randn(D, generator=gen, device=dev)).float()
    kn = (1 + 0.02 * torch.randn(D, generator=gen, device=dev)).float()
    cfg = AttnConfig(Hq, Hkv, D, q_norm=qn, k_norm=kn, rope=rope)
    q8 = c.get("kv") == "q8"
    kv = KvCache(eng.ctx, layers, B, Hkv, D, P, q8=q8)
    q_in = torch.randn((layers, nch, B, CH, Hq, D), generator=gen, device=dev)
    k_in = torch.randn((layers, nch, B, CH, Hkv, D), generator=gen, device=dev)
    v_in = torch.randn((layers, nch, B, CH, Hkv, D), generator=gen, device=dev)
    q_work = torch.empty((B, CH, Hq, D), dtype=torch.float32, device=dev)
    q16_work = torch.empty((B, CH, Hq, D), dtype=torch.float16, device=dev)
    out = torch.empty((layers, nch, B, CH, Hq, D), dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream()
    flops = prefill_flops(c, B)

    def step(ev=None, qi=q_in, ki=k_in, vi=v_in, oo=out):
        for layer in range(layers):
            for ci in range(nch):
                pos = [ci * CH] * B
                if ev is None:
                    # The product path: K/V append + tensor-core kernel with the q prologue fused.
                    eng.prefillStep(kv, layer, cfg, qi[layer, ci], ki[layer, ci], vi[layer, ci], oo[layer, ci], pos)
                else:
                    # Roofline pass: the attention kernel alone, on pre-rotated q -- fp16 rows loaded
                    # with TMA as in the product path (fp16 cache), or f32 rows it stages (int8).
                    eng.appendKv(kv, layer, cfg, qi[layer, ci], ki[layer, ci], vi[layer, ci], q_work, pos)
                    if not q8:
                        q16_work.copy_(q_work)
                    ev[layer][ci][0].record(stream)
                    if q8:
                        eng.recAttention(kv, layer, cfg, q_work, oo[layer, ci], pos, kernel="prefill")
                    else:
                        eng.prefillHalfQ(kv, layer, cfg, q16_work, oo[layer, ci], pos)
                    ev[layer][ci][1].record(stream)

    def barrier():
        if world > 1:
            dist.barrier()

    for _ in range(args.warmup):
        step()
    eng.ctx.check()
    barrier()
    torch.cuda.synchronize()
    vis = os.environ.get("CUDA_VISIBLE_DEVICES", "").split(",")
    sampler = ClockSampler(int(vis[local]) if len(vis) > local and vis[local].strip().isdigit() else local)
    sampler.start()
    time.sleep(0.3)
    n0 = eng.ctx.launches
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        step()
    e1.record(stream)
    torch.cuda.synchronize()
    launches = eng.ctx.launches - n0
    clocks = sampler.stop()
    eng.ctx.check()
    barrier()
    ms_total = e0.elapsed_time(e1)
    rsteps = max(2, min(args.steps, 3))
    ev = [[[[torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)] for _ in range(nch)]
           for _ in range(layers)] for _ in range(rsteps)]
    for si in range(rsteps):
        step(ev[si])
    torch.cuda.synchronize()
    eng.ctx.check()
    kern_ms = sum(ev[si][l][ci][0].elapsed_time(ev[si][l][ci][1]) for si in range(rsteps) for l in range(layers)
                  for ci in range(nch)) / rsteps
    if world > 1:
        t = torch.tensor([ms_total], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms_total = float(t.item())
    ms_step = ms_total / args.steps
    step_flops = sum(flops) * layers
    value = world * step_flops / (ms_step * 1e-3) / 1e12
    sus, burst, kind = load_tflops_peak()
    achieved = step_flops / (kern_ms * 1e-3) / 1e12
    e2e = None
    if not args.no_e2e:
        hq, hk, hv = q_in.cpu().pin_memory(), k_in.cpu().pin_memory(), v_in.cpu().pin_memory()
        hout = torch.empty(out.shape, dtype=torch.float32, pin_memory=True)
        dq, dk, dv, do = torch.empty_like(q_in), torch.empty_like(k_in), torch.empty_like(v_in), torch.empty_like(out)

        units = [(layer, ci) for layer in range(layers) for ci in range(nch)]
        pipe = CopyPipeline(dev, len(units))

        def h2d(i):
            layer, ci = units[i]
            dq[layer, ci].copy_(hq[layer, ci], non_blocking=True)
            dk[layer, ci].copy_(hk[layer, ci], non_blocking=True)
            dv[layer, ci].copy_(hv[layer, ci], non_blocking=True)

        def compute(i):
            layer, ci = units[i]
            eng.prefillStep(kv, layer, cfg, dq[layer, ci], dk[layer, ci], dv[layer, ci], do[layer, ci], [ci * CH] * B)

        def d2h(i):
            layer, ci = units[i]
            hout[layer, ci].copy_(do[layer, ci], non_blocking=True)

        def e2e_step():
            pipe.run(stream, len(units), h2d, compute, d2h)

        e2e_step()
        torch.cuda.synchronize()
        f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        esteps = max(1, min(args.steps, 3))
        f0.record(stream)
        for _ in range(esteps):
            e2e_step()
        f1.record(stream)
        torch.cuda.synchronize()
        e_ms = f0.elapsed_time(f1) / esteps
        e2e = {"value": round(world * step_flops / (e_ms * 1e-3) / 1e12, 2), "unit": "TFLOP/s",
               "h2d_bytes_per_step": int((hq.numel() + hk.numel() + hv.numel()) * 4),
               "d2h_bytes_per_step": int(hout.numel() * 4), "ms_per_step": round(e_ms, 3)}
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        tf, used, desc = cpu_prefill_sample(c, 8.0)
        cpu = {"value": round(tf, 6), "unit": "TFLOP/s", "cores": used, "kind": "port", "sample": desc}
    line = None
    if rank == 0:
        line = {
            "metric": "prefill-attn TFLOP/s (causal-exact)", "value": round(value, 2), "unit": "TFLOP/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": ("int8 KV codes dequantized to an fp16 stage per call, f16 MMA / f32 accumulate" if q8 else
                      "f16 in / f32 accumulate"),
            "data": "synthetic",
            "config": {"workload": workload, "kv_cache": "int8" if q8 else "fp16", "global_batch": B * world,
                       "prompt": P, "chunk": CH, "layers": layers,
                       "heads": f"{Hq}q/{Hkv}kv", "head_dim": D, "parallelism": f"batch-sharded x{world}",
                       "l2": "no flush: KV + inputs of a step are 4.2 GB > L2"},
            "tokens_per_s": round(world * B * P / (ms_step * 1e-3), 1),
            "roofline": {"bound": "tensor", "achieved": round(achieved, 1), "peak": sus, "unit": "TFLOP/s",
                         "frac": round(achieved / sus, 4), "frac_of_burst": round(achieved / burst, 4),
                         "traffic": None, "peak_kind": kind + " sustained bf16 (fp16 runs at the same rate)",
                         "kernel": "prefill_attn_kernel", "timing": (f"CUDA events around each prefill launch, {rsteps} steps; q given pre-rotated "
                                    + ("as f32 rows it stages" if q8 else "as fp16 rows it loads with TMA, as in the step")),
                         "flops_per_step": step_flops, "kernel_ms_per_step": round(kern_ms, 4)},
            "cpu_baseline": cpu, "e2e": e2e, "gpu_launches": int(launches), "clocks": clocks,
        }
        if emit:
            print(json.dumps(line), flush=True)
    kv.close()
    rope.close()
    if not own_engine:
        return line
    eng.close()
    if world > 1:
        dist.destroy_process_group()
    return 0


def run_sharded(args, c, workload):
    """Config 5 on N GPUs: the KV sequence is split across ranks (ShardPlan), each rank decodes
    its slice to (m, l, o) partials that its decode kernel stores straight into every rank's
    exchange area over NVLink (--sharded-nccl: one NCCL all-gather per layer instead), LSE combine
    on every rank.  Strong scaling: the context (and total KV bytes) is fixed, N GPUs share it."""
    import datetime

    import torch
    import torch.distributed as dist

    from brimkern_b200.engine import AttentionEngine, AttnConfig, RopeTable, llama3_rope_factors
    from brimkern_b200.sharded import ShardedDecoder, ShardPlan

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    B, Lkv, layers = args.batch, c["L"], c["layers"]
    Hq, Hkv, D = c["Hq"], c["Hkv"], c["D"]
    context = Lkv - 1                      # cached positions; the step appends position Lkv - 1
    plan = ShardPlan(context, world, rank)
    eng = AttentionEngine(local)
    ff = llama3_rope_factors(D, c["base"], *c["ff"]) if c["ff"] else None
    rope = RopeTable(eng.ctx, D, c["base"], ff, Lkv)
    cfg = AttnConfig(Hq, Hkv, D, scale=c["scale"], softcap=c["softcap"], rope=rope)
    fused = not args.sharded_nccl
    dec = ShardedDecoder(eng, plan, layers, B, Hkv, D, extra=1, fused=fused, max_rows=B * Hq)
    gen = torch.Generator(device=dev)
    gen.manual_seed(3000 + rank)
    rows = plan.hi - plan.lo
    if rows > 0:
        tmp_k = torch.empty((rows, Hkv, D), dtype=torch.float32, device=dev)
        tmp_v = torch.empty_like(tmp_k)
        for layer in range(layers):
            for b in range(B):
                tmp_k.normal_(generator=gen)
                tmp_v.normal_(generator=gen)
                dec.kv.write_rows(layer, b, 0, tmp_k, tmp_v)
        del tmp_k, tmp_v
    shared = torch.Generator(device=dev)
    shared.manual_seed(4000)  # q / k / v inputs replicated on every rank
    q_in = torch.randn((layers, B, 1, Hq, D), generator=shared, device=dev)
    k_in = torch.randn((layers, B, 1, Hkv, D), generator=shared, device=dev)
    v_in = torch.randn((layers, B, 1, Hkv, D), generator=shared, device=dev)
    q_work = torch.empty((B, 1, Hq, D), dtype=torch.float32, device=dev)
    out = torch.empty((layers, B, 1, Hq, D), dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream()
    position = Lkv - 1

    def step():
        for layer in range(layers):
            dec.step(layer, cfg, q_in[layer], k_in[layer], v_in[layer], position, q_work, out[layer])

    for _ in range(args.warmup):
        step()
    eng.ctx.check()
    dist.barrier()
    torch.cuda.synchronize()
    vis = os.environ.get("CUDA_VISIBLE_DEVICES", "").split(",")
    sampler = ClockSampler(int(vis[local]) if len(vis) > local and vis[local].strip().isdigit() else local)
    sampler.start()
    time.sleep(0.3)
    n0 = eng.ctx.launches
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        step()
    e1.record(stream)
    torch.cuda.synchronize()
    launches = eng.ctx.launches - n0
    clocks = sampler.stop()
    eng.ctx.check()
    dist.barrier()
    t = torch.tensor([e0.elapsed_time(e1)], device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_step = float(t.item()) / args.steps
    bytes_step = kv_bytes_per_step(c, B)
    value = bytes_step / (ms_step * 1e-3) / 1e9
    peak, peak_kind = load_peak()
    if rank == 0:
        line = {
            "metric": "decode-attn KV-read GB/s", "value": round(value, 2), "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 4), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f16 KV / f32 accumulate", "data": "synthetic",
            "config": {"workload": workload, "global_batch": B, "kv_len": Lkv, "layers": layers,
                       "heads": f"{Hq}q/{Hkv}kv", "head_dim": D,
                       "parallelism": (f"sequence-sharded x{world}: the decode kernel stores its (m, l, o) partials "
                                       "into every rank's exchange area over NVLink (CUDA IPC), flag-synchronised "
                                       "combine" if fused else
                                       f"sequence-sharded x{world}: per-layer NCCL all-gather of (m, l, o) partials"),
                       "l2": f"no flush: each step streams {bytes_step / 1e9:.1f} GB of KV > L2"},
            "tokens_per_s": round(B / (ms_step * 1e-3), 1),
            "frac_of_measured_hbm_per_gpu": round(value / world / peak, 4),
            "allgather_bytes_per_rank_per_layer": B * Hq * (D + 2) * 4,
            "roofline": None, "cpu_baseline": None, "e2e": None, "gpu_launches": int(launches), "clocks": clocks,
        }
        print(json.dumps(line), flush=True)
    dec.close()
    eng.close()
    dist.destroy_process_group()
    return 0


def load_peak():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as fh:
            return float(json.load(fh)["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def read_traffic(workload, batch, bytes_launch):
    """DRAM bytes per decode launch from the committed ncu summary of this workload: the capture at
    this batch if one exists, else the default capture scaled by the algorithmic bytes (the
    kernel's traffic grows with the KV it streams).  Returns (bytes or None, note)."""
    for name in (f"decode_{workload}_b{batch}.md", f"decode_{workload}.md"):
        path = os.path.join(ROOT, "profiles", name)
        dram = alg = None
        try:
            for line in open(path):
                if line.startswith("dram_bytes_per_launch:"):
                    dram = float(line.split(":", 1)[1].strip().split()[0])
                elif line.startswith("algorithmic_bytes_per_launch:"):
                    alg = float(line.split(":", 1)[1].strip().split()[0])
        except OSError:
            continue
        if dram is None or alg is None:
            continue
        if abs(alg - bytes_launch) < 1:
            return dram, f"ncu capture profiles/{name}"
        return round(dram * bytes_launch / alg), f"ncu capture profiles/{name} scaled by algorithmic bytes"
    return None, "no ncu capture of this workload"


class ClockSampler:
    """nvidia-smi clock / throttle sampling during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu_index = gpu_index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "100", "-i", str(self.gpu_index)], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.thread.join(timeout=5)
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = max(mx, float(parts[2]))
            except ValueError:
                continue
            for name, val in zip(names, parts[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(name)
        if not sm:
            return None
        sm.sort()
        return {"sm_mhz": sm[len(sm) // 2], "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


def cpu_reference_sample(c, batch, target_s, threads=0, seed=7, with_time=False):
    """Time the CPU attention (oracle restatement of attentionCpu) on a bounded sample of the
    workload: whole (layer, sequence) decode units at the configured KV length, repeated over a
    pool of 8 sequences until about target_s seconds of work.  Returns (GB/s, threads, desc), and
    the timed seconds as a fourth value with with_time."""
    import numpy as np

    from oracle import oracle as O

    rng = np.random.default_rng(seed)
    keys = c["L"]
    per_seq = keys * c["Hkv"] * c["D"] * 4 * 2
    pool = max(1, min(batch, 8, (1 << 30) // per_seq))
    k = rng.standard_normal(pool * keys * c["Hkv"] * c["D"], dtype=np.float32)
    v = rng.standard_normal(pool * keys * c["Hkv"] * c["D"], dtype=np.float32)
    q = rng.standard_normal(pool * c["Hq"] * c["D"], dtype=np.float32)
    past = [keys - 1] * pool
    stride = keys * c["Hkv"] * c["D"]
    t0 = time.perf_counter()
    _, used = O.attention_batch(q, k, v, pool, stride, 1, c["Hq"], c["Hkv"], c["D"], past, c["scale"], c["softcap"],
                                0, threads)
    first = time.perf_counter() - t0
    reps = max(1, int(target_s / max(first, 1e-3)))
    t0 = time.perf_counter()
    for _ in range(reps):
        O.attention_batch(q, k, v, pool, stride, 1, c["Hq"], c["Hkv"], c["D"], past, c["scale"], c["softcap"], 0,
                          threads)
    dt = time.perf_counter() - t0
    units = reps * pool
    q8 = c.get("kv") == "q8"
    row_bytes = c["D"] + 4 if q8 else c["D"] * 2
    gbs = units * keys * c["Hkv"] * row_bytes * 2 / dt / 1e9  # K+V bytes of those units in the cache type
    desc = (f"{units} (layer, sequence) decode units at KV length {keys} ({c['Hq']}q/{c['Hkv']}kv, D {c['D']}), "
            f"JS-faithful double arithmetic over f32 K/V, {used} threads, {dt:.1f} s; bytes counted as the "
            f"{'int8 codes + scales' if q8 else 'fp16 KV'} of those units")
    return (gbs, used, desc, dt) if with_time else (gbs, used, desc)


def cpu_slice_sample(c, target_s, pool=8, seed=11):
    """CPU attention slice (oracle rmsnormCpu + matmulCpu + attentionCpu + matmulCpu) of one layer
    for `pool` sequences, repeated for about target_s seconds.  Returns (GB/s, threads, desc) with
    the bytes counted as the fp16 weights of the layer plus the fp16 KV of those sequences."""
    import numpy as np

    from oracle import oracle as O

    rng = np.random.default_rng(seed)
    d, Hq, Hkv, D, keys = c["d_model"], c["Hq"], c["Hkv"], c["D"], c["L"]
    qd, kvd = Hq * D, Hkv * D
    w_qkv = (rng.standard_normal((qd + 2 * kvd, d), dtype=np.float32) / np.sqrt(d)).astype(np.float32)
    w_o = (rng.standard_normal((d, qd), dtype=np.float32) / np.sqrt(qd)).astype(np.float32)
    g = np.ones(d, np.float32)
    x = rng.standard_normal((pool, d), dtype=np.float32)
    k = rng.standard_normal(pool * keys * kvd, dtype=np.float32)
    v = rng.standard_normal(pool * keys * kvd, dtype=np.float32)
    stride = keys * kvd

    def once():
        n1 = O.rmsnorm(x.ravel(), g, pool, d, 1e-6)
        qkv = O.matmul_t(n1, w_qkv, pool, d, qd + 2 * kvd).reshape(pool, -1)
        q = np.ascontiguousarray(qkv[:, :qd]).ravel()
        att, used = O.attention_batch(q, k, v, pool, stride, 1, Hq, Hkv, D, [keys - 1] * pool, c["scale"],
                                      c["softcap"], 0, 0)
        O.matmul_t(att, w_o, pool, qd, d)
        return used

    t0 = time.perf_counter()
    used = once()
    reps = max(1, int(target_s / max(time.perf_counter() - t0, 1e-3)))
    t0 = time.perf_counter()
    for _ in range(reps):
        once()
    dt = time.perf_counter() - t0
    units = reps
    byts = units * ((qd + 2 * kvd + qd) * d * 2 + pool * keys * kvd * 2 * 2)
    desc = (f"{units} single-layer slices of {pool} sequences at KV length {keys}: rmsnormCpu + matmulCpu "
            f"(double sums, one thread) + attentionCpu ({used} threads) + matmulCpu, {dt:.1f} s; bytes counted as "
            f"the fp16 weights of the layer + the fp16 KV of those sequences")
    return byts / dt / 1e9, used, desc


def run_slice(args, c, workload):
    """The attention slice of a decode step (recordLayerKV, kernels.ts:1700-1736): per layer,
    RMSNorm + q/k/v projections, QK-norm + RoPE + append + decode attention, output projection +
    residual.  value = (fp16 weights + KV) bytes per step / step time."""
    import torch

    from brimkern_b200.engine import AttentionEngine, AttnConfig, KvCache, RopeTable, llama3_rope_factors

    if int(os.environ.get("WORLD_SIZE", "1")) > 1:
        raise SystemExit("--slice runs on one GPU")
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    B, Lkv, layers = args.batch, c["L"], c["layers"]
    Hq, Hkv, D, d = c["Hq"], c["Hkv"], c["D"], c["d_model"]
    qd, kvd = Hq * D, Hkv * D
    eng = AttentionEngine(0)
    ff = llama3_rope_factors(D, c["base"], *c["ff"]) if c["ff"] else None
    rope = RopeTable(eng.ctx, D, c["base"], ff, Lkv)
    gen = torch.Generator(device=dev)
    gen.manual_seed(3000)
    qn = kn = None
    if c["qk_norm"]:
        qn = (1 + 0.02 * torch.randn(D, generator=gen, device=dev)).float()
        kn = (1 + 0.02 * torch.randn(D, generator=gen, device=dev)).float()
    cfgs = [AttnConfig(Hq, Hkv, D, scale=c["scale"], softcap=c["softcap"],
                       window=c["window_even"] if (c["window_even"] and l % 2 == 0) else 0, q_norm=qn, k_norm=kn,
                       rope=rope) for l in range(layers)]

    def w(n, k):
        return (torch.randn((n, k), generator=gen, device=dev) / k ** 0.5).half()

    wq = [w(qd, d) for _ in range(layers)]
    wk = [w(kvd, d) for _ in range(layers)]
    wv = [w(kvd, d) for _ in range(layers)]
    wo = [w(d, qd) for _ in range(layers)]
    g1 = [(1 + 0.02 * torch.randn(d, generator=gen, device=dev)).float() for _ in range(layers)]
    kv = KvCache(eng.ctx, layers, B, Hkv, D, Lkv)
    tmp_k = torch.empty((Lkv, Hkv, D), dtype=torch.float32, device=dev)
    tmp_v = torch.empty_like(tmp_k)
    for layer in range(layers):
        for b in range(B):
            tmp_k.normal_(generator=gen)
            tmp_v.normal_(generator=gen)
            kv.write_rows(layer, b, 0, tmp_k, tmp_v)
    del tmp_k, tmp_v
    past = [Lkv - 1] * B
    x = torch.randn((layers, B, d), generator=gen, device=dev)
    h = torch.empty_like(x)
    q = torch.empty((B, qd), device=dev)
    k = torch.empty((B, kvd), device=dev)
    v = torch.empty_like(k)
    q_work = torch.empty((B, 1, Hq, D), device=dev)
    att = torch.empty((B, 1, Hq, D), device=dev)
    eng.ctx.reserve(64 << 20)
    stream = torch.cuda.current_stream()

    def layer_slice(layer, xi, hi, ev=None):
        if ev is not None:
            ev[0].record(stream)
        eng.projQkv(xi, wq[layer], wk[layer], wv[layer], q, k, v, attn_norm=g1[layer], eps=1e-6)
        if ev is None:
            eng.attentionLayer(kv, layer, cfgs[layer], q.view(B, 1, Hq, D), k.view(B, 1, Hkv, D),
                               v.view(B, 1, Hkv, D), past, q_work, att)
        else:
            ev[1].record(stream)
            eng.appendKv(kv, layer, cfgs[layer], q.view(B, 1, Hq, D), k.view(B, 1, Hkv, D), v.view(B, 1, Hkv, D),
                         q_work, past)
            ev[2].record(stream)
            eng.recAttention(kv, layer, cfgs[layer], q_work, att, past)
            ev[3].record(stream)
        eng.projOut(att.view(B, qd), wo[layer], xi, hi)
        if ev is not None:
            ev[4].record(stream)

    def step(ev=None):
        for layer in range(layers):
            layer_slice(layer, x[layer], h[layer], None if ev is None else ev[layer])

    for _ in range(args.warmup):
        step()
    eng.ctx.check()
    torch.cuda.synchronize()

    def capture(fn):
        side = torch.cuda.Stream(device=dev)
        side.wait_stream(stream)
        with torch.cuda.stream(side):
            fn()
        stream.wait_stream(side)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        n0 = eng.ctx.launches
        with torch.cuda.graph(g):
            fn()
        g.launches = eng.ctx.launches - n0  # kernels one replay launches
        g.replay()
        torch.cuda.synchronize()
        eng.ctx.check()
        return g

    def timed(g, reps):
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record(stream)
        for _ in range(reps):
            g.replay()
        t1.record(stream)
        torch.cuda.synchronize()
        return t0.elapsed_time(t1) / reps

    graph = None if args.eager else capture(step)
    sampler = ClockSampler(0)
    sampler.start()
    time.sleep(0.3)
    n0 = eng.ctx.launches
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        if graph is None:
            step()
        else:
            graph.replay()
    e1.record(stream)
    torch.cuda.synchronize()
    # Per layer: cast + GEMM for q/k/v, append + decode, cast + GEMM for the output.
    launches = eng.ctx.launches - n0 if graph is None else args.steps * graph.launches
    clocks = sampler.stop()
    eng.ctx.check()
    ms_step = e0.elapsed_time(e1) / args.steps
    rsteps = max(2, min(args.steps, 5))
    if args.eager:
        ev = [[[torch.cuda.Event(enable_timing=True) for _ in range(5)] for _ in range(layers)]
              for _ in range(rsteps)]
        for si in range(rsteps):
            step(ev[si])
        torch.cuda.synchronize()
        eng.ctx.check()
        n = rsteps * layers
        proj_ms = sum(e[0].elapsed_time(e[1]) + e[3].elapsed_time(e[4]) for es in ev for e in es) / n
        attn_ms = sum(e[2].elapsed_time(e[3]) for es in ev for e in es) / n
    else:
        # The projections alone and the decode kernels alone, each as a graph of every layer's
        # launches back to back (inputs from the warm-up steps).
        def projections():
            for layer in range(layers):
                eng.projQkv(x[layer], wq[layer], wk[layer], wv[layer], q, k, v, attn_norm=g1[layer], eps=1e-6)
                eng.projOut(att.view(B, qd), wo[layer], x[layer], h[layer])

        def decodes():
            for layer in range(layers):
                eng.recAttention(kv, layer, cfgs[layer], q_work, att, past)

        gp, gd = capture(projections), capture(decodes)
        proj_ms = timed(gp, rsteps) / layers
        attn_ms = timed(gd, rsteps) / layers
        del gp, gd
    wbytes = weight_bytes_per_step(c)
    kbytes = kv_bytes_per_step(c, B)
    value = (wbytes + kbytes) / (ms_step * 1e-3) / 1e9
    peak, peak_kind = load_peak()
    wl = wbytes / layers
    proj_ach = wl / (proj_ms * 1e-3) / 1e9
    attn_ach = kbytes / layers / (attn_ms * 1e-3) / 1e9
    e2e = None
    if not args.no_e2e:
        hx = x.cpu().pin_memory()
        hh = torch.empty(h.shape, dtype=torch.float32, pin_memory=True)
        dx, dh = torch.empty_like(x), torch.empty_like(h)
        pipe = CopyPipeline(dev, layers)

        def e2e_step():
            pipe.run(stream, layers, lambda l: dx[l].copy_(hx[l], non_blocking=True),
                     lambda l: layer_slice(l, dx[l], dh[l]), lambda l: hh[l].copy_(dh[l], non_blocking=True))

        for _ in range(args.warmup):
            e2e_step()
        torch.cuda.synchronize()
        f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        f0.record(stream)
        for _ in range(args.steps):
            e2e_step()
        f1.record(stream)
        torch.cuda.synchronize()
        e_step = f0.elapsed_time(f1) / args.steps
        e2e = {"value": round((wbytes + kbytes) / (e_step * 1e-3) / 1e9, 2), "unit": "GB/s",
               "h2d_bytes_per_step": int(hx.numel() * 4), "d2h_bytes_per_step": int(hh.numel() * 4),
               "ms_per_step": round(e_step, 4), "tokens_per_s": round(B / (e_step * 1e-3), 1)}
        eng.ctx.check()
    cpu = None
    if not args.no_cpu:
        gbs, used, desc = cpu_slice_sample(c, 10.0)
        cpu = {"value": round(gbs, 4), "unit": "GB/s", "cores": used, "kind": "port", "sample": desc}
    line = {
        "metric": "decode attention-slice GB/s (weights + KV)", "value": round(value, 2), "unit": "GB/s",
        "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "f16 weights + f16 KV / f32 accumulate", "data": "synthetic (random-init weights)",
        "config": {"workload": workload + "-slice", "global_batch": B, "kv_len": Lkv, "layers": layers,
                   "d_model": d, "heads": f"{Hq}q/{Hkv}kv", "head_dim": D, "parallelism": "single GPU",
                   "launch": "host launches" if args.eager else "CUDA-graph replay of the step",
                   "l2": f"no flush: each step streams {(wbytes + kbytes) / 1e9:.1f} GB > 126 MB L2"},
        "tokens_per_s": round(B / (ms_step * 1e-3), 1),
        "roofline": {"bound": "hbm", "achieved": round(proj_ach, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(proj_ach / peak, 4), "traffic": None, "peak_kind": peak_kind,
                     "kernel": "projections (norm_cast + proj_kernel, q/k/v and output)",
                     "timing": (f"CUDA events around projQkv and projOut, {rsteps} steps" if args.eager else
                                f"CUDA events around {rsteps} replays of a graph of every layer's projections"),
                     "bytes_per_layer": wl, "proj_ms_per_layer": round(proj_ms, 5),
                     "attention_ms_per_layer": round(attn_ms, 5), "attention_achieved_gbs": round(attn_ach, 1)},
        "cpu_baseline": cpu, "e2e": e2e, "gpu_launches": int(launches), "clocks": clocks,
    }
    print(json.dumps(line), flush=True)
    eng.close()
    return 0


def decode_config(c, workload, B, world, scaling):
    """The `config` object of a decode line, shared by this build's arm and the reference arm so
    that both name the same workload with the same keys (how the GPU arm launches its kernels is
    a key of its line, not of the workload)."""
    bytes_step = kv_bytes_per_step(c, B)
    q8 = c.get("kv") == "q8"
    cfg = {"workload": workload, "kv_cache": "int8" if q8 else "fp16", "global_batch": B * world,
           "batch_per_gpu": B, "kv_len": c["L"], "layers": c["layers"], "heads": f"{c['Hq']}q/{c['Hkv']}kv",
           "head_dim": c["D"],
           "parallelism": (f"batch-sharded x{world}: {B} of {B * world} sequences per GPU, no communication "
                           f"({scaling} scaling)"),
           "l2": f"no flush: each step streams {bytes_step / 1e9:.1f} GB of KV per GPU > 126 MB L2"}
    return cfg


def run_reference(args, c, workload):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    per_step_s = 2.0
    vals, secs = [], []
    for i in range(args.warmup + args.steps):
        gbs, used, desc, dt = cpu_reference_sample(c, args.batch, per_step_s, threads=0, seed=100 + i,
                                                   with_time=True)
        if i >= args.warmup:
            vals.append(gbs)
            secs.append(dt)
    value = sum(vals) / len(vals)
    world = max(1, args.gpus)
    tok_s = value * 1e9 / (kv_bytes_per_step(c, 1))
    line = {
        "metric": "decode-attn KV-read GB/s", "value": round(value, 4), "unit": "GB/s", "impl": "reference",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        # A whole step of the workload would take minutes on the host cores, so a step here is a
        # bounded sample of it: ~2 s of whole (layer, sequence) decode units, timed.  The time a
        # whole step would take at that rate is reported beside it.
        "ms_per_step": round(sum(secs) / len(secs) * 1e3, 3),
        "step_kind": "one timed sample of the workload: whole (layer, sequence) decode units for about 2 s",
        "ms_per_full_step_extrapolated": round(kv_bytes_per_step(c, args.batch * world) / (value * 1e9) * 1e3, 3),
        "sampled": {"seconds_per_step": per_step_s, "rates_gbs": [round(v, 4) for v in vals]},
        "higher_is_better": True, "scaling": args.scaling, "vs_baseline": None, "dtype": "f64",
        "data": "synthetic",
        "config": decode_config(c, workload, args.batch, world, args.scaling),
        "tokens_per_s": round(tok_s, 3),
        "cpu_baseline": {"value": round(value, 4), "unit": "GB/s", "cores": used, "kind": "port", "sample": desc},
        "e2e": {"value": round(value, 4), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def workload_sharded(workload):
    # The long-context workload shards the KV sequence over the ranks (config 5).
    return workload == "llama3.2-1b-long"


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=list(CONFIGS), default="qwen3-4b")
    ap.add_argument("--batch", type=int, default=None,
                    help="decode: global batch split over the GPUs (per GPU with --weak); prefill: per GPU")
    ap.add_argument("--weak", action="store_true",
                    help="decode on N GPUs: every GPU runs the full batch (weak scaling) instead of 1/N of it")
    ap.add_argument("--no-prefill", action="store_true",
                    help="default decode run: skip the embedded config-3 prefill measurement")
    ap.add_argument("--layers", type=int, default=None, help="override the layer count (tests only)")
    ap.add_argument("--kv-len", type=int, default=None, help="override the KV length (tests only)")
    ap.add_argument("--softcap", type=float, default=None, help="override the logit softcap (diagnostics)")
    ap.add_argument("--window", type=int, default=None, help="override the even-layer window (diagnostics)")
    ap.add_argument("--kv", choices=["f16", "q8"], default="f16",
                    help="KV cache type: fp16, or the reference's int8 mode (setKvQuant)")
    ap.add_argument("--sharded-nccl", action="store_true",
                    help="llama3.2-1b-long on N>1 GPUs: exchange partials with NCCL all-gathers (baseline)")
    ap.add_argument("--slice", action="store_true",
                    help="decode workloads: the whole attention slice (RMSNorm + q/k/v projections, attention, "
                         "output projection + residual) on one GPU")
    ap.add_argument("--eager", action="store_true",
                    help="decode: launch every kernel from the host in the timed loop instead of replaying a CUDA "
                         "graph of the step (host launch cost then dominates small batches)")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    args = ap.parse_args()
    c = dict(CONFIGS[args.workload])
    if args.layers:
        c["layers"] = args.layers
    if args.kv_len:
        c["L"] = args.kv_len
    if args.softcap is not None:
        c["softcap"] = args.softcap
    if args.window is not None:
        c["window_even"] = args.window
    c["kv"] = args.kv
    workload = args.workload
    world = int(os.environ.get("WORLD_SIZE", str(max(1, args.gpus) if args.impl == "reference" else 1)))
    decode = not c.get("prefill") and not args.slice and not (workload_sharded(workload) and world > 1)
    if decode and not args.weak:
        # Strong scaling: the global batch is split over the ranks.
        glob = args.batch or c["batch"]
        if glob % world:
            print(json.dumps({"error": f"global batch {glob} is not a multiple of {world} GPUs (use --weak)"}))
            return 2
        args.batch = glob // world
        args.scaling = "strong"
    else:
        args.batch = args.batch or c["batch"]
        args.scaling = "weak"
    args.warmup = max(args.warmup, 3)
    if args.impl == "reference":
        return run_reference(args, c, workload)
    if c.get("prefill"):
        return run_prefill(args, c, workload)
    if args.slice:
        return run_slice(args, c, workload)
    if workload == "llama3.2-1b-long" and int(os.environ.get("WORLD_SIZE", "1")) > 1:
        return run_sharded(args, c, workload)

    import numpy as np
    import torch
    import torch.distributed as dist

    from brimkern_b200.engine import AttentionEngine, AttnConfig, KvCache, RopeTable, llama3_rope_factors

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        torch.cuda.set_device(local)
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    B, Lkv, layers = args.batch, c["L"], c["layers"]
    Hq, Hkv, D = c["Hq"], c["Hkv"], c["D"]

    eng = AttentionEngine(local)
    ff = llama3_rope_factors(D, c["base"], *c["ff"]) if c["ff"] else None
    rope = RopeTable(eng.ctx, D, c["base"], ff, Lkv)
    gen = torch.Generator(device=dev)
    gen.manual_seed(1000 + rank)
    qn = kn = None
    if c["qk_norm"]:
        qn = (1 + 0.02 * torch.randn(D, generator=gen, device=dev)).float()
        kn = (1 + 0.02 * torch.randn(D, generator=gen, device=dev)).float()
    cfgs = []
    for layer in range(layers):
        window = c["window_even"] if (c["window_even"] and layer % 2 == 0) else 0
        cfgs.append(AttnConfig(Hq, Hkv, D, scale=c["scale"], softcap=c["softcap"], window=window, q_norm=qn,
                               k_norm=kn, rope=rope))
    q8 = c["kv"] == "q8"
    kv = KvCache(eng.ctx, layers, B, Hkv, D, Lkv, q8=q8)
    tmp_k = torch.empty((Lkv, Hkv, D), dtype=torch.float32, device=dev)
    tmp_v = torch.empty_like(tmp_k)
    for layer in range(layers):
        for b in range(B):
            tmp_k.normal_(generator=gen)
            tmp_v.normal_(generator=gen)
            kv.write_rows(layer, b, 0, tmp_k, tmp_v)
    del tmp_k, tmp_v
    past = [Lkv - 1] * B  # KV length Lkv including the token appended each step
    q_in = torch.randn((layers, B, 1, Hq, D), generator=gen, device=dev)
    k_in = torch.randn((layers, B, 1, Hkv, D), generator=gen, device=dev)
    v_in = torch.randn((layers, B, 1, Hkv, D), generator=gen, device=dev)
    q_work = torch.empty((layers, B, 1, Hq, D), dtype=torch.float32, device=dev)
    out = torch.empty((layers, B, 1, Hq, D), dtype=torch.float32, device=dev)
    eng.ctx.reserve(64 << 20)
    stream = torch.cuda.current_stream()

    def step(ev=None, qi=q_in, ki=k_in, vi=v_in, oo=out):
        for layer in range(layers):
            if ev is None:
                eng.attentionLayer(kv, layer, cfgs[layer], qi[layer], ki[layer], vi[layer], past, q_work[layer],
                                   oo[layer])
            else:
                # Roofline timing brackets the decode kernel alone (separate launches, no overlap).
                eng.appendKv(kv, layer, cfgs[layer], qi[layer], ki[layer], vi[layer], q_work[layer], past)
                ev[layer][0].record(stream)
                eng.recAttention(kv, layer, cfgs[layer], q_work[layer], oo[layer], past)
                ev[layer][1].record(stream)

    def barrier():
        if world > 1:
            dist.barrier()

    for _ in range(args.warmup):
        step()
    eng.ctx.check()
    barrier()
    torch.cuda.synchronize()

    def capture(fn):
        """A CUDA graph of fn's launches (the same kernels and arguments), captured on a side
        stream after the warm-up has sized every workspace."""
        side = torch.cuda.Stream(device=dev)
        side.wait_stream(stream)
        with torch.cuda.stream(side):
            fn()
        stream.wait_stream(side)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        n0 = eng.ctx.launches
        with torch.cuda.graph(g):
            fn()
        g.launches = eng.ctx.launches - n0  # kernels one replay launches
        g.replay()
        torch.cuda.synchronize()
        eng.ctx.check()
        return g

    graph = None if args.eager else capture(step)
    import ctypes

    from brimkern_b200 import _lib as L
    _p = cfgs[-1].params()
    nsplit = L.lib().brk_attn_decode_splits(eng.ctx.handle, kv.handle, ctypes.byref(_p), B, 1,
                                            (ctypes.c_int32 * B)(*past))
    vis = os.environ.get("CUDA_VISIBLE_DEVICES", "").split(",")
    phys = int(vis[local]) if len(vis) > local and vis[local].strip().isdigit() else local
    sampler = ClockSampler(phys)
    sampler.start()
    time.sleep(0.3)
    n0 = eng.ctx.launches
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for s in range(args.steps):
        if graph is None:
            step()
        else:
            graph.replay()
    stop.record(stream)
    torch.cuda.synchronize()
    # Kernels launched in the timed region (a replay launches the captured step's kernels).
    launches = eng.ctx.launches - n0 if graph is None else args.steps * graph.launches
    clocks = sampler.stop()
    eng.ctx.check()
    barrier()
    ms_total = start.elapsed_time(stop)
    # Roofline pass: the decode kernel alone (no append overlap), every layer's launch back to
    # back in a CUDA graph timed by CUDA events around the replays (so no host launch gap is
    # counted); --eager brackets each host-launched decode kernel with events instead.
    rsteps = max(2, min(args.steps, 5))

    def decode_only():
        for layer in range(layers):
            eng.recAttention(kv, layer, cfgs[layer], q_work[layer], out[layer], past)

    if args.eager:
        layer_ev = [[[torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)]
                     for _ in range(layers)] for _ in range(rsteps)]
        for s in range(rsteps):
            step(layer_ev[s])
        torch.cuda.synchronize()
        eng.ctx.check()
        attn_ms = [layer_ev[s][l][0].elapsed_time(layer_ev[s][l][1]) for s in range(rsteps) for l in range(layers)]
    else:
        dgraph = capture(decode_only)
        r0, r1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        r0.record(stream)
        for _ in range(rsteps):
            dgraph.replay()
        r1.record(stream)
        torch.cuda.synchronize()
        eng.ctx.check()
        attn_ms = [r0.elapsed_time(r1) / (rsteps * layers)]
        del dgraph
    if world > 1:
        t = torch.tensor([ms_total], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms_total = float(t.item())
    ms_step = ms_total / args.steps
    bytes_step = kv_bytes_per_step(c, B)
    value = world * bytes_step / (ms_step * 1e-3) / 1e9
    tok_s = world * B / (ms_step * 1e-3)

    # Roofline of the decode attention launches (decode kernel + its split combine).
    peak, peak_kind = load_peak()
    attn_avg_ms = sum(attn_ms) / len(attn_ms)
    bytes_launch = bytes_step / layers
    achieved = bytes_launch / (attn_avg_ms * 1e-3) / 1e9
    traffic, traffic_src = read_traffic(workload + ("-q8" if q8 else ""), B, bytes_launch)
    roofline = {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                "frac": round(achieved / peak, 4), "traffic": traffic, "traffic_source": traffic_src,
                "peak_kind": peak_kind,
                "kernel": "decode_kernel<int8>" if q8 else "decode_kernel<fp16>",
                "timing": (f"CUDA events around each host-launched decode kernel, {rsteps} steps" if args.eager else
                           f"CUDA events around {rsteps} replays of a graph of the {layers} layers' decode launches"),
                "bytes_per_launch": bytes_launch,
                "avg_launch_ms": round(attn_avg_ms, 5), "frac_of_8TBs": round(achieved / 8000.0, 4)}

    # End to end through the host API: pinned host inputs -> device, step, outputs -> host.
    e2e = None
    if not args.no_e2e:
        hq = q_in.cpu().pin_memory()
        hk = k_in.cpu().pin_memory()
        hv = v_in.cpu().pin_memory()
        hout = torch.empty(out.shape, dtype=torch.float32, pin_memory=True)
        dq, dk, dv, do = torch.empty_like(q_in), torch.empty_like(k_in), torch.empty_like(v_in), torch.empty_like(out)

        pipe = CopyPipeline(dev, layers)

        def h2d(layer):
            dq[layer].copy_(hq[layer], non_blocking=True)
            dk[layer].copy_(hk[layer], non_blocking=True)
            dv[layer].copy_(hv[layer], non_blocking=True)

        def compute(layer):
            eng.attentionLayer(kv, layer, cfgs[layer], dq[layer], dk[layer], dv[layer], past, q_work[layer], do[layer])

        def d2h(layer):
            hout[layer].copy_(do[layer], non_blocking=True)

        def e2e_step():
            pipe.run(stream, layers, h2d, compute, d2h)

        for _ in range(args.warmup):
            e2e_step()
        barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.steps):
            e2e_step()
        e1.record(stream)
        torch.cuda.synchronize()
        e_ms = e0.elapsed_time(e1)
        if world > 1:
            t = torch.tensor([e_ms], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            e_ms = float(t.item())
        e_step = e_ms / args.steps
        e2e = {"value": round(world * bytes_step / (e_step * 1e-3) / 1e9, 2), "unit": "GB/s",
               "h2d_bytes_per_step": int((hq.numel() + hk.numel() + hv.numel()) * 4),
               "d2h_bytes_per_step": int(hout.numel() * 4), "ms_per_step": round(e_step, 4),
               "tokens_per_s": round(world * B / (e_step * 1e-3), 1)}
        eng.ctx.check()

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        gbs, used, desc = cpu_reference_sample(c, B, 10.0)
        cpu = {"value": round(gbs, 4), "unit": "GB/s", "cores": used, "kind": "port", "sample": desc}

    line = None
    if rank == 0:
        line = {
            "metric": "decode-attn KV-read GB/s", "value": round(value, 2), "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 4), "higher_is_better": True,
            "scaling": args.scaling, "vs_baseline": None,
            "dtype": "int8 KV + f32 row scales / f32 accumulate" if q8 else "f16 KV / f32 accumulate",
            "data": "synthetic",
            "config": decode_config(c, workload, B, world, args.scaling),
            "launch": "host launches" if args.eager else "CUDA-graph replay of the step",
            "tokens_per_s": round(tok_s, 1),
            "frac_of_measured_hbm": round(value / world / peak, 4),
            "decode_splits": nsplit,
            "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e, "gpu_launches": int(launches),
            "clocks": clocks,
        }
    if world == 1 and not args.no_prefill and not q8 and workload == "qwen3-4b" and args.batch == 64:
        # BASELINE config 3 in the same run: the tensor-core prefill, with its own roofline and CPU
        # baseline, nested under "prefill" (the decode step's buffers are released first).
        if graph is not None:
            del graph
        kv.close()
        del q_in, k_in, v_in, q_work, out
        torch.cuda.empty_cache()
        pc = dict(CONFIGS["qwen3-4b-prefill"])
        pargs = argparse.Namespace(**vars(args))
        pargs.batch, pargs.steps, pargs.warmup, pargs.no_e2e = pc["batch"], 5, 3, args.no_e2e
        line["prefill"] = run_prefill(pargs, pc, "qwen3-4b-prefill", eng=eng, emit=False)
    if rank == 0:
        print(json.dumps(line), flush=True)
    eng.close()
    if world > 1:
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
