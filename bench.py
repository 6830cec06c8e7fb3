#!/usr/bin/env python
"""bench.py - phone-attn partial attention on B200: BASELINE.json's decode workload (config 1).

One step = one decode step of a 64-layer, Qwen3-27B-shaped model over its offloaded KV: per layer, 40 query heads
(8 KV heads, GQA 5), head dim 128, one query token with fresh seeded Q, against 131,072 Q8_0 key/value positions;
softmax scale 1/sqrt(128). The KV is sharded by position across the N GPUs (one process per GPU, rank r holds
positions [r*S, (r+1)*S) of every layer); every step each rank computes its partial (O, m, l) for all 64 layers
(one decode-kernel launch + one merge launch), the partials are exchanged with ONE NCCL all-gather (N > 1) and
folded by log-sum-exp on every rank.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    (N > 1: python -m torch.distributed.run --nnodes=1 --nproc-per-node N --master-addr 127.0.0.1 ... bench.py ...)

Prints ONE JSON line (rank 0). `value` is whole-job GB/s of algorithmic bytes (quantised K+V read, f16 Q read,
(O, m, l) written) with inputs resident in HBM, timed with CUDA events over K steps, max over ranks; `e2e` is the
same metric through the host-buffer path (pinned Q in, O/m/l out, copies inside the timed region). The per-step KV
(18.3 GB) is far larger than L2, so no flush is needed. `--impl reference` times the CPU restatement of the
reference's own kernel (the oracle's fp32 port of sme_attn_partial) on all host threads instead.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

LAYERS, KEYS, NKV, GQA, HD = 64, 131072, 8, 5, 128
Q_HEADS = NKV * GQA
SEED = 20260127
GEN_CHUNK = 16384   # keys per generator draw (the data does not depend on the number of GPUs)


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=256)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--layers", type=int, default=LAYERS)
    ap.add_argument("--keys", type=int, default=KEYS)
    ap.add_argument("--e2e-steps", type=int, default=16)
    ap.add_argument("--chunk-keys", type=int, default=0,
                    help="keys per decode job (0: the plan's own choice); lets a small capture keep the full run's job size")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--prefill-steps", type=int, default=5)
    ap.add_argument("--prefill-layers", type=int, default=LAYERS)
    ap.add_argument("--hd", type=int, choices=[128, 256], default=HD,
                    help="head dim of the decode workload (256: the reference server's wire geometry)")
    ap.add_argument("--gqa", type=int, default=GQA, help="query rows per KV head of the decode workload")
    args = ap.parse_args()
    set_geometry(args.hd, args.gqa)
    return args


def set_geometry(hd: int, gqa: int):
    """The decode workload's head dim and query rows per KV head (128 and 5)."""
    global HD, GQA, Q_HEADS
    HD, GQA, Q_HEADS = hd, gqa, NKV * gqa


def decode_metric(layers: int, keys: int) -> str:
    """The metric name: BASELINE config 1's, or the same measure at another geometry."""
    if (HD, GQA, layers, keys) == (128, 5, LAYERS, KEYS):
        return "decode KV-attn GB/s (config 1: 64 layers x 131072 Q8_0 keys, 40q/8kv, d128)"
    return f"decode KV-attn GB/s ({layers} layers x {keys} Q8_0 keys, {Q_HEADS}q/{NKV}kv, d{HD})"


def layer_bytes(keys: int) -> dict:
    """Algorithmic bytes of one layer's partial over `keys` positions (the roofline's unit)."""
    kv = 2 * keys * NKV * (HD // 32 * 34)
    q = Q_HEADS * HD * 2                    # f16(q * scale) read
    oml = Q_HEADS * (HD + 2) * 4            # (O, m, l) written
    return dict(kv=kv, q=q, oml=oml, total=kv + q + oml)


def measured_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def measured_tensor_peak(sustained: bool = False):
    """bf16 dense TFLOP/s from MEASURED_PEAKS.json: the burst figure, or the power-capped sustained one."""
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        if sustained:
            return float(d["bf16_tflops_sustained"]), "measured (sustained)"
        return float(d["bf16_tflops"]), "measured (burst)"
    except Exception:
        return (1400.0, "fallback (sustained)") if sustained else (1590.0, "fallback")


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device = device
        self.proc = None
        self.path = None
        self.skip = 0

    def _lines(self) -> int:
        try:
            with open(self.path) as f:
                return sum(1 for _ in f)
        except Exception:
            return 0

    def __enter__(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.device}", f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
        # nvidia-smi takes a few hundred ms to start: wait for its first sample, so that a short timed region (an
        # 8-GPU run's is ~0.15 s) is sampled too, and count only the samples taken from here on
        t0 = time.time()
        while self.proc and self._lines() == 0 and time.time() - t0 < 3.0:
            time.sleep(0.02)
        self.skip = self._lines()
        return self

    def __exit__(self, *a):
        if self.proc:
            t0 = time.time()
            while self._lines() <= self.skip and time.time() - t0 < 0.5:   # at least one sample of the region
                time.sleep(0.02)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        rows = []
        try:
            for i, line in enumerate(open(self.path)):
                parts = [x.strip() for x in line.split(",")]
                if i >= self.skip and len(parts) >= 9:
                    rows.append(parts)
        except Exception:
            pass
        finally:
            try:
                os.unlink(self.path)
            except Exception:
                pass
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        load = [x for x in sm if mx and x > 0.5 * max(mx)] or sm
        return {"sm_mhz": statistics.median(load) if load else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


# --------------------------------------------------------------------------------------------- data
def make_layer(torch, pa, layer: int, k0: int, nk: int, device):
    """Quantised K and V rows [nk][NKV*HD/32*34] for positions [k0, k0+nk) of `layer`: N(0,1) values, 4 K channels
    per head scaled x8, Q8_0 (the BASELINE distributions)."""
    g = torch.Generator(device=device)
    g.manual_seed(SEED * 1000 + layer)
    ch = torch.stack([torch.randperm(HD, generator=g, device=device)[:4] for _ in range(NKV)])   # [NKV, 4]
    out_k, out_v = [], []
    c0 = (k0 // GEN_CHUNK) * GEN_CHUNK
    for c in range(c0, k0 + nk, GEN_CHUNK):
        g.manual_seed((SEED * 1000 + layer) * 4096 + c // GEN_CHUNK)
        kf = torch.randn((GEN_CHUNK, NKV, HD), generator=g, device=device)
        vf = torch.randn((GEN_CHUNK, NKV, HD), generator=g, device=device)
        for h in range(NKV):
            kf[:, h, ch[h]] *= 8.0
        a, b = max(k0, c) - c, min(k0 + nk, c + GEN_CHUNK) - c
        out_k.append(pa.quantize_q8_0(kf[a:b]).reshape(b - a, -1))
        out_v.append(pa.quantize_q8_0(vf[a:b]).reshape(b - a, -1))
    return torch.cat(out_k), torch.cat(out_v)


def make_q(torch, steps: int, layers: int, device):
    """Fresh seeded Q per step: f16(q * scale) [steps][layers][NKV][GQA][HD] with q ~ N(0,1)."""
    g = torch.Generator(device=device)
    g.manual_seed(SEED + 7)
    q = torch.randn((steps, layers, NKV, GQA, HD), generator=g, device=device)
    return (q * (1.0 / HD ** 0.5)).to(torch.float16)


# --------------------------------------------------------------------------------------------- CPU baseline
def cpu_baseline(target_s: float = 10.0):
    """The oracle's fp32 restatement of the reference's own kernel (block online softmax of
    scripts/sme/sme_attn.c:274-306) on all host threads, on a bounded sample of the workload: 32,768 positions of one
    layer (8 KV heads, GQA 5, Q8_0), computed repeatedly for ~target_s seconds. Returns the cpu_baseline object."""
    from oracle import oracle as orc
    threads = os.cpu_count() or 1
    nk = 32768
    c = orc.gen_case(SEED, HD, NKV, GQA, nk, orc.Q8_0)
    chunk = max(512, nk // (threads * 4) // 512 * 512)
    orc.partial_f32_mt(c["shape"], c["Qs"], c["K"], c["V"], nk, threads, chunk)
    reps, t0 = 0, time.perf_counter()
    while True:
        orc.partial_f32_mt(c["shape"], c["Qs"], c["K"], c["V"], nk, threads, chunk)
        reps += 1
        dt = time.perf_counter() - t0
        if dt >= target_s:
            break
    b = layer_bytes(nk)["total"] * reps
    return {"value": round(b / dt / 1e9, 3), "unit": "GB/s", "cores": threads, "kind": "port",
            "sample": f"{reps} x (1 layer x {nk} Q8_0 positions x {NKV} KV heads x {GQA} rows (GQA {GQA}), d{HD}, "
                      f"{layer_bytes(nk)['total'] / 1e6:.1f} MB) in {dt:.1f} s; oracle fp32 block-online port of "
                      f"sme_attn_partial on {threads} threads"}


def run_reference(args, rank: int, world: int):
    """--impl reference: the CPU restatement of the reference path on the host cores (rank 0 only)."""
    if rank != 0:
        return
    import numpy as np
    from oracle import oracle as orc
    threads = os.cpu_count() or 1
    nk = 8192       # each step: a bounded sample of one layer's positions
    cases = [orc.gen_case(SEED + i, HD, NKV, GQA, nk, orc.Q8_0) for i in range(2)]
    for i in range(args.warmup):
        c = cases[i % 2]
        orc.partial_f32_mt(c["shape"], c["Qs"], c["K"], c["V"], nk, threads, 512)
    t0 = time.perf_counter()
    for i in range(args.steps):
        c = cases[i % 2]
        orc.partial_f32_mt(c["shape"], c["Qs"], c["K"], c["V"], nk, threads, 512)
    dt = time.perf_counter() - t0
    b = layer_bytes(nk)["total"] * args.steps
    v = b / dt / 1e9
    sample = (f"each step: 1 layer x {nk} Q8_0 positions x {NKV} KV heads x {GQA} rows, d{HD} "
              f"({layer_bytes(nk)['total'] / 1e6:.1f} MB); oracle fp32 block-online port of sme_attn_partial (the "
              f"reference CPU kernel is ARM SME2-only)")
    line = {
        "impl": "reference", "metric": decode_metric(args.layers, args.keys),
        "value": round(v, 3), "unit": "GB/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(dt / args.steps * 1e3, 3), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": ("config 1 decode" if (HD, GQA) == (128, 5) else "decode") + " (bounded CPU sample per step)",
                   "layers": args.layers, "keys": args.keys,
                   "nkv": NKV, "q_heads": Q_HEADS, "hd": HD, "quant": "q8_0"},
        "cpu_baseline": {"value": round(v, 3), "unit": "GB/s", "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": round(v, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# --------------------------------------------------------------------------------------------- config 2
PF_TOKENS, PF_KEYS = 512, 65536


def bench_prefill(torch, pa, ctx, device, stream, layers: int, steps: int):
    """Config 2: a 512-token query batch (40 q / 8 KV heads, d128) against 65,536 older Q8_0 positions per layer, no
    mask, all `layers` layers per step in one plan (the tcgen05 kernel: 2,560 rows per KV head). Device-timed."""
    rows = PF_TOKENS * GQA
    shape = pa.shape_for(HD, NKV, rows, pa.Q8_0)
    K = torch.empty((layers, PF_KEYS, shape.rs), dtype=torch.uint8, device=device)
    V = torch.empty_like(K)
    for layer in range(layers):
        k, v = make_layer(torch, pa, 1000 + layer, 0, PF_KEYS, device)
        K[layer].copy_(k)
        V[layer].copy_(v)
        del k, v
    g = torch.Generator(device=device)
    g.manual_seed(SEED + 11)
    Qs = (torch.randn((layers, NKV, rows, HD), generator=g, device=device) / HD ** 0.5).to(torch.float16)
    segs = [pa.Seg(K[i].data_ptr(), V[i].data_ptr(), PF_KEYS, i) for i in range(layers)]
    plan = pa.Plan(ctx, shape, layers, segs)
    O = torch.empty((layers, NKV, rows, HD), dtype=torch.float32, device=device)
    m = torch.empty((layers, NKV, rows), dtype=torch.float32, device=device)
    l = torch.empty_like(m)
    for _ in range(2):
        plan.run(Qs, O, m, l, stream)
    ctx.status(stream)
    torch.cuda.synchronize()
    plan.profile(steps)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(device.index if device.index is not None else 0) as clk:
        e0.record(stream)
        for _ in range(steps):
            plan.run(Qs, O, m, l, stream)
        e1.record(stream)
        torch.cuda.synchronize()
    ctx.status(stream)
    ms = e0.elapsed_time(e1) / steps
    kms, kn = plan.kernel_ms()
    kms /= max(1, kn)
    kname = plan.kernel
    flops = 4.0 * PF_TOKENS * Q_HEADS * HD * PF_KEYS * layers
    peak, kind = measured_tensor_peak()
    peak_s, _ = measured_tensor_peak(sustained=True)
    plan.close()
    del K, V, Qs, O
    torch.cuda.empty_cache()
    return {"metric": "prefill attn TFLOP/s (config 2: 512 tokens x 65536 Q8_0 keys, 40q/8kv, d128)",
            "value": round(flops / (ms * 1e-3) / 1e12, 1), "unit": "TFLOP/s", "ms_per_step": round(ms, 3),
            "layers": layers, "steps": steps,
            "roofline": {"bound": "tensor", "achieved": round(flops / (kms * 1e-3) / 1e12, 1), "peak": peak,
                         "unit": "TFLOP/s", "frac": round(flops / (kms * 1e-3) / 1e12 / peak, 4), "peak_kind": kind,
                         "frac_of_sustained": round(flops / (kms * 1e-3) / 1e12 / peak_s, 4),
                         "kernel": kname, "kernel_ms": round(kms, 3),
                         "algorithmic_flops_per_launch": flops}, "clocks": clk.summary()}


# --------------------------------------------------------------------------------------------- GPU arm
def main():
    args = parse()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        return run_reference(args, rank, world)

    import torch
    import torch.distributed as dist
    import backburner_b200 as pa

    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", init_method="env://", rank=rank, world_size=world,
                                timeout=__import__("datetime").timedelta(seconds=120), device_id=device)
    if not pa.available():
        raise RuntimeError("libpacuda.so did not load on this GPU (build it with python -m backburner_b200.build)")
    ctx = pa.Context(local)
    L = args.layers
    shard = args.keys // world
    k0 = rank * shard
    nk = shard if rank < world - 1 else args.keys - k0
    shape = pa.shape_for(HD, NKV, GQA, pa.Q8_0)
    rows = L * NKV * GQA

    # ---- resident inputs: this rank's positions of every layer
    Kall = torch.empty((L, nk, shape.rs), dtype=torch.uint8, device=device)
    Vall = torch.empty_like(Kall)
    for layer in range(L):
        k, v = make_layer(torch, pa, layer, k0, nk, device)
        Kall[layer].copy_(k)
        Vall[layer].copy_(v)
        del k, v
    torch.cuda.synchronize()
    total_steps = args.warmup + args.steps
    Qs = make_q(torch, total_steps, L, device)            # [steps][L][NKV][GQA][HD]
    segs = [pa.Seg(Kall[i].data_ptr(), Vall[i].data_ptr(), nk, i) for i in range(L)]
    plan = pa.Plan(ctx, shape, L, segs, chunk_keys=args.chunk_keys)
    packed = torch.empty((rows * (HD + 2),), dtype=torch.float32, device=device)   # this rank's (O, m, l)
    Op, mp, lp = pa.packed_views(packed, rows, HD)
    gathered = torch.empty((world, rows * (HD + 2)), dtype=torch.float32, device=device) if world > 1 else None
    Of = torch.empty((rows, HD), dtype=torch.float32, device=device)
    mf = torch.empty((rows,), dtype=torch.float32, device=device)
    lf = torch.empty_like(mf)
    stream = torch.cuda.current_stream(device)

    def step(i):
        plan.run(Qs[i], Op, mp, lp, stream)
        if world > 1:
            dist.all_gather_into_tensor(gathered, packed)
            pa.merge_gathered(ctx, HD, rows, gathered, world, out=(Of, mf, lf), stream=stream)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])

    for i in range(args.warmup):
        step(i)
    ctx.status(stream)
    barrier()
    torch.cuda.synchronize()
    launches0 = ctx.launches
    plan.profile(args.steps)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        barrier()
        torch.cuda.synchronize()
        ev0.record(stream)
        for i in range(args.steps):
            step(args.warmup + i)
        ev1.record(stream)
        torch.cuda.synchronize()
        barrier()
    launches = ctx.launches - launches0
    ctx.status(stream)
    ms = ev0.elapsed_time(ev1)
    kern_ms, kern_runs = plan.kernel_ms()
    plan.profile(0)
    t = torch.tensor([ms], device=device)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    per_step_bytes = L * layer_bytes(args.keys)["total"]      # the whole job's algorithmic bytes per step
    value = per_step_bytes * args.steps / (ms * 1e-3) / 1e9

    # ---- roofline of the dominant kernel (the decode kernel; one launch = this rank's 64-layer shard)
    peak, peak_kind = measured_peaks()
    kb = layer_bytes(nk)
    launch_bytes = L * kb["total"]
    kern_avg_ms = kern_ms / max(1, kern_runs)
    achieved = launch_bytes / (kern_avg_ms * 1e-3) / 1e9
    traffic = None
    try:
        with open(os.path.join(ROOT, "profiles", "decode_traffic.json")) as f:
            tr = json.load(f)
        # ncu DRAM bytes of a smaller capture, scaled to this launch: reads by key positions, writes by jobs (slots)
        if (HD, GQA) == (128, 5):   # the capture's geometry (config 1)
            traffic = round(tr["dram_read_bytes_per_key_position"] * nk * L + tr["dram_write_bytes_per_job"] * plan.jobs)
    except Exception:
        pass
    roofline = {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                "frac": round(achieved / peak, 4), "traffic": traffic, "peak_kind": peak_kind,
                "kernel": plan.kernel, "kernel_ms": round(kern_avg_ms, 4),
                "algorithmic_bytes_per_launch": launch_bytes}

    # ---- end to end through the host-buffer path (pinned Q in, O/m/l out, copies inside the timed region)
    e2e = None
    if args.e2e_steps > 0:
        qh = torch.empty((args.e2e_steps, L, NKV, GQA, HD), dtype=torch.float16).pin_memory()
        qh.copy_(Qs[:args.e2e_steps].cpu())
        Oh = torch.empty((rows, HD), dtype=torch.float32).pin_memory()
        mh = torch.empty((rows,), dtype=torch.float32).pin_memory()
        lh = torch.empty_like(mh).pin_memory()
        qd = torch.empty((L, NKV, GQA, HD), dtype=torch.float16, device=device)

        def e2e_step(i):
            if world == 1:
                plan.run_host(qh[i], Oh, mh, lh, stream)     # the C ABI host path: H2D, kernels, D2H, sync
            else:
                qd.copy_(qh[i], non_blocking=True)
                plan.run(qd, Op, mp, lp, stream)
                dist.all_gather_into_tensor(gathered, packed)
                pa.merge_gathered(ctx, HD, rows, gathered, world, out=(Of, mf, lf), stream=stream)
                Oh.copy_(Of, non_blocking=True)
                mh.copy_(mf, non_blocking=True)
                lh.copy_(lf, non_blocking=True)
                stream.synchronize()

        for i in range(min(3, args.e2e_steps)):
            e2e_step(i)
        barrier()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for i in range(args.e2e_steps):
            e2e_step(i)
        dt = time.perf_counter() - t0
        tt = torch.tensor([dt], device=device)
        if world > 1:
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        dt = float(tt.item())
        e2e = {"value": round(per_step_bytes * args.e2e_steps / dt / 1e9, 1), "unit": "GB/s",
               "h2d_bytes_per_step": L * NKV * GQA * HD * 2, "d2h_bytes_per_step": rows * (HD + 2) * 4,
               "ms_per_step": round(dt / args.e2e_steps * 1e3, 3)}

    # ---- config 2 (prefill): 512 tokens x 40 q heads against 65,536 Q8_0 positions per layer, all layers per step
    prefill = None
    if world == 1 and args.prefill_steps > 0 and (HD, GQA) == (128, 5):
        del Kall, Vall
        torch.cuda.empty_cache()
        prefill = bench_prefill(torch, pa, ctx, device, stream, args.prefill_layers, args.prefill_steps)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline()

    clocks = clk.summary()
    if rank == 0:
        line = {
            "metric": decode_metric(L, args.keys),
            "value": round(value, 1), "unit": "GB/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms / args.steps, 4), "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f16", "data": "synthetic",
            "config": {"workload": ("config 1: decode" if (HD, GQA) == (128, 5) else "decode") +
                                   ", 1 token/step, fresh seeded Q per step", "layers": L,
                       "keys": args.keys, "keys_per_gpu": shard, "nkv": NKV, "q_heads": Q_HEADS, "hd": HD,
                       "quant": "q8_0", "parallelism": f"sequence shards x{world}, 1 NCCL all-gather of (O,m,l)/step",
                       "l2": f"inputs larger than L2 ({per_step_bytes / 1e9:.1f} GB of KV per step), no flush",
                       "bytes_per_step": per_step_bytes},
            "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e, "gpu_launches": launches, "clocks": clocks,
            "prefill": prefill,
        }
        print(json.dumps(line), flush=True)
    plan.close()
    ctx.close()
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
