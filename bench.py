#!/usr/bin/env python
"""bench.py - phone-attn partial attention on B200: BASELINE.json's decode workload (config 1), with the prefill (config
2) and speculative-verify (config 3) workloads measured the same way.

One step = one decode step of a 64-layer, Qwen3-27B-shaped model over its offloaded KV: per layer, 40 query heads
(8 KV heads, GQA 5), head dim 128, one query token with fresh seeded Q, against 131,072 Q8_0 key/value positions;
softmax scale 1/sqrt(128). The KV is sharded by position across the N GPUs (one process per GPU, rank r holds
positions [r*S, (r+1)*S) of every layer); every step each rank computes its partial (O, m, l) for all 64 layers
(one attention-kernel launch + one merge launch), and for N > 1 the library's own position-shard call
(pa_cuda_shard_attn_allgather_merge over its NCCL communicator, include/pa_cuda.h) exchanges the partials and folds
them by log-sum-exp on every rank.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    (N > 1: python -m torch.distributed.run --nnodes=1 --nproc-per-node N --master-addr 127.0.0.1 ... bench.py ...)

Prints ONE JSON line (rank 0). `value` is whole-job GB/s of algorithmic bytes (quantised K+V read, f16 Q read,
(O, m, l) written) with inputs resident in HBM, timed with CUDA events over K steps, max over ranks; `e2e` is the
same metric through the host-buffer path (pinned Q in, O/m/l out, copies inside the timed region). The per-step KV
(18.3 GB) is far larger than L2, so no flush is needed. `parity` checks the merged output of the last timed step
against an fp64 attention over all positions computed on the device with torch (exact dequantisation; pa-tool's 5e-3
gate). `prefill` (config 2) and `verify` (config 3) are the same kind of measurement for those workloads, sharded the
same way. `--impl reference` times the CPU restatement of the reference's own kernel (the oracle's fp32 port of
sme_attn_partial) on all host threads instead.
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
PF_TOKENS, PF_KEYS = 512, 65536          # config 2
VF_TOKENS, VF_KEYS = 16, 196608          # config 3
PARITY_TOL = 5e-3                        # against exact fp64 (pa-tool's gate, phone-attn/pa-tool.cpp:150-173)


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
    ap.add_argument("--verify-steps", type=int, default=20)
    ap.add_argument("--verify-layers", type=int, default=LAYERS)
    ap.add_argument("--engine-calls", type=int, default=200)
    ap.add_argument("--uneven-steps", type=int, default=20, help="config-4 decode steps (0: no config-4 legs)")
    ap.add_argument("--uneven-prefill-steps", type=int, default=2)
    ap.add_argument("--uneven-layers", type=int, default=LAYERS)
    ap.add_argument("--only", choices=["all", "decode", "prefill", "verify", "uneven"], default="all",
                    help="run one workload only (profiling captures); the default line has all of them")
    ap.add_argument("--hd", type=int, choices=[128, 256], default=HD,
                    help="head dim of the decode workload (256: the reference server's wire geometry)")
    ap.add_argument("--gqa", type=int, default=GQA, help="query rows per KV head of the decode workload")
    ap.add_argument("--qk", choices=["f16", "int8"], default="f16",
                    help="QK arithmetic of the config-1 decode workload: f16 (default) or the reference's int8-domain QK "
                         "(scripts/sme/sme_attn.c:465-508; its fp64 error is past the 5e-3 parity gate)")
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


def head_bytes(quant: int, hd: int = None) -> int:
    hd = HD if hd is None else hd
    return hd // 32 * (34 if quant == 1 else 18)


def layer_bytes(keys: int, rows: int = None, quant: int = 1) -> dict:
    """Algorithmic bytes of one layer's partial over `keys` positions for `rows` query rows per KV head (the roofline's
    unit): quantised K + V read (scales included), f16 Q read, (O, m, l) written."""
    rows = GQA if rows is None else rows
    kv = 2 * keys * NKV * head_bytes(quant)
    q = NKV * rows * HD * 2
    oml = NKV * rows * (HD + 2) * 4
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
    """nvidia-smi clocks / throttle reasons sampled every 25 ms during the timed region (a 20-step decode region at N=1
    lasts ~75 ms)."""

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
                                          "--format=csv,noheader,nounits", "-lms", "25"],
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
def make_layer(torch, pa, layer: int, k0: int, nk: int, device, quant: int = 1, student_t: bool = False):
    """Quantised K and V rows [nk][NKV*hb] for positions [k0, k0+nk) of `layer`: N(0,1) values, 4 K channels per head
    scaled x8, Q8_0 or Q4_0 (the BASELINE distributions); student_t: V from Student-t with 3 degrees of freedom
    (config 4: z / sqrt(chi2_3 / 3) from the same seeded generator). The values of a position do not depend on the
    range asked for, so every rank's shard and the parity check's full layer agree."""
    quantize = pa.quantize_q8_0 if quant == pa.Q8_0 else pa.quantize_q4_0
    g = torch.Generator(device=device)
    g.manual_seed(SEED * 1000 + layer)
    ch = torch.stack([torch.randperm(HD, generator=g, device=device)[:4] for _ in range(NKV)])   # [NKV, 4]
    out_k, out_v = [], []
    c0 = (k0 // GEN_CHUNK) * GEN_CHUNK
    for c in range(c0, k0 + nk, GEN_CHUNK):
        g.manual_seed((SEED * 1000 + layer) * 4096 + c // GEN_CHUNK)
        kf = torch.randn((GEN_CHUNK, NKV, HD), generator=g, device=device)
        vf = torch.randn((GEN_CHUNK, NKV, HD), generator=g, device=device)
        if student_t:
            chi = torch.randn((3, GEN_CHUNK, NKV, HD), generator=g, device=device).square().sum(0)
            vf = vf / (chi / 3.0).sqrt()
        for h in range(NKV):
            kf[:, h, ch[h]] *= 8.0
        a, b = max(k0, c) - c, min(k0 + nk, c + GEN_CHUNK) - c
        out_k.append(quantize(kf[a:b]).reshape(b - a, -1))
        out_v.append(quantize(vf[a:b]).reshape(b - a, -1))
    return torch.cat(out_k), torch.cat(out_v)


def make_q(torch, steps: int, layers: int, rows: int, device, seed: int):
    """Seeded Q per step: f16(q * scale) [steps][layers][NKV][rows][HD] with q ~ N(0,1)."""
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    q = torch.randn((steps, layers, NKV, rows, HD), generator=g, device=device)
    return (q * (1.0 / HD ** 0.5)).to(torch.float16)


def shard_inputs(torch, pa, device, layers: int, keys: int, rank: int, world: int, quant: int, layer_base: int,
                 shares=None, student_t: bool = False):
    """This rank's contiguous positions [k0, k0+nk) of every layer (equal shards, or `shares` positions per rank),
    resident on the device."""
    from backburner_b200 import shard
    k0, nk = shard.shard_range(keys, world, rank, shares)
    rs = NKV * head_bytes(quant)
    K = torch.empty((layers, nk, rs), dtype=torch.uint8, device=device)
    V = torch.empty_like(K)
    for layer in range(layers):
        k, v = make_layer(torch, pa, layer_base + layer, k0, nk, device, quant, student_t)
        K[layer].copy_(k)
        V[layer].copy_(v)
        del k, v
    return K, V, k0, nk


# --------------------------------------------------------------------------------------------- parity
def parity_fp64(torch, pa, device, quant: int, keys: int, layer_ids, layer_base: int, Q, O, m, l, rows_sample,
                student_t: bool = False):
    """The merged (O, m, l) of the sampled layers and rows against an fp64 attention over ALL `keys` positions on the
    device (exact dequantisation of the same rows, f16(q*scale) as the kernels read it): max |O/l - ref| / max |ref|
    and max |lse - lse_ref| over the sampled rows, with pa-tool's 5e-3 gate. Q: f16 [layers][NKV][rows][HD]."""
    hb = head_bytes(quant)
    eo_w, el_w = 0.0, 0.0
    for li in layer_ids:
        Kf, Vf = make_layer(torch, pa, layer_base + li, 0, keys, device, quant, student_t)
        for h in range(NKV):
            kf = pa.dequantize(Kf[:, h * hb:(h + 1) * hb], quant, HD).double()
            vf = pa.dequantize(Vf[:, h * hb:(h + 1) * hb], quant, HD).double()
            qs = Q[li, h, rows_sample].double()
            s = qs @ kf.T
            mx = s.max(dim=1, keepdim=True).values
            p = torch.exp(s - mx)
            lr = p.sum(dim=1)
            ref = (p @ vf) / lr[:, None]
            del s, p, kf, vf
            og, lg, mg = O[li, h, rows_sample].double(), l[li, h, rows_sample].double(), m[li, h, rows_sample].double()
            got = og / lg[:, None]
            eo = float((got - ref).abs().max() / ref.abs().max().clamp_min(1e-30))
            el = float(((mg + torch.log(lg)) - (mx[:, 0] + torch.log(lr))).abs().max())
            eo_w, el_w = max(eo_w, eo), max(el_w, el)
        del Kf, Vf
    torch.cuda.empty_cache()
    n_rows = len(layer_ids) * NKV * len(rows_sample)
    return {"max_rel_O": float(f"{eo_w:.3e}"), "max_abs_lse": float(f"{el_w:.3e}"), "tol": PARITY_TOL,
            "ok": bool(eo_w <= PARITY_TOL and el_w <= PARITY_TOL), "layers": list(layer_ids), "rows": n_rows,
            "positions": keys, "reference": "fp64 attention on the device over all positions of the layer (exact "
                                            "dequantisation), rank 0, against the merged output of the last timed step"}


# --------------------------------------------------------------------------------------------- one sharded workload
class Leg:
    """One workload (layers x keys x rows per KV head) sharded by position over the ranks: this rank's inputs, its plan
    (one output set per layer) and the step: the plan alone at N = 1, the library's position-shard call at N > 1."""

    def __init__(self, torch, dist, pa, ctx, comm, device, stream, world, rank, local, layers, keys, rows, quant,
                 layer_base, exchange=0, groups=0, chunk_keys=0, shares=None, student_t=False, inputs=None):
        self.torch, self.dist, self.pa, self.ctx, self.comm = torch, dist, pa, ctx, comm
        self.device, self.stream, self.world, self.rank, self.local = device, stream, world, rank, local
        self.layers, self.keys, self.rows, self.quant, self.layer_base = layers, keys, rows, quant, layer_base
        self.exchange, self.groups = exchange, groups
        # inputs: another leg's (K, V, k0, nk) of the same positions (a second query shape over the same keys)
        self.K, self.V, self.k0, self.nk = inputs if inputs is not None else shard_inputs(
            torch, pa, device, layers, keys, rank, world, quant, layer_base, shares, student_t)
        torch.cuda.synchronize()
        self.shape = pa.shape_for(HD, NKV, rows, quant)
        segs = [pa.Seg(self.K[i].data_ptr(), self.V[i].data_ptr(), self.nk, i) for i in range(layers)]
        self.plan = pa.Plan(ctx, self.shape, layers, segs, chunk_keys=chunk_keys)
        self.O = torch.empty((layers, NKV, rows, HD), dtype=torch.float32, device=device)
        self.m = torch.empty((layers, NKV, rows), dtype=torch.float32, device=device)
        self.l = torch.empty_like(self.m)

    def step(self, Q, out=None):
        O, m, l = out if out is not None else (self.O, self.m, self.l)
        if self.world == 1:
            self.plan.run(Q, O, m, l, self.stream)
        else:
            self.pa.shard_attn_allgather_merge(self.plan, Q, self.comm, O, m, l, self.stream)

    def barrier(self):
        if self.world > 1:
            self.dist.barrier(device_ids=[self.local])

    def max_over_ranks(self, x: float) -> float:
        t = self.torch.tensor([x], device=self.device)
        if self.world > 1:
            self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return float(t.item())

    def timed(self, q_of, steps: int, warmup: int, plan_only_steps: int = 0):
        """W untimed steps, then exactly `steps` steps between a barrier + synchronize on both sides, CUDA events on the
        step stream (one after every step), max over ranks; the attention kernel's own time from events around its
        launches; the clocks of the timed region. plan_only_steps > 0 (N > 1): also the plan alone (kernel + in-plan
        merge), to split the step into kernel, merge and exchange."""
        torch = self.torch
        self.ctx.set_shard_exchange(self.exchange)
        self.ctx.set_shard_groups(self.groups)
        for i in range(warmup):
            self.step(q_of(i))
        self.ctx.status(self.stream)
        self.barrier()
        torch.cuda.synchronize()
        launches0 = self.ctx.launches
        self.plan.profile(steps * 16)    # up to 16 set groups per step
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(steps + 1)]
        with ClockSampler(self.local) as clk:
            self.barrier()
            torch.cuda.synchronize()
            ev[0].record(self.stream)
            for i in range(steps):
                self.step(q_of(warmup + i))
                ev[i + 1].record(self.stream)
            torch.cuda.synchronize()
            self.barrier()
        launches = self.ctx.launches - launches0
        self.ctx.status(self.stream)
        kern_total, _ = self.plan.kernel_ms()
        self.plan.profile(0)
        per = [ev[i].elapsed_time(ev[i + 1]) for i in range(steps)]
        ms = self.max_over_ranks(ev[0].elapsed_time(ev[-1]))
        kern = self.max_over_ranks(kern_total / steps)
        res = {"ms": ms, "kernel_ms": kern, "launches": launches, "clocks": clk.summary(), "exchange": self.ctx.shard_last(),
               "step_ms": {"min": round(min(per), 4), "median": round(statistics.median(per), 4),
                           "max": round(max(per), 4)}}
        if plan_only_steps > 0 and self.world > 1:
            # into separate outputs: (O, m, l) keep the last timed step's merged result for the parity check
            Ox, mx, lx = torch.empty_like(self.O), torch.empty_like(self.m), torch.empty_like(self.l)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            self.barrier()
            torch.cuda.synchronize()
            e0.record(self.stream)
            for i in range(plan_only_steps):
                self.plan.run(q_of(warmup + i), Ox, mx, lx, self.stream)
            e1.record(self.stream)
            torch.cuda.synchronize()
            res["plan_ms"] = self.max_over_ranks(e0.elapsed_time(e1) / plan_only_steps)
            del Ox, mx, lx
        return res

    def close(self):
        self.plan.close()
        del self.K, self.V, self.O, self.m, self.l
        self.torch.cuda.empty_cache()


def breakdown(r: dict, steps: int) -> dict:
    """Per-step split of the timed step: attention kernel, in-plan merge (and launch gaps), and what the exchange adds
    on top (the exposed part of the exchange and the fold), all from CUDA events, max over ranks."""
    step = r["ms"] / steps
    b = {"step_ms": round(step, 4), "kernel_ms": round(r["kernel_ms"], 4)}
    if "plan_ms" in r:
        b["merge_and_gaps_ms"] = round(max(0.0, r["plan_ms"] - r["kernel_ms"]), 4)
        b["exchange_and_fold_ms"] = round(max(0.0, step - r["plan_ms"]), 4)
    else:
        b["merge_and_gaps_ms"] = round(max(0.0, step - r["kernel_ms"]), 4)
    return b


def exchange_name(world: int, used) -> str:
    """The exchange the library's shard call used (pa_cuda_shard_last): mode, set groups."""
    if world == 1:
        return "none (one GPU)"
    mode, groups = used
    kind = {1: "NCCL all-gather of (O,m,l) + LSE fold", 2: "NCCL all-reduce MAX of m + SUM of rescaled (O,l)",
            3: "peer stores of the merged (O,m,l) over NVLink into every rank + bounded-wait LSE fold"}.get(mode, "?")
    return kind + (f", {groups} set groups overlapped with the kernels" if groups > 1 else "")


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


# --------------------------------------------------------------------------------------------- config 2 and 3 legs
def bench_prefill(torch, dist, pa, ctx, comm, device, stream, world, rank, local, layers: int, steps: int):
    """Config 2: a 512-token query batch (40 q / 8 KV heads, d128) against 65,536 older Q8_0 positions per layer, no
    mask, all `layers` layers per step in one plan (the tcgen05 CTA-pair kernel: 2,560 rows per KV head); the positions
    sharded over the ranks like the decode workload (each rank 65,536/N of every layer)."""
    rows = PF_TOKENS * GQA
    leg = Leg(torch, dist, pa, ctx, comm, device, stream, world, rank, local, layers, PF_KEYS, rows, pa.Q8_0,
              1000)
    g = torch.Generator(device=device)
    g.manual_seed(SEED + 11)
    Qs = (torch.randn((layers, NKV, rows, HD), generator=g, device=device) / HD ** 0.5).to(torch.float16)
    r = leg.timed(lambda i: Qs, steps, 2, plan_only_steps=steps)
    kname = leg.plan.kernel
    flops_layer = 4.0 * PF_TOKENS * Q_HEADS * HD * PF_KEYS
    flops = flops_layer * layers                                  # the whole job per step
    flops_launch = 4.0 * PF_TOKENS * Q_HEADS * HD * leg.nk * layers   # this rank's kernel launches per step
    peak, kind = measured_tensor_peak()
    peak_s, _ = measured_tensor_peak(sustained=True)
    ms = r["ms"] / steps
    achieved = flops_launch / (r["kernel_ms"] * 1e-3) / 1e12
    parity = None
    if rank == 0:
        sample = torch.arange(0, rows, rows // 32, device=device)[:32]
        parity = parity_fp64(torch, pa, device, pa.Q8_0, PF_KEYS, [0], 1000, Qs, leg.O, leg.m, leg.l, sample)
    leg.close()
    del Qs
    torch.cuda.empty_cache()
    return {"metric": "prefill attn TFLOP/s (config 2: 512 tokens x 65536 Q8_0 keys, 40q/8kv, d128)",
            "value": round(flops / (ms * 1e-3) / 1e12, 1), "unit": "TFLOP/s", "ms_per_step": round(ms, 3),
            "layers": layers, "steps": steps, "keys_per_gpu": leg.nk,
            "exchange": exchange_name(world, r["exchange"]),
            "roofline": {"bound": "tensor", "achieved": round(achieved, 1), "peak": peak,
                         "unit": "TFLOP/s", "frac": round(achieved / peak, 4), "peak_kind": kind,
                         "frac_of_sustained": round(achieved / peak_s, 4),
                         "kernel": kname, "kernel_ms": round(r["kernel_ms"], 3),
                         "algorithmic_flops_per_launch": flops_launch,
                         "traffic": prefill_traffic(leg.nk, layers)},
            "breakdown": breakdown(r, steps), "parity": parity, "clocks": r["clocks"], "step_ms": r["step_ms"]}


U_KEYS, U_SHARDS, U_SEED = 229376, 8, 41   # config 4


def uneven_shares(world: int):
    """Config 4's 8 seeded uneven shards (10-20% of the positions each, as tests/test_configs_gpu.py draws them),
    grouped onto `world` ranks (1, 2, 4 or 8): rank r holds shards [r*8/world, (r+1)*8/world), contiguous positions."""
    import numpy as np
    w = np.random.default_rng(U_SEED).uniform(0.10, 0.20, U_SHARDS)
    shares = np.floor(w / w.sum() * U_KEYS).astype(int)
    shares[-1] += U_KEYS - shares.sum()
    per = U_SHARDS // world
    return [int(shares[r * per:(r + 1) * per].sum()) for r in range(world)]


def bench_uneven(torch, dist, pa, ctx, comm, device, stream, world, rank, local, layers: int, steps: int,
                 prefill_steps: int):
    """Config 4: 229,376 Q8_0 positions per layer with Student-t(3) V, split by position into 8 seeded uneven shards of
    10-20% each (grouped onto the ranks), 64 layers: a 1-token decode (fresh seeded Q per step) and a 512-token prefill
    over the same positions. The step time is the slowest rank's, so the uneven split shows in the whole-job rate."""
    if U_SHARDS % world:
        return {"skipped": f"config 4's 8 shards do not group onto {world} ranks"}
    shares = uneven_shares(world)
    out = {"keys": U_KEYS, "layers": layers, "shares_per_rank": shares}
    # decode
    leg = Leg(torch, dist, pa, ctx, comm, device, stream, world, rank, local, layers, U_KEYS, GQA, pa.Q8_0, 4000,
              shares=shares, student_t=True)
    Qs = make_q(torch, 16, layers, GQA, device, SEED + 17)
    r = leg.timed(lambda i: Qs[i % 16], steps, 3, plan_only_steps=min(steps, 20))
    ms = r["ms"] / steps
    lb = layer_bytes(U_KEYS)["total"] * layers
    lb_launch = layer_bytes(leg.nk)["total"] * layers
    parity = None
    if rank == 0:
        last = (3 + steps - 1) % 16   # the last timed step's Q (3 warm-up steps first)
        parity = parity_fp64(torch, pa, device, pa.Q8_0, U_KEYS, [0, layers - 1], 4000, Qs[last], leg.O, leg.m, leg.l,
                             torch.arange(GQA, device=device), student_t=True)
    out["decode"] = {
        "metric": "uneven decode KV-attn GB/s (config 4: 229376 Q8_0 keys in 8 seeded shards of 10-20%, Student-t V)",
        "value": round(lb / (ms * 1e-3) / 1e9, 1), "unit": "GB/s", "ms_per_step": round(ms, 4), "steps": steps,
        "keys_per_gpu": leg.nk, "exchange": exchange_name(world, r["exchange"]),
        "roofline": {"bound": "hbm", "achieved": round(lb_launch / (r["kernel_ms"] * 1e-3) / 1e9, 1),
                     "peak": measured_peaks()[0], "unit": "GB/s",
                     "frac": round(lb_launch / (r["kernel_ms"] * 1e-3) / 1e9 / measured_peaks()[0], 4),
                     "kernel": leg.plan.kernel, "kernel_ms": round(r["kernel_ms"], 4)},
        "breakdown": breakdown(r, steps), "parity": parity, "clocks": r["clocks"]}
    inputs = (leg.K, leg.V, leg.k0, leg.nk)
    leg.plan.close()
    del Qs
    # prefill over the same positions
    if prefill_steps > 0:
        rows = PF_TOKENS * GQA
        leg2 = Leg(torch, dist, pa, ctx, comm, device, stream, world, rank, local, layers, U_KEYS, rows, pa.Q8_0, 4000,
                   inputs=inputs)
        g = torch.Generator(device=device)
        g.manual_seed(SEED + 19)
        Qp = (torch.randn((layers, NKV, rows, HD), generator=g, device=device) / HD ** 0.5).to(torch.float16)
        r2 = leg2.timed(lambda i: Qp, prefill_steps, 2, plan_only_steps=prefill_steps)
        ms2 = r2["ms"] / prefill_steps
        flops = 4.0 * PF_TOKENS * Q_HEADS * HD * U_KEYS * layers
        flops_launch = 4.0 * PF_TOKENS * Q_HEADS * HD * leg2.nk * layers
        peak, kind = measured_tensor_peak()
        parity2 = None
        if rank == 0:
            sample = torch.arange(0, rows, rows // 32, device=device)[:32]
            parity2 = parity_fp64(torch, pa, device, pa.Q8_0, U_KEYS, [0], 4000, Qp, leg2.O, leg2.m, leg2.l, sample,
                                  student_t=True)
        out["prefill"] = {
            "metric": "uneven prefill attn TFLOP/s (config 4: 512 tokens x 229376 Q8_0 keys in 8 seeded shards)",
            "value": round(flops / (ms2 * 1e-3) / 1e12, 1), "unit": "TFLOP/s", "ms_per_step": round(ms2, 3),
            "steps": prefill_steps, "keys_per_gpu": leg2.nk, "exchange": exchange_name(world, r2["exchange"]),
            "roofline": {"bound": "tensor", "achieved": round(flops_launch / (r2["kernel_ms"] * 1e-3) / 1e12, 1),
                         "peak": peak, "unit": "TFLOP/s",
                         "frac": round(flops_launch / (r2["kernel_ms"] * 1e-3) / 1e12 / peak, 4), "peak_kind": kind,
                         "kernel": leg2.plan.kernel, "kernel_ms": round(r2["kernel_ms"], 3)},
            "breakdown": breakdown(r2, prefill_steps), "parity": parity2, "clocks": r2["clocks"]}
        leg2.close()
        del Qp
    del inputs, leg
    torch.cuda.empty_cache()
    return out


def prefill_traffic(nk: int, layers: int):
    """ncu DRAM bytes of the prefill kernel (profiles/prefill_traffic.json, a smaller capture of the same kernel)
    scaled to this launch by key positions, or None when no capture is committed."""
    try:
        with open(os.path.join(ROOT, "profiles", "prefill_traffic.json")) as f:
            tr = json.load(f)
        return round(tr["dram_bytes_per_key_position_per_layer"] * nk * layers)
    except Exception:
        return None


def bench_verify(torch, dist, pa, ctx, comm, device, stream, world, rank, local, layers: int, steps: int):
    """Config 3: a speculative-verify batch of 16 draft tokens (80 rows per KV head, GQA 5) against 196,608 offloaded
    Q4_0 positions per layer, 64 layers per step. The causal mask applies among the 16 new tokens only, i.e. to the
    host's local partial: the offloaded keys are fully visible to every draft token, so the offloaded partial has no
    mask. Fresh seeded Q per step. Roofline: the slower of HBM (quantised K/V bytes) and tensor (4 n_tok q_heads d keys
    flops) for this rank's launch."""
    rows = VF_TOKENS * GQA
    leg = Leg(torch, dist, pa, ctx, comm, device, stream, world, rank, local, layers, VF_KEYS, rows, pa.Q4_0,
              3000)
    Qs = make_q(torch, steps + 3, layers, rows, device, SEED + 13)
    r = leg.timed(lambda i: Qs[i % Qs.shape[0]], steps, 3, plan_only_steps=min(steps, 20))
    ms = r["ms"] / steps
    lb = layer_bytes(VF_KEYS, rows, pa.Q4_0)["total"] * layers
    flops = 4.0 * VF_TOKENS * Q_HEADS * HD * VF_KEYS * layers
    lb_launch = layer_bytes(leg.nk, rows, pa.Q4_0)["total"] * layers
    fl_launch = 4.0 * VF_TOKENS * Q_HEADS * HD * leg.nk * layers
    hbm, _ = measured_peaks()
    ten, _ = measured_tensor_peak()
    t_hbm, t_ten = lb_launch / (hbm * 1e9), fl_launch / (ten * 1e12)
    bound = "tensor" if t_ten >= t_hbm else "hbm"
    kt = r["kernel_ms"] * 1e-3
    parity = None
    if rank == 0:
        last = (3 + steps - 1) % Qs.shape[0]
        parity = parity_fp64(torch, pa, device, pa.Q4_0, VF_KEYS, [0, layers - 1], 3000, Qs[last], leg.O, leg.m, leg.l,
                             torch.arange(rows, device=device))
    kname = leg.plan.kernel
    nk = leg.nk
    leg.close()
    del Qs
    torch.cuda.empty_cache()
    return {"metric": "verify KV-attn GB/s (config 3: 16 tokens x 196608 Q4_0 keys, 40q/8kv, d128, 64 layers)",
            "value": round(lb / (ms * 1e-3) / 1e9, 1), "unit": "GB/s", "tflops": round(flops / (ms * 1e-3) / 1e12, 1),
            "ms_per_step": round(ms, 4), "layers": layers, "steps": steps, "keys_per_gpu": nk,
            "exchange": exchange_name(world, r["exchange"]),
            "roofline": {"bound": bound, "unit": "TFLOP/s" if bound == "tensor" else "GB/s",
                         "achieved": round((fl_launch / kt / 1e12) if bound == "tensor" else (lb_launch / kt / 1e9), 1),
                         "peak": ten if bound == "tensor" else hbm,
                         "frac": round(max(t_hbm, t_ten) / kt, 4),
                         "achieved_gbs": round(lb_launch / kt / 1e9, 1), "achieved_tflops": round(fl_launch / kt / 1e12, 1),
                         "roofline_ms": round(max(t_hbm, t_ten) * 1e3, 4), "kernel": kname,
                         "kernel_ms": round(r["kernel_ms"], 4), "algorithmic_bytes_per_launch": lb_launch,
                         "algorithmic_flops_per_launch": fl_launch},
            "breakdown": breakdown(r, steps), "parity": parity, "clocks": r["clocks"], "step_ms": r["step_ms"]}


# --------------------------------------------------------------------------------------------- the engine path
def bench_engine(pa, ctx, calls: int):
    """pa::engine calls as the reference server makes them (phone-attn/phone-attn.h:527-697) and as pa-tool times them
    (phone-attn/pa-tool.cpp:245-263): pa-tool's geometry (HD 256, 4 KV heads, 48 rows per KV head, Q8_0 pages of 4,096
    keys), 8 layers of 32,768 keys, calls cycling the layers, each followed by arm() for the next layer as the server's
    arm_after_reply does. p50 / p90 of begin-to-end (pa_cuda_end's milliseconds: plan lookup, Q packing, upload, kernels,
    readback, unpacking) and of the GPU time, for 8-token and 1-token calls."""
    import numpy as np
    import torch
    hd, nkv, nr, layers, nk, page = 256, 4, 48, 8, 32768, 4096
    shape = pa.shape_for(hd, nkv, nr, pa.Q8_0)
    g = torch.Generator()
    g.manual_seed(SEED + 17)
    k = pa.quantize_q8_0(torch.randn((nk, nkv, hd), generator=g) * 1.5).reshape(nk, -1).numpy()
    v = pa.quantize_q8_0(torch.randn((nk, nkv, hd), generator=g)).reshape(nk, -1).numpy()
    eng = pa.Engine(ctx)
    pages = []
    for _ in range(layers):
        lp = []
        for p0 in range(0, nk, page):
            pg = eng.alloc_page(page * shape.rs)
            eng.page_view(pg, page * shape.rs, "k")[:] = k[p0:p0 + page].reshape(-1)
            eng.page_view(pg, page * shape.rs, "v")[:] = v[p0:p0 + page].reshape(-1)
            lp.append(pg)
        pages.append(lp)
    nkeys = [page] * (nk // page)
    q = (np.random.default_rng(SEED + 19).standard_normal((nkv, nr, hd)) / 16).astype(np.float16).view(np.uint16)
    O = np.empty((nkv * nr, hd), np.float32)
    m = np.empty((nkv * nr,), np.float32)
    l = np.empty_like(m)
    out = {}
    for ntok in (8, 1):
        qt = q.copy()
        qt.reshape(nkv, 6, 8, hd)[:, :, ntok:, :] = 0
        wall, gpu = [], []
        for it in range(calls + 10):
            L = it % layers
            eng.begin(pages[L], nkeys, qt, shape, 1, ntok)
            ms = eng.end(O, m, l)
            if it >= 10:
                wall.append(ms)
                gpu.append(eng.exec_ms)
            eng.arm(pages[(L + 1) % layers], nkeys, shape, ntok)
        wall.sort()
        gpu.sort()
        out[f"tokens_{ntok}"] = {"p50_ms": round(wall[len(wall) // 2], 4), "p90_ms": round(wall[len(wall) * 9 // 10], 4),
                                 "gpu_p50_ms": round(gpu[len(gpu) // 2], 4), "calls": len(wall)}
    out["graph_calls"] = eng.graph_calls
    for lp in pages:
        for pg in lp:
            eng.free_page(pg)
    out["workload"] = (f"pa::engine begin/end (C ABI), one layer per call: {nk} Q8_0 keys in {nk // page} pages, "
                       f"HD {hd}, {nkv} KV heads, 48 rows per KV head, armed for the next layer after each call")
    return out


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
    comm = None
    if world > 1:
        # the library's own communicator; torch only carries its unique id from rank 0 to the others
        obj = [pa.nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        comm = pa.NcclComm(ctx, obj[0], rank, world)
    stream = torch.cuda.current_stream(device)
    L = args.layers

    # ---- config 1: decode
    decode = None
    if args.only in ("all", "decode"):
        # --qk int8: the config-1 decode plan only (the other workloads keep the f16-domain QK and their kernels)
        ctx.set_qk_domain(pa.QK_INT8 if args.qk == "int8" else pa.QK_F16)
        leg = Leg(torch, dist, pa, ctx, comm, device, stream, world, rank, local, L, args.keys, GQA, pa.Q8_0, 0,
                  chunk_keys=args.chunk_keys)
        ctx.set_qk_domain(pa.QK_F16)
        total_steps = args.warmup + args.steps
        Qs = make_q(torch, total_steps, L, GQA, device, SEED + 7)      # [steps][L][NKV][GQA][HD]
        r = leg.timed(lambda i: Qs[i], args.steps, args.warmup, plan_only_steps=min(args.steps, 64))
        ms = r["ms"]
        per_step_bytes = L * layer_bytes(args.keys)["total"]      # the whole job's algorithmic bytes per step
        value = per_step_bytes * args.steps / (ms * 1e-3) / 1e9
        peak, peak_kind = measured_peaks()
        launch_bytes = L * layer_bytes(leg.nk)["total"]
        achieved = launch_bytes / (r["kernel_ms"] * 1e-3) / 1e9
        traffic = None
        try:
            with open(os.path.join(ROOT, "profiles", "decode_traffic.json")) as f:
                tr = json.load(f)
            # ncu DRAM bytes of a smaller capture, scaled to this launch: reads by key positions, writes by jobs (slots)
            if (HD, GQA) == (128, 5):   # the capture's geometry (config 1)
                traffic = round(tr["dram_read_bytes_per_key_position"] * leg.nk * L + tr["dram_write_bytes_per_job"] *
                                leg.plan.jobs)
        except Exception:
            pass
        roofline = {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                    "frac": round(achieved / peak, 4), "traffic": traffic, "peak_kind": peak_kind,
                    "kernel": leg.plan.kernel, "kernel_ms": round(r["kernel_ms"], 4),
                    "algorithmic_bytes_per_launch": launch_bytes}
        parity = None
        if rank == 0:
            last = args.warmup + args.steps - 1
            parity = parity_fp64(torch, pa, device, pa.Q8_0, args.keys, sorted({0, L - 1}), 0, Qs[last], leg.O, leg.m,
                                 leg.l, torch.arange(GQA, device=device))

        # ---- end to end through the public API with host buffers (pinned Q in, O/m/l out, copies inside the region)
        e2e = None
        if args.e2e_steps > 0:
            rows = L * NKV * GQA
            qh = torch.empty((args.e2e_steps, L, NKV, GQA, HD), dtype=torch.float16).pin_memory()
            qh.copy_(Qs[:args.e2e_steps].cpu())
            Oh = torch.empty((rows, HD), dtype=torch.float32).pin_memory()
            mh = torch.empty((rows,), dtype=torch.float32).pin_memory()
            lh = torch.empty_like(mh).pin_memory()
            qd = torch.empty((L, NKV, GQA, HD), dtype=torch.float16, device=device)

            def e2e_step(i):
                if world == 1:
                    leg.plan.run_host(qh[i], Oh, mh, lh, stream)     # the C ABI host path: H2D, kernels, D2H, sync
                else:
                    qd.copy_(qh[i], non_blocking=True)
                    leg.step(qd)
                    Oh.copy_(leg.O.view(rows, HD), non_blocking=True)
                    mh.copy_(leg.m.view(rows), non_blocking=True)
                    lh.copy_(leg.l.view(rows), non_blocking=True)
                    stream.synchronize()

            for i in range(min(3, args.e2e_steps)):
                e2e_step(i)
            leg.barrier()
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            for i in range(args.e2e_steps):
                e2e_step(i)
            dt = leg.max_over_ranks(time.perf_counter() - t0)
            e2e = {"value": round(per_step_bytes * args.e2e_steps / dt / 1e9, 1), "unit": "GB/s",
                   "h2d_bytes_per_step": L * NKV * GQA * HD * 2, "d2h_bytes_per_step": rows * (HD + 2) * 4,
                   "ms_per_step": round(dt / args.e2e_steps * 1e3, 3)}
        decode = dict(value=value, ms=ms, roofline=roofline, parity=parity, e2e=e2e, r=r, keys_per_gpu=leg.nk,
                      bytes_per_step=per_step_bytes)
        leg.close()
        del Qs
        torch.cuda.empty_cache()

    # ---- config 3 (verify) and config 2 (prefill), sharded the same way
    verify = None
    if args.only in ("all", "verify") and args.verify_steps > 0 and (HD, GQA) == (128, 5):
        verify = bench_verify(torch, dist, pa, ctx, comm, device, stream, world, rank, local, args.verify_layers,
                              args.verify_steps)
    prefill = None
    if args.only in ("all", "prefill") and args.prefill_steps > 0 and (HD, GQA) == (128, 5):
        prefill = bench_prefill(torch, dist, pa, ctx, comm, device, stream, world, rank, local, args.prefill_layers,
                                args.prefill_steps)

    uneven = None
    if args.only in ("all", "uneven") and args.uneven_steps > 0 and (HD, GQA) == (128, 5):
        uneven = bench_uneven(torch, dist, pa, ctx, comm, device, stream, world, rank, local, args.uneven_layers,
                              args.uneven_steps, args.uneven_prefill_steps)

    engine = None
    if rank == 0 and world == 1 and args.only == "all" and args.engine_calls > 0:
        engine = bench_engine(pa, ctx, args.engine_calls)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline and args.only == "all":
        cpu = cpu_baseline()

    if rank == 0:
        if decode is not None:
            r = decode["r"]
            line = {
                "metric": decode_metric(L, args.keys),
                "value": round(decode["value"], 1), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": round(decode["ms"] / args.steps, 4), "higher_is_better": True,
                "scaling": "strong", "vs_baseline": None, "dtype": "f16", "data": "synthetic",
                "config": {"workload": ("config 1: decode" if (HD, GQA) == (128, 5) else "decode") +
                                       ", 1 token/step, fresh seeded Q per step", "layers": L,
                           "keys": args.keys, "keys_per_gpu": decode["keys_per_gpu"], "nkv": NKV, "q_heads": Q_HEADS,
                           "hd": HD, "quant": "q8_0", "qk": args.qk,
                           "parallelism": f"sequence shards x{world}" + (
                               ", pa_cuda_shard_attn_allgather_merge: " + exchange_name(world, r["exchange"])
                               if world > 1 else ""),
                           "l2": f"inputs larger than L2 ({decode['bytes_per_step'] / 1e9:.1f} GB of KV per step), "
                                 f"no flush",
                           "bytes_per_step": decode["bytes_per_step"]},
                "roofline": decode["roofline"], "cpu_baseline": cpu, "e2e": decode["e2e"],
                "gpu_launches": r["launches"], "clocks": r["clocks"], "step_ms": r["step_ms"],
                "breakdown": breakdown(r, args.steps), "parity": decode["parity"],
                "verify": verify, "prefill": prefill, "uneven": uneven, "engine": engine,
            }
        else:
            line = {"metric": "partial run (--only)", "verify": verify, "prefill": prefill, "uneven": uneven,
                    "n_gpus": world}
        print(json.dumps(line), flush=True)
    ctx.set_shard_exchange(0)
    if comm is not None:
        comm.close()
    ctx.close()
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
