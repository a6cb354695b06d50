#!/usr/bin/env python
"""Benchmark of the B200 distillation loss (fwd + bwd) on BASELINE's metric
configuration, printing one JSON line.

Workload (the metric's config): Precomputed teacher
logits, BT=8192 rows per GPU, H=4096, V=131072, bf16 inputs, kd=0.4, T=1.5,
INT8 row-wise grad_W round trip; resolver plan 16 chunks x 512 rows. Synthetic
seeded inputs (h ~ N(0,1), W ~ N(0,0.02), teacher logits ~ N(0,2) read as
variance 2, labels uniform). A step is one `distillation_loss` call over the
rank's rows. Inputs (W 1 GiB, teacher logits 2 GiB per GPU) are larger than
the 126 MB L2, so no flush is needed between steps.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

N>1 runs under torchrun (one rank per GPU, NCCL): rows are sharded across
ranks (weak scaling, 8192 rows per GPU) and the grad_W reduce-scatter is fused
into the wgrad GEMM (peer stores into the owners' slot buffers; `--reduce
nccl` uses an NCCL reduce-scatter instead; `--balance` redistributes rows to
the GPUs' measured speed). `--config c5` runs BASELINE configs[4] (Tied
teacher, H=8192, V=152064) with `--shard rows` or `--shard vocab`.
`--impl reference` times the reference's CPU path (the oracle restatement,
all host threads) on a bounded row sample of the same workload.
"""
from __future__ import annotations

import argparse
import ctypes as C
import json
import os
import re
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import numpy as np

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO / "orda-cutile-rs_b200"))
sys.path.insert(0, str(REPO / "oracle"))

METRIC = "distillation fwd+bwd tokens/sec at BT=8192,H=4096,V=131072; % bf16 tensor peak"
CFG = dict(bt=8192, h=4096, v=131072, kd=0.4, temperature=1.5, teacher_std=2.0 ** 0.5, w_std=0.02)
WORKLOAD = ("c4: Precomputed teacher logits, BT=8192 rows/GPU, H=4096, V=131072, bf16 inputs, "
            "kd=0.4, T=1.5, INT8 grad_W round trip, chunks 16x512")


def algorithmic_flops(bt, h, v):
    """2*BT*V*(3*H_s) for the Precomputed teacher: logits, dgrad, wgrad."""
    return 2.0 * bt * v * 3 * h


def balanced_rows(total: int, speeds: list, quantum: int, lo: int, hi: int) -> list:
    """Rows per rank proportional to each rank's measured rows/ms, in whole
    `quantum`s within [lo, hi], summing to `total` (a multiple of quantum)."""
    n = len(speeds)
    units, lo_u, hi_u = total // quantum, lo // quantum, hi // quantum
    want = [units * sp / sum(speeds) for sp in speeds]
    got = [min(max(int(x), lo_u), hi_u) for x in want]
    # hand out (or take back) the remaining quanta by largest (smallest) residual
    order = sorted(range(n), key=lambda i: want[i] - got[i], reverse=True)
    k = 0
    while sum(got) != units and k < 4 * n * units:
        i = order[k % n]
        if sum(got) < units and got[i] < hi_u:
            got[i] += 1
        elif sum(got) > units and got[order[n - 1 - k % n]] > lo_u:
            got[order[n - 1 - k % n]] -= 1
        k += 1
    if sum(got) != units:
        raise ValueError("cannot balance rows within the bounds")
    return [g * quantum for g in got]


def load_peaks():
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d["bf16_tflops"], d.get("bf16_tflops_sustained"), d["hbm_gbs"], "measured"
    return 1590.0, 1400.0, 6650.0, "fallback"


def host_cores():
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


# ------------------------------------------------------------------ clocks

class ClockSampler:
    """nvidia-smi clock / throttle sampling during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_id: str):
        self.gpu_id = gpu_id
        self.proc = None
        self.f = None

    def start(self):
        try:
            self.f = tempfile.TemporaryFile(mode="w+")
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "50",
                 "-i", self.gpu_id], stdout=self.f, stderr=subprocess.DEVNULL)
        except (FileNotFoundError, OSError):
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.f.seek(0)
        rows = [r.split(",") for r in self.f.read().strip().splitlines() if r.count(",") >= 8]
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].strip().replace(".", "").isdigit()]
        smax = [float(r[2]) for r in rows if r[2].strip().replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].strip() == "Active"})
        power = [float(r[3]) for r in rows if r[3].strip().replace(".", "").isdigit()]
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(smax) if smax else None,
                "reasons": reasons, "samples": len(rows), "power_w_max": max(power) if power else None}


# ------------------------------------------------------------- CPU baselines

def cpu_reference_sample(rows, nthreads, seed=77):
    """Times the reference CPU path (oracle restatement of src/api.rs) on
    `rows` rows of the workload (full H and V, Precomputed teacher, INT8
    round trip). Returns seconds."""
    import torch

    import oracle
    import orda_b200 as ob

    gen = torch.Generator().manual_seed(seed)
    h, v = CFG["h"], CFG["v"]
    hs = torch.randn(rows, h, generator=gen).bfloat16().float().numpy()
    w = (CFG["w_std"] * torch.randn(v, h, generator=gen)).bfloat16().float().numpy()
    tl = (CFG["teacher_std"] * torch.randn(rows, v, generator=gen)).bfloat16().float().numpy()
    labels = torch.randint(0, v, (rows,), generator=gen).tolist()
    opts = ob.LossOptions(kd_weight=CFG["kd"], temperature=CFG["temperature"],
                          config=ob.KernelConfig(quantize_grad_weight=True))
    s, wm, t = ob.Mat.from_array(hs), ob.Mat.from_array(w), ob.Teacher.Precomputed(ob.Mat.from_array(tl))
    t0 = time.perf_counter()
    out = oracle.distillation_loss(s, wm, labels, t, opts, nthreads=nthreads)
    dt = time.perf_counter() - t0
    assert np.isfinite(out.loss)
    return dt


def extrapolate(samples, bt=8192, chunk_rows=512):
    """Least-squares fit t = a*rows + b over (rows, seconds) samples of one
    reference call each (one chunk per call), then the reference's own plan
    for the full workload: 16 chunks x 512 rows -> T = 16 * (a*512 + b).
    b holds the per-call O(V*H) work (grad_W-sized zero/add/scale/quantise
    passes); at full size the per-row GEMM term a dominates."""
    r = np.array([x for x, _ in samples], dtype=np.float64)
    t = np.array([y for _, y in samples], dtype=np.float64)
    a, b = np.polyfit(r, t, 1)
    a = max(a, 1e-12)
    b = max(b, 0.0)
    chunks = bt // chunk_rows
    total = chunks * (a * chunk_rows + b)
    return bt / total, a, b, total


def cpu_baseline_line(nthreads, rows_pair, reps=1):
    samples = []
    for _ in range(reps):
        for rows in rows_pair:
            samples.append((rows, cpu_reference_sample(rows, nthreads, seed=200 + len(samples))))
    value, a, b, total = extrapolate(samples)
    desc = (f"reference CPU path (oracle restatement), {nthreads} thread(s): calls of "
            f"{'/'.join(str(x) for x in rows_pair)} rows at full H=4096, V=131072 (Precomputed, INT8 round trip) "
            f"timed {', '.join(f'{t:.1f}s' for _, t in samples)}; fit t = {a:.3f} s/row + {b:.2f} s/call, "
            f"extrapolated to the 16 x 512-row plan ({total / 3600:.2f} h for 8192 rows)")
    return value, desc, samples


def run_reference_arm(args):
    """--impl reference: the reference's CPU path with all host threads."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    cores = host_cores()
    # Two sample sizes: 1 row (mostly the per-call O(V*H) passes) and the
    # smallest power of two whose call takes about twice as long, so the
    # per-row GEMM term is resolved by the fit.
    t1 = cpu_reference_sample(1, cores)
    rows = 2
    t = cpu_reference_sample(rows, cores)
    while t < 2.0 * t1 and t < 30.0 and rows < 512:
        rows *= 2
        t = cpu_reference_sample(rows, cores)
    for _ in range(max(0, args.warmup - 2)):
        cpu_reference_sample(rows, cores)
    samples = []
    for i in range(max(2, args.steps)):
        r = 1 if i % 2 == 0 else rows
        samples.append((r, cpu_reference_sample(r, cores, seed=100 + i)))
    value, a, b, total = extrapolate(samples)
    per = statistics.mean(t for _, t in samples)
    sample = (f"per step one reference call on 1 or {rows} of 8192 rows (alternating), full H=4096 and "
              f"V=131072, Precomputed teacher, INT8 round trip; fit t = {a:.4f} s/row + {b:.2f} s/call, "
              f"extrapolated to the reference's 16 x 512-row plan ({total / 3600:.2f} h for 8192 rows)")
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": per * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32 (CPU reference path: f32 GEMMs, f64 softmax)",
        "data": "synthetic", "config": {"workload": WORKLOAD, "sample_rows_per_step": [rows, 2 * rows]},
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": cores, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ----------------------------------------------------- c5 (large vocabulary)

C5 = dict(rows=8192, h=8192, v=152064, kd=0.4, temperature=1.5, w_std=0.02)


def run_c5(args):
    """BASELINE config c5: Tied teacher, H=8192, V=152064, 8192 rows per GPU
    (weak scaling). --shard rows: each rank its own 8192 rows, grad_W
    reduce-scatter fused into the wgrad GEMM. --shard vocab: every rank holds
    all 8192*N rows and V/N vocabulary rows of W; one all-gather of per-row
    statistics, all-reduce of grad_hidden and the scalars. No e2e / CPU
    baseline (those are measured on the metric config c4)."""
    import torch
    import torch.distributed as dist

    import orda_b200 as ob
    from orda_b200 import shard
    from orda_b200.device import DeviceContext, distillation_loss_device

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    h, v = C5["h"], C5["v"]
    vocab = world > 1 and args.shard == "vocab"
    rows = C5["rows"] * (world if vocab else 1)
    gen = torch.Generator(device=dev).manual_seed(2000 + (0 if vocab else rank))
    hs = torch.randn(rows, h, generator=gen, device=dev).bfloat16()
    ht = (hs.float() + 0.1 * torch.randn(rows, h, generator=gen, device=dev)).bfloat16()
    labels = torch.randint(0, v, (rows,), generator=gen, device=dev)
    v0, v1 = shard.vocab_slice_bounds(v, world, rank) if vocab else (0, v)
    wgen = torch.Generator(device=dev).manual_seed(7 + v0)
    w = (C5["w_std"] * torch.randn(v1 - v0, h, generator=wgen, device=dev)).bfloat16()
    opts = ob.LossOptions(kd_weight=C5["kd"], temperature=C5["temperature"])
    ctx = DeviceContext(local)
    stream = torch.cuda.current_stream(dev)
    out = {"grad_student_hidden": torch.empty(rows, h, device=dev),
           "grad_teacher_hidden": torch.empty(rows, h, device=dev), "scalars": torch.empty(4, device=dev)}
    fused = None
    if world > 1 and not vocab:
        fused = shard.SlotReduceScatter(ctx, v, h)
        gw_slice = torch.empty(v // world, h, device=dev)
        n_global = shard.global_non_ignore(labels, -100)
    else:
        out["grad_weight"] = torch.empty(v1 - v0, h, device=dev)

    # vocabulary-sharded: grad_hidden reduce-scattered by the dgrad GEMMs
    # (each rank keeps its 8192 rows) unless --reduce nccl (all-reduce)
    hslots = shard.HiddenSlots(ctx, rows, h, teacher=True) if vocab and args.reduce == "fused" else None

    def step():
        if vocab:
            return shard.vocab_sharded_step(ctx, hs, w, labels, ob.TeacherMode.Tied, v, v0, teacher_hidden=ht,
                                            opts=opts, out=out, stream=stream, hidden_slots=hslots)
        if fused:
            def compute(n):
                r = distillation_loss_device(ctx, hs, w, labels, ob.TeacherMode.Tied, teacher_hidden=ht, opts=opts,
                                             out=out, global_non_ignore=n, scatter_grad_weight=True, stream=stream)
                return r.scalars, r.grad_student_hidden

            return fused.step(compute, labels, -100, n_global, gw_slice, stream=stream)
        return distillation_loss_device(ctx, hs, w, labels, ob.TeacherMode.Tied, teacher_hidden=ht, opts=opts,
                                        out=out, stream=stream)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    ctx.check()
    sampler = None
    if rank == 0 and not args.no_clocks:
        uuid = getattr(torch.cuda.get_device_properties(dev), "uuid", None)
        sampler = ClockSampler(f"GPU-{uuid}" if uuid is not None else str(local))
        sampler.start()
        time.sleep(0.3)
    ctx.reset_timing()
    ctx.enable_timing(True)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    ev0.record(stream)
    for _ in range(args.steps):
        step()
    ev1.record(stream)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    ms_total = ev0.elapsed_time(ev1)
    phases = ctx.phase_times()
    ctx.enable_timing(False)
    clocks = sampler.stop() if sampler else None
    ctx.check()
    if world > 1:
        t = torch.tensor([ms_total], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms_total = float(t.item())
    ms_step = ms_total / args.steps
    tokens = C5["rows"] * world
    peak, peak_sus, hbm, peak_kind = load_peaks()
    # Tied teacher with teacher CE weight 1: 12 * rows * V * H per GPU
    flops = 12.0 * C5["rows"] * v * h
    gemm_ms = sum(phases[p][0] for p in ("logits_gemm", "dgrad_gemm", "wgrad_gemm")) / args.steps
    achieved = flops / (gemm_ms / 1e3) / 1e12
    if rank == 0:
        line = {
            "metric": "distillation fwd+bwd tokens/sec, c5 (Tied, H=8192, V=152064)", "value": tokens / (ms_step / 1e3),
            "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "c5: Tied teacher, 8192 rows per GPU, H=8192, V=152064, kd=0.4, T=1.5",
                       "parallelism": (("vocabulary sharded (V/N per GPU, all rows on every GPU), grad_hidden "
                                        + ("reduce-scattered by the dgrad GEMMs" if hslots else "all-reduced"))
                                       if vocab else
                                       "rows sharded, grad_W reduce-scatter fused into the wgrad GEMM"
                                       if world > 1 else "single GPU")},
            "phases_ms_per_step": {k: v_[0] / args.steps for k, v_ in phases.items()},
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                         "frac": achieved / peak, "kernel": "gemm_kernel (tcgen05 cta_group::2)",
                         "gemm_ms_per_step": gemm_ms},
            "step_tflops_per_gpu": flops / (ms_step / 1e3) / 1e12, "clocks": clocks,
        }
        print(json.dumps(line), flush=True)
    ctx.close()
    if world > 1:
        dist.destroy_process_group()
    return 0


# --------------------------------------------------------------- our arm

def run_ours(args):
    import torch
    import torch.distributed as dist

    import orda_b200 as ob
    from orda_b200 import shard
    from orda_b200.device import DeviceContext, distillation_loss_device, quantize_grad_w

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        print(f"warning: --gpus {args.gpus} but WORLD_SIZE {world}", file=sys.stderr)
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)

    bt, h, v = args.rows, CFG["h"], CFG["v"]
    # N > 1 with balancing: room for up to 25 % more rows on a faster GPU
    balance = world > 1 and args.balance
    cap = bt + (bt // 4 if balance else 0)
    gen = torch.Generator(device=dev).manual_seed(1000 + rank)
    wgen = torch.Generator(device=dev).manual_seed(7)
    hs_all = torch.randn(cap, h, generator=gen, device=dev).bfloat16()
    w = (CFG["w_std"] * torch.randn(v, h, generator=wgen, device=dev)).bfloat16()
    tl_all = torch.empty(cap, v, device=dev, dtype=torch.bfloat16)
    for r0 in range(0, cap, 1024):  # generate in slabs to bound the fp32 temporary
        tl_all[r0:r0 + 1024] = (CFG["teacher_std"] * torch.randn(min(1024, cap - r0), v, generator=gen, device=dev))
    labels_all = torch.randint(0, v, (cap,), generator=gen, device=dev)
    gsh_all = torch.empty(cap, h, device=dev)
    opts = ob.LossOptions(kd_weight=CFG["kd"], temperature=CFG["temperature"],
                          config=ob.KernelConfig(quantize_grad_weight=True))
    out = {"grad_weight": torch.empty(v, h, device=dev), "scalars": torch.empty(4, device=dev)}

    def use_rows(n):
        """This rank's rows: the first n of the generated inputs."""
        nonlocal hs, tl, labels
        hs, tl, labels = hs_all[:n], tl_all[:n], labels_all[:n]
        out["grad_student_hidden"] = gsh_all[:n]

    hs = tl = labels = None
    use_rows(bt)
    rows_per_rank = None
    q = torch.empty(v // world, h, device=dev, dtype=torch.int8)
    qs = torch.empty(v // world, device=dev)
    stream = torch.cuda.current_stream(dev)
    ctx = DeviceContext(local)
    n_global = bt * world if world == 1 else shard.global_non_ignore(labels, -100)

    # N > 1: the grad_W reduce-scatter is fused into the wgrad GEMM (peer
    # stores into the owners' slot buffers) unless --reduce nccl
    fused = (shard.SlotReduceScatter(ctx, v, h, label_capacity=cap)
             if world > 1 and args.reduce == "fused" else None)
    gw_slice = torch.empty(v // world, h, device=dev) if fused else None
    if fused:
        del out["grad_weight"]  # the local full grad_W is never materialised
    marks = []  # (after compute, end of step) events of the timed steps

    def step():
        if world == 1:
            out["grad_weight_q"], out["grad_weight_scale"] = q, qs
            return distillation_loss_device(ctx, hs, w, labels, ob.TeacherMode.Precomputed, teacher_logits=tl,
                                            opts=opts, out=out, want_int8=True, stream=stream)
        # events: [0] device entry done, [1] step done, [2] barrier passed,
        # [3] slot reduction done, [4] step start
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(5)]
        ev[4].record(stream)

        if fused:
            def compute_scatter(n):
                r = distillation_loss_device(ctx, hs, w, labels, ob.TeacherMode.Precomputed, teacher_logits=tl,
                                             opts=opts, out=out, global_non_ignore=n, scatter_grad_weight=True,
                                             stream=stream)
                ev[0].record(stream)
                return r.scalars, r.grad_student_hidden

            res = fused.step(compute_scatter, labels, -100, n_global, gw_slice, quantize=True, q=q, scale=qs,
                             stream=stream, marks=ev[2:4])
        else:
            def compute(n):
                r = distillation_loss_device(ctx, hs, w, labels, ob.TeacherMode.Precomputed, teacher_logits=tl,
                                             opts=opts, out=out, global_non_ignore=n, skip_quantize=True,
                                             stream=stream)
                ev[0].record(stream)
                return r.scalars, r.grad_student_hidden, r.grad_weight

            def quant(sl, shifted):
                quantize_grad_w(ctx, sl, shifted, -100, False, 0, q, qs, stream=stream)

            res = shard.row_sharded_step(compute, labels, -100, n_global, quantize=quant, label_capacity=cap)
        ev[1].record(stream)
        marks.append(ev)
        return res

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    ctx.check()
    if balance:
        # Power-capped GPUs of one node settle at different clocks, so equal
        # row blocks finish at different times and every step waits for the
        # slowest rank. Redistribute the global batch (8192 x N rows, as
        # before) in proportion to each rank's rows per ms of device time in
        # the warm-up steps after the first, then warm up again.
        t_mine = statistics.mean(ev[4].elapsed_time(ev[0]) for ev in marks[1:])
        tt = torch.tensor([t_mine], device=dev, dtype=torch.float64)
        all_t = [torch.empty_like(tt) for _ in range(world)]
        dist.all_gather(all_t, tt)
        speeds = [bt / float(x) for x in all_t]
        rows_per_rank = balanced_rows(bt * world, speeds, 16, bt - bt // 4, cap)
        use_rows(rows_per_rank[rank])
        n_global = shard.global_non_ignore(labels, -100)
        for _ in range(args.warmup):
            step()
        torch.cuda.synchronize()
        ctx.check()

    # ---------------- timed region
    sampler = None
    if not args.no_clocks:  # every rank samples its own GPU; rank 0's is the line's `clocks`
        uuid = getattr(torch.cuda.get_device_properties(dev), "uuid", None)
        sampler = ClockSampler(f"GPU-{uuid}" if uuid is not None else str(local))
        sampler.start()
        time.sleep(0.3)
    ctx.reset_timing()
    ctx.enable_timing(True)
    launches0 = ctx.launch_count()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    marks.clear()
    ev0.record(stream)
    h0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    host_ms = (time.perf_counter() - h0) * 1e3 / args.steps
    ev1.record(stream)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    ms_total = ev0.elapsed_time(ev1)
    # N > 1: time from the end of the device entry to the end of the step
    # (scalar all-reduce, grad_W reduction and the slice's INT8 round trip)
    collective_ms = statistics.mean(ev[0].elapsed_time(ev[1]) for ev in marks) if marks else None
    rank_split = None
    if world > 1:
        # per rank: device-entry time, then (fused path) the wait at the
        # barrier and the slot reduction, averaged over the timed steps
        mine = [statistics.mean(ev[4].elapsed_time(ev[0]) for ev in marks)]
        if fused:
            mine += [statistics.mean(ev[0].elapsed_time(ev[2]) for ev in marks),
                     statistics.mean(ev[2].elapsed_time(ev[3]) for ev in marks)]
        t = torch.tensor(mine, device=dev, dtype=torch.float64)
        allt = [torch.empty_like(t) for _ in range(world)]
        dist.all_gather(allt, t)
        rank_split = [[round(x, 3) for x in a.tolist()] for a in allt]
    phases = ctx.phase_times()
    ctx.enable_timing(False)
    launches = ctx.launch_count() - launches0
    clocks = sampler.stop() if sampler else None
    ctx.check()
    if world > 1:
        t = torch.tensor([ms_total], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms_total = float(t.item())
        if clocks is not None or sampler is not None:
            mine = torch.tensor([float((clocks or {}).get("sm_mhz") or 0.0), float((clocks or {}).get("power_w_max")
                                                                                   or 0.0)], device=dev)
            allc = [torch.empty_like(mine) for _ in range(world)]
            dist.all_gather(allc, mine)
            if rank_split is not None:
                rank_split = [r + [round(float(c[0]), 1), round(float(c[1]), 1)] for r, c in zip(rank_split, allc)]
    ms_step = ms_total / args.steps
    tokens = bt * world
    value = tokens / (ms_step / 1e3)

    # ---------------- roofline of the dominant kernel family (tcgen05 GEMM)
    peak, peak_sus, hbm, peak_kind = load_peaks()
    gemm_ms = sum(phases[p][0] for p in ("logits_gemm", "dgrad_gemm", "wgrad_gemm")) / args.steps
    gemm_launches = sum(phases[p][1] for p in ("logits_gemm", "dgrad_gemm", "wgrad_gemm")) / args.steps
    flops = algorithmic_flops(bt, h, v)
    achieved = flops / (gemm_ms / 1e3) / 1e12
    # DRAM bytes of the step's GEMM launches from the committed ncu launch list
    # of this workload (dram__bytes_read.sum + dram__bytes_write.sum)
    traffic = None
    tfile = REPO / "profiles" / "launch_list_c4_bench.md"
    if tfile.exists() and bt == CFG["bt"]:
        m = re.search(r"traffic_bytes_per_step_gemm = (\d+)", tfile.read_text())
        traffic = int(m.group(1)) if m else None
    roofline = {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s", "frac": achieved / peak,
                "traffic": traffic, "traffic_scope": "DRAM bytes of the step's 3 GEMM launches (ncu launch list, "
                "profiles/launch_list_c4_bench.md)", "kernel": "gemm_kernel (tcgen05 cta_group::2, 3 layouts)",
                "launches_per_step": gemm_launches, "gemm_ms_per_step": gemm_ms,
                "peak_kind": f"{peak_kind} burst bf16 (MEASURED_PEAKS.json bf16_tflops)",
                "frac_of_sustained": achieved / peak_sus if peak_sus else None}
    step_tflops = flops * world / (ms_step / 1e3) / 1e12 / world

    line = {
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": WORKLOAD if bt == CFG["bt"] else f"{WORKLOAD} [profiling size: {bt} rows]",
                   "global_batch": tokens, "seq_len": None, "rows_per_gpu": bt,
                   "rows_per_rank": rows_per_rank,
                   "balance": ("rows redistributed in proportion to each GPU's measured speed (warm-up); "
                               "the global batch is unchanged") if rows_per_rank else None,
                   "parallelism": (f"rows sharded, grad_W reduce-scatter "
                                   f"({'fused into the wgrad GEMM' if args.reduce == 'fused' else 'NCCL'})"
                                   if world > 1 else "single GPU"),
                   "l2": "inputs larger than L2 (W 1 GiB, teacher logits 2 GiB per GPU); no flush"},
        "step_tflops_per_gpu": step_tflops, "step_frac_of_peak": step_tflops / peak,
        "phases_ms_per_step": {k: v_[0] / args.steps for k, v_ in phases.items()},
        "host_enqueue_ms_per_step": host_ms, "collective_ms_per_step": collective_ms,
        "per_rank_ms": ({"fields": (["device_entry", "barrier_wait", "slot_reduce_quant"] if fused
                                    else ["device_entry"]) + ([] if args.no_clocks else ["sm_mhz", "power_w_max"]),
                         "ranks": rank_split} if rank_split else None),
        "roofline": roofline, "gpu_launches": int(launches), "clocks": clocks,
    }

    # ---------------- e2e through the host-Mat C ABI (HOST buffers)
    if not args.no_e2e:
        line["e2e"] = e2e_measure(args, ob, hs_all[:bt], w, tl_all[:bt], labels_all[:bt], opts, rank, world, dist)
    else:
        line["e2e"] = None

    # ---------------- CPU baseline (rank 0, N=1 only)
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        val, desc, _ = cpu_baseline_line(1, (1, args.cpu_rows))
        line["cpu_baseline"] = {"value": val, "unit": "tokens/s", "cores": 1, "kind": "port", "sample": desc}
    else:
        line["cpu_baseline"] = None

    ctx.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)
    return 0


def e2e_measure(args, ob, hs, w, tl, labels, opts, rank, world, dist):
    """The reference-facing host entry (orda_distillation_loss) with pinned
    f32 host inputs; every step copies the inputs host->device and the
    gradients device->host inside the call."""
    import torch

    from orda_b200 import _abi

    lib = ob.load_library()
    hs_h = hs.float().cpu().pin_memory()
    w_h = w.float().cpu().pin_memory()
    tl_h = torch.empty(tl.shape, dtype=torch.float32, pin_memory=True)
    for r0 in range(0, tl.shape[0], 1024):
        tl_h[r0:r0 + 1024].copy_(tl[r0:r0 + 1024].float())
    lab_h = labels.cpu().contiguous()
    s, wm = ob.Mat.from_array(hs_h.numpy()), ob.Mat.from_array(w_h.numpy())
    t = ob.Teacher.Precomputed(ob.Mat.from_array(tl_h.numpy()))
    sc, wc, tc, oc = s._c(), wm._c(), t._c(), opts._c()
    lab_p = C.cast(lab_h.data_ptr(), C.POINTER(C.c_int64))
    buf = _abi.err_buf()

    def call():
        o = _abi.OrdaOutput()
        rc = lib.orda_distillation_loss(C.byref(sc), C.byref(wc), lab_p, lab_h.numel(), C.byref(tc), C.byref(oc),
                                        C.byref(o), buf, len(buf))
        if rc:
            raise ob.OrdaError(rc, buf.value.decode())
        loss = o.loss
        lib.orda_output_free(C.byref(o))
        return loss

    call()  # warm-up (allocates the staging buffers)
    if world > 1:
        dist.barrier()
    times = []
    for _ in range(args.e2e_steps):
        t0 = time.perf_counter()
        call()
        times.append(time.perf_counter() - t0)
    per = statistics.mean(times)
    if world > 1:
        tt = torch.tensor([per], device="cuda", dtype=torch.float64)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        per = float(tt.item())
    bt, h, v = hs.shape[0], CFG["h"], CFG["v"]
    h2d = bt * h * 4 + v * h * 4 + bt * v * 4 + bt * 8
    d2h = bt * h * 4 + v * h * 4 + 16
    return {"value": bt * world / per, "unit": "tokens/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
            "ms_per_step": per * 1e3, "api": "orda_distillation_loss (f32 host Mats, pinned inputs)",
            "scope": "per-rank local shard" if world > 1 else "full"}


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--e2e-steps", type=int, default=2)
    ap.add_argument("--rows", type=int, default=CFG["bt"],
                    help="rows per GPU (default 8192, the metric's config; smaller values are for profiling only)")
    ap.add_argument("--cpu-rows", type=int, default=3)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-clocks", action="store_true")
    ap.add_argument("--config", choices=["c4", "c5"], default="c4",
                    help="c4: the metric configuration (default); c5: the large-vocabulary Tied configuration")
    ap.add_argument("--shard", choices=["rows", "vocab"], default="rows", help="c5 with N > 1: partitioning")
    ap.add_argument("--balance", action="store_true",
                    help="N > 1: redistribute rows to each GPU's speed measured in warm-up (off by default: "
                         "warm-up clocks do not predict the power-capped steady state)")
    ap.add_argument("--reduce", choices=["fused", "nccl"], default="fused",
                    help="N > 1: grad_W reduce-scatter fused into the wgrad GEMM, or an NCCL reduce-scatter")
    args = ap.parse_args()
    if args.warmup < 3:
        print("note: at least 3 warm-up steps are required for a valid number; using 3", file=sys.stderr)
        args.warmup = 3
    if args.impl == "reference":
        return run_reference_arm(args)
    if args.config == "c5":
        return run_c5(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
