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
the GPUs' measured speed).

Besides the headline, the line carries:
  parity     checks of the timed path, outside the timed region. N=1: sampled
             grad_hidden rows against the reference CPU path (the same oracle
             calls the CPU baseline times), the full call against the sum of 8
             row-block calls, and the INT8 grad_W against the reference
             quantiser on the same fp32 grad_W. N>1: one small step through
             the same sharded path against the same problem on one GPU.
  c5_rows    BASELINE configs[4] (Tied, H=8192, V=152064, 8192 rows per GPU),
             rows sharded with the fused grad_W reduce-scatter at N>1;
  c5_vocab   the same configuration vocabulary-sharded (V/N rows of W per
             GPU, every GPU all 8192*N rows, grad_hidden reduce-scattered by
             the dgrad GEMMs); at N=1 the vocabulary phases on one GPU.
  c4_fast    N=1: the c4 workload under Profile::Fast, with its agreement
             with the Balanced call.
Each c5 object has its own timing, roofline and parity.
`--config c5` runs only c5 (`--shard rows|vocab`).
`--impl reference` times the reference's CPU path (the oracle restatement,
all host threads) on a bounded row sample of the same workload.
"""
from __future__ import annotations

import argparse
import ctypes as C
import datetime
import json
import os
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
C5 = dict(rows=8192, h=8192, v=152064, kd=0.4, temperature=1.5, w_std=0.02)
C5_WORKLOAD = "c5: Tied teacher, 8192 rows per GPU, H=8192, V=152064, kd=0.4, T=1.5"

# Tolerances of the parity checks (the GPU parity tests state the same ones).
TOL = dict(
    rows_rel_l2=1e-2,       # grad rows vs the reference CPU path: bf16 logit gradients feed the GEMMs
    blocks_rel=1e-5,        # full call vs the sum of row-block calls: fp32 sums in another order
    shard_rel=1e-5,         # sharded path vs one GPU: fp32 sums in another order
    int8_code_diff=1,       # sharded INT8 codes: a scale from a row that differs in the last bits
    int8_identical=0.999,   # can move a value across a rounding boundary
)


def ksum_tol(k_terms):
    """Tolerance (rel-L2) between two fp32 evaluations of a GEMM output whose
    K sums (k_terms products per element) are associated differently: grad_W
    summed over row blocks or ranks (K = rows, x2 for a Tied teacher's second
    K segment), grad_hidden summed over vocabulary shards (K = V). With
    rounding of random sign the difference grows like sqrt(K) * 2^-24 relative
    to the result (six times that is allowed); the tensor-core accumulator
    rounds once per 16-product MMA step, and where that rounding leans one way
    the difference grows like (K / 16) * 2^-24 instead. The tolerance is the
    larger of the two, and never below the 1e-5 of the other quantities:
    6.1e-5 at K = 16384, 5.7e-4 at K = 152064."""
    return max(TOL["shard_rel"], 6.0 * (k_terms ** 0.5) * 2.0 ** -24, k_terms / 16.0 * 2.0 ** -24)


def algorithmic_flops(bt, h, v):
    """2*BT*V*(3*H_s) for the Precomputed teacher: logits, dgrad, wgrad."""
    return 2.0 * bt * v * 3 * h


def c5_flops(rows, h, v):
    """Tied teacher with teacher CE weight 1: 2*rows*V*(3H + H + 2H)."""
    return 12.0 * rows * v * h


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


class RowBalancer:
    """Feedback load balancing of the global batch (per_rank x world rows)
    across ranks whose GPUs run at different speeds: power-capped B200s of one
    node settle at different SM clocks, and with equal row blocks every step
    waits for the slowest. After each step a rank records the device time of
    its device entry (CUDA events); `lag` steps later (so reading the events
    waits for nothing the host still needs to enqueue) the ranks exchange
    rows / ms over a CPU (gloo) group, smooth it, and give the next step
    rows in proportion, in whole `quantum`s (the GEMM's M tile, so no rank
    computes a partly empty tile) within [lo, hi]. Every rank computes the
    same allocation from the same gathered numbers. The global row count is
    unchanged; n_global comes from prefix counts exchanged once."""

    def __init__(self, dist, group, world, rank, per_rank, quantum, lo, hi, smoothing=0.5, lag=2):
        self.dist, self.group, self.world, self.rank = dist, group, world, rank
        self.total = per_rank * world
        self.quantum, self.lo, self.hi = quantum, lo, hi
        self.smoothing, self.lag = smoothing, lag
        self.rows = [per_rank] * world
        self.speed = None
        self.pending = []
        self.history = []

    def mine(self):
        return self.rows[self.rank]

    def record(self, ev_start, ev_end, rows):
        self.pending.append((ev_start, ev_end, rows))
        if len(self.pending) > self.lag:
            a, b, n = self.pending.pop(0)
            b.synchronize()
            mine = n / max(a.elapsed_time(b), 1e-3)
            speeds = [None] * self.world
            self.dist.all_gather_object(speeds, mine, group=self.group)
            if self.speed is None:
                self.speed = speeds
            else:
                k = self.smoothing
                self.speed = [k * x + (1 - k) * y for x, y in zip(speeds, self.speed)]
            self.rows = balanced_rows(self.total, self.speed, self.quantum, self.lo, self.hi)
            self.history.append(list(self.rows))


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


def start_clocks(torch, dev, local):
    uuid = getattr(torch.cuda.get_device_properties(dev), "uuid", None)
    s = ClockSampler(f"GPU-{uuid}" if uuid is not None else str(local))
    s.start()
    time.sleep(0.3)
    return s


# ------------------------------------------------------- synthetic workloads
# Seeded generators shared with the full-size GPU parity tests. Every rank
# can regenerate any rank's inputs from the seeds alone.

def c4_weight(torch, dev):
    g = torch.Generator(device=dev).manual_seed(7)
    return (CFG["w_std"] * torch.randn(CFG["v"], CFG["h"], generator=g, device=dev)).bfloat16()


def c4_rows(torch, rows, dev, seed):
    """Student hidden [rows, H] bf16, teacher logits [rows, V] bf16 (std
    sqrt 2), labels uniform in [0, V)."""
    g = torch.Generator(device=dev).manual_seed(seed)
    h, v = CFG["h"], CFG["v"]
    hs = torch.randn(rows, h, generator=g, device=dev).bfloat16()
    tl = torch.empty(rows, v, device=dev, dtype=torch.bfloat16)
    for r0 in range(0, rows, 1024):  # slabs bound the fp32 temporary
        tl[r0:r0 + 1024] = CFG["teacher_std"] * torch.randn(min(1024, rows - r0), v, generator=g, device=dev)
    labels = torch.randint(0, v, (rows,), generator=g, device=dev)
    return hs, tl, labels


def c4_opts(ob, quantize=True):
    return ob.LossOptions(kd_weight=CFG["kd"], temperature=CFG["temperature"],
                          config=ob.KernelConfig(quantize_grad_weight=quantize))


def c5_weight_slice(torch, v0, v1, dev):
    """Rows [v0, v1) of the c5 W (each slice has its own seed, so the full W
    is the concatenation of the slices of any partition that was generated)."""
    g = torch.Generator(device=dev).manual_seed(7 + v0)
    return (C5["w_std"] * torch.randn(v1 - v0, C5["h"], generator=g, device=dev)).bfloat16()


def c5_rows(torch, rows, dev, seed):
    """Student hidden [rows, H] bf16, teacher hidden = student + N(0, 0.1),
    labels uniform."""
    g = torch.Generator(device=dev).manual_seed(seed)
    hs = torch.randn(rows, C5["h"], generator=g, device=dev).bfloat16()
    ht = (hs.float() + 0.1 * torch.randn(rows, C5["h"], generator=g, device=dev)).bfloat16()
    labels = torch.randint(0, C5["v"], (rows,), generator=g, device=dev)
    return hs, ht, labels


def c5_opts(ob):
    return ob.LossOptions(kd_weight=C5["kd"], temperature=C5["temperature"])


# ------------------------------------------------------------ parity checks

def rel_l2_dev(torch, a, b, slab=1 << 24):
    """||a - b|| / ||b|| of two device tensors of the same shape, accumulated
    in f64 over slabs (bounded temporaries)."""
    a = a.reshape(-1)
    b = b.reshape(-1)
    num = den = 0.0
    for i in range(0, b.numel(), slab):
        x = a[i:i + slab].double()
        y = b[i:i + slab].double()
        num += float(((x - y) ** 2).sum())
        den += float((y ** 2).sum())
    return (num ** 0.5) / (den ** 0.5 if den > 0 else 1.0)


def scalars_rel(a, b, atol=1e-7):
    """Largest |a_i - b_i| / (|b_i| + atol) over the four scalars."""
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return float(np.max(np.abs(a - b) / (np.abs(b) + atol)))


def check_row_blocks(torch, call, bt, n_global, v, blocks=8, k_segments=1):
    """The full call against the sum of `blocks` row-block calls.

    call(r0, r1, n) runs the device entry on rows [r0, r1) with mean
    denominator n (0: the call's own count) and skip_quantize, returning
    (scalars, grad_student_hidden, grad_weight, grad_teacher_hidden or None)
    as device tensors. The per-row terms, grad_hidden rows and the grad_W
    partials of the blocks must add up to the full call (src/api.rs:188-422
    is a sum over rows with one global mean); the partials are summed in f64
    so that only the GEMMs' own fp32 order differs (ksum_tol of the
    bt * k_segments summed products). grad_hidden rows are sums over the
    vocabulary (K = v) that the dgrad GEMM may split into two K halves in
    one call (the tiles of a partial last wave) and not in the other, so
    they get ksum_tol(v)."""
    sc_f, gh_f, gw_f, gth_f = [None if t is None else t.clone() for t in call(0, bt, n_global)]
    sc_sum = np.zeros(4)
    gw_sum = torch.zeros(gw_f.shape, device=gw_f.device, dtype=torch.float64)
    gh_b = torch.empty_like(gh_f)
    gth_b = None if gth_f is None else torch.empty_like(gth_f)
    step = -(-bt // blocks)
    for r0 in range(0, bt, step):
        r1 = min(bt, r0 + step)
        sc, gh, gw, gth = call(r0, r1, n_global)
        sc_sum += sc.double().cpu().numpy()
        gw_sum += gw
        gh_b[r0:r1] = gh
        if gth_b is not None:
            gth_b[r0:r1] = gth
    torch.cuda.synchronize()
    tol_w = ksum_tol(bt * k_segments)
    tol_h = ksum_tol(v)
    res = {"blocks": blocks, "scalars_rel": scalars_rel(sc_sum, sc_f.double().cpu().numpy()),
           "grad_weight_rel_l2": rel_l2_dev(torch, gw_sum, gw_f),
           "grad_hidden_rel_l2": rel_l2_dev(torch, gh_b, gh_f), "tol": TOL["blocks_rel"], "tol_grad_weight": tol_w,
           "tol_grad_hidden": tol_h}
    del gw_sum
    ok_h = res["grad_hidden_rel_l2"] <= tol_h
    if gth_b is not None:
        res["grad_teacher_hidden_rel_l2"] = rel_l2_dev(torch, gth_b, gth_f)
        ok_h = ok_h and res["grad_teacher_hidden_rel_l2"] <= tol_h
    res["pass"] = res["scalars_rel"] <= TOL["blocks_rel"] and res["grad_weight_rel_l2"] <= tol_w and ok_h
    return res, gw_f


def check_rows_vs_oracle(ref_out, gpu_rows, labels_rows, n_full, ignore_index=-100):
    """Sampled gradient rows of a full GPU call against the reference CPU
    path run on those rows alone (TEST / CPU-BASELINE CHECKER: `ref_out` is
    the oracle's output). Under the mean reduction a row's gradient is
    G_row / n, with n the non-ignored count of the call, so the GPU rows
    (n = n_full) are compared as G_row = grad * n with the oracle's
    (n = the sample's count). gpu_rows: {name: host array of the rows}."""
    n_sub = int(sum(1 for y in labels_rows if y != ignore_index))
    res = {"rows_checked": len(labels_rows), "tol": TOL["rows_rel_l2"]}
    ok = True
    for name, arr in gpu_rows.items():
        ref = getattr(ref_out, name)
        a = np.asarray(arr, dtype=np.float64) * n_full
        b = ref.a.astype(np.float64) * max(n_sub, 1)
        e = float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))
        res[f"{name}_rel_l2"] = e
        res[f"{name}_max_abs"] = float(np.max(np.abs(a - b)) / n_full)
        ok = ok and e <= TOL["rows_rel_l2"]
    res["pass"] = ok
    return res


def check_int8_vs_oracle(gw_raw, labels, q, scale, deq, nthreads, ignore_index=-100):
    """The GPU's INT8 grad_W (codes, scales, dequantised matrix) against the
    reference quantiser (src/quant.rs:157-202, oracle restatement) applied to
    the GPU's own fp32 grad_W (TEST / CPU-BASELINE CHECKER). Host arrays."""
    import oracle

    q_ref, s_ref, deq_ref = oracle.quantize_grad_w(gw_raw, labels, ignore_index, nthreads=nthreads)
    res = {"rows": int(gw_raw.shape[0]), "codes_identical": bool(np.array_equal(q, q_ref)),
           "scales_identical": bool(np.array_equal(scale.view(np.uint32), s_ref.view(np.uint32))),
           "dequantised_identical": bool(np.array_equal(deq.view(np.uint32), deq_ref.view(np.uint32)))}
    res["pass"] = res["codes_identical"] and res["scales_identical"] and res["dequantised_identical"]
    return res


def sample_rows(bt, k=32):
    """k rows spread over [0, bt), the last row included."""
    return sorted({int(round(i * (bt - 1) / (k - 1))) for i in range(k)})


# ------------------------------------------------------------- CPU baselines

def cpu_reference_sample(rows, nthreads, seed=77, inputs=None):
    """Times the reference CPU path (oracle restatement of src/api.rs) on
    `rows` rows of the workload (full H and V, Precomputed teacher, INT8
    round trip). inputs: (hidden rows, W, teacher logits rows, labels) as
    host f32 arrays (default: fresh seeded ones). Returns (seconds, output)."""
    import torch

    import oracle
    import orda_b200 as ob

    if inputs is None:
        gen = torch.Generator().manual_seed(seed)
        h, v = CFG["h"], CFG["v"]
        hs = torch.randn(rows, h, generator=gen).bfloat16().float().numpy()
        w = (CFG["w_std"] * torch.randn(v, h, generator=gen)).bfloat16().float().numpy()
        tl = (CFG["teacher_std"] * torch.randn(rows, v, generator=gen)).bfloat16().float().numpy()
        labels = torch.randint(0, v, (rows,), generator=gen).tolist()
    else:
        hs, w, tl, labels = inputs
    s, wm, t = ob.Mat.from_array(hs), ob.Mat.from_array(w), ob.Teacher.Precomputed(ob.Mat.from_array(tl))
    t0 = time.perf_counter()
    out = oracle.distillation_loss(s, wm, list(labels), t, c4_opts(ob), nthreads=nthreads)
    dt = time.perf_counter() - t0
    assert np.isfinite(out.loss)
    return dt, out


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


def run_reference_arm(args):
    """--impl reference: the reference's CPU path with all host threads."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    cores = host_cores()
    # Two sample sizes: 1 row (mostly the per-call O(V*H) passes) and the
    # smallest power of two whose call takes about twice as long, so the
    # per-row GEMM term is resolved by the fit.
    t1, _ = cpu_reference_sample(1, cores)
    rows = 2
    t, _ = cpu_reference_sample(rows, cores)
    while t < 2.0 * t1 and t < 30.0 and rows < 512:
        rows *= 2
        t, _ = cpu_reference_sample(rows, cores)
    for _ in range(max(0, args.warmup - 2)):
        cpu_reference_sample(rows, cores)
    samples = []
    for i in range(max(2, args.steps)):
        r = 1 if i % 2 == 0 else rows
        samples.append((r, cpu_reference_sample(r, cores, seed=100 + i)[0]))
    value, a, b, total = extrapolate(samples)
    per = statistics.mean(t for _, t in samples)
    sample = (f"per step one reference call on 1 or {rows} of 8192 rows (alternating), full H=4096 and "
              f"V=131072, Precomputed teacher, INT8 round trip; fit t = {a:.4f} s/row + {b:.2f} s/call, "
              f"extrapolated to the reference's 16 x 512-row plan ({total / 3600:.2f} h for 8192 rows)")
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": per * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32 (CPU reference path: f32 GEMMs, f64 softmax)",
        "data": "synthetic", "config": {"workload": WORKLOAD, "sample_rows_per_step": [1, rows]},
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": cores, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ------------------------------------------------------------ distributed

class Dist:
    """World, rank and the process group (NCCL) of one bench process."""

    def __init__(self, torch):
        import torch.distributed as dist

        self.dist = dist
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        torch.cuda.set_device(self.local)
        self.dev = torch.device("cuda", self.local)
        if self.world > 1:
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=self.dev)

    def barrier(self):
        if self.world > 1:
            self.dist.barrier()

    def max(self, torch, x):
        if self.world == 1:
            return x
        t = torch.tensor([x], device=self.dev, dtype=torch.float64)
        self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return float(t.item())

    def sum(self, torch, xs):
        t = torch.tensor(xs, device=self.dev, dtype=torch.float64)
        if self.world > 1:
            self.dist.all_reduce(t)
        return t.tolist()

    def close(self):
        if self.world > 1:
            self.dist.barrier()
            self.dist.destroy_process_group()


def timed(torch, D, stream, step, steps, ctx=None, clocks=True):
    """Runs `steps` steps bracketed by a barrier and a device synchronize on
    both sides; returns (ms per step as the max over ranks, phase times of
    ctx, clocks, kernel launches of ctx, host enqueue ms per step)."""
    sampler = start_clocks(torch, D.dev, D.local) if clocks else None
    if ctx is not None:
        ctx.reset_timing()
        ctx.enable_timing(True)
        launches0 = ctx.launch_count()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    D.barrier()
    torch.cuda.synchronize()
    ev0.record(stream)
    h0 = time.perf_counter()
    for _ in range(steps):
        step()
    host_ms = (time.perf_counter() - h0) * 1e3 / steps
    ev1.record(stream)
    torch.cuda.synchronize()
    D.barrier()
    ms = D.max(torch, ev0.elapsed_time(ev1)) / steps
    phases = launches = None
    if ctx is not None:
        phases = ctx.phase_times()
        ctx.enable_timing(False)
        launches = ctx.launch_count() - launches0
    cl = sampler.stop() if sampler else None
    return ms, phases, cl, launches, host_ms


def gemm_roofline(phases, steps, flops, kernel):
    peak, peak_sus, _hbm, kind = load_peaks()
    gemm_ms = sum(phases[p][0] for p in ("logits_gemm", "dgrad_gemm", "wgrad_gemm")) / steps
    achieved = flops / (gemm_ms / 1e3) / 1e12
    return {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s", "frac": achieved / peak,
            "kernel": kernel, "gemm_ms_per_step": gemm_ms,
            "launches_per_step": sum(phases[p][1] for p in ("logits_gemm", "dgrad_gemm", "wgrad_gemm")) / steps,
            "peak_kind": f"{kind} burst bf16 (MEASURED_PEAKS.json bf16_tflops)",
            "frac_of_sustained": achieved / peak_sus if peak_sus else None}


# ----------------------------------------------------------------- c4 arm

# DRAM bytes (read + write) per c4 step of the three GEMM launches, from a
# one-pass ncu capture of exactly those launches at full size
# (profiles/gemm_traffic_c4.md, which gives the command and the spread
# between boxes).
GEMM_TRAFFIC_C4 = 32474239488


def run_ours(args):
    import torch

    import orda_b200 as ob
    from orda_b200 import shard
    from orda_b200.device import DeviceContext, distillation_loss_device, quantize_grad_w

    D = Dist(torch)
    world, rank, dev = D.world, D.rank, D.dev
    if world != args.gpus:
        print(f"warning: --gpus {args.gpus} but WORLD_SIZE {world}", file=sys.stderr)
    bt, h, v = args.rows, CFG["h"], CFG["v"]
    # N > 1 with balancing: room for up to 25 % more rows on a faster GPU
    balance = args.balance if world > 1 else "off"
    cap = bt + (bt // 4 if balance != "off" else 0)
    hs_all, tl_all, labels_all = c4_rows(torch, cap, dev, 1000 + rank)
    w = c4_weight(torch, dev)
    gsh_all = torch.empty(cap, h, device=dev)
    opts = c4_opts(ob)
    out = {"grad_weight": torch.empty(v, h, device=dev), "scalars": torch.empty(4, device=dev)}
    hs = tl = labels = None

    def use_rows(n):
        """This rank's rows: the first n of the generated inputs."""
        nonlocal hs, tl, labels
        hs, tl, labels = hs_all[:n], tl_all[:n], labels_all[:n]
        out["grad_student_hidden"] = gsh_all[:n]

    use_rows(bt)
    rows_per_rank = None
    vs0, vs1 = shard.vocab_slice(v, world, rank) if world > 1 else (0, v)
    q = torch.empty(vs1 - vs0, h, device=dev, dtype=torch.int8)
    qs = torch.empty(vs1 - vs0, device=dev)
    stream = torch.cuda.current_stream(dev)
    ctx = DeviceContext(D.local)
    n_global = bt * world if world == 1 else shard.global_non_ignore(labels, -100)

    # N > 1: the grad_W reduce-scatter is fused into the wgrad GEMM (peer
    # stores into the owners' slot buffers) unless --reduce nccl
    fused = (shard.SlotReduceScatter(ctx, v, h, label_capacity=cap)
             if world > 1 and args.reduce == "fused" else None)
    gw_slice = torch.empty(vs1 - vs0, h, device=dev) if fused else None
    if fused:
        del out["grad_weight"]  # the local full grad_W is never materialised
    marks = []  # (after compute, end of step) events of the timed steps

    balancer = None
    if balance == "dynamic":
        quantum = 256
        gl = D.dist.new_group(backend="gloo")
        balancer = RowBalancer(D.dist, gl, world, rank, bt, quantum, bt - bt // 4, cap)
        # non-ignored labels among this rank's first k * quantum rows, for every k
        valid = (labels_all != -100).to(torch.int64).cumsum(0)
        mine = [0] + [int(x) for x in valid[quantum - 1::quantum].tolist()]
        prefix = [None] * world
        D.dist.all_gather_object(prefix, mine, group=gl)

    def step():
        nonlocal n_global
        if balancer is not None:
            rows_now = balancer.rows
            use_rows(rows_now[rank])
            n_global = sum(prefix[r][rows_now[r] // quantum] for r in range(world))
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
        if balancer is not None:
            balancer.record(ev[4], ev[0], hs.shape[0])
        return res

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    ctx.check()
    if balance == "once":
        # Power-capped GPUs of one node settle at different clocks, so equal
        # row blocks finish at different times and every step waits for the
        # slowest rank. Redistribute the global batch (8192 x N rows, as
        # before) in proportion to each rank's rows per ms of device time in
        # the warm-up steps after the first, then warm up again.
        t_mine = statistics.mean(ev[4].elapsed_time(ev[0]) for ev in marks[1:])
        tt = torch.tensor([t_mine], device=dev, dtype=torch.float64)
        all_t = [torch.empty_like(tt) for _ in range(world)]
        D.dist.all_gather(all_t, tt)
        speeds = [bt / float(x) for x in all_t]
        rows_per_rank = balanced_rows(bt * world, speeds, 16, bt - bt // 4, cap)
        use_rows(rows_per_rank[rank])
        n_global = shard.global_non_ignore(labels, -100)
        for _ in range(args.warmup):
            step()
        torch.cuda.synchronize()
        ctx.check()

    # ---------------- timed region
    marks.clear()
    ms_step, phases, clocks, launches, host_ms = timed(torch, D, stream, step, args.steps, ctx,
                                                        clocks=not args.no_clocks)
    ctx.check()
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
        mine += [float((clocks or {}).get("sm_mhz") or 0.0), float((clocks or {}).get("power_w_max") or 0.0)]
        t = torch.tensor(mine, device=dev, dtype=torch.float64)
        allt = [torch.empty_like(t) for _ in range(world)]
        D.dist.all_gather(allt, t)
        rank_split = [[round(x, 3) for x in a.tolist()] for a in allt]
    tokens = bt * world
    value = tokens / (ms_step / 1e3)
    flops = algorithmic_flops(bt, h, v)
    peak = load_peaks()[0]
    roofline = gemm_roofline(phases, args.steps, flops, "gemm_kernel (tcgen05 cta_group::2, 3 layouts)")
    roofline["traffic"] = GEMM_TRAFFIC_C4 if bt == CFG["bt"] else None
    roofline["traffic_scope"] = ("DRAM bytes (read + write) per step of the 3 GEMM launches, one-pass ncu "
                                 "capture of those launches at full size (profiles/gemm_traffic_c4.md; "
                                 "algorithmic 13.2 GB)")
    step_tflops = flops / (ms_step / 1e3) / 1e12

    line = {
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": WORKLOAD if bt == CFG["bt"] else f"{WORKLOAD} [profiling size: {bt} rows]",
                   "global_batch": tokens, "seq_len": None, "rows_per_gpu": bt,
                   "rows_per_rank": rows_per_rank,
                   "balance": ("rows redistributed in proportion to each GPU's measured speed (warm-up); "
                               "the global batch is unchanged") if rows_per_rank else
                              ("rows redistributed every step in proportion to each GPU's smoothed speed "
                               "(256-row quanta, 0.75x-1.25x); the global batch is unchanged; allocations of the "
                               "timed steps in `rows_per_step`") if balancer is not None else None,
                   "parallelism": (f"rows sharded, grad_W reduce-scatter "
                                   f"({'fused into the wgrad GEMM' if args.reduce == 'fused' else 'NCCL'})"
                                   if world > 1 else "single GPU"),
                   "l2": "inputs larger than L2 (W 1 GiB, teacher logits 2 GiB per GPU); no flush"},
        "step_tflops_per_gpu": step_tflops, "step_frac_of_peak": step_tflops / peak,
        "phases_ms_per_step": {k: v_[0] / args.steps for k, v_ in phases.items()},
        "host_enqueue_ms_per_step": host_ms, "collective_ms_per_step": collective_ms,
        "per_rank_ms": ({"fields": (["device_entry", "barrier_wait", "slot_reduce_quant"] if fused
                                    else ["device_entry"]) + ["sm_mhz", "power_w_max"],
                         "ranks": rank_split} if rank_split else None),
        "roofline": roofline, "gpu_launches": int(launches), "clocks": clocks,
    }
    if balancer is not None:
        line["config"]["rows_per_step"] = balancer.history[-args.steps:]

    # ---------------- parity of the timed path (outside the timed region)
    parity = {}
    if not args.no_parity:
        if world == 1:
            parity["row_blocks"] = c4_row_blocks(torch, ob, ctx, hs, w, tl, labels, opts, dev, stream, parity)
        else:
            parity["sharded_vs_one_gpu"] = verify_c4_sharded(torch, ob, shard, D, ctx, fused, w, q, qs, args)
    raw_gw = parity.pop("_raw_grad_weight", None)

    # ---------------- e2e: inputs from pinned host memory, results back to host
    if not args.no_e2e:
        line["e2e"] = (e2e_host_entry(args, ob, hs_all[:bt], w, tl_all[:bt], labels_all[:bt], opts, D)
                       if world == 1 else
                       e2e_sharded(torch, ob, shard, D, ctx, fused, hs_all[:bt], w, tl_all[:bt], labels_all[:bt],
                                   opts, args))
    else:
        line["e2e"] = None

    # ---------------- CPU baseline (rank 0, N=1 only); its oracle calls run on
    # rows of this workload and double as the row check of the parity object
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        val, desc, checks = cpu_baseline_leg(torch, ob, args, hs, w, tl, labels, out, q, qs, raw_gw)
        line["cpu_baseline"] = {"value": val, "unit": "tokens/s", "cores": 1, "kind": "port", "sample": desc}
        parity.update(checks)
    else:
        line["cpu_baseline"] = None
    # ---------------- Profile::Fast on the same workload (N=1)
    if world == 1 and not args.no_fast:
        line["c4_fast"] = run_c4_fast(torch, ob, D, ctx, hs, w, tl, labels, out, stream, args, raw_gw)
    del raw_gw
    if parity:
        parity["pass"] = all(p.get("pass", True) for p in parity.values() if isinstance(p, dict))
    line["parity"] = parity or None

    # ---------------- c5 at this N, both partitionings
    ctx.close()
    del hs_all, tl_all, labels_all, gsh_all, out, q, qs, w
    hs = tl = labels = gw_slice = None
    torch.cuda.empty_cache()
    if not args.no_c5:
        line["c5_rows"] = run_c5_part(torch, ob, shard, D, args, "rows")
        torch.cuda.empty_cache()
        line["c5_vocab"] = run_c5_part(torch, ob, shard, D, args, "vocab")
    D.close()
    if rank == 0:
        print(json.dumps(line), flush=True)
    return 0


def run_c4_fast(torch, ob, D, ctx, hs, w, tl, labels, ref_out, stream, args, raw_gw):
    """Profile::Fast (fp16 logits storage, exact label logits, a quarter of
    the logits epilogue's tempered exp2 on the FMA pipe) on the c4 workload: timing and roofline as the
    headline, and its agreement with the Balanced call of the timed steps
    (scalars, grad_hidden; grad_W before the INT8 round trip). The Fast
    tolerances against the reference are stated in include/orda.h."""
    from orda_b200.device import distillation_loss_device

    h, v = CFG["h"], CFG["v"]
    dev = hs.device
    opts = ob.LossOptions(kd_weight=CFG["kd"], temperature=CFG["temperature"],
                          config=ob.KernelConfig(quantize_grad_weight=True, fast_math=True))
    out_f = {"grad_weight": torch.empty(v, h, device=dev), "grad_student_hidden": torch.empty(hs.shape[0], h, device=dev),
             "scalars": torch.empty(4, device=dev), "grad_weight_q": torch.empty(v, h, device=dev, dtype=torch.int8),
             "grad_weight_scale": torch.empty(v, device=dev)}

    def step():
        return distillation_loss_device(ctx, hs, w, labels, ob.TeacherMode.Precomputed, teacher_logits=tl, opts=opts,
                                        out=out_f, want_int8=True, stream=stream)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    ctx.check()
    ms, phases, clocks, launches, _ = timed(torch, D, stream, step, args.steps, ctx, clocks=not args.no_clocks)
    ctx.check()
    flops = algorithmic_flops(hs.shape[0], h, v)
    res = {"profile": "Fast (KernelConfig.fast_math)", "value": hs.shape[0] / (ms / 1e3), "unit": "tokens/s",
           "ms_per_step": ms, "steps": args.steps,
           "phases_ms_per_step": {k: v_[0] / args.steps for k, v_ in phases.items()},
           "roofline": gemm_roofline(phases, args.steps, flops, "gemm_kernel (tcgen05 cta_group::2, fp16 logits)"),
           "gpu_launches": int(launches), "clocks": clocks}
    if raw_gw is not None:
        r = distillation_loss_device(ctx, hs, w, labels, ob.TeacherMode.Precomputed, teacher_logits=tl, opts=opts,
                                     skip_quantize=True, stream=stream)
        torch.cuda.synchronize()
        res["vs_balanced"] = {
            "scalars_rel": scalars_rel(out_f["scalars"].cpu().numpy(), ref_out["scalars"].cpu().numpy()),
            "grad_hidden_rel_l2": rel_l2_dev(torch, out_f["grad_student_hidden"], ref_out["grad_student_hidden"]),
            "grad_weight_rel_l2": rel_l2_dev(torch, r.grad_weight, raw_gw),
            "tol": {"scalars_rel": 1e-3, "grad_rel_l2": 2e-2}}
        vb = res["vs_balanced"]
        vb["pass"] = (vb["scalars_rel"] <= 1e-3 and vb["grad_hidden_rel_l2"] <= 2e-2
                      and vb["grad_weight_rel_l2"] <= 2e-2)
        del r
    del out_f
    torch.cuda.empty_cache()
    return res


def c4_row_blocks(torch, ob, ctx, hs, w, tl, labels, opts, dev, stream, keep):
    """Row-block check of the c4 path on one GPU; also keeps the full call's
    fp32 grad_W (before the INT8 round trip) for the INT8 check."""
    from orda_b200.device import distillation_loss_device

    bt = hs.shape[0]
    n_all = int((labels != -100).sum())

    def call(r0, r1, n):
        r = distillation_loss_device(ctx, hs[r0:r1], w, labels[r0:r1], ob.TeacherMode.Precomputed,
                                     teacher_logits=tl[r0:r1], opts=opts, global_non_ignore=n, skip_quantize=True,
                                     stream=stream)
        return r.scalars, r.grad_student_hidden, r.grad_weight, None

    res, gw_full = check_row_blocks(torch, call, bt, n_all, CFG["v"])
    ctx.check()
    keep["_raw_grad_weight"] = gw_full
    return res


def cpu_baseline_leg(torch, ob, args, hs, w, tl, labels, out, q, qs, raw_gw):
    """The reference CPU path (oracle restatement, 1 thread) timed on rows of
    the bench workload itself: one call on the last row and one on
    args.cpu_rows rows spread over the batch, fitted as t = a*rows + b and
    extrapolated to the reference's plan. The same oracle outputs check the
    GPU's grad_hidden rows of the timed call; the reference quantiser checks
    the GPU's INT8 grad_W on the GPU's own fp32 grad_W (all host threads)."""
    bt = hs.shape[0]
    w_h = w.float().cpu().numpy()
    picks = [[bt - 1], sample_rows(bt, args.cpu_rows)]
    samples, rows_checked, gh_ref, gh_gpu = [], [], [], []
    n_full = int((labels != -100).sum())
    gsh = out["grad_student_hidden"]
    lab_h = labels.cpu().numpy()
    for rows in picks:
        idx = torch.tensor(rows, device=hs.device)
        inp = (hs[idx].float().cpu().numpy(), w_h, tl[idx].float().cpu().numpy(), lab_h[rows].tolist())
        dt, ref = cpu_reference_sample(len(rows), 1, inputs=inp)
        samples.append((len(rows), dt))
        rows_checked += rows
        gh_ref.append(ref.grad_student_hidden.a * max(1, int(sum(1 for y in inp[3] if y != -100))))
        gh_gpu.append(gsh[idx].cpu().numpy().astype(np.float64) * n_full)
    value, a, b, total = extrapolate(samples)
    desc = (f"reference CPU path (oracle restatement), 1 thread: calls on rows {picks[0]} and {len(picks[1])} rows "
            f"spread over the batch of this workload (full H=4096, V=131072, Precomputed, INT8 round trip) timed "
            f"{', '.join(f'{t:.1f}s' for _, t in samples)}; fit t = {a:.3f} s/row + {b:.2f} s/call, extrapolated "
            f"to the 16 x 512-row plan ({total / 3600:.2f} h for 8192 rows)")
    ga, gb = np.concatenate(gh_gpu), np.concatenate(gh_ref)
    e = float(np.linalg.norm(ga - gb) / max(np.linalg.norm(gb), 1e-30))
    checks = {"rows_vs_reference_cpu": {"rows": rows_checked, "grad_student_hidden_rel_l2": e,
                                        "max_abs": float(np.max(np.abs(ga - gb)) / n_full),
                                        "tol": TOL["rows_rel_l2"], "pass": e <= TOL["rows_rel_l2"]}}
    if raw_gw is not None:
        checks["int8_vs_reference_quantiser"] = check_int8_vs_oracle(
            raw_gw.cpu().numpy(), lab_h, q.cpu().numpy(), qs.cpu().numpy(), out["grad_weight"].cpu().numpy(),
            host_cores())
    return value, desc, checks


def verify_c4_sharded(torch, ob, shard, D, ctx, fused, w, q, qs, args, rows=256):
    """One small step (rows per rank, c4's H and V) through the same sharded
    path as the timed steps, against the whole problem on one GPU (rank 0
    regenerates every rank's rows from their seeds, computes, and broadcasts
    the reference). Raw reduced grad_W slice and scalars within 1e-5; INT8
    codes within one step, >= 99.9 % identical."""
    from orda_b200.device import distillation_loss_device, quantize_grad_w

    world, rank, dev = D.world, D.rank, D.dev
    v, h = CFG["v"], CFG["h"]
    hs, tl, labels = c4_rows(torch, rows, dev, 5000 + rank)
    labels[::29] = -100
    n_global = shard.global_non_ignore(labels, -100)
    opts = c4_opts(ob)
    st = torch.cuda.current_stream(dev)
    sc_v = torch.empty(4, device=dev)
    gh = torch.empty(rows, h, device=dev)
    v0, v1 = shard.vocab_slice(v, world, rank)
    sl_raw = torch.empty(v1 - v0, h, device=dev)
    sl_q = torch.empty(v1 - v0, h, device=dev)
    if fused:
        def compute(n):
            r = distillation_loss_device(ctx, hs, w, labels, ob.TeacherMode.Precomputed, teacher_logits=tl,
                                         opts=opts, out={"grad_student_hidden": gh, "scalars": sc_v},
                                         global_non_ignore=n, scatter_grad_weight=True, stream=st)
            return r.scalars, r.grad_student_hidden

        fused.step(compute, labels, -100, n_global, sl_raw, stream=st)
        res = fused.step(compute, labels, -100, n_global, sl_q, quantize=True, q=q, scale=qs, stream=st)
    else:
        def compute(n):
            r = distillation_loss_device(ctx, hs, w, labels, ob.TeacherMode.Precomputed, teacher_logits=tl,
                                         opts=opts, out={"grad_student_hidden": gh, "scalars": sc_v},
                                         global_non_ignore=n, skip_quantize=True, stream=st)
            return r.scalars, r.grad_student_hidden, r.grad_weight

        raw = {}

        def quant(sl, shifted):
            raw["sl"] = sl.clone()
            quantize_grad_w(ctx, sl, shifted, -100, False, 0, q, qs, stream=st)

        res = shard.row_sharded_step(compute, labels, -100, n_global, quantize=quant)
        sl_raw.copy_(raw["sl"])
        sl_q.copy_(res.grad_weight_slice)
    torch.cuda.synchronize()
    ctx.check()
    # reference on one GPU (rank 0), broadcast to every rank
    gw_ref = torch.empty(v, h, device=dev)
    q_ref = torch.empty(v, h, device=dev, dtype=torch.int8)
    gh_ref = torch.empty(rows * world, h, device=dev)
    sc_ref = torch.empty(4, device=dev)
    if rank == 0:
        parts = [c4_rows(torch, rows, dev, 5000 + r) for r in range(world)]
        for p in parts:
            p[2][::29] = -100
        hs_a = torch.cat([p[0] for p in parts])
        tl_a = torch.cat([p[1] for p in parts])
        lab_a = torch.cat([p[2] for p in parts])
        r = distillation_loss_device(ctx, hs_a, w, lab_a, ob.TeacherMode.Precomputed, teacher_logits=tl_a,
                                     opts=opts, out={"grad_weight": gw_ref, "grad_student_hidden": gh_ref,
                                                     "scalars": sc_ref}, skip_quantize=True, stream=st)
        deq = gw_ref.clone()
        quantize_grad_w(ctx, deq, lab_a, -100, False, 0, q_ref, torch.empty(v, device=dev), stream=st)
        del deq, parts, hs_a, tl_a
        torch.cuda.synchronize()
        ctx.check()
    for t in (gw_ref, q_ref, gh_ref, sc_ref):
        D.dist.broadcast(t, src=0)
    ref_sl = gw_ref[v0:v1]
    dq = (q.int() - q_ref[v0:v1].int()).abs()
    stats = D.sum(torch, [
        float(((sl_raw.double() - ref_sl.double()) ** 2).sum()), float((ref_sl.double() ** 2).sum()),
        float(((gh.double() - gh_ref[rank * rows:(rank + 1) * rows].double()) ** 2).sum()),
        float((gh_ref[rank * rows:(rank + 1) * rows].double() ** 2).sum()),
        float((dq == 0).sum()), float(dq.numel()),
    ])
    worst = D.max(torch, float(dq.max()))
    sc_err = scalars_rel(res.scalars.cpu().numpy(), sc_ref.cpu().numpy())
    sc_err = D.max(torch, sc_err)
    tol_w = ksum_tol(rows * world)
    out = {"rows_per_rank": rows, "path": "fused wgrad scatter + slot reduce" if fused else "NCCL reduce-scatter",
           "scalars_rel": sc_err, "grad_weight_slice_rel_l2": (stats[0] ** 0.5) / (stats[1] ** 0.5),
           "grad_hidden_rel_l2": (stats[2] ** 0.5) / (stats[3] ** 0.5), "int8_max_code_diff": worst,
           "int8_identical_frac": stats[4] / stats[5], "tol": TOL["shard_rel"], "tol_grad_weight": tol_w}
    out["pass"] = (out["scalars_rel"] <= TOL["shard_rel"] and out["grad_weight_slice_rel_l2"] <= tol_w
                   and out["grad_hidden_rel_l2"] <= TOL["shard_rel"] and worst <= TOL["int8_code_diff"]
                   and out["int8_identical_frac"] >= TOL["int8_identical"])
    del gw_ref, q_ref
    torch.cuda.empty_cache()
    return out


# ---------------------------------------------------------------- e2e

def e2e_host_entry(args, ob, hs, w, tl, labels, opts, D):
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

    call()  # warm-up (allocates the staging and page-locked buffers)
    call()  # a fresh host touches its memory for the first time during the first calls
    times, moved = [], []
    up, down = C.c_uint64(0), C.c_uint64(0)
    for _ in range(args.e2e_steps):
        t0 = time.perf_counter()
        call()
        times.append(time.perf_counter() - t0)
        lib.orda_last_call_bytes(C.byref(up), C.byref(down))  # what the call actually copied
        moved.append((up.value, down.value))
    per = statistics.mean(times)
    bt, h, v = hs.shape[0], CFG["h"], CFG["v"]
    # bytes over PCIe, as the library counted them per call: h and W cross as
    # bf16 or (when the copy engine would otherwise idle) fp32, the teacher
    # logits as bf16 where they hold bf16 values, grad_W as INT8 codes + scales
    # + exact target rows with the INT8 round trip; mean over the timed calls
    h2d = int(round(statistics.mean(m[0] for m in moved)))
    d2h = int(round(statistics.mean(m[1] for m in moved)))
    compressed = bool(opts.config.quantize_grad_weight) and os.environ.get("ORDA_HOST_DEQUANT", "1")[:1] != "0"
    return {"value": bt / per, "unit": "tokens/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
            "ms_per_step": per * 1e3, "calls_ms": [round(t * 1e3, 2) for t in times],
            "api": "orda_distillation_loss (f32 host Mats, pinned inputs)", "scope": "full", "grad_weight_download": ("int8 codes + row scales + exact target rows, dequantised "
                                                      "on the host" if compressed else "fp32")}


def e2e_sharded(torch, ob, shard, D, ctx, fused, hs, w, tl, labels, opts, args):
    """N > 1: the sharded flow end to end. Every step each rank copies its
    f32 host inputs (its rows' hidden states and teacher logits, W, labels)
    from pinned memory to the device, runs the row-sharded step (device
    entry + fused grad_W reduce-scatter + INT8 round trip of its slice) and
    copies its results (grad_W slice, grad_hidden rows, scalars) back to
    pinned host memory. Wall time per step, max over ranks."""
    from orda_b200.device import distillation_loss_device, quantize_grad_w

    dev = D.dev
    bt, h, v = hs.shape[0], CFG["h"], CFG["v"]
    world = D.world
    hs_h = hs.float().cpu().pin_memory()
    w_h = w.float().cpu().pin_memory()
    tl_h = torch.empty(tl.shape, dtype=torch.float32, pin_memory=True)
    for r0 in range(0, bt, 1024):
        tl_h[r0:r0 + 1024].copy_(tl[r0:r0 + 1024].float())
    lab_h = labels.cpu().pin_memory()
    v0, v1 = shard.vocab_slice(v, world, D.rank)
    gw_h = torch.empty(v1 - v0, h, pin_memory=True)
    gh_h = torch.empty(bt, h, pin_memory=True)
    sc_h = torch.empty(4, pin_memory=True)
    st = torch.cuda.current_stream(dev)
    hs_f = torch.empty(bt, h, device=dev)
    w_f = torch.empty(v, h, device=dev)
    tl_d = torch.empty(bt, v, device=dev)
    lab_d = torch.empty(bt, dtype=torch.int64, device=dev)
    gh = torch.empty(bt, h, device=dev)
    sc = torch.empty(4, device=dev)
    sl = torch.empty(v1 - v0, h, device=dev)
    q = torch.empty(v1 - v0, h, device=dev, dtype=torch.int8)
    qs = torch.empty(v1 - v0, device=dev)
    n_global = shard.global_non_ignore(labels, -100)

    def one():
        hs_f.copy_(hs_h, non_blocking=True)
        w_f.copy_(w_h, non_blocking=True)
        tl_d.copy_(tl_h, non_blocking=True)
        lab_d.copy_(lab_h, non_blocking=True)
        hs_b, w_b = hs_f.bfloat16(), w_f.bfloat16()  # the tensor-core operand type
        if fused:
            def compute(n):
                r = distillation_loss_device(ctx, hs_b, w_b, lab_d, ob.TeacherMode.Precomputed, teacher_logits=tl_d,
                                             opts=opts, out={"grad_student_hidden": gh, "scalars": sc},
                                             global_non_ignore=n, scatter_grad_weight=True, stream=st)
                return r.scalars, r.grad_student_hidden

            res = fused.step(compute, lab_d, -100, n_global, sl, quantize=True, q=q, scale=qs, stream=st)
        else:
            def compute(n):
                r = distillation_loss_device(ctx, hs_b, w_b, lab_d, ob.TeacherMode.Precomputed, teacher_logits=tl_d,
                                             opts=opts, out={"grad_student_hidden": gh, "scalars": sc},
                                             global_non_ignore=n, skip_quantize=True, stream=st)
                return r.scalars, r.grad_student_hidden, r.grad_weight

            def quant(s_, shifted):
                quantize_grad_w(ctx, s_, shifted, -100, False, 0, q, qs, stream=st)

            res = shard.row_sharded_step(compute, lab_d, -100, n_global, quantize=quant)
        gw_h.copy_(res.grad_weight_slice, non_blocking=True)
        gh_h.copy_(gh, non_blocking=True)
        sc_h.copy_(res.scalars, non_blocking=True)
        torch.cuda.synchronize()
        return float(sc_h[0])

    one()
    D.barrier()
    times = []
    for _ in range(args.e2e_steps):
        t0 = time.perf_counter()
        one()
        times.append(time.perf_counter() - t0)
    per = D.max(torch, statistics.mean(times))
    ctx.check()
    h2d = bt * h * 4 + v * h * 4 + bt * v * 4 + bt * 8
    d2h = (v1 - v0) * h * 4 + bt * h * 4 + 16
    return {"value": bt * world / per, "unit": "tokens/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
            "ms_per_step": per * 1e3, "scope": "sharded (per rank: its rows, W and its grad_W slice)",
            "api": "orda_b200.shard.SlotReduceScatter + orda_distillation_loss_device (f32 pinned host inputs)"}


# ----------------------------------------------------- c5 (large vocabulary)

def run_c5_part(torch, ob, shard, D, args, part):
    """BASELINE configs[4] at this N. part "rows": each rank its own 8192
    rows (grad_W reduce-scatter fused into the wgrad GEMM at N>1); "vocab":
    every rank all 8192*N rows and V/N rows of W (one all-gather of per-row
    statistics, grad_hidden reduce-scattered by the dgrad GEMMs); at N=1 the
    two vocabulary phases run on one GPU. Returns the sub-object."""
    from orda_b200.device import DeviceContext, distillation_loss_device, vocab_backward_device, vocab_forward_device

    world, rank, dev = D.world, D.rank, D.dev
    h, v = C5["h"], C5["v"]
    vocab = part == "vocab"
    rows = C5["rows"] * (world if vocab else 1)
    hs, ht, labels = c5_rows(torch, rows, dev, 2000 + (0 if vocab else rank))
    v0, v1 = shard.vocab_slice_bounds(v, world, rank) if vocab else (0, v)
    w = c5_weight_slice(torch, v0, v1, dev)
    opts = c5_opts(ob)
    ctx = DeviceContext(D.local)
    stream = torch.cuda.current_stream(dev)
    out = {"grad_student_hidden": torch.empty(rows, h, device=dev),
           "grad_teacher_hidden": torch.empty(rows, h, device=dev), "scalars": torch.empty(4, device=dev)}
    fused = gw_slice = hslots = None
    if world > 1 and not vocab:
        fused = shard.SlotReduceScatter(ctx, v, h, int8_wire=args.int8_wire)
        gw_slice = torch.empty(fused.v1 - fused.v0, h, device=dev)
        n_global = shard.global_non_ignore(labels, -100)
    else:
        out["grad_weight"] = torch.empty(v1 - v0, h, device=dev)
    if vocab and world > 1:
        hslots = shard.HiddenSlots(ctx, rows, h, teacher=True)

    def step():
        if vocab and world > 1:
            return shard.vocab_sharded_step(ctx, hs, w, labels, ob.TeacherMode.Tied, v, v0, teacher_hidden=ht,
                                            opts=opts, out=out, stream=stream, hidden_slots=hslots)
        if vocab:
            part_ = vocab_forward_device(ctx, hs, w, labels, ob.TeacherMode.Tied, v, v0, teacher_hidden=ht,
                                         opts=opts, stream=stream)
            return vocab_backward_device(ctx, hs, w, labels, ob.TeacherMode.Tied, v, v0, part_.unsqueeze(0),
                                         include_rows=True, teacher_hidden=ht, opts=opts, out=out, stream=stream)
        if fused:
            def compute(n):
                r = distillation_loss_device(ctx, hs, w, labels, ob.TeacherMode.Tied, teacher_hidden=ht, opts=opts,
                                             out=out, global_non_ignore=n, scatter_grad_weight=True, stream=stream,
                                             int8_wire=args.int8_wire)
                return r.scalars, r.grad_student_hidden

            return fused.step(compute, labels, -100, n_global, gw_slice, stream=stream)
        return distillation_loss_device(ctx, hs, w, labels, ob.TeacherMode.Tied, teacher_hidden=ht, opts=opts,
                                        out=out, stream=stream)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    ctx.check()
    steps = args.c5_steps
    ms, phases, clocks, launches, _ = timed(torch, D, stream, step, steps, ctx, clocks=not args.no_clocks)
    ctx.check()
    flops = c5_flops(C5["rows"], h, v)  # per GPU: the same work in both partitionings
    res = {"metric": "distillation fwd+bwd tokens/sec, c5 (Tied, H=8192, V=152064)",
           "value": C5["rows"] * world / (ms / 1e3), "unit": "tokens/s", "ms_per_step": ms, "steps": steps,
           "workload": C5_WORKLOAD,
           "parallelism": ({"rows": "rows sharded, grad_W reduce-scatter fused into the wgrad GEMM",
                            "vocab": "vocabulary sharded (V/N rows of W per GPU, all rows on every GPU), "
                                     "per-row statistics all-gathered, grad_hidden reduce-scattered by the dgrad "
                                     "GEMMs"}[part] if world > 1 else
                           ("single GPU" if not vocab else "single GPU, vocabulary phases (one slice)")),
           "phases_ms_per_step": {k: v_[0] / steps for k, v_ in phases.items()},
           "roofline": gemm_roofline(phases, steps, flops, "gemm_kernel (tcgen05 cta_group::2, 3 layouts)"),
           "step_tflops_per_gpu": flops / (ms / 1e3) / 1e12, "gpu_launches": int(launches), "clocks": clocks}
    if not args.no_parity:
        if world == 1 and not vocab:
            def call(r0, r1, n):
                r = distillation_loss_device(ctx, hs[r0:r1], w, labels[r0:r1], ob.TeacherMode.Tied,
                                             teacher_hidden=ht[r0:r1], opts=opts, global_non_ignore=n, stream=stream)
                return r.scalars, r.grad_student_hidden, r.grad_weight, r.grad_teacher_hidden

            res["parity"] = {"row_blocks": check_row_blocks(torch, call, rows, int((labels != -100).sum()), C5["v"],
                                                            k_segments=2)[0]}
        elif world == 1:
            res["parity"] = {"vocab_phases_vs_device_entry": verify_c5_vocab_one_gpu(torch, ob, ctx, hs, ht, w,
                                                                                      labels, opts, out, stream)}
        else:
            del out
            out = None
            torch.cuda.empty_cache()
            res["parity"] = {"sharded_vs_one_gpu": verify_c5_sharded(torch, ob, shard, D, ctx, part, args,
                                                                     int8_wire=args.int8_wire and not vocab)}
            if args.int8_wire and not vocab:
                res["grad_w_exchange"] = "INT8 wire format (row-wise codes + fp32 scales)"
        res["parity"]["pass"] = all(p.get("pass", True) for p in res["parity"].values())
    ctx.close()
    del hs, ht, labels, w, out
    torch.cuda.empty_cache()
    return res


def verify_c5_vocab_one_gpu(torch, ob, ctx, hs, ht, w, labels, opts, out, stream):
    """N=1: the vocabulary phases on one slice (the whole vocabulary) against
    the device entry on the same inputs."""
    from orda_b200.device import distillation_loss_device

    a = {k: t.clone() for k, t in out.items()}
    r = distillation_loss_device(ctx, hs, w, labels, ob.TeacherMode.Tied, teacher_hidden=ht, opts=opts,
                                 stream=stream)
    torch.cuda.synchronize()
    res = {"scalars_rel": scalars_rel(a["scalars"].cpu().numpy(), r.scalars.cpu().numpy()),
           "grad_weight_rel_l2": rel_l2_dev(torch, a["grad_weight"], r.grad_weight),
           "grad_hidden_rel_l2": rel_l2_dev(torch, a["grad_student_hidden"], r.grad_student_hidden),
           "grad_teacher_hidden_rel_l2": rel_l2_dev(torch, a["grad_teacher_hidden"], r.grad_teacher_hidden),
           "tol": TOL["shard_rel"]}
    res["pass"] = all(v <= TOL["shard_rel"] for k, v in res.items() if k != "tol")
    return res


def verify_c5_sharded(torch, ob, shard, D, ctx, part, args, rows=256, int8_wire=False):
    """One small c5 step (H, V of c5) through the sharded path of `part`
    against the whole problem on one GPU (rank 0 computes, then broadcasts):
    scalars, this rank's grad_W rows and grad_hidden rows within 1e-5 (with
    the INT8 wire format, grad_W within its stated 2e-2)."""
    from orda_b200.device import distillation_loss_device

    world, rank, dev = D.world, D.rank, D.dev
    h, v = C5["h"], C5["v"]
    st = torch.cuda.current_stream(dev)
    opts = c5_opts(ob)
    bounds = [shard.vocab_slice_bounds(v, world, r) for r in range(world)]
    if part == "vocab":
        total = rows * world
        hs, ht, labels = c5_rows(torch, total, dev, 6000)
        v0, v1 = bounds[rank]
        w = c5_weight_slice(torch, v0, v1, dev)
        hsl = shard.HiddenSlots(ctx, total, h, teacher=True)
        res = shard.vocab_sharded_step(ctx, hs, w, labels, ob.TeacherMode.Tied, v, v0, teacher_hidden=ht, opts=opts,
                                       stream=st, hidden_slots=hsl)
        my_gw, r0, r1 = res.grad_weight, hsl.r0, hsl.r1
        my_gh, my_gth = res.grad_student_hidden, res.grad_teacher_hidden
    else:
        hs, ht, labels = c5_rows(torch, rows, dev, 6000 + rank)
        w = c5_weight_slice(torch, 0, v, dev)
        fused = shard.SlotReduceScatter(ctx, v, h, int8_wire=int8_wire)
        n_global = shard.global_non_ignore(labels, -100)
        gth = {}

        def compute(n):
            r = distillation_loss_device(ctx, hs, w, labels, ob.TeacherMode.Tied, teacher_hidden=ht, opts=opts,
                                         global_non_ignore=n, scatter_grad_weight=True, stream=st,
                                         int8_wire=int8_wire)
            gth["t"] = r.grad_teacher_hidden
            return r.scalars, r.grad_student_hidden

        v0, v1 = shard.vocab_slice(v, world, rank)
        my_gw = torch.empty(v1 - v0, h, device=dev)
        res = fused.step(compute, labels, -100, n_global, my_gw, stream=st)
        r0, r1 = rank * rows, (rank + 1) * rows
        my_gh, my_gth = res.grad_student_hidden, gth["t"]
    torch.cuda.synchronize()
    ctx.check()
    gw_ref = torch.empty(v, h, device=dev)
    gh_ref = torch.empty(rows * world, h, device=dev)
    gth_ref = torch.empty(rows * world, h, device=dev)
    sc_ref = torch.empty(4, device=dev)
    if rank == 0:
        if part == "vocab":
            hs_a, ht_a, lab_a = hs, ht, labels
            w_a = torch.cat([c5_weight_slice(torch, a, b, dev) for a, b in bounds])
        else:
            parts = [c5_rows(torch, rows, dev, 6000 + r) for r in range(world)]
            hs_a, ht_a, lab_a = (torch.cat([p[i] for p in parts]) for i in range(3))
            w_a = w
        distillation_loss_device(ctx, hs_a, w_a, lab_a, ob.TeacherMode.Tied, teacher_hidden=ht_a, opts=opts,
                                 out={"grad_weight": gw_ref, "grad_student_hidden": gh_ref,
                                      "grad_teacher_hidden": gth_ref, "scalars": sc_ref}, stream=st)
        torch.cuda.synchronize()
        ctx.check()
        del w_a
    for t in (gw_ref, gh_ref, gth_ref, sc_ref):
        D.dist.broadcast(t, src=0)
    ref_gw = gw_ref[v0:v1]
    stats = D.sum(torch, [
        float(((my_gw.double() - ref_gw.double()) ** 2).sum()), float((ref_gw.double() ** 2).sum()),
        float(((my_gh.double() - gh_ref[r0:r1].double()) ** 2).sum()), float((gh_ref[r0:r1].double() ** 2).sum()),
        float(((my_gth.double() - gth_ref[r0:r1].double()) ** 2).sum()), float((gth_ref[r0:r1].double() ** 2).sum()),
    ])
    sc_err = D.max(torch, scalars_rel(res.scalars.cpu().numpy(), sc_ref.cpu().numpy()))
    tol_w = 2e-2 if int8_wire else ksum_tol(2 * rows * world)  # Tied: student and teacher rows
    # vocabulary sharding sums grad_hidden over the ranks' V slices: its K
    # (= V) is associated differently from the one-GPU GEMM's
    tol_h = ksum_tol(v) if part == "vocab" else TOL["shard_rel"]
    out = {"rows": rows * world, "scalars_rel": sc_err, "grad_weight_rel_l2": (stats[0] / stats[1]) ** 0.5,
           "grad_hidden_rel_l2": (stats[2] / stats[3]) ** 0.5,
           "grad_teacher_hidden_rel_l2": (stats[4] / stats[5]) ** 0.5, "tol": TOL["shard_rel"],
           "tol_grad_weight": tol_w, "tol_grad_hidden": tol_h}
    out["pass"] = (out["scalars_rel"] <= TOL["shard_rel"] and out["grad_weight_rel_l2"] <= tol_w
                   and out["grad_hidden_rel_l2"] <= tol_h and out["grad_teacher_hidden_rel_l2"] <= tol_h)
    del gw_ref, gh_ref, gth_ref
    torch.cuda.empty_cache()
    return out


def run_c5_only(args):
    import torch

    import orda_b200 as ob
    from orda_b200 import shard

    D = Dist(torch)
    res = run_c5_part(torch, ob, shard, D, args, args.shard)
    D.close()
    if D.rank == 0:
        line = dict(res)
        line.update({"n_gpus": D.world, "warmup": args.warmup, "higher_is_better": True, "scaling": "weak",
                     "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
                     "config": {"workload": C5_WORKLOAD, "parallelism": res["parallelism"]}})
        print(json.dumps(line), flush=True)
    return 0


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--e2e-steps", type=int, default=4)
    ap.add_argument("--c5-steps", type=int, default=10)
    ap.add_argument("--rows", type=int, default=CFG["bt"],
                    help="rows per GPU (default 8192, the metric's config; smaller values are for profiling only)")
    ap.add_argument("--cpu-rows", type=int, default=3)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-clocks", action="store_true")
    ap.add_argument("--no-parity", action="store_true")
    ap.add_argument("--no-c5", action="store_true", help="leave out the c5 sub-objects")
    ap.add_argument("--no-fast", action="store_true", help="leave out the Profile::Fast sub-object (N=1)")
    ap.add_argument("--config", choices=["c4", "c5"], default="c4",
                    help="c4: the metric configuration with c5 sub-objects (default); c5: only c5")
    ap.add_argument("--shard", choices=["rows", "vocab"], default="rows", help="--config c5: partitioning")
    ap.add_argument("--balance", choices=["off", "once", "dynamic"], default="off",
                    help="N > 1: redistribute the global batch to the GPUs' measured speeds: once after warm-up, "
                         "or every step by feedback (RowBalancer)")
    ap.add_argument("--reduce", choices=["fused", "nccl"], default="fused",
                    help="N > 1: grad_W reduce-scatter fused into the wgrad GEMM, or an NCCL reduce-scatter")
    ap.add_argument("--int8-wire", action="store_true",
                    help="--config c5 --shard rows, N > 1: grad_W partials exchanged as row-wise INT8 + scales "
                         "(lossy; the verification then reports its error against the fp32 exchange)")
    args = ap.parse_args()
    if args.warmup < 3:
        print("note: at least 3 warm-up steps are required for a valid number; using 3", file=sys.stderr)
        args.warmup = 3
    if args.impl == "reference":
        return run_reference_arm(args)
    if args.config == "c5":
        return run_c5_only(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
