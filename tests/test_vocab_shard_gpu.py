"""Vocabulary-sharded distillation (W split by vocabulary rows, every rank
sees all tokens) against the full-vocabulary device call.

The single-GPU tests emulate the ranks: one context per vocabulary slice runs
orda_vocab_forward_device, the per-row partial statistics of all slices are
stacked (the all-gather), every slice runs orda_vocab_backward_device, and
the partial grad_hidden / scalars are summed (the all-reduce) while the grad_W
slices are concatenated. The two-GPU test runs the same flow over NCCL with
shard.vocab_sharded_step.

Tolerances: the sharded path merges the row statistics in another order and
splits the dgrad K dimension over the slices, so values agree to fp32
rounding, not bit for bit: scalars within 1e-5 relative, gradients within
rel-L2 1e-5, INT8 codes within one code (a scale from a grad_W row that
differs in the last bits can move a value across a rounding boundary) with
at least 99.9 % identical, per-row scales within 1e-3 relative.
"""
from __future__ import annotations

import os
import socket
import sys
from pathlib import Path

import pytest
import torch

from conftest import rel_l2

REPO = Path(__file__).resolve().parent.parent
pytestmark = pytest.mark.gpu

BT, H, HT, V = 256, 512, 384, 8192


def _case(ob, mode, dev, stochastic=False):
    g = torch.Generator(device=dev).manual_seed(31 + int(mode))
    hs = torch.randn(BT, H, generator=g, device=dev).bfloat16()
    w = (0.02 * torch.randn(V, H, generator=g, device=dev)).bfloat16()
    labels = torch.randint(0, V, (BT,), generator=g, device=dev)
    labels[::13] = -100
    kw = {}
    if mode == ob.TeacherMode.Tied:
        kw["teacher_hidden"] = (hs.float() + 0.1 * torch.randn(BT, H, generator=g, device=dev)).bfloat16()
        opts = ob.LossOptions(kd_weight=0.4, temperature=1.5, label_smoothing=0.1)
    elif mode == ob.TeacherMode.Separate:
        kw["teacher_hidden"] = torch.randn(BT, HT, generator=g, device=dev).bfloat16()
        kw["teacher_weight"] = (0.02 * torch.randn(V, HT, generator=g, device=dev)).bfloat16()
        opts = ob.LossOptions(kd_weight=0.5, temperature=2.0, teacher_ce_weight=0.7)
    else:
        kw["teacher_logits"] = (2.0 ** 0.5 * torch.randn(BT, V, generator=g, device=dev)).bfloat16()
        cfg = (ob.KernelConfig(quantize_grad_weight=True, stochastic_rounding=True, stochastic_seed=12345)
               if stochastic else ob.KernelConfig(quantize_grad_weight=True))
        opts = ob.LossOptions(kd_weight=0.4, temperature=1.5, config=cfg)
    return hs, w, labels, kw, opts


def _slice_kw(kw, v0, v1):
    out = {}
    if "teacher_hidden" in kw:
        out["teacher_hidden"] = kw["teacher_hidden"]
    if "teacher_weight" in kw:
        out["teacher_weight_slice"] = kw["teacher_weight"][v0:v1]
    if "teacher_logits" in kw:
        out["teacher_logits_slice"] = kw["teacher_logits"][:, v0:v1]
    return out


def _check_against_full(ob, full, sc, gsh, gth, gw, gtw, q, qs):
    assert torch.allclose(sc, full.scalars, rtol=1e-5, atol=1e-6), (sc, full.scalars)
    assert rel_l2(gsh.cpu().numpy(), full.grad_student_hidden.cpu().numpy()) < 1e-5
    assert rel_l2(gw.cpu().numpy(), full.grad_weight.cpu().numpy()) < 1e-5
    assert (gth is None) == (full.grad_teacher_hidden is None)
    if gth is not None:
        assert rel_l2(gth.cpu().numpy(), full.grad_teacher_hidden.cpu().numpy()) < 1e-5
    assert (gtw is None) == (full.grad_teacher_weight is None)
    if gtw is not None:
        assert rel_l2(gtw.cpu().numpy(), full.grad_teacher_weight.cpu().numpy()) < 1e-5
    if q is not None:
        d = (q.int() - full.grad_weight_q.int()).abs()
        assert int(d.max()) <= 1
        assert float((d == 0).float().mean()) >= 0.999
        # scales follow each row's absmax: in rows with tiny gradients one bf16
        # logit gradient that rounds the other way moves the absmax visibly
        rel = ((qs - full.grad_weight_scale).abs() / full.grad_weight_scale).max()
        assert float(rel) < 1e-3


@pytest.mark.parametrize("mode", ["Tied", "Separate", "Precomputed", "PrecomputedStochastic"])
@pytest.mark.parametrize("bounds", [[0, 2048, 5120, 8192], [0, 4096, 8192]])
def test_vocab_shards_emulated_on_one_gpu_match_full(ob, mode, bounds):
    """PrecomputedStochastic: stochastic INT8 rounding, whose draws are indexed
    by the global grad_W row, so each slice must offset its rows by v0."""
    from orda_b200.device import DeviceContext, distillation_loss_device, vocab_backward_device, vocab_forward_device

    stochastic = mode.endswith("Stochastic")
    mode = getattr(ob.TeacherMode, mode.replace("Stochastic", ""))
    dev = torch.device("cuda", 0)
    hs, w, labels, kw, opts = _case(ob, mode, dev, stochastic)
    quant = opts.config.quantize_grad_weight
    with DeviceContext(0) as ctx:
        full = distillation_loss_device(ctx, hs, w, labels, mode, opts=opts, want_int8=quant, **kw)
        torch.cuda.synchronize()
        ctx.check()

    slices = list(zip(bounds[:-1], bounds[1:]))
    ctxs = [DeviceContext(0) for _ in slices]
    try:
        parts = [vocab_forward_device(c, hs, w[v0:v1], labels, mode, V, v0, opts=opts, **_slice_kw(kw, v0, v1))
                 for c, (v0, v1) in zip(ctxs, slices)]
        every = torch.stack(parts)
        res = [vocab_backward_device(c, hs, w[v0:v1], labels, mode, V, v0, every, include_rows=(r == 0), opts=opts,
                                     want_int8=quant, **_slice_kw(kw, v0, v1))
               for r, (c, (v0, v1)) in enumerate(zip(ctxs, slices))]
        torch.cuda.synchronize()
        for c in ctxs:
            c.check()
    finally:
        for c in ctxs:
            c.close()
    sc = sum(r.scalars for r in res)
    gsh = sum(r.grad_student_hidden for r in res)
    gth = sum(r.grad_teacher_hidden for r in res) if res[0].grad_teacher_hidden is not None else None
    gw = torch.cat([r.grad_weight for r in res])
    gtw = torch.cat([r.grad_teacher_weight for r in res]) if res[0].grad_teacher_weight is not None else None
    q = torch.cat([r.grad_weight_q for r in res]) if quant else None
    qs = torch.cat([r.grad_weight_scale for r in res]) if quant else None
    for r in res:
        assert r.chunk_plan == full.chunk_plan
    _check_against_full(ob, full, sc, gsh, gth, gw, gtw, q, qs)


def test_vocab_backward_requires_the_forward_phase(ob):
    from orda_b200.device import DeviceContext, vocab_backward_device

    dev = torch.device("cuda", 0)
    hs, w, labels, kw, opts = _case(ob, ob.TeacherMode.Tied, dev)
    every = torch.zeros(2, BT, 12, device=dev)
    with DeviceContext(0) as ctx:
        with pytest.raises(ob.OrdaError, match="must follow orda_vocab_forward_device"):
            vocab_backward_device(ctx, hs, w[:4096], labels, ob.TeacherMode.Tied, V, 0, every, True, opts=opts,
                                  **_slice_kw(kw, 0, 4096))
        # another call on the context between the phases reuses the workspace
        # that held the slice logits: the backward phase is refused
        from orda_b200.device import distillation_loss_device, vocab_forward_device

        vocab_forward_device(ctx, hs, w[:4096], labels, ob.TeacherMode.Tied, V, 0, opts=opts, **_slice_kw(kw, 0, 4096))
        distillation_loss_device(ctx, hs, w, labels, ob.TeacherMode.Tied, opts=opts, **kw)
        with pytest.raises(ob.OrdaError, match="must follow orda_vocab_forward_device"):
            vocab_backward_device(ctx, hs, w[:4096], labels, ob.TeacherMode.Tied, V, 0, every, True, opts=opts,
                                  **_slice_kw(kw, 0, 4096))
        torch.cuda.synchronize()


# --------------------------------------------------------------- two GPUs

def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, outdir, scatter=False):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    if scatter == "wide":
        # the scattering dgrad GEMMs on wide (256 x 512) pair tiles, which the
        # default rule takes for long vocabulary slices (1024 K blocks)
        os.environ["ORDA_GEMM_WIDE"] = "2"
    import datetime

    import torch.distributed as dist

    sys.path.insert(0, str(REPO / "orda-cutile-rs_b200"))
    import orda_b200 as ob
    from orda_b200 import shard
    from orda_b200.device import DeviceContext

    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        mode = ob.TeacherMode.Tied
        hs, w, labels, kw, opts = _case(ob, mode, dev)
        v0, v1 = shard.vocab_slice_bounds(V, world, rank)
        with DeviceContext(rank) as ctx:
            slots = shard.HiddenSlots(ctx, BT, H, teacher=True) if scatter else None
            rows = (slots.r0, slots.r1) if scatter else (0, BT)
            # two steps in a row: the second reuses the slot buffers
            for _ in range(2 if scatter else 1):
                r = shard.vocab_sharded_step(ctx, hs, w[v0:v1], labels, mode, V, v0, opts=opts, hidden_slots=slots,
                                             **_slice_kw(kw, v0, v1))
            torch.cuda.synchronize()
            ctx.check()
            torch.save({"scalars": r.scalars.cpu(), "gsh": r.grad_student_hidden.cpu(),
                        "gth": r.grad_teacher_hidden.cpu(), "gw": r.grad_weight.cpu(), "vocab": (v0, v1),
                        "rows": rows}, os.path.join(outdir, f"rank{rank}.pt"))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("scatter", [False, True, "wide"])
def test_vocab_sharded_two_gpus_match_single_gpu(ob, tmp_path, scatter):
    """grad_hidden all-reduced (full on every rank), or reduce-scattered by
    the dgrad GEMMs into the owners' slot buffers (each rank its rows)."""
    import torch.multiprocessing as mp

    from orda_b200.device import DeviceContext, distillation_loss_device

    world = 2
    port = _free_port()
    ctxm = mp.get_context("spawn")
    procs = [ctxm.Process(target=_worker, args=(r, world, port, str(tmp_path), scatter)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    codes = [p.exitcode for p in procs]
    for p in procs:
        if p.is_alive():
            p.kill()
    assert codes == [0, 0], f"rank exit codes {codes}"

    dev = torch.device("cuda", 0)
    mode = ob.TeacherMode.Tied
    hs, w, labels, kw, opts = _case(ob, mode, dev)
    with DeviceContext(0) as ctx:
        full = distillation_loss_device(ctx, hs, w, labels, mode, opts=opts, **kw)
        torch.cuda.synchronize()
    parts = [torch.load(tmp_path / f"rank{r}.pt") for r in range(world)]
    for p in parts:
        assert torch.allclose(p["scalars"], full.scalars.cpu(), rtol=1e-5, atol=1e-6)
        r0, r1 = p["rows"]
        assert rel_l2(p["gsh"].numpy(), full.grad_student_hidden[r0:r1].cpu().numpy()) < 1e-5
        assert rel_l2(p["gth"].numpy(), full.grad_teacher_hidden[r0:r1].cpu().numpy()) < 1e-5
        v0, v1 = p["vocab"]
        assert rel_l2(p["gw"].numpy(), full.grad_weight[v0:v1].cpu().numpy()) < 1e-5
