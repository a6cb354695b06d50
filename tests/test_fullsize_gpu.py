"""Parity at the full shapes the bench times (BASELINE configs[3] = c4 and
configs[4] = c5 on one GPU), through the C ABI, against the reference CPU
path (the oracle restatement) where that can finish in seconds.

Each case runs the exact call the bench times (c4: 8192 rows, V=131072,
H=4096, one forward group with a 4 GiB fp32 logits buffer, INT8 round trip;
c5: 8192 rows, V=152064, H=8192, Tied teacher, whose teacher logits rows
lie past element 2^31 of the logits buffer from row 5931 on) and checks:

  (i)   32 gradient rows spread over the batch (the last row included)
        against the oracle run on those rows alone; under the mean reduction
        a row's gradient is G_row / n, so both sides are compared as G_row
        (rel-L2 <= 1e-2, the bf16 logit-gradient tolerance);
  (ii)  the full call against the sum of 8 row-block calls given the global
        mean denominator: scalars within 1e-5, grad_W within bench.ksum_tol
        of its K (fp32 sums of the same products in another order: 3.2e-5
        at K=8192), grad_hidden within ksum_tol(V) (the dgrad GEMM splits the
        V sum of the tiles of a partial last wave into two halves);
  (iii) c4: the GPU's fp32 grad_W (skip_quantize), quantised by the oracle's
        restatement of src/quant.rs:157-202, bit-identical to the GPU's INT8
        codes, scales and dequantised grad_W of the timed call.

The checks are the ones bench.py prints in its `parity` object.
"""
from __future__ import annotations

import os
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

sys.path.insert(0, str(Path(__file__).resolve().parent.parent))
import bench  # noqa: E402

pytestmark = pytest.mark.gpu
NT = os.cpu_count() or 1


def _host(t):
    return t.float().cpu().numpy()


def test_c4_full_batch_matches_reference(ob, oracle):
    from orda_b200.device import DeviceContext, distillation_loss_device

    dev = torch.device("cuda", 0)
    hs, tl, labels = bench.c4_rows(torch, bench.CFG["bt"], dev, 1000)  # the bench's rank-0 rows
    w = bench.c4_weight(torch, dev)
    opts = bench.c4_opts(ob)
    bt = hs.shape[0]
    n_full = int((labels != -100).sum())
    with DeviceContext(0) as ctx:
        r = distillation_loss_device(ctx, hs, w, labels, ob.TeacherMode.Precomputed, teacher_logits=tl, opts=opts,
                                     want_int8=True)
        torch.cuda.synchronize()
        ctx.check()
        assert r.chunk_plan == ob.ChunkPlan(512, 16)

        # (ii) row blocks; gw_raw is the full call's fp32 grad_W
        def call(r0, r1, n):
            x = distillation_loss_device(ctx, hs[r0:r1], w, labels[r0:r1], ob.TeacherMode.Precomputed,
                                         teacher_logits=tl[r0:r1], opts=opts, global_non_ignore=n, skip_quantize=True)
            return x.scalars, x.grad_student_hidden, x.grad_weight, None

        blocks, gw_raw = bench.check_row_blocks(torch, call, bt, n_full, bench.CFG["v"])
        ctx.check()
    assert blocks["pass"], blocks

    # (iii) INT8 of the timed call vs the reference quantiser on the same fp32 grad_W
    int8 = bench.check_int8_vs_oracle(gw_raw.cpu().numpy(), labels.cpu().numpy(), r.grad_weight_q.cpu().numpy(),
                                      r.grad_weight_scale.cpu().numpy(), r.grad_weight.cpu().numpy(), NT)
    del gw_raw
    assert int8["pass"], int8

    # (i) sampled rows vs the oracle on those rows
    rows = bench.sample_rows(bt, 32)
    idx = torch.tensor(rows, device=dev)
    lab_rows = labels[idx].cpu().tolist()
    s, wm = ob.Mat.from_array(_host(hs[idx])), ob.Mat.from_array(_host(w))
    t = ob.Teacher.Precomputed(ob.Mat.from_array(_host(tl[idx])))
    ref = oracle.distillation_loss(s, wm, lab_rows, t, bench.c4_opts(ob, quantize=False), nthreads=NT)
    chk = bench.check_rows_vs_oracle(ref, {"grad_student_hidden": r.grad_student_hidden[idx].cpu().numpy()},
                                     lab_rows, n_full)
    assert chk["pass"], chk


def test_c5_full_batch_one_gpu_matches_reference(ob, oracle):
    from orda_b200.device import DeviceContext, distillation_loss_device

    dev = torch.device("cuda", 0)
    h, v = bench.C5["h"], bench.C5["v"]
    hs, ht, labels = bench.c5_rows(torch, bench.C5["rows"], dev, 2000)  # the bench's rank-0 rows
    w = bench.c5_weight_slice(torch, 0, v, dev)
    opts = bench.c5_opts(ob)
    bt = hs.shape[0]
    n_full = int((labels != -100).sum())
    with DeviceContext(0) as ctx:
        r = distillation_loss_device(ctx, hs, w, labels, ob.TeacherMode.Tied, teacher_hidden=ht, opts=opts)
        torch.cuda.synchronize()
        ctx.check()
        assert r.chunk_plan == ob.ChunkPlan(512, 16)
        # the teacher logits of the rows from 5931 on start past element 2^31
        rows = bench.sample_rows(bt, 32)
        assert sum(1 for x in rows if (bt + x) * v >= 2 ** 31) >= 8
        idx = torch.tensor(rows, device=dev)
        gsh_rows = r.grad_student_hidden[idx].cpu().numpy()
        gth_rows = r.grad_teacher_hidden[idx].cpu().numpy()
        del r

        def call(r0, r1, n):
            x = distillation_loss_device(ctx, hs[r0:r1], w, labels[r0:r1], ob.TeacherMode.Tied,
                                         teacher_hidden=ht[r0:r1], opts=opts, global_non_ignore=n)
            return x.scalars, x.grad_student_hidden, x.grad_weight, x.grad_teacher_hidden

        blocks, gw = bench.check_row_blocks(torch, call, bt, n_full, v, k_segments=2)
        del gw
        ctx.check()
    assert blocks["pass"], blocks

    lab_rows = labels[idx].cpu().tolist()
    s, wm = ob.Mat.from_array(_host(hs[idx])), ob.Mat.from_array(_host(w))
    t = ob.Teacher.Tied(ob.Mat.from_array(_host(ht[idx])))
    del w
    torch.cuda.empty_cache()
    ref = oracle.distillation_loss(s, wm, lab_rows, t, opts, nthreads=NT)
    chk = bench.check_rows_vs_oracle(ref, {"grad_student_hidden": gsh_rows, "grad_teacher_hidden": gth_rows},
                                     lab_rows, n_full)
    assert chk["pass"], chk
