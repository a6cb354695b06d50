"""Row-sharded data parallelism (orda_b200/shard.py) with world-size-2 gloo
ranks on CPU.

Each rank runs the oracle on its block of rows with the global mean
denominator (what the device entry does with OrdaShardOptions), then the
shard module's collectives combine the ranks: all-reduce of the scalars,
reduction of grad_W to each rank's vocabulary slice, label all-gather for the
INT8 round trip on the slice. The combined result must equal the single-rank
oracle on the whole batch.
"""
from __future__ import annotations

import os
import socket
import sys
from pathlib import Path

import numpy as np
import pytest

REPO = Path(__file__).resolve().parent.parent


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _problem(bt=12):
    sys.path.insert(0, str(REPO / "orda-cutile-rs_b200"))
    sys.path.insert(0, str(REPO / "oracle"))
    import oracle
    import orda_b200 as ob

    h, v = 8, 16
    hs = oracle.lcg_fill(bt * h, 5, 0.5).reshape(bt, h)
    ht = oracle.lcg_fill(bt * h, 6, 0.5).reshape(bt, h)
    w = oracle.lcg_fill(v * h, 7, 0.4).reshape(v, h)
    labels = oracle.e2e_labels(bt, v, 5, -100)
    return bt, h, v, hs, ht, w, labels


def _opts(ob, reduction, quant):
    return ob.LossOptions(kd_weight=0.4, temperature=1.5, teacher_ce_weight=0.5, label_smoothing=0.05,
                          reduction=reduction, config=ob.KernelConfig(quantize_grad_weight=quant))


def _worker(rank, world, port, quant, q, bt=12):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime

    import torch
    import torch.distributed as dist

    sys.path.insert(0, str(REPO / "orda-cutile-rs_b200"))
    sys.path.insert(0, str(REPO / "oracle"))
    import oracle
    import orda_b200 as ob
    from orda_b200 import shard

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        bt, h, v, hs, ht, w, labels = _problem(bt)
        r0, r1 = shard.shard_rows(bt, world, rank)
        cap = shard.shard_rows(bt, world, 0)[1]  # rank 0 holds the most rows
        lab_local = torch.tensor(labels[r0:r1], dtype=torch.int64)
        n_global = shard.global_non_ignore(lab_local, -100)

        def compute(n):
            # local rows, Sum reduction, then the global mean scale (f32), which is
            # what the device entry applies given global_non_ignore = n
            out = oracle.distillation_loss(ob.Mat.from_array(hs[r0:r1]), ob.Mat.from_array(w), labels[r0:r1],
                                           ob.Teacher.Tied(ob.Mat.from_array(ht[r0:r1])),
                                           _opts(ob, ob.Reduction.Sum, False))
            ms = np.float32(1.0) / np.float32(max(n, 1))
            sc = torch.tensor([out.loss, out.student_ce, out.teacher_ce, out.kl], dtype=torch.float32) * float(ms)
            return (sc, torch.from_numpy(out.grad_student_hidden.a * ms),
                    torch.from_numpy(np.ascontiguousarray(out.grad_weight.a * ms)))

        def quantize(sl, shifted):
            _q, _s, deq = oracle.quantize_grad_w(sl.numpy(), shifted.numpy(), -100)
            sl.copy_(torch.from_numpy(deq))

        res = shard.row_sharded_step(compute, lab_local, -100, n_global, quantize=quantize if quant else None,
                                     label_capacity=cap)
        q.put((rank, res.scalars.numpy(), res.grad_student_hidden.numpy(), res.grad_weight_slice.numpy().copy(),
               res.vocab_range, (r0, r1)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("quant,bt", [(False, 12), (True, 12), (True, 13)])
def test_row_sharded_matches_single_rank(quant, bt):
    """bt=13 gives the ranks 7 and 6 rows: the label gather pads to the
    larger count."""
    import torch.multiprocessing as mp

    sys.path.insert(0, str(REPO / "orda-cutile-rs_b200"))
    sys.path.insert(0, str(REPO / "oracle"))
    import oracle
    import orda_b200 as ob

    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, quant, q, bt)) for r in range(world)]
    for p in procs:
        p.start()
    results = sorted([q.get(timeout=120) for _ in range(world)], key=lambda x: x[0])
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0

    bt, h, v, hs, ht, w, labels = _problem(bt)
    full = oracle.distillation_loss(ob.Mat.from_array(hs), ob.Mat.from_array(w), labels,
                                    ob.Teacher.Tied(ob.Mat.from_array(ht)), _opts(ob, ob.Reduction.Mean, quant))
    sc = results[0][1]
    assert np.allclose(sc, results[1][1])  # all-reduced on every rank
    ref = np.array([full.loss, full.student_ce, full.teacher_ce, full.kl], np.float32)
    assert np.allclose(sc, ref, rtol=1e-5, atol=1e-6), (sc, ref)
    gh = np.concatenate([r[2] for r in results])
    assert np.allclose(gh, full.grad_student_hidden.a, rtol=1e-5, atol=1e-7)
    gw = np.concatenate([r[3] for r in results])
    assert [r[4] for r in results] == [(0, v // 2), (v // 2, v)]
    if quant:
        # INT8 round trip on each reduced slice: error bounded by half a
        # quantisation step of the full-batch result's rows
        _q, s, _d = oracle.quantize_grad_w(full.grad_weight.a, labels, -100)
        assert np.all(np.abs(gw - full.grad_weight.a) <= s[:, None] * 0.5 + 1e-6)
    else:
        assert np.allclose(gw, full.grad_weight.a, rtol=1e-5, atol=1e-7)


def test_shard_rows_and_vocab_slices():
    sys.path.insert(0, str(REPO / "orda-cutile-rs_b200"))
    from orda_b200 import shard

    assert [shard.shard_rows(10, 3, r) for r in range(3)] == [(0, 4), (4, 7), (7, 10)]
    assert [shard.shard_rows(8192 * 8, 8, r) for r in (0, 7)] == [(0, 8192), (57344, 65536)]
    assert shard.vocab_slice(131072, 8, 3) == (49152, 65536)
    # V not divisible by the world size: slices of ceil(V / N) rounded up to
    # 8 rows, the last owner holds the rest (ceil(50257 / 8) = 6283 -> 6288;
    # rank 7 holds 50257 - 7 x 6288 = 6241 rows)
    b = [shard.vocab_slice(50257, 8, r) for r in range(8)]
    assert b[0] == (0, 6288) and b[7] == (44016, 50257)
    assert all(b[i][1] == b[i + 1][0] for i in range(7))
    assert shard.vocab_slice(32001, 2, 1) == (16008, 32001)
    with pytest.raises(ValueError):
        shard.owner_rows(17, 8, 7)  # slices of 8: ranks 3.. hold no rows


def test_vocab_slice_bounds_cover_the_vocabulary_once():
    sys.path.insert(0, str(REPO / "orda-cutile-rs_b200"))
    from orda_b200 import shard

    for v, world in ((152064, 8), (131072, 8), (8192, 3), (1000, 4), (40, 2)):
        b = [shard.vocab_slice_bounds(v, world, r) for r in range(world)]
        assert b[0][0] == 0 and b[-1][1] == v
        assert all(b[i][1] == b[i + 1][0] for i in range(world - 1))
        assert all(v0 % 8 == 0 and v1 > v0 for v0, v1 in b)
    assert shard.vocab_slice_bounds(152064, 8, 3) == (57024, 76032)
    with pytest.raises(ValueError):
        shard.vocab_slice_bounds(16, 4, 3)  # slices of 8: rank 2 ends the vocabulary


def _failing_worker(rank, world, port, q):
    """Rank 1 fails before the step's first collective; rank 0 must end with
    an error from the process-group timeout instead of waiting for good."""
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime
    import time

    import torch
    import torch.distributed as dist

    sys.path.insert(0, str(REPO / "orda-cutile-rs_b200"))
    from orda_b200 import shard

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    t0 = time.monotonic()
    try:
        if rank == 1:
            raise RuntimeError("injected failure on rank 1")
        lab = torch.zeros(4, dtype=torch.int64)

        def compute(n):
            return torch.zeros(4), torch.zeros(4, 2), torch.zeros(8, 2)

        shard.row_sharded_step(compute, lab, -100, 8)
        q.put((rank, "no error", time.monotonic() - t0))
    except Exception as e:  # noqa: BLE001 - the test reports what the rank saw
        q.put((rank, type(e).__name__, time.monotonic() - t0))


def test_failed_rank_ends_the_step_with_an_error():
    import torch.multiprocessing as mp

    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_failing_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    seen = dict((r, (what, dt)) for r, what, dt in [q.get(timeout=120) for _ in range(world)])
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert seen[1][0] == "RuntimeError"
    what, dt = seen[0]
    assert what != "no error", "rank 0 completed a collective its peer never joined"
    assert dt < 60.0
