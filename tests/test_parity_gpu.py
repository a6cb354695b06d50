"""Parity of the B200 path with the CPU oracle (the reference's CPU path
restated), through the C ABI, on the same seeded inputs.

Inputs are rounded to bf16 first (the tensor-core operand type) and the same
values are given to both sides as f32.

Stated tolerances:
  * loss and the three components: |gpu - ref| <= 1e-4 * |ref| + 1e-6
  * gradients: relative L2 error <= 1e-2 (the logit gradients are bf16
    operands of the backward GEMMs); max-abs error is reported on failure
  * INT8 grad_W quantisation: bit-exact on the same fp32 grad_W.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np
import pytest
import torch

from conftest import bf16_round, rel_l2

pytestmark = pytest.mark.gpu

LOSS_RTOL = 1e-4
LOSS_ATOL = 1e-6
GRAD_REL_L2 = 1e-2
NT = os.cpu_count() or 1


def assert_parity(gpu, ref, what=""):
    for name in ("loss", "student_ce", "teacher_ce", "kl"):
        a, b = getattr(gpu, name), getattr(ref, name)
        assert abs(a - b) <= LOSS_RTOL * abs(b) + LOSS_ATOL, f"{what} {name}: gpu {a!r} ref {b!r}"
    for name in ("grad_student_hidden", "grad_weight", "grad_teacher_hidden", "grad_teacher_weight"):
        a, b = getattr(gpu, name), getattr(ref, name)
        assert (a is None) == (b is None), f"{what} {name} presence differs"
        if a is None:
            continue
        assert a.shape() == b.shape()
        e = rel_l2(a.a, b.a)
        mx = float(np.max(np.abs(a.a.astype(np.float64) - b.a))) if a.a.size else 0.0
        assert e <= GRAD_REL_L2, f"{what} {name}: rel L2 {e:.3e} (max abs {mx:.3e})"
    assert gpu.chunk_plan == ref.chunk_plan


def lcg_mat(ob, oracle, rows, cols, seed, scale):
    return ob.Mat.from_array(bf16_round(oracle.lcg_fill(rows * cols, seed, scale).reshape(rows, cols)))


def randn_mat(ob, rows, cols, gen, std=1.0):
    return ob.Mat.from_array(bf16_round((torch.randn(rows, cols, generator=gen) * std).numpy()))


# --------------------------------------------------------- small exact cases

def test_tied_small_matches_oracle(ob, oracle):
    """Shapes and options of tests/end_to_end.rs:89-128 (Tied, smoothing,
    ignored rows, teacher CE)."""
    bt, h, v = 6, 5, 7
    s = lcg_mat(ob, oracle, bt, h, 1, 0.3)
    w = lcg_mat(ob, oracle, v, h, 2, 0.2)
    th = lcg_mat(ob, oracle, bt, h, 3, 0.3)
    labs = oracle.e2e_labels(bt, v, 4, -100)
    t = ob.Teacher.Tied(th)
    opts = ob.LossOptions(kd_weight=0.5, temperature=1.5, teacher_ce_weight=1.0, label_smoothing=0.1)
    assert_parity(ob.distillation_loss(s, w, labs, t, opts), oracle.distillation_loss(s, w, labs, t, opts), "tied")


def test_separate_small_matches_oracle(ob, oracle):
    """tests/end_to_end.rs:130-178 shapes (Separate teacher, H_t != H)."""
    bt, h, ht, v = 6, 5, 4, 7
    s = lcg_mat(ob, oracle, bt, h, 11, 0.3)
    w = lcg_mat(ob, oracle, v, h, 12, 0.2)
    th = lcg_mat(ob, oracle, bt, ht, 13, 0.3)
    tw = lcg_mat(ob, oracle, v, ht, 14, 0.2)
    labs = oracle.e2e_labels(bt, v, None, -100)
    t = ob.Teacher.Separate(th, tw)
    opts = ob.LossOptions(kd_weight=0.5, temperature=1.5, teacher_ce_weight=0.7)
    assert_parity(ob.distillation_loss(s, w, labs, t, opts), oracle.distillation_loss(s, w, labs, t, opts), "sep")


def test_precomputed_small_matches_oracle(ob, oracle):
    """tests/end_to_end.rs:180-204 shapes; also with a teacher CE weight
    (reported, no teacher gradient)."""
    bt, h, v = 6, 5, 7
    s = lcg_mat(ob, oracle, bt, h, 21, 0.3)
    w = lcg_mat(ob, oracle, v, h, 22, 0.2)
    tl = ob.Mat.from_array(oracle.lcg_fill(bt * v, 23, 0.5).reshape(bt, v))
    labs = oracle.e2e_labels(bt, v, 5, -100)
    t = ob.Teacher.Precomputed(tl)
    for opts in (ob.LossOptions(kd_weight=0.5, temperature=1.5),
                 ob.LossOptions(kd_weight=0.5, temperature=1.5, teacher_ce_weight=0.3, label_smoothing=0.2)):
        g = ob.distillation_loss(s, w, labs, t, opts)
        assert g.grad_teacher_hidden is None and g.grad_teacher_weight is None
        assert_parity(g, oracle.distillation_loss(s, w, labs, t, opts), "pre")


def test_pure_student_ce(ob, oracle):
    """tests/end_to_end.rs:206-228: kd = 0, w_t = 0."""
    bt, h, v = 8, 4, 6
    s = lcg_mat(ob, oracle, bt, h, 31, 0.3)
    w = lcg_mat(ob, oracle, v, h, 32, 0.2)
    labs = oracle.e2e_labels(bt, v, None, -100)
    t = ob.Teacher.Tied(ob.Mat.zeros(bt, h))
    opts = ob.LossOptions(kd_weight=0.0, teacher_ce_weight=0.0)
    g = ob.distillation_loss(s, w, labs, t, opts)
    assert g.teacher_ce == 0.0 and g.kl == 0.0
    assert_parity(g, oracle.distillation_loss(s, w, labs, t, opts), "ce")


def test_all_rows_ignored(ob, oracle):
    """Every label equals ignore_index: zero loss and zero gradients, mean
    denominator clamped to 1 (src/api.rs:225-230)."""
    bt, h, v = 5, 16, 40
    gen = torch.Generator().manual_seed(3)
    s, w, th = randn_mat(ob, bt, h, gen), randn_mat(ob, v, h, gen, 0.1), randn_mat(ob, bt, h, gen)
    labs = [-100] * bt
    t = ob.Teacher.Tied(th)
    opts = ob.LossOptions(kd_weight=0.4, temperature=1.5)
    g = ob.distillation_loss(s, w, labs, t, opts)
    assert g.loss == 0.0 and g.kl == 0.0
    assert np.all(g.grad_weight.a == 0.0) and np.all(g.grad_student_hidden.a == 0.0)
    assert_parity(g, oracle.distillation_loss(s, w, labs, t, opts), "ignored")


# ----------------------------------------------------------------- c1 config

@pytest.fixture(scope="module")
def c1(ob):
    """Tied, BT=256, H=512, V=8192, h_t = h_s + N(0,0.1),
    W ~ N(0, 0.02), labels uniform, kd=0.4, T=1.5, fixed seed."""
    gen = torch.Generator().manual_seed(20261201)
    bt, h, v = 256, 512, 8192
    hs = torch.randn(bt, h, generator=gen)
    ht = hs + 0.1 * torch.randn(bt, h, generator=gen)
    w = 0.02 * torch.randn(v, h, generator=gen)
    labs = torch.randint(0, v, (bt,), generator=gen).tolist()
    return (ob.Mat.from_array(bf16_round(hs.numpy())), ob.Mat.from_array(bf16_round(w.numpy())), labs,
            ob.Teacher.Tied(ob.Mat.from_array(bf16_round(ht.numpy()))))


@pytest.mark.parametrize("chunk", [None, 64])
def test_c1_matches_oracle(ob, oracle, c1, chunk):
    s, w, labs, t = c1
    cs = ob.ChunkSize.Auto() if chunk is None else ob.ChunkSize.Fixed(chunk)
    opts = ob.LossOptions(kd_weight=0.4, temperature=1.5, chunk_size=cs)
    g = ob.distillation_loss(s, w, labs, t, opts)
    r = oracle.distillation_loss(s, w, labs, t, opts, nthreads=NT)
    assert_parity(g, r, f"c1 chunk={chunk}")
    assert g.chunk_plan == (ob.ChunkPlan(256, 1) if chunk is None else ob.ChunkPlan(64, 4))


def test_c1_chunk_invariance_on_gpu(ob, c1):
    """tests/end_to_end.rs:230-278 on the GPU: single chunk vs 4 chunks vs 256
    chunks give identical results (the backward GEMMs run once per group)."""
    s, w, labs, t = c1
    outs = [ob.distillation_loss(s, w, labs, t, ob.LossOptions(kd_weight=0.4, temperature=1.5,
                                                               chunk_size=ob.ChunkSize.Fixed(c)))
            for c in (256, 64, 1)]
    for o in outs[1:]:
        assert abs(o.loss - outs[0].loss) <= 1e-6 * abs(outs[0].loss)
        assert rel_l2(o.grad_weight.a, outs[0].grad_weight.a) < 1e-6
        assert rel_l2(o.grad_student_hidden.a, outs[0].grad_student_hidden.a) < 1e-6


def test_c1_sum_is_mean_times_count(ob, c1):
    """tests/end_to_end.rs:313-358 on the GPU."""
    s, w, labs, t = c1
    labs = [(-100 if i % 4 == 0 else y) for i, y in enumerate(labs)]
    n_valid = sum(1 for y in labs if y != -100)
    mean = ob.distillation_loss(s, w, labs, t, ob.LossOptions(kd_weight=0.4, temperature=1.5))
    summ = ob.distillation_loss(s, w, labs, t, ob.LossOptions(kd_weight=0.4, temperature=1.5,
                                                              reduction=ob.Reduction.Sum))
    assert abs(summ.loss - mean.loss * n_valid) <= 1e-5 * abs(summ.loss)
    assert rel_l2(summ.grad_weight.a, mean.grad_weight.a * n_valid) < 1e-5


def test_c1_device_entry_matches_host_entry(ob, c1):
    """The timed device entry and the reference-facing host entry agree."""
    from orda_b200.device import DeviceContext, distillation_loss_device

    s, w, labs, t = c1
    opts = ob.LossOptions(kd_weight=0.4, temperature=1.5)
    host = ob.distillation_loss(s, w, labs, t, opts)
    with DeviceContext(0) as ctx:
        d = distillation_loss_device(
            ctx, torch.from_numpy(s.a).cuda().bfloat16(), torch.from_numpy(w.a).cuda().bfloat16(),
            torch.tensor(labs, dtype=torch.int64, device="cuda"), ob.TeacherMode.Tied,
            teacher_hidden=torch.from_numpy(t.hidden.a).cuda().bfloat16(), opts=opts)
        torch.cuda.synchronize()
        ctx.check()
        sc = d.scalars.cpu().numpy()
    assert np.allclose(sc, [host.loss, host.student_ce, host.teacher_ce, host.kl], rtol=1e-6, atol=0)
    assert rel_l2(d.grad_weight.cpu().numpy(), host.grad_weight.a) < 1e-6
    assert rel_l2(d.grad_student_hidden.cpu().numpy(), host.grad_student_hidden.a) < 1e-6
    assert rel_l2(d.grad_teacher_hidden.cpu().numpy(), host.grad_teacher_hidden.a) < 1e-6


def test_oom_ladder_on_device(ob, c1):
    """An injected workspace-allocation failure moves the device entry to the
    next rung of the chunk-doubling schedule; results are unchanged."""
    from orda_b200.device import DeviceContext, distillation_loss_device

    s, w, labs, t = c1
    opts = ob.LossOptions(kd_weight=0.4, temperature=1.5)
    args = (torch.from_numpy(s.a).cuda().bfloat16(), torch.from_numpy(w.a).cuda().bfloat16(),
            torch.tensor(labs, dtype=torch.int64, device="cuda"), ob.TeacherMode.Tied)
    kw = dict(teacher_hidden=torch.from_numpy(t.hidden.a).cuda().bfloat16(), opts=opts)
    with DeviceContext(0) as ctx:
        a = distillation_loss_device(ctx, *args, **kw)
        torch.cuda.synchronize()
        ctx.inject_alloc_failures(1)
        b = distillation_loss_device(ctx, *args, **kw)
        torch.cuda.synchronize()
        ctx.check()
        ctx.inject_alloc_failures(10)
        with pytest.raises(ob.OrdaError, match="OOM ladder"):
            distillation_loss_device(ctx, *args, **kw)
        ctx.inject_alloc_failures(0)
    assert a.chunk_plan == ob.ChunkPlan(256, 1)
    assert b.chunk_plan == ob.ChunkPlan(128, 2)
    assert torch.allclose(a.scalars, b.scalars, rtol=1e-6, atol=0)
    assert rel_l2(b.grad_weight.cpu().numpy(), a.grad_weight.cpu().numpy()) < 1e-6


def test_device_label_range_error(ob):
    """Out-of-range labels on the device entry are reported by the device
    label check (no out-of-bounds access; the rows are skipped)."""
    from orda_b200.device import DeviceContext, distillation_loss_device

    bt, h, v = 16, 64, 256
    gen = torch.Generator(device="cuda").manual_seed(1)
    hs = torch.randn(bt, h, generator=gen, device="cuda").bfloat16()
    w = (0.02 * torch.randn(v, h, generator=gen, device="cuda")).bfloat16()
    labs = torch.randint(0, v, (bt,), generator=gen, device="cuda")
    labs[3] = v + 5
    with DeviceContext(0) as ctx:
        distillation_loss_device(ctx, hs, w, labs, ob.TeacherMode.Tied, teacher_hidden=hs,
                                 opts=ob.LossOptions(kd_weight=0.4))
        torch.cuda.synchronize()
        with pytest.raises(ob.OrdaError, match="out of range"):
            ctx.check()


def test_bounded_wait_expiry_is_reported_and_context_survives(ob, c1):
    """A device wait that nothing completes gives up after its limit (50 ms
    here), the context reports a timeout, and the same context then computes
    a correct loss: failure detection without a GPU fault."""
    import time

    from orda_b200.device import DeviceContext, distillation_loss_device

    s, w, labs, t = c1
    opts = ob.LossOptions(kd_weight=0.4, temperature=1.5)
    host = ob.distillation_loss(s, w, labs, t, opts)
    with DeviceContext(0) as ctx:
        t0 = time.perf_counter()
        ctx.selftest_bounded_wait(50000)
        with pytest.raises(ob.OrdaError, match="bounded device wait expired"):
            ctx.check()
        waited = time.perf_counter() - t0
        d = distillation_loss_device(
            ctx, torch.from_numpy(s.a).cuda().bfloat16(), torch.from_numpy(w.a).cuda().bfloat16(),
            torch.tensor(labs, dtype=torch.int64, device="cuda"), ob.TeacherMode.Tied,
            teacher_hidden=torch.from_numpy(t.hidden.a).cuda().bfloat16(), opts=opts)
        torch.cuda.synchronize()
        ctx.check()
        sc = d.scalars.cpu().numpy()
    assert 0.04 <= waited < 5.0
    assert np.allclose(sc, [host.loss, host.student_ce, host.teacher_ce, host.kl], rtol=1e-6, atol=0)


# ------------------------------------------------------- BASELINE subsets

def _subset_case(ob, cfg, rows, gen):
    if cfg == "c2":
        bt, h, v = rows, 4096, 32000
        hs = torch.randn(bt, h, generator=gen)
        ht = hs + 0.1 * torch.randn(bt, h, generator=gen)
        w = 0.02 * torch.randn(v, h, generator=gen)
        labs = torch.randint(0, v, (bt,), generator=gen).tolist()
        t = ob.Teacher.Tied(ob.Mat.from_array(bf16_round(ht.numpy())))
        opts = ob.LossOptions(kd_weight=0.4, temperature=1.5)
        return ob.Mat.from_array(bf16_round(hs.numpy())), ob.Mat.from_array(bf16_round(w.numpy())), labs, t, opts
    if cfg == "c3":
        bt, hs_d, ht_d, v = rows, 2048, 4096, 128256
        hs = torch.randn(bt, hs_d, generator=gen)
        ht = torch.randn(bt, ht_d, generator=gen)
        ws = 0.02 * torch.randn(v, hs_d, generator=gen)
        wt = 0.02 * torch.randn(v, ht_d, generator=gen)
        labs = torch.randint(0, v, (bt,), generator=gen)
        labs[torch.rand(bt, generator=gen) < 0.05] = -100
        t = ob.Teacher.Separate(ob.Mat.from_array(bf16_round(ht.numpy())), ob.Mat.from_array(bf16_round(wt.numpy())))
        opts = ob.LossOptions(kd_weight=0.5, temperature=2.0, label_smoothing=0.1)
        return (ob.Mat.from_array(bf16_round(hs.numpy())), ob.Mat.from_array(bf16_round(ws.numpy())),
                labs.tolist(), t, opts)
    if cfg == "c4":
        bt, h, v = rows, 4096, 131072
        hs = torch.randn(bt, h, generator=gen)
        w = 0.02 * torch.randn(v, h, generator=gen)
        tl = np.sqrt(2.0) * torch.randn(bt, v, generator=gen)
        labs = torch.randint(0, v, (bt,), generator=gen).tolist()
        t = ob.Teacher.Precomputed(ob.Mat.from_array(bf16_round(tl.numpy())))
        opts = ob.LossOptions(kd_weight=0.4, temperature=1.5, config=ob.KernelConfig(quantize_grad_weight=True))
        return ob.Mat.from_array(bf16_round(hs.numpy())), ob.Mat.from_array(bf16_round(w.numpy())), labs, t, opts
    if cfg == "c5":
        bt, h, v = rows, 8192, 152064
        hs = torch.randn(bt, h, generator=gen)
        ht = hs + 0.1 * torch.randn(bt, h, generator=gen)
        w = 0.02 * torch.randn(v, h, generator=gen)
        labs = torch.randint(0, v, (bt,), generator=gen).tolist()
        t = ob.Teacher.Tied(ob.Mat.from_array(bf16_round(ht.numpy())))
        opts = ob.LossOptions(kd_weight=0.4, temperature=1.5)
        return ob.Mat.from_array(bf16_round(hs.numpy())), ob.Mat.from_array(bf16_round(w.numpy())), labs, t, opts
    raise ValueError(cfg)


@pytest.mark.parametrize("cfg,rows", [("c2", 64), ("c3", 16), ("c4", 16), ("c5", 4)])
def test_baseline_config_row_subsets_match_oracle(ob, oracle, cfg, rows):
    """Full H and V of BASELINE configs c2-c5 on a row subset the oracle can
    finish in seconds (c4 includes the INT8 grad_W round trip; c5 is the
    large-vocab Tied configuration, H=8192, V=152064, whose tail of 64 rows
    past the last 128-row block exercises the ragged tile edges)."""
    gen = torch.Generator().manual_seed(7 + rows)
    s, w, labs, t, opts = _subset_case(ob, cfg, rows, gen)
    g = ob.distillation_loss(s, w, labs, t, opts)
    r = oracle.distillation_loss(s, w, labs, t, opts, nthreads=NT)
    assert_parity(g, r, cfg)


# ------------------------------------------------------------ INT8 parity

@pytest.mark.parametrize("stochastic", [False, True])
def test_quantizer_bit_exact_on_same_grad_w(ob, oracle, stochastic):
    """`quantize_grad_w` + `dequantize_grad_w` (src/quant.rs:157-202) on the
    GPU vs the oracle on the same fp32 grad_W: q, scales and the dequantised
    matrix are bit-identical."""
    from orda_b200.device import DeviceContext, quantize_grad_w

    gen = torch.Generator().manual_seed(11)
    v, h = 1000, 515
    gw = (torch.randn(v, h, generator=gen) * torch.rand(v, 1, generator=gen) ** 3 * 1e-3).numpy()
    gw[7, :] = 0.0  # amax = 0 -> scale from the 1e-12 floor
    gw[9, 3] = 2.5e-3  # exact .5 ties after scaling are handled by rint
    labels = torch.randint(0, v, (300,), generator=gen)
    labels[::7] = -100
    q_ref, s_ref, deq_ref = oracle.quantize_grad_w(gw, labels.numpy(), -100, stochastic=stochastic, seed=12345)
    with DeviceContext(0) as ctx:
        g = torch.from_numpy(gw).cuda()
        q = torch.empty(v, h, dtype=torch.int8, device="cuda")
        sc = torch.empty(v, device="cuda")
        quantize_grad_w(ctx, g, labels.cuda(), -100, stochastic, 12345, q, sc)
        torch.cuda.synchronize()
        ctx.check()
    assert np.array_equal(q.cpu().numpy(), q_ref)
    assert np.array_equal(sc.cpu().numpy().view(np.uint32), s_ref.view(np.uint32))
    assert np.array_equal(g.cpu().numpy().view(np.uint32), deq_ref.view(np.uint32))


def test_end_to_end_int8_close_but_lossy(ob, oracle, c1):
    """tests/end_to_end.rs:360-417 on the GPU: the loss is unchanged by the
    INT8 round trip, grad_W changes slightly."""
    s, w, labs, t = c1
    exact = ob.distillation_loss(s, w, labs, t, ob.LossOptions(kd_weight=0.4, temperature=1.5))
    quant = ob.distillation_loss(s, w, labs, t, ob.LossOptions(
        kd_weight=0.4, temperature=1.5, config=ob.KernelConfig(quantize_grad_weight=True)))
    assert abs(exact.loss - quant.loss) < 1e-6
    d = np.abs(exact.grad_weight.a - quant.grad_weight.a)
    assert 0.0 < d.max() < 0.05
    # the GPU quantiser applied to the GPU's own fp32 grad_W equals the oracle
    # quantiser on that same matrix
    _q, _s, deq = oracle.quantize_grad_w(exact.grad_weight.a, labs, -100)
    assert np.array_equal(deq.view(np.uint32), quant.grad_weight.a.view(np.uint32))


def test_l2_persisting_carveout_keeps_results_and_is_restored(ob, c1):
    """orda_context_set_l2_persisting changes where lines live in L2, not the
    arithmetic: results are identical with and without it, and destroying the
    context restores the process's previous limit."""
    from cuda.bindings import runtime as cudart

    from orda_b200.device import DeviceContext, distillation_loss_device

    s, w, labs, t = c1
    opts = ob.LossOptions(kd_weight=0.4, temperature=1.5)
    args = (torch.from_numpy(s.a).cuda().bfloat16(), torch.from_numpy(w.a).cuda().bfloat16(),
            torch.tensor(labs, dtype=torch.int64, device="cuda"), ob.TeacherMode.Tied)
    kw = dict(teacher_hidden=torch.from_numpy(t.hidden.a).cuda().bfloat16(), opts=opts)
    before = cudart.cudaDeviceGetLimit(cudart.cudaLimit.cudaLimitPersistingL2CacheSize)[1]
    with DeviceContext(0) as ctx:
        a = distillation_loss_device(ctx, *args, **kw)
        torch.cuda.synchronize()
    ctx = DeviceContext(0)
    granted = ctx.set_l2_persisting(64 << 20)
    assert granted > 0  # the driver rounds the request to its granularity
    assert cudart.cudaDeviceGetLimit(cudart.cudaLimit.cudaLimitPersistingL2CacheSize)[1] == granted
    b = distillation_loss_device(ctx, *args, **kw)
    torch.cuda.synchronize()
    ctx.check()
    ctx.close()
    assert cudart.cudaDeviceGetLimit(cudart.cudaLimit.cudaLimitPersistingL2CacheSize)[1] == before
    assert torch.equal(a.scalars, b.scalars)
    assert torch.equal(a.grad_weight, b.grad_weight)
    assert torch.equal(a.grad_student_hidden, b.grad_student_hidden)


# ------------------------------------------------------------ edge cases

@pytest.mark.parametrize("case", ["large_logits", "single_row", "same_label", "odd_vocab"])
def test_edge_cases_match_oracle(ob, oracle, case):
    """large_logits: logits of magnitude ~50 (softmax far in saturation, the
    online merge of per-part statistics and ex2.approx must stay exact to the
    tolerance); single_row: BT = 1; same_label: every row has the same label
    (one target row for the INT8 round trip, stochastic); odd_vocab: V = 1001
    (not a multiple of 8: unvectorised gradient path, ragged last tile)."""
    gen = torch.Generator().manual_seed(sum(map(ord, case)))  # fixed per case (str hash is salted)
    bt, h, v = 64, 256, 4096
    w_std, h_std = 0.02, 1.0
    cfg = ob.KernelConfig()
    if case == "large_logits":
        w_std, h_std = 0.25, 2.0
    elif case == "single_row":
        bt = 1
    elif case == "same_label":
        cfg = ob.KernelConfig(quantize_grad_weight=True, stochastic_rounding=True, stochastic_seed=7)
    elif case == "odd_vocab":
        v = 1001
    hs = randn_mat(ob, bt, h, gen, h_std)
    ht = randn_mat(ob, bt, h, gen, h_std)
    w = randn_mat(ob, v, h, gen, w_std)
    labs = torch.randint(0, v, (bt,), generator=gen).tolist()
    if case == "same_label":
        labs = [17] * bt
    opts = ob.LossOptions(kd_weight=0.4, temperature=1.5, label_smoothing=0.05, config=cfg)
    t = ob.Teacher.Tied(ht)
    g = ob.distillation_loss(hs, w, labs, t, opts)
    r = oracle.distillation_loss(hs, w, labs, t, opts, nthreads=NT)
    if case == "same_label":
        # INT8: compare the non-target rows within one quantisation step of the
        # oracle's (the fp32 grad_W differs in the last bits, so codes may move
        # by one); the target row is kept exact in both
        for name in ("loss", "student_ce", "teacher_ce", "kl"):
            a, b = getattr(g, name), getattr(r, name)
            assert abs(a - b) <= LOSS_RTOL * abs(b) + LOSS_ATOL, f"{name}: gpu {a!r} ref {b!r}"
        assert rel_l2(g.grad_weight.a, r.grad_weight.a) < 2e-2
        assert rel_l2(g.grad_weight.a[17], r.grad_weight.a[17]) < GRAD_REL_L2
        return
    assert_parity(g, r, case)


# ------------------------------------------------- host entry copy pipeline

@pytest.mark.parametrize("quantize", [False, True])
def test_host_entry_slab_pipeline_matches_oracle(ob, oracle, quantize):
    """orda_distillation_loss with the teacher-logit copy pipeline engaged
    (slabs shrunk to 512 KiB, so 256 rows x V=4096 f32 run as 8 forward /
    backward groups of 32 rows while later slabs are in flight): parity with
    the oracle, and with the same call in one group (grad_W summed over the
    groups in another fp32 order: rel-L2 1e-5)."""
    lib = ob.load_library()
    gen = torch.Generator().manual_seed(404)
    bt, h, v = 256, 256, 4096
    s = randn_mat(ob, bt, h, gen)
    w = randn_mat(ob, v, h, gen, 0.05)
    tl = ob.Mat.from_array((np.sqrt(2.0) * torch.randn(bt, v, generator=gen)).numpy())
    labs = torch.randint(0, v, (bt,), generator=gen).tolist()
    labs[3] = labs[100] = -100
    t = ob.Teacher.Precomputed(tl)
    opts = ob.LossOptions(kd_weight=0.4, temperature=1.5, label_smoothing=0.05, chunk_size=ob.ChunkSize.Fixed(32),
                          config=ob.KernelConfig(quantize_grad_weight=quantize))
    try:
        lib.orda_set_host_slab_bytes(512 << 10)
        piped = ob.distillation_loss(s, w, labs, t, opts)
    finally:
        lib.orda_set_host_slab_bytes(0)
    whole = ob.distillation_loss(s, w, labs, t, opts)
    assert piped.chunk_plan == ob.ChunkPlan(32, 8)
    assert abs(piped.loss - whole.loss) <= 1e-6 * abs(whole.loss)
    assert rel_l2(piped.grad_student_hidden.a, whole.grad_student_hidden.a) < 1e-6
    if quantize:
        # codes may move by one where the summation order changes a scale
        assert rel_l2(piped.grad_weight.a, whole.grad_weight.a) < 1e-2
    else:
        assert rel_l2(piped.grad_weight.a, whole.grad_weight.a) < 1e-5
    assert_parity(piped, oracle.distillation_loss(s, w, labs, t, opts, nthreads=NT), "pipelined")


@pytest.mark.parametrize("mode,h,stochastic", [("Precomputed", 256, False), ("Tied", 250, True)])
def test_host_entry_compressed_grad_w_download_is_bit_identical(ob, monkeypatch, mode, h, stochastic):
    """With the INT8 round trip the host-Mat entry copies grad_W back as its
    INT8 codes, row scales and exact target rows and forms q * s on the host;
    the result equals the fp32 download (ORDA_HOST_DEQUANT=0) bit for bit,
    with ignored and repeated labels, an odd H (scalar row gather) and a Tied
    teacher whose CE term adds to grad_W."""
    gen = torch.Generator().manual_seed(505)
    bt, v = 192, 5000
    s = randn_mat(ob, bt, h, gen)
    w = randn_mat(ob, v, h, gen, 0.05)
    labs = torch.randint(0, v, (bt,), generator=gen).tolist()
    labs[5] = labs[6] = -100
    labs[11] = labs[10]
    if mode == "Tied":
        t = ob.Teacher.Tied(randn_mat(ob, bt, h, gen))
        extra = dict(teacher_ce_weight=0.5)
    else:
        t = ob.Teacher.Precomputed(ob.Mat.from_array((np.sqrt(2.0) * torch.randn(bt, v, generator=gen)).numpy()))
        extra = {}
    cfg = ob.KernelConfig(quantize_grad_weight=True, stochastic_rounding=stochastic,
                          stochastic_seed=7 if stochastic else None)
    opts = ob.LossOptions(kd_weight=0.4, temperature=1.5, config=cfg, **extra)
    res = {}
    for flag in ("1", "0"):
        monkeypatch.setenv("ORDA_HOST_DEQUANT", flag)
        res[flag] = ob.distillation_loss(s, w, labs, t, opts)
    a, b = res["1"], res["0"]
    assert np.array_equal(a.grad_weight.a.view(np.uint32), b.grad_weight.a.view(np.uint32))
    assert np.array_equal(a.grad_student_hidden.a, b.grad_student_hidden.a)
    assert (a.loss, a.student_ce, a.teacher_ce, a.kl) == (b.loss, b.student_ce, b.teacher_ce, b.kl)
    # not vacuous: non-target rows lie on the INT8 grid of their row scale
    gw = a.grad_weight.a.astype(np.float64)
    rows = [r for r in range(v) if r not in set(labs)][:50]
    for r in rows:
        sc = max(np.abs(gw[r]).max(), 1e-30) / 127.0
        assert np.allclose(gw[r] / sc, np.round(gw[r] / sc), atol=1e-3)


@pytest.mark.parametrize("teacher", ["bf16_values", "fp32_values", "mixed"])
def test_host_entry_bf16_uploads_are_bit_identical(ob, monkeypatch, teacher):
    """The host-Mat entry rounds hidden states and weights to bf16 on the host
    (the device's rounding, ties to even: W holds exact ties here) and sends
    teacher-logit chunks of bf16 values as bf16, widened exactly on the
    device; any other chunk, and every chunk after it, crosses as fp32. Each
    case, with every chunk through the host passes (ORDA_HOST_CONVERT=2; by
    default a chunk crosses as fp32 whenever the copy engine is idle), equals
    the same call with the device-side conversion (ORDA_HOST_CONVERT=0) bit
    for bit. V = 70000 gives chunks of 479 rows,
    so 1024 rows take three; "mixed" turns inexact from row 500 on (inside
    the second chunk)."""
    gen = torch.Generator().manual_seed(606)
    bt, h, v = 1024, 128, 70000
    s_ = randn_mat(ob, bt, h, gen)
    wa = (0.05 * torch.randn(v, h, generator=gen)).numpy()
    bits = wa.view(np.uint32)
    bits[:64, :8] = (bits[:64, :8] & 0xFFFF0000) | 0x8000  # exact ties between two bf16 values
    w = ob.Mat.from_array(wa)
    tl = (np.sqrt(2.0) * torch.randn(bt, v, generator=gen)).numpy().astype(np.float32)
    assert tl.dtype == np.float32  # the bit masking below works on fp32 words
    if teacher in ("bf16_values", "mixed"):
        tb = tl.view(np.uint32)
        r1 = bt if teacher == "bf16_values" else 500
        tb[:r1] &= 0xFFFF0000
    t = ob.Teacher.Precomputed(ob.Mat.from_array(tl))
    labs = torch.randint(0, v, (bt,), generator=gen).tolist()
    opts = ob.LossOptions(kd_weight=0.4, temperature=1.5, config=ob.KernelConfig(quantize_grad_weight=True))
    res, moved = {}, {}
    lib = ob.load_library()
    up, down = C.c_uint64(0), C.c_uint64(0)
    for flag in ("2", "1", "0"):  # 2: every chunk through the host conversion; 1: the default split
        monkeypatch.setenv("ORDA_HOST_CONVERT", flag)
        res[flag] = ob.distillation_loss(s_, w, labs, t, opts)
        lib.orda_last_call_bytes(C.byref(up), C.byref(down))
        moved[flag] = up.value
    # bytes over PCIe as counted by the library: labels, the exact-row index
    # of the compressed download, then h and W (bf16 or fp32) and the teacher
    # logits (bf16 for the chunks of bf16 values before the first other one)
    fixed = bt * 8 + 4 * len({x for x in labs if x != -100})
    assert moved["0"] == fixed + (bt * h + v * h + bt * v) * 4
    bf16_rows = {"bf16_values": bt, "fp32_values": 0, "mixed": 479}[teacher]
    assert moved["2"] == fixed + (bt * h + v * h) * 2 + bf16_rows * v * 2 + (bt - bf16_rows) * v * 4
    assert moved["2"] <= moved["1"] <= moved["0"]
    b = res["0"]
    for a in (res["2"], res["1"]):
        assert (a.loss, a.student_ce, a.teacher_ce, a.kl) == (b.loss, b.student_ce, b.teacher_ce, b.kl)
        assert np.array_equal(a.grad_student_hidden.a.view(np.uint32), b.grad_student_hidden.a.view(np.uint32))
        assert np.array_equal(a.grad_weight.a.view(np.uint32), b.grad_weight.a.view(np.uint32))


# ------------------------------------------------------------ Profile::Fast

# Stated tolerances of Profile::Fast (include/orda.h, OrdaProfile): the CE
# terms come from the fp32 statistics and exact label logits (as Balanced);
# the KL cross term and the logit gradients read fp16 logits.
FAST_CE_RTOL = 1e-4
FAST_KL_RTOL = 1e-3
FAST_GRAD_REL_L2 = 2e-2


def assert_parity_fast(gpu, ref, what=""):
    for name, tol in (("student_ce", FAST_CE_RTOL), ("teacher_ce", FAST_CE_RTOL), ("kl", FAST_KL_RTOL),
                      ("loss", FAST_KL_RTOL)):
        a, b = getattr(gpu, name), getattr(ref, name)
        assert abs(a - b) <= tol * abs(b) + LOSS_ATOL, f"{what} {name}: gpu {a!r} ref {b!r}"
    for name in ("grad_student_hidden", "grad_weight", "grad_teacher_hidden", "grad_teacher_weight"):
        a, b = getattr(gpu, name), getattr(ref, name)
        assert (a is None) == (b is None), f"{what} {name} presence differs"
        if a is not None:
            e = rel_l2(a.a, b.a)
            assert e <= FAST_GRAD_REL_L2, f"{what} {name}: rel L2 {e:.3e}"
    assert gpu.chunk_plan == ref.chunk_plan


@pytest.mark.parametrize("case", ["tied", "separate", "precomputed", "piped"])
def test_wide_tiles_match_oracle(ob, oracle, monkeypatch, case):
    """Every store-epilogue GEMM on wide 256 x 512 pair tiles
    (ORDA_GEMM_WIDE=2; by default only the large ones take them): student and
    teacher dgrad (one tile, split into two K halves), wgrad (16 tiles, split),
    the Tied wgrad over two K segments (not split), the Separate teacher's
    H_t = 384 (an N tail inside the wide tile), and in "piped" the host entry
    in 3 forward groups whose wgrads reduce-add into grad_W (not split)."""
    monkeypatch.setenv("ORDA_GEMM_WIDE", "2")
    gen = torch.Generator().manual_seed(sum(map(ord, case)) + 11)
    bt, h, ht_, v = 96, 512, 384, 4096
    s = randn_mat(ob, bt, h, gen)
    w = randn_mat(ob, v, h, gen, 0.05)
    labs = torch.randint(0, v, (bt,), generator=gen).tolist()
    labs[9] = -100
    kw = dict(kd_weight=0.4, temperature=1.5, label_smoothing=0.05,
              config=ob.KernelConfig(quantize_grad_weight=True))
    if case == "separate":
        t = ob.Teacher.Separate(randn_mat(ob, bt, ht_, gen), randn_mat(ob, v, ht_, gen, 0.05))
        kw["teacher_ce_weight"] = 0.5
    elif case in ("precomputed", "piped"):
        t = ob.Teacher.Precomputed(ob.Mat.from_array((np.sqrt(2.0) * torch.randn(bt, v, generator=gen)).numpy()))
    else:
        t = ob.Teacher.Tied(randn_mat(ob, bt, h, gen))
        kw["teacher_ce_weight"] = 0.5
    if case == "piped":
        kw["chunk_size"] = ob.ChunkSize.Fixed(32)
    opts = ob.LossOptions(**kw)
    lib = ob.load_library()
    try:
        if case == "piped":
            lib.orda_set_host_slab_bytes(512 << 10)
        g = ob.distillation_loss(s, w, labs, t, opts)
    finally:
        lib.orda_set_host_slab_bytes(0)
    # the INT8 codes of grad_W may differ by one step where a scale moves, so
    # grad_W is compared within the bf16 gradient tolerance
    assert_parity(g, oracle.distillation_loss(s, w, labs, t, opts, nthreads=NT), case)


@pytest.mark.parametrize("case", ["tied", "separate", "precomputed", "large_logits", "odd_vocab"])
def test_fast_profile_matches_oracle_and_differs_from_balanced(ob, oracle, case):
    """Profile::Fast (config.rs:35-42, 81-93): fp16 logits storage, exact label
    logits, part of the epilogue's exp2 on the FMA pipe; within its stated
    tolerances of the oracle, and not byte-identical to Balanced."""
    gen = torch.Generator().manual_seed(sum(map(ord, case)) + 1)
    bt, h, ht_, v = 96, 256, 192, 4096
    w_std, h_std = 0.05, 1.0
    if case == "large_logits":
        w_std, h_std = 0.25, 2.0
    if case == "odd_vocab":
        v = 1001
    s = randn_mat(ob, bt, h, gen, h_std)
    w = randn_mat(ob, v, h, gen, w_std)
    labs = torch.randint(0, v, (bt,), generator=gen).tolist()
    labs[7] = -100
    kw = dict(kd_weight=0.4, temperature=1.5, label_smoothing=0.05)
    if case == "separate":
        t = ob.Teacher.Separate(randn_mat(ob, bt, ht_, gen), randn_mat(ob, v, ht_, gen, 0.05))
        kw["teacher_ce_weight"] = 0.5
    elif case == "precomputed":
        t = ob.Teacher.Precomputed(ob.Mat.from_array((np.sqrt(2.0) * torch.randn(bt, v, generator=gen)).numpy()))
        kw["teacher_ce_weight"] = 0.3
    else:
        t = ob.Teacher.Tied(randn_mat(ob, bt, h, gen, h_std))
    fast = ob.LossOptions(config=ob.KernelConfig.from_profile(ob.Profile.Fast), **kw)
    bal = ob.LossOptions(**kw)
    assert fast.config.fast_math and not bal.config.fast_math
    g = ob.distillation_loss(s, w, labs, t, fast)
    r = oracle.distillation_loss(s, w, labs, t, fast, nthreads=NT)
    assert_parity_fast(g, r, case)
    b = ob.distillation_loss(s, w, labs, t, bal)
    assert not np.array_equal(g.grad_weight.a, b.grad_weight.a)
    # the CE terms share Balanced's fp32 statistics and exact label logits
    assert abs(g.student_ce - b.student_ce) <= 1e-6 * abs(b.student_ce) + 1e-7


def test_exp2_fma_accuracy_on_device(ob):
    """The Fast profile's FMA-pipe exp2 against float64 2^x over its range
    [-125, 126]: within 2 ulp (the SFU's ex2.approx is reported beside it)."""
    from orda_b200 import _abi

    lib = ob.load_library()
    x = torch.cat([torch.linspace(-125.0, 126.0, 1 << 20), torch.rand(1 << 20) * -40.0,
                   torch.arange(-125, 126, dtype=torch.float32) + 0.5]).cuda()
    yf, ys = torch.empty_like(x), torch.empty_like(x)
    buf = _abi.err_buf()
    rc = lib.orda_selftest_exp2(x.data_ptr(), yf.data_ptr(), ys.data_ptr(), x.numel(),
                                torch.cuda.current_stream().cuda_stream, buf, len(buf))
    assert rc == 0, buf.value
    torch.cuda.synchronize()
    ref = torch.exp2(x.double())
    ef = ((yf.double() / ref) - 1.0).abs().max().item()
    es = ((ys.double() / ref) - 1.0).abs().max().item()
    assert ef < 2 * 2.0 ** -23, (ef, es)


def test_concurrent_schedule_is_bit_identical_to_serial(ob):
    """orda_context_set_concurrency: teacher statistics beside the logits GEMM
    and the INT8 round trip beside dgrad (on an auxiliary stream, the GEMMs on
    all SMs but the spare ones) give the same bits as the serial schedule."""
    from orda_b200.device import DeviceContext, distillation_loss_device

    gen = torch.Generator(device="cuda").manual_seed(77)
    bt, h, v = 512, 512, 8192
    hs = torch.randn(bt, h, generator=gen, device="cuda").bfloat16()
    w = (0.02 * torch.randn(v, h, generator=gen, device="cuda")).bfloat16()
    tl = (2.0 ** 0.5 * torch.randn(bt, v, generator=gen, device="cuda")).bfloat16()
    labels = torch.randint(0, v, (bt,), generator=gen, device="cuda")
    opts = ob.LossOptions(kd_weight=0.4, temperature=1.5, config=ob.KernelConfig(quantize_grad_weight=True))
    res = []
    with DeviceContext(0) as ctx:
        for spare in (0, 4, 8, 0):
            ctx.set_concurrency(spare)
            r = distillation_loss_device(ctx, hs, w, labels, ob.TeacherMode.Precomputed, teacher_logits=tl,
                                         opts=opts, want_int8=True)
            torch.cuda.synchronize()
            ctx.check()
            res.append(r)
    for r in res[1:]:
        for name in ("scalars", "grad_student_hidden", "grad_weight", "grad_weight_q", "grad_weight_scale"):
            assert torch.equal(getattr(r, name), getattr(res[0], name)), name
