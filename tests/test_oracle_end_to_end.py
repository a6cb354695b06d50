"""Restates tests/end_to_end.rs of the reference against the CPU oracle.

The central check is the reference's finite-difference gradient test: the
analytic gradients of `distillation_loss` must match central differences of
the independent f64 forward `forward_loss_f64` (with the detached KL teacher),
for all three teacher modes. Plus chunk invariance, component consistency,
Sum vs Mean and the INT8 round trip. Data comes from the reference's LCG
`fill` and `labels` helpers (tests/end_to_end.rs:14-36).
"""
from __future__ import annotations

import numpy as np


def _mat(ob, oracle, rows, cols, seed, scale):
    return ob.Mat.from_vec(rows, cols, oracle.lcg_fill(rows * cols, seed, scale))


def check_grad(param, analytic, eps, atol, rtol, loss_at):
    """`check_grad` tests/end_to_end.rs:43-78."""
    assert param.shape() == analytic.shape()
    work = param.clone()
    max_rel = 0.0
    for idx in range(param.data.size):
        base = param.data[idx]
        work.data[idx] = np.float32(base + np.float32(eps))
        lp = loss_at(work)
        work.data[idx] = np.float32(base - np.float32(eps))
        lm = loss_at(work)
        work.data[idx] = base
        num = (lp - lm) / (2.0 * eps)
        ana = float(analytic.data[idx])
        assert abs(ana - num) <= atol + rtol * max(abs(ana), abs(num)), f"grad mismatch at {idx}: {ana} vs {num}"
        if max(abs(ana), abs(num)) > 1e-3:
            max_rel = max(max_rel, abs(ana - num) / max(abs(ana), abs(num)))
    assert max_rel < 0.05, f"max relative grad error too high: {max_rel}"


def base_opts(ob, **kw):
    """`base_opts` tests/end_to_end.rs:80-87."""
    d = dict(student_ce_weight=1.0, kd_weight=0.5, temperature=1.5)
    d.update(kw)
    return ob.LossOptions(**d)


def test_tied_teacher_gradients_match_finite_difference(ob, oracle):
    """tests/end_to_end.rs:89-128."""
    bt, h, v = 6, 5, 7
    student = _mat(ob, oracle, bt, h, 1, 0.3)
    weight = _mat(ob, oracle, v, h, 2, 0.2)
    t_hidden = _mat(ob, oracle, bt, h, 3, 0.3)
    labs = oracle.e2e_labels(bt, v, 4, -100)
    teacher = ob.Teacher.Tied(t_hidden.clone())
    opts = base_opts(ob, teacher_ce_weight=1.0, label_smoothing=0.1)
    out = oracle.distillation_loss(student, weight, labs, teacher, opts)
    kt = oracle.teacher_logits(teacher, weight)
    check_grad(student, out.grad_student_hidden, 1e-3, 1e-3, 1e-2,
               lambda s: oracle.forward_loss_f64(s, weight, labs, teacher, opts, kt))
    check_grad(weight, out.grad_weight, 1e-3, 1e-3, 1e-2,
               lambda w: oracle.forward_loss_f64(student, w, labs, teacher, opts, kt))
    assert out.grad_teacher_hidden is not None
    check_grad(t_hidden, out.grad_teacher_hidden, 1e-3, 1e-3, 1e-2,
               lambda th: oracle.forward_loss_f64(student, weight, labs, ob.Teacher.Tied(th.clone()), opts, kt))


def test_separate_teacher_gradients_match_finite_difference(ob, oracle):
    """tests/end_to_end.rs:130-178."""
    bt, h, ht, v = 6, 5, 4, 7
    student = _mat(ob, oracle, bt, h, 11, 0.3)
    weight = _mat(ob, oracle, v, h, 12, 0.2)
    t_hidden = _mat(ob, oracle, bt, ht, 13, 0.3)
    t_weight = _mat(ob, oracle, v, ht, 14, 0.2)
    labs = oracle.e2e_labels(bt, v, None, -100)
    opts = base_opts(ob, teacher_ce_weight=0.7)
    teacher = ob.Teacher.Separate(t_hidden.clone(), t_weight.clone())
    out = oracle.distillation_loss(student, weight, labs, teacher, opts)
    kt = oracle.teacher_logits(teacher, weight)
    check_grad(student, out.grad_student_hidden, 1e-3, 1e-3, 1e-2,
               lambda s: oracle.forward_loss_f64(s, weight, labs, teacher, opts, kt))
    check_grad(weight, out.grad_weight, 1e-3, 1e-3, 1e-2,
               lambda w: oracle.forward_loss_f64(student, w, labs, teacher, opts, kt))
    check_grad(t_hidden, out.grad_teacher_hidden, 1e-3, 1e-3, 1e-2,
               lambda th: oracle.forward_loss_f64(student, weight, labs, ob.Teacher.Separate(th.clone(), t_weight),
                                                  opts, kt))
    check_grad(t_weight, out.grad_teacher_weight, 1e-3, 1e-3, 1e-2,
               lambda tw: oracle.forward_loss_f64(student, weight, labs, ob.Teacher.Separate(t_hidden, tw.clone()),
                                                  opts, kt))


def test_precomputed_teacher_gradients_match_finite_difference(ob, oracle):
    """tests/end_to_end.rs:180-204."""
    bt, h, v = 6, 5, 7
    student = _mat(ob, oracle, bt, h, 21, 0.3)
    weight = _mat(ob, oracle, v, h, 22, 0.2)
    t_logits = _mat(ob, oracle, bt, v, 23, 0.5)
    labs = oracle.e2e_labels(bt, v, 5, -100)
    opts = base_opts(ob)
    teacher = ob.Teacher.Precomputed(t_logits.clone())
    out = oracle.distillation_loss(student, weight, labs, teacher, opts)
    assert out.grad_teacher_hidden is None
    assert out.grad_teacher_weight is None
    check_grad(student, out.grad_student_hidden, 1e-3, 1e-3, 1e-2,
               lambda s: oracle.loss_only_f64(s, weight, labs, teacher, opts))
    check_grad(weight, out.grad_weight, 1e-3, 1e-3, 1e-2,
               lambda w: oracle.loss_only_f64(student, w, labs, teacher, opts))


def test_pure_student_ce_no_teacher_term(ob, oracle):
    """tests/end_to_end.rs:206-228."""
    bt, h, v = 8, 4, 6
    student = _mat(ob, oracle, bt, h, 31, 0.3)
    weight = _mat(ob, oracle, v, h, 32, 0.2)
    labs = oracle.e2e_labels(bt, v, None, -100)
    teacher = ob.Teacher.Tied(ob.Mat.zeros(bt, h))
    opts = ob.LossOptions(kd_weight=0.0, teacher_ce_weight=0.0)
    out = oracle.distillation_loss(student, weight, labs, teacher, opts)
    assert out.teacher_ce == 0.0
    assert out.kl == 0.0
    check_grad(student, out.grad_student_hidden, 1e-3, 1e-3, 1e-2,
               lambda s: oracle.loss_only_f64(s, weight, labs, teacher, opts))


def test_chunking_is_exact_invariant(ob, oracle):
    """tests/end_to_end.rs:230-278."""
    bt, h, v = 16, 5, 9
    student = _mat(ob, oracle, bt, h, 41, 0.3)
    weight = _mat(ob, oracle, v, h, 42, 0.2)
    t_hidden = _mat(ob, oracle, bt, h, 43, 0.3)
    labs = oracle.e2e_labels(bt, v, 3, -100)
    teacher = ob.Teacher.Tied(t_hidden)

    def mk(cs):
        return oracle.distillation_loss(student, weight, labs, teacher, base_opts(ob, chunk_size=cs, teacher_ce_weight=1.0))

    full = mk(ob.ChunkSize.Fixed(bt))
    for other in (mk(ob.ChunkSize.Fixed(1)), mk(ob.ChunkSize.Fixed(3)), mk(ob.ChunkSize.Auto())):
        assert abs(full.loss - other.loss) < 1e-5
        assert np.all(np.abs(full.grad_weight.data - other.grad_weight.data) < 1e-5)
        assert np.all(np.abs(full.grad_student_hidden.data - other.grad_student_hidden.data) < 1e-5)


def test_loss_components_and_total_are_consistent(ob, oracle):
    """tests/end_to_end.rs:280-311."""
    bt, h, v = 10, 4, 8
    student = _mat(ob, oracle, bt, h, 51, 0.3)
    weight = _mat(ob, oracle, v, h, 52, 0.2)
    t_hidden = _mat(ob, oracle, bt, h, 53, 0.3)
    labs = oracle.e2e_labels(bt, v, None, -100)
    teacher = ob.Teacher.Tied(t_hidden)
    w_s, w_t, kd = np.float32(1.0), np.float32(0.8), np.float32(0.5)
    opts = ob.LossOptions(student_ce_weight=1.0, teacher_ce_weight=0.8, kd_weight=0.5, temperature=2.0)
    out = oracle.distillation_loss(student, weight, labs, teacher, opts)
    recon = w_s * np.float32(out.student_ce) + w_t * np.float32(out.teacher_ce) + kd * np.float32(out.kl)
    assert abs(recon - np.float32(out.loss)) < 1e-4
    orc = np.float32(oracle.loss_only_f64(student, weight, labs, teacher, opts))
    assert abs(orc - np.float32(out.loss)) < 1e-3


def test_sum_reduction_is_mean_times_token_count(ob, oracle):
    """tests/end_to_end.rs:313-358."""
    bt, h, v = 8, 4, 6
    student = _mat(ob, oracle, bt, h, 61, 0.3)
    weight = _mat(ob, oracle, v, h, 62, 0.2)
    t_hidden = _mat(ob, oracle, bt, h, 63, 0.3)
    labs = oracle.e2e_labels(bt, v, 4, -100)
    teacher = ob.Teacher.Tied(t_hidden)
    n_valid = np.float32(sum(1 for t in labs if t != -100))
    mean = oracle.distillation_loss(student, weight, labs, teacher,
                                    base_opts(ob, reduction=ob.Reduction.Mean, teacher_ce_weight=1.0))
    summ = oracle.distillation_loss(student, weight, labs, teacher,
                                    base_opts(ob, reduction=ob.Reduction.Sum, teacher_ce_weight=1.0))
    assert abs(np.float32(summ.loss) - np.float32(mean.loss) * n_valid) < 1e-3
    assert np.all(np.abs(summ.grad_weight.data - mean.grad_weight.data * n_valid) < 1e-3)


def test_int8_quant_grad_w_is_close_but_lossy(ob, oracle):
    """tests/end_to_end.rs:360-417."""
    bt, h, v = 8, 4, 20
    student = _mat(ob, oracle, bt, h, 71, 0.3)
    weight = _mat(ob, oracle, v, h, 72, 0.2)
    t_hidden = _mat(ob, oracle, bt, h, 73, 0.3)
    labs = oracle.e2e_labels(bt, v, None, -100)
    teacher = ob.Teacher.Tied(t_hidden)
    exact = oracle.distillation_loss(student, weight, labs, teacher, base_opts(ob, teacher_ce_weight=1.0))
    cfg = ob.KernelConfig(quantize_grad_weight=True)
    quant = oracle.distillation_loss(student, weight, labs, teacher, base_opts(ob, config=cfg, teacher_ce_weight=1.0))
    assert abs(exact.loss - quant.loss) < 1e-6
    max_abs = float(np.max(np.abs(exact.grad_weight.data - quant.grad_weight.data)))
    assert 0.0 < max_abs < 0.05


def test_oracle_thread_count_invariance(ob, oracle):
    """The threaded oracle (used for the CPU baseline and large parity cases)
    is bit-identical to the sequential restatement."""
    bt, h, v = 12, 16, 40
    student = _mat(ob, oracle, bt, h, 81, 0.5)
    weight = _mat(ob, oracle, v, h, 82, 0.3)
    t_hidden = _mat(ob, oracle, bt, h, 83, 0.5)
    labs = oracle.e2e_labels(bt, v, 5, -100)
    teacher = ob.Teacher.Tied(t_hidden)
    opts = base_opts(ob, teacher_ce_weight=1.0, label_smoothing=0.05, chunk_size=ob.ChunkSize.Fixed(5))
    a = oracle.distillation_loss(student, weight, labs, teacher, opts, nthreads=1)
    b = oracle.distillation_loss(student, weight, labs, teacher, opts, nthreads=4)
    assert a.loss == b.loss and a.kl == b.kl
    assert np.array_equal(a.grad_weight.data, b.grad_weight.data)
    assert np.array_equal(a.grad_student_hidden.data, b.grad_student_hidden.data)
    assert np.array_equal(a.grad_teacher_hidden.data, b.grad_teacher_hidden.data)


def test_demo_main_runs(ob, oracle):
    """The demo of src/main.rs:30-72 (Tied, BT=32, H=64, V=128, kd=0.4,
    T=1.5) runs and yields finite values with a 1 x 32 chunk plan."""
    bt, h, v = 32, 64, 128
    student = _mat(ob, oracle, bt, h, 1, 0.2)
    teacher = ob.Teacher.Tied(_mat(ob, oracle, bt, h, 2, 0.2))
    weight = _mat(ob, oracle, v, h, 3, 0.05)
    labs = [(i * 7) % v for i in range(bt)]
    out = oracle.distillation_loss(student, weight, labs, teacher, ob.LossOptions(kd_weight=0.4, temperature=1.5))
    assert (out.chunk_plan.num_chunks, out.chunk_plan.chunk_size) == (1, 32)
    assert np.isfinite(out.loss) and out.kl >= 0.0
    # near-uniform logits: CE close to ln(V)
    assert abs(out.student_ce - np.log(v)) < 0.05
