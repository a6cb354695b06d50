"""Python binding of the CPU parity oracle (liborda_oracle.so).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the
CPU-baseline legs of bench.py, as the checker or as the timed CPU baseline of
the reference's CPU path. It is never part of the product path.

Each function mirrors the reference item named in its docstring (paths inside
malcolmgreaves/orda-cutile-rs). Types (`Mat`, `Teacher`, `LossOptions`) are
the orda_b200 mirrors so the same test inputs feed both sides.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parent
sys.path.insert(0, str(REPO / "orda-cutile-rs_b200"))

import orda_b200 as ob  # noqa: E402
from orda_b200 import _abi  # noqa: E402

LIB_PATH = HERE / "liborda_oracle.so"
_LIB = None

f32p = C.POINTER(C.c_float)
f64p = C.POINTER(C.c_double)
i64p = C.POINTER(C.c_int64)
i8p = C.POINTER(C.c_int8)
szp = C.POINTER(C.c_size_t)


def build() -> Path:
    """Compiles the oracle with its Makefile (IEEE flags, OpenMP)."""
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB_PATH


def lib():
    global _LIB
    if _LIB is None:
        if not LIB_PATH.exists():
            build()
        L = C.CDLL(str(LIB_PATH))
        sig = {
            "oref_matmul_nt": (None, [f32p, f32p, f32p, C.c_size_t, C.c_size_t, C.c_size_t, C.c_int]),
            "oref_matmul_nn": (None, [f32p, f32p, f32p, C.c_size_t, C.c_size_t, C.c_size_t, C.c_int]),
            "oref_matmul_tn": (None, [f32p, f32p, f32p, C.c_size_t, C.c_size_t, C.c_size_t, C.c_int]),
            "oref_softmax_logsoftmax": (None, [f32p, C.c_size_t, C.c_double, f64p, f64p]),
            "oref_forward_kl_row": (C.c_double, [f32p, f32p, C.c_size_t, C.c_double]),
            "oref_kl_chunk": (
                C.c_float,
                [f32p, C.c_size_t, i64p, C.c_size_t, C.c_float, C.c_float, C.c_int64, C.c_float, f32p, C.c_int],
            ),
            "oref_ce_fwdbwd_row": (C.c_float, [f32p, C.c_size_t, C.c_int64, C.c_int64, C.c_float, C.c_float, f32p]),
            "oref_chunks_from_raw": (C.c_size_t, [C.c_double]),
            "oref_resolve_chunk_size": (
                None,
                [C.c_size_t, C.c_int, C.c_size_t, C.c_int, C.c_size_t, C.c_int, C.c_size_t,
                 C.POINTER(_abi.OrdaChunkPlan)],
            ),
            "oref_default_max_chunks_limit": (C.c_size_t, [C.c_size_t]),
            "oref_chunk_doubling_schedule": (C.c_size_t, [C.c_size_t, C.c_size_t, C.c_size_t, szp, C.c_size_t]),
            "oref_rng_f32_stream": (None, [C.c_uint64, f32p, C.c_size_t]),
            "oref_round_half_even": (C.c_float, [C.c_float]),
            "oref_quantize_rowwise_int8": (None, [f32p, C.c_size_t, C.c_size_t, i8p, f32p, C.c_int]),
            "oref_quantize_rowwise_int8_stochastic": (None, [f32p, C.c_size_t, C.c_size_t, C.c_uint64, i8p, f32p]),
            "oref_unique_targets": (C.c_size_t, [i64p, C.c_size_t, C.c_int64, C.c_size_t, szp]),
            "oref_quantize_grad_w": (
                None,
                [f32p, C.c_size_t, C.c_size_t, i64p, C.c_size_t, C.c_int64, C.c_int, C.c_uint64, C.c_float, i8p,
                 f32p, f32p, C.c_int],
            ),
            "oref_is_power_of_two": (C.c_int, [C.c_size_t]),
            "oref_kernel_config_from_profile": (None, [C.c_int, C.POINTER(_abi.OrdaKernelConfig)]),
            "oref_loss_options_default": (None, [C.POINTER(_abi.OrdaLossOptions)]),
            "oref_kernel_config_validate": (C.c_int, [C.POINTER(_abi.OrdaKernelConfig), C.c_char_p, C.c_size_t]),
            "oref_default_teacher_ce_weight": (C.c_float, [C.c_int]),
            "oref_validate": (
                C.c_int,
                [C.POINTER(_abi.OrdaMatF32), C.POINTER(_abi.OrdaMatF32), i64p, C.c_size_t,
                 C.POINTER(_abi.OrdaTeacher), C.POINTER(_abi.OrdaLossOptions), szp, szp, szp, C.c_char_p,
                 C.c_size_t],
            ),
            "oref_distillation_loss": (
                C.c_int,
                [C.POINTER(_abi.OrdaMatF32), C.POINTER(_abi.OrdaMatF32), i64p, C.c_size_t,
                 C.POINTER(_abi.OrdaTeacher), C.POINTER(_abi.OrdaLossOptions), C.c_int, f32p, f32p, f32p, f32p,
                 f32p, C.POINTER(C.c_int), C.POINTER(C.c_int), f32p, C.POINTER(_abi.OrdaChunkPlan), C.c_char_p,
                 C.c_size_t],
            ),
            "oref_forward_loss_f64": (
                C.c_int,
                [C.POINTER(_abi.OrdaMatF32), C.POINTER(_abi.OrdaMatF32), i64p, C.c_size_t,
                 C.POINTER(_abi.OrdaTeacher), C.POINTER(_abi.OrdaLossOptions), f32p, f64p, C.c_char_p,
                 C.c_size_t],
            ),
            "oref_teacher_logits": (None, [C.POINTER(_abi.OrdaTeacher), C.POINTER(_abi.OrdaMatF32), f32p, C.c_int]),
            "oref_lcg_fill": (None, [f32p, C.c_size_t, C.c_uint64, C.c_float]),
            "oref_format_f32": (None, [C.c_float, C.c_char_p, C.c_size_t]),
            "oref_max_threads": (C.c_int, []),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _LIB = L
    return _LIB


def _f(a):
    return a.ctypes.data_as(f32p)


def _c32(a):
    return np.ascontiguousarray(np.asarray(a, dtype=np.float32))


def max_threads() -> int:
    return int(lib().oref_max_threads())


# ------------------------------------------------------------------ mat.rs
def matmul_nt(a, b, nthreads=1):
    """`matmul_nt` src/mat.rs:63-80."""
    a, b = _c32(a), _c32(b)
    out = np.empty((a.shape[0], b.shape[0]), np.float32)
    lib().oref_matmul_nt(_f(a), _f(b), _f(out), a.shape[0], a.shape[1], b.shape[0], nthreads)
    return out


def matmul_nn(a, b, nthreads=1):
    """`matmul_nn` src/mat.rs:86-105."""
    a, b = _c32(a), _c32(b)
    out = np.empty((a.shape[0], b.shape[1]), np.float32)
    lib().oref_matmul_nn(_f(a), _f(b), _f(out), a.shape[0], a.shape[1], b.shape[1], nthreads)
    return out


def matmul_tn(a, b, nthreads=1):
    """`matmul_tn` src/mat.rs:111-130 (a [k,m], b [k,n])."""
    a, b = _c32(a), _c32(b)
    out = np.empty((a.shape[1], b.shape[1]), np.float32)
    lib().oref_matmul_tn(_f(a), _f(b), _f(out), a.shape[0], a.shape[1], b.shape[1], nthreads)
    return out


# ---------------------------------------------------------- reference/kl.rs
def softmax_logsoftmax(x, inv_t):
    """`softmax_logsoftmax` src/reference/kl.rs:20-41."""
    x = _c32(x)
    p = np.empty(x.size, np.float64)
    lp = np.empty(x.size, np.float64)
    lib().oref_softmax_logsoftmax(_f(x), x.size, inv_t, p.ctypes.data_as(f64p), lp.ctypes.data_as(f64p))
    return p, lp


def forward_kl_row(s, t, temperature):
    """`forward_kl_row` src/reference/kl.rs:45-54."""
    s, t = _c32(s), _c32(t)
    return float(lib().oref_forward_kl_row(_f(s), _f(t), s.size, temperature))


def kl_chunk(logits, targets, n_rows, kl_weight, temperature, ignore_index, grad_denom, compute_grad, nthreads=1):
    """`kl_chunk` src/reference/kl.rs:66-127 -> (f32 kl sum, grad or None)."""
    logits = _c32(logits)
    tg = np.ascontiguousarray(np.asarray(targets, dtype=np.int64))
    v = logits.shape[1]
    grad = np.empty((n_rows, v), np.float32) if compute_grad else None
    kl = lib().oref_kl_chunk(
        _f(logits), v, tg.ctypes.data_as(i64p), n_rows, kl_weight, temperature, ignore_index, grad_denom,
        _f(grad) if grad is not None else None, nthreads,
    )
    return np.float32(kl), grad


def kl_reference_chunk(logits, targets, n_rows, kl_weight, temperature, n_non_ignore, ignore_index, compute_grad):
    """`kl_reference_chunk` src/reference/kl.rs:132-153."""
    denom = np.float32(max(n_non_ignore, 1))
    return kl_chunk(logits, targets, n_rows, kl_weight, temperature, ignore_index, denom, compute_grad)


# ------------------------------------------------ reference/cross_entropy.rs
def ce_fwdbwd_row(x, y, ignore_index, label_smoothing, scale):
    """`ce_fwdbwd_row` src/reference/cross_entropy.rs:20-74."""
    x = _c32(x).copy()
    g = np.empty_like(x)
    nll = lib().oref_ce_fwdbwd_row(_f(x), x.size, y, ignore_index, label_smoothing, scale, _f(g))
    return np.float32(nll), g


def ce_loss_row(x, y, ignore_index, label_smoothing):
    """`ce_loss_row` src/reference/cross_entropy.rs:77-79."""
    return ce_fwdbwd_row(x, y, ignore_index, label_smoothing, 1.0)[0]


# ------------------------------------------------------------- resolver.rs
def chunks_from_raw(raw):
    return int(lib().oref_chunks_from_raw(raw))


def resolve_chunk_size(bt, chunk_size: "ob.ChunkSize", v=None, max_chunks=None):
    p = _abi.OrdaChunkPlan()
    lib().oref_resolve_chunk_size(
        bt, int(chunk_size.fixed is not None), int(chunk_size.fixed or 0), int(v is not None), int(v or 0),
        int(max_chunks is not None), int(max_chunks or 0), C.byref(p),
    )
    return ob.ChunkPlan(int(p.chunk_size), int(p.num_chunks))


def default_max_chunks_limit(bt):
    return int(lib().oref_default_max_chunks_limit(bt))


def chunk_doubling_schedule(bt, start, limit):
    cap = 128
    arr = (C.c_size_t * cap)()
    n = int(lib().oref_chunk_doubling_schedule(bt, start, limit, arr, cap))
    return [int(arr[i]) for i in range(min(n, cap))]


# ---------------------------------------------------------------- quant.rs
def rng_f32_stream(seed, n):
    out = np.empty(n, np.float32)
    lib().oref_rng_f32_stream(seed, _f(out), n)
    return out


def round_half_even(x):
    return float(lib().oref_round_half_even(x))


def quantize_rowwise_int8(m, nthreads=1):
    m = _c32(m)
    q = np.empty(m.shape, np.int8)
    s = np.empty(m.shape[0], np.float32)
    lib().oref_quantize_rowwise_int8(_f(m), m.shape[0], m.shape[1], q.ctypes.data_as(i8p), _f(s), nthreads)
    return q, s


def quantize_rowwise_int8_stochastic(m, seed):
    m = _c32(m)
    q = np.empty(m.shape, np.int8)
    s = np.empty(m.shape[0], np.float32)
    lib().oref_quantize_rowwise_int8_stochastic(_f(m), m.shape[0], m.shape[1], seed, q.ctypes.data_as(i8p), _f(s))
    return q, s


def unique_targets(target, ignore_index, rows):
    t = np.ascontiguousarray(np.asarray(target, dtype=np.int64))
    out = (C.c_size_t * max(t.size, 1))()
    n = int(lib().oref_unique_targets(t.ctypes.data_as(i64p), t.size, ignore_index, rows, out))
    return [int(out[i]) for i in range(n)]


def quantize_grad_w(grad_w, target, ignore_index, stochastic=False, seed=0, grad_output=1.0, nthreads=1):
    """`quantize_grad_w` + `dequantize_grad_w` src/quant.rs:157-202."""
    g = _c32(grad_w)
    t = np.ascontiguousarray(np.asarray(target, dtype=np.int64))
    q = np.empty(g.shape, np.int8)
    s = np.empty(g.shape[0], np.float32)
    deq = np.empty_like(g)
    lib().oref_quantize_grad_w(
        _f(g), g.shape[0], g.shape[1], t.ctypes.data_as(i64p), t.size, ignore_index, int(stochastic), seed,
        grad_output, q.ctypes.data_as(i8p), _f(s), _f(deq), nthreads,
    )
    return q, s, deq


# ------------------------------------------------------------------ api.rs
class OracleError(RuntimeError):
    def __init__(self, code, message):
        super().__init__(message)
        self.code = code
        self.message = message


def _labels(labels):
    lab = np.ascontiguousarray(np.asarray(labels, dtype=np.int64))
    return lab, lab.ctypes.data_as(i64p)


def validate(student_hidden, weight, labels, teacher, opts):
    lab, lp = _labels(labels)
    v, h, bt = C.c_size_t(), C.c_size_t(), C.c_size_t()
    buf = C.create_string_buffer(1024)
    rc = lib().oref_validate(
        C.byref(student_hidden._c()), C.byref(weight._c()), lp, lab.size, C.byref(teacher._c()),
        C.byref(opts._c()), C.byref(v), C.byref(h), C.byref(bt), buf, len(buf),
    )
    if rc:
        raise OracleError(rc, buf.value.decode())
    return int(v.value), int(h.value), int(bt.value)


def distillation_loss(student_hidden, weight, labels, teacher, opts=None, nthreads=1, return_raw_grad_w=False):
    """`distillation_loss` src/api.rs:188-422 (the reference CPU path)."""
    opts = opts or ob.LossOptions()
    lab, lp = _labels(labels)
    bt, h = student_hidden.shape()
    v = weight.rows
    ht = teacher.hidden.cols if teacher.kind == ob.TeacherMode.Separate else h
    gh = np.empty((bt, h), np.float32)
    gw = np.empty((v, h), np.float32)
    gth = np.empty((bt, ht), np.float32)
    gtw = np.empty((v, ht), np.float32)
    raw = np.empty((v, h), np.float32) if return_raw_grad_w else None
    sc = np.zeros(4, np.float32)
    has_t, has_w = C.c_int(), C.c_int()
    plan = _abi.OrdaChunkPlan()
    buf = C.create_string_buffer(1024)
    rc = lib().oref_distillation_loss(
        C.byref(student_hidden._c()), C.byref(weight._c()), lp, lab.size, C.byref(teacher._c()), C.byref(opts._c()),
        nthreads, _f(sc), _f(gh), _f(gw), _f(gth), _f(gtw), C.byref(has_t), C.byref(has_w),
        _f(raw) if raw is not None else None, C.byref(plan), buf, len(buf),
    )
    if rc:
        raise OracleError(rc, buf.value.decode())
    out = ob.DistillationLossOutput(
        loss=float(sc[0]),
        student_ce=float(sc[1]),
        teacher_ce=float(sc[2]),
        kl=float(sc[3]),
        grad_student_hidden=ob.Mat.from_array(gh),
        grad_weight=ob.Mat.from_array(gw),
        grad_teacher_hidden=ob.Mat.from_array(gth) if has_t.value else None,
        grad_teacher_weight=ob.Mat.from_array(gtw) if has_w.value else None,
        chunk_plan=ob.ChunkPlan(int(plan.chunk_size), int(plan.num_chunks)),
    )
    if return_raw_grad_w:
        return out, raw
    return out


def forward_loss_f64(student_hidden, weight, labels, teacher, opts, kl_teacher_logits=None):
    """`forward_loss_f64` src/api.rs:511-572."""
    lab, lp = _labels(labels)
    res = C.c_double()
    buf = C.create_string_buffer(1024)
    kt = _c32(kl_teacher_logits.a) if kl_teacher_logits is not None else None
    rc = lib().oref_forward_loss_f64(
        C.byref(student_hidden._c()), C.byref(weight._c()), lp, lab.size, C.byref(teacher._c()), C.byref(opts._c()),
        _f(kt) if kt is not None else None, C.byref(res), buf, len(buf),
    )
    if rc:
        raise OracleError(rc, buf.value.decode())
    return float(res.value)


def loss_only_f64(student_hidden, weight, labels, teacher, opts):
    """`loss_only_f64` src/api.rs:576-584."""
    return forward_loss_f64(student_hidden, weight, labels, teacher, opts, None)


def teacher_logits(teacher, weight, nthreads=1):
    """`teacher_logits` src/api.rs:490-496."""
    if teacher.kind == ob.TeacherMode.Precomputed:
        return teacher.logits.clone()
    rows = teacher.hidden.rows
    out = np.empty((rows, weight.rows), np.float32)
    lib().oref_teacher_logits(C.byref(teacher._c()), C.byref(weight._c()), _f(out), nthreads)
    return ob.Mat.from_array(out)


# ------------------------------------------------------------ test helpers
def lcg_fill(n, seed, scale):
    """`fill` of tests/end_to_end.rs:14-27 (and src/main.rs:11-24)."""
    out = np.empty(n, np.float32)
    lib().oref_lcg_fill(_f(out), n, seed, scale)
    return out


def e2e_labels(bt, v, ignore_every, ignore_index):
    """`labels` of tests/end_to_end.rs:29-36."""
    return [ignore_index if (ignore_every and i % ignore_every == 0) else (i * 7 + 3) % v for i in range(bt)]


def format_f32(x):
    buf = C.create_string_buffer(64)
    lib().oref_format_f32(x, buf, len(buf))
    return buf.value.decode()
