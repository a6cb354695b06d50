"""Device entry points of the C ABI for torch tensors (torch is used only for
device memory and streams; every computation runs in liborda_b200.so).
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass
from typing import Optional

import torch

from . import ChunkPlan, LossOptions, TeacherMode, _abi, _check
from ._abi import load_library


def _lib():
    return load_library()


class DeviceContext:
    """Owns an `OrdaContext` (device workspace + status word)."""

    def __init__(self, device: int = 0):
        self.device = device
        h = C.c_void_p()
        buf = _abi.err_buf()
        _check(_lib().orda_context_create(device, C.byref(h), buf, len(buf)), buf)
        self.handle = h

    def close(self) -> None:
        if self.handle:
            _lib().orda_context_destroy(self.handle)
            self.handle = C.c_void_p()

    def check(self) -> None:
        buf = _abi.err_buf()
        _check(_lib().orda_context_check(self.handle, buf, len(buf)), buf)

    def workspace_bytes(self) -> int:
        return int(_lib().orda_context_workspace_bytes(self.handle))

    def inject_alloc_failures(self, count: int) -> None:
        _lib().orda_context_inject_alloc_failures(self.handle, count)

    def enable_timing(self, on: bool = True) -> None:
        _lib().orda_context_enable_timing(self.handle, int(on))

    def reset_timing(self) -> None:
        _lib().orda_context_reset_timing(self.handle)

    def phase_times(self) -> dict:
        """Milliseconds and kernel launches per phase since the last reset
        (events recorded on the launch stream; synchronizes)."""
        ms = (C.c_double * _abi.NUM_PHASES)()
        n = (C.c_uint64 * _abi.NUM_PHASES)()
        _lib().orda_context_phase_times(self.handle, ms, n)
        return {name: (float(ms[i]), int(n[i])) for i, name in enumerate(_abi.PHASE_NAMES)}

    def set_concurrency(self, spare_sms: int) -> None:
        """`orda_context_set_concurrency`: SMs the persistent GEMMs leave to the
        teacher statistics and the INT8 quantiser running beside them on an
        auxiliary stream (0, the default = every kernel serial on the caller's
        stream)."""
        _lib().orda_context_set_concurrency(self.handle, int(spare_sms))

    def launch_count(self) -> int:
        return int(_lib().orda_context_launch_count(self.handle))

    def slots_create(self, world: int, rank: int, total_rows: int, h: int, copies: int = 1) -> bytes:
        """`orda_context_slots_create`: allocates this rank's slot buffer for
        `total_rows` rows split over the owners (shard.owner_rows; `copies`
        sets of [world][slice][h] fp32) for the fused reduce-scatters;
        returns its 64-byte IPC handle."""
        hd = _abi.OrdaIpcHandle()
        buf = _abi.err_buf()
        _check(_lib().orda_context_slots_create(self.handle, world, rank, total_rows, h, copies, C.byref(hd), buf,
                                                len(buf)), buf)
        return C.string_at(C.addressof(hd), C.sizeof(hd))

    def slots_attach(self, handles: list) -> None:
        """`orda_context_slots_attach` with every rank's handle, by rank."""
        arr = (_abi.OrdaIpcHandle * len(handles))()
        for i, b in enumerate(handles):
            b = bytes(b)
            if len(b) != C.sizeof(_abi.OrdaIpcHandle):
                raise ValueError(f"IPC handle {i} has {len(b)} bytes")
            C.memmove(C.addressof(arr[i]), b, len(b))
        buf = _abi.err_buf()
        _check(_lib().orda_context_slots_attach(self.handle, arr, buf, len(buf)), buf)

    def reduce_slots(self, grad_w_slice: torch.Tensor, labels: torch.Tensor, ignore_index: int = -100,
                     quantize: bool = False, stochastic: bool = False, seed: int = 0,
                     q: Optional[torch.Tensor] = None, scale: Optional[torch.Tensor] = None, stream=None,
                     int8_wire: bool = False) -> None:
        """`orda_reduce_slots_device`: this rank's grad_W rows, summed over
        the ranks' partials (and INT8 round trip when quantize); int8_wire
        when the partials were sent in the INT8 wire format."""
        buf = _abi.err_buf()
        _check(_lib().orda_reduce_slots_device(
            self.handle, grad_w_slice.data_ptr(), grad_w_slice.stride(0), labels.data_ptr(), labels.numel(),
            ignore_index, int(quantize), int(stochastic), seed, _ptr(q), _ptr(scale), int(int8_wire),
            _stream(stream), buf, len(buf)), buf)

    def reduce_slot_set(self, copy: int, out: torch.Tensor, stream=None) -> None:
        """`orda_reduce_slot_set_device`: rank-ordered sum of slot set `copy`."""
        buf = _abi.err_buf()
        _check(_lib().orda_reduce_slot_set_device(self.handle, copy, out.data_ptr(), out.stride(0), _stream(stream),
                                                  buf, len(buf)), buf)

    def set_l2_persisting(self, nbytes: int) -> int:
        """`orda_context_set_l2_persisting`: persisting-L2 carve-out for the
        evict-last GEMM operands; returns the bytes granted."""
        got = C.c_size_t()
        buf = _abi.err_buf()
        _check(_lib().orda_context_set_l2_persisting(self.handle, nbytes, C.byref(got), buf, len(buf)), buf)
        return int(got.value)

    def selftest_bounded_wait(self, limit_us: int = 50000, stream=None) -> None:
        """Runs the bounded-wait self-test kernel (a wait that expires)."""
        buf = _abi.err_buf()
        _check(_lib().orda_context_selftest_bounded_wait(self.handle, limit_us, _stream(stream), buf, len(buf)), buf)

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()


def dev_mat(t: Optional[torch.Tensor]) -> _abi.OrdaDeviceMat:
    m = _abi.OrdaDeviceMat()
    if t is None:
        return m
    if t.dim() != 2 or t.stride(1) != 1:
        raise ValueError("device matrices must be 2-D with unit column stride")
    if t.dtype == torch.bfloat16:
        m.dtype = _abi.DTYPE_BF16
    elif t.dtype == torch.float32:
        m.dtype = _abi.DTYPE_F32
    else:
        raise ValueError(f"unsupported dtype {t.dtype}")
    m.data = t.data_ptr()
    m.rows, m.cols = t.shape
    m.ld = t.stride(0)
    return m


def _ptr(t: Optional[torch.Tensor]):
    return None if t is None else t.data_ptr()


def _stream(stream) -> int:
    if stream is None:
        return torch.cuda.current_stream().cuda_stream
    if isinstance(stream, torch.cuda.Stream):
        return stream.cuda_stream
    return int(stream)


@dataclass
class DeviceLossResult:
    scalars: torch.Tensor  # device float[4]: loss, student_ce, teacher_ce, kl
    grad_student_hidden: Optional[torch.Tensor]
    grad_weight: Optional[torch.Tensor]
    grad_teacher_hidden: Optional[torch.Tensor]
    grad_teacher_weight: Optional[torch.Tensor]
    grad_weight_q: Optional[torch.Tensor]
    grad_weight_scale: Optional[torch.Tensor]
    chunk_plan: ChunkPlan


def _teacher_struct(teacher_mode, teacher_hidden, teacher_weight, teacher_logits):
    t = _abi.OrdaDeviceTeacher()
    t.mode = int(teacher_mode)
    t.hidden = dev_mat(teacher_hidden)
    t.weight = dev_mat(teacher_weight)
    t.logits = dev_mat(teacher_logits)
    return t


def _outputs(opts, teacher_mode, bt, h, v, ht, dev, out, want_int8, with_grad_weight=True, with_grad_hidden=True):
    """Output tensors (from `out` or newly allocated) and their C struct."""
    w_t = opts.teacher_ce_weight
    if w_t is None:
        w_t = 1.0 if teacher_mode == TeacherMode.Tied else 0.0
    live = teacher_mode in (TeacherMode.Tied, TeacherMode.Separate)
    out = dict(out or {})
    f32 = dict(device=dev, dtype=torch.float32)
    gsh = out.get("grad_student_hidden") if with_grad_hidden else None
    if gsh is None and with_grad_hidden:
        gsh = torch.empty(bt, h, **f32)
    gw = out.get("grad_weight") if with_grad_weight else None
    if gw is None and with_grad_weight:
        gw = torch.empty(v, h, **f32)
    gth = out.get("grad_teacher_hidden") if with_grad_hidden else None
    if gth is None and w_t > 0 and live and with_grad_hidden:
        gth = torch.empty(bt, ht, **f32)
    gtw = out.get("grad_teacher_weight")
    if gtw is None and w_t > 0 and teacher_mode == TeacherMode.Separate:
        gtw = torch.empty(v, ht, **f32)
    q = out.get("grad_weight_q")
    sc = out.get("grad_weight_scale")
    if want_int8 and opts.config.quantize_grad_weight:
        if q is None:
            q = torch.empty(v, h, device=dev, dtype=torch.int8)
        if sc is None:
            sc = torch.empty(v, **f32)
    scal = out.get("scalars")
    if scal is None:
        scal = torch.empty(4, **f32)
    o = _abi.OrdaDeviceOutputs()
    if gsh is not None:
        o.grad_student_hidden = gsh.data_ptr()
        o.ld_grad_student_hidden = gsh.stride(0)
    if gw is not None:
        o.grad_weight = gw.data_ptr()
        o.ld_grad_weight = gw.stride(0)
    if gth is not None:
        o.grad_teacher_hidden = gth.data_ptr()
        o.ld_grad_teacher_hidden = gth.stride(0)
    if gtw is not None:
        o.grad_teacher_weight = gtw.data_ptr()
        o.ld_grad_teacher_weight = gtw.stride(0)
    o.grad_weight_q = _ptr(q)
    o.grad_weight_scale = _ptr(sc)
    o.scalars = scal.data_ptr()
    tensors = dict(scalars=scal, grad_student_hidden=gsh, grad_weight=gw, grad_teacher_hidden=gth,
                   grad_teacher_weight=gtw, grad_weight_q=q, grad_weight_scale=sc)
    return o, tensors


def distillation_loss_device(
    ctx: DeviceContext,
    student_hidden: torch.Tensor,
    weight: torch.Tensor,
    labels: torch.Tensor,
    teacher_mode: TeacherMode,
    teacher_hidden: Optional[torch.Tensor] = None,
    teacher_weight: Optional[torch.Tensor] = None,
    teacher_logits: Optional[torch.Tensor] = None,
    opts: Optional[LossOptions] = None,
    out: Optional[dict] = None,
    global_non_ignore: int = 0,
    skip_quantize: bool = False,
    want_int8: bool = False,
    stream=None,
    scatter_grad_weight: bool = False,
    int8_wire: bool = False,
) -> DeviceLossResult:
    """`orda_distillation_loss_device`: bf16 device inputs, fp32 device grads.
    With scatter_grad_weight the grad_W partial goes to the slot buffers
    (see DeviceContext.slots_create) and the returned grad_weight is None;
    int8_wire sends it there as row-wise INT8 codes and scales."""
    opts = opts or LossOptions()
    bt, h = student_hidden.shape
    v = weight.shape[0]
    ht = teacher_hidden.shape[1] if teacher_mode == TeacherMode.Separate else h
    o, tensors = _outputs(opts, teacher_mode, bt, h, v, ht, student_hidden.device, out, want_int8,
                          with_grad_weight=not scatter_grad_weight)
    t = _teacher_struct(teacher_mode, teacher_hidden, teacher_weight, teacher_logits)
    shard = _abi.OrdaShardOptions(int(global_non_ignore), int(skip_quantize), int(scatter_grad_weight),
                                  int(int8_wire), 0)
    plan = _abi.OrdaChunkPlan()
    buf = _abi.err_buf()
    rc = _lib().orda_distillation_loss_device(
        ctx.handle,
        C.byref(dev_mat(student_hidden)),
        C.byref(dev_mat(weight)),
        labels.data_ptr(),
        labels.numel(),
        C.byref(t),
        C.byref(opts._c()),
        C.byref(o),
        C.byref(shard),
        _stream(stream),
        C.byref(plan),
        buf,
        len(buf),
    )
    _check(rc, buf)
    return DeviceLossResult(chunk_plan=ChunkPlan(int(plan.chunk_size), int(plan.num_chunks)), **tensors)


def vocab_forward_device(
    ctx: DeviceContext,
    student_hidden: torch.Tensor,
    weight_slice: torch.Tensor,
    labels: torch.Tensor,
    teacher_mode: TeacherMode,
    v_total: int,
    v0: int,
    teacher_hidden: Optional[torch.Tensor] = None,
    teacher_weight_slice: Optional[torch.Tensor] = None,
    teacher_logits_slice: Optional[torch.Tensor] = None,
    opts: Optional[LossOptions] = None,
    partials: Optional[torch.Tensor] = None,
    stream=None,
) -> torch.Tensor:
    """`orda_vocab_forward_device`: logits of this rank's vocabulary rows
    [v0, v0 + len(weight_slice)); returns the per-row partial statistics
    [bt, VOCAB_TUPLE] to all-gather."""
    opts = opts or LossOptions()
    bt = student_hidden.shape[0]
    if partials is None:
        partials = torch.empty(bt, _abi.VOCAB_TUPLE, device=student_hidden.device, dtype=torch.float32)
    t = _teacher_struct(teacher_mode, teacher_hidden, teacher_weight_slice, teacher_logits_slice)
    vs = _abi.OrdaVocabShard(int(v_total), int(v0), 1, 0, 0, 0)
    buf = _abi.err_buf()
    rc = _lib().orda_vocab_forward_device(
        ctx.handle, C.byref(dev_mat(student_hidden)), C.byref(dev_mat(weight_slice)), labels.data_ptr(),
        labels.numel(), C.byref(t), C.byref(opts._c()), C.byref(vs), partials.data_ptr(), _stream(stream), buf,
        len(buf))
    _check(rc, buf)
    return partials


def vocab_backward_device(
    ctx: DeviceContext,
    student_hidden: torch.Tensor,
    weight_slice: torch.Tensor,
    labels: torch.Tensor,
    teacher_mode: TeacherMode,
    v_total: int,
    v0: int,
    all_partials: torch.Tensor,
    include_rows: bool,
    teacher_hidden: Optional[torch.Tensor] = None,
    teacher_weight_slice: Optional[torch.Tensor] = None,
    teacher_logits_slice: Optional[torch.Tensor] = None,
    opts: Optional[LossOptions] = None,
    out: Optional[dict] = None,
    want_int8: bool = False,
    stream=None,
    scatter_grad_hidden: bool = False,
) -> DeviceLossResult:
    """`orda_vocab_backward_device`: all_partials [world, bt, VOCAB_TUPLE]
    are every rank's tuples by rank. grad_weight (and grad_teacher_weight)
    hold this slice's rows; grad_student_hidden, grad_teacher_hidden and
    scalars are this rank's partial sums (add them over the ranks)."""
    opts = opts or LossOptions()
    bt, h = student_hidden.shape
    v = weight_slice.shape[0]
    ht = teacher_hidden.shape[1] if teacher_mode == TeacherMode.Separate else h
    o, tensors = _outputs(opts, teacher_mode, bt, h, v, ht, student_hidden.device, out, want_int8,
                          with_grad_hidden=not scatter_grad_hidden)
    t = _teacher_struct(teacher_mode, teacher_hidden, teacher_weight_slice, teacher_logits_slice)
    vs = _abi.OrdaVocabShard(int(v_total), int(v0), int(all_partials.shape[0]), int(include_rows),
                             int(scatter_grad_hidden), 0)
    plan = _abi.OrdaChunkPlan()
    buf = _abi.err_buf()
    rc = _lib().orda_vocab_backward_device(
        ctx.handle, C.byref(dev_mat(student_hidden)), C.byref(dev_mat(weight_slice)), labels.data_ptr(),
        labels.numel(), C.byref(t), C.byref(opts._c()), C.byref(vs), all_partials.data_ptr(), C.byref(o),
        _stream(stream), C.byref(plan), buf, len(buf))
    _check(rc, buf)
    return DeviceLossResult(chunk_plan=ChunkPlan(int(plan.chunk_size), int(plan.num_chunks)), **tensors)


def gemm_bf16(
    ctx: DeviceContext,
    a: torch.Tensor,
    a_kind: int,
    b: torch.Tensor,
    b_kind: int,
    c: torch.Tensor,
    m: int,
    n: int,
    k: int,
    alpha: float = 1.0,
    beta: float = 0.0,
    stream=None,
) -> torch.Tensor:
    """`orda_gemm_bf16_device`: C = alpha * op(A) @ op(B) + beta * C."""
    buf = _abi.err_buf()
    rc = _lib().orda_gemm_bf16_device(
        ctx.handle, a.data_ptr(), a.stride(0), a_kind, b.data_ptr(), b.stride(0), b_kind, c.data_ptr(), c.stride(0),
        m, n, k, alpha, beta, _stream(stream), buf, len(buf),
    )
    _check(rc, buf)
    return c


def quantize_grad_w(
    ctx: DeviceContext,
    grad_w: torch.Tensor,
    labels: torch.Tensor,
    ignore_index: int = -100,
    stochastic: bool = False,
    seed: int = 0,
    q: Optional[torch.Tensor] = None,
    scale: Optional[torch.Tensor] = None,
    stream=None,
):
    """`orda_quantize_grad_w_device`; grad_w is overwritten with the
    dequantised values, q / scale receive the INT8 body and scales."""
    v, h = grad_w.shape
    buf = _abi.err_buf()
    rc = _lib().orda_quantize_grad_w_device(
        ctx.handle, grad_w.data_ptr(), v, h, grad_w.stride(0), labels.data_ptr(), labels.numel(), ignore_index,
        int(stochastic), int(seed) & ((1 << 64) - 1), _ptr(q), _ptr(scale), _stream(stream), buf, len(buf),
    )
    _check(rc, buf)
    return grad_w, q, scale
