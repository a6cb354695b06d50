"""orda_b200 -- Python mirror of the reference crate's public API, backed by
the B200 C ABI (include/orda.h, liborda_b200.so).

The names follow malcolmgreaves/orda-cutile-rs (src/lib.rs:57-64):
`distillation_loss`, `LossOptions`, `Teacher.{Tied,Separate,Precomputed}`,
`DistillationLossOutput`, `KernelConfig`, `Profile`, `Reduction`, `Backend`,
`ChunkSize`, `ChunkPlan`, `Mat`, `is_available`, plus the resolver helpers of
src/resolver.rs. Errors that the crate returns as `Err(String)` are raised as
`OrdaError` with the same message. Every call goes through the C ABI; the
package has no Python or CPU fallback for the loss.
"""
from __future__ import annotations

import ctypes as C
import enum
from dataclasses import dataclass, field
from typing import Optional, Sequence

import numpy as np

from . import _abi
from ._abi import load_library

__all__ = [
    "Mat",
    "Teacher",
    "TeacherMode",
    "Reduction",
    "Backend",
    "Profile",
    "KernelConfig",
    "ChunkSize",
    "ChunkPlan",
    "LossOptions",
    "DistillationLossOutput",
    "OrdaError",
    "distillation_loss",
    "resolve_chunk_size",
    "chunks_from_raw",
    "default_max_chunks_limit",
    "chunk_doubling_schedule",
    "chunk_retry",
    "is_available",
    "is_power_of_two",
    "DEFAULT_MAX_FUSED_SIZE",
    "load_library",
]

DEFAULT_MAX_FUSED_SIZE = 65536 // 2  # src/config.rs:66


class OrdaError(RuntimeError):
    """The `Err(String)` of the reference API; `.code` is the C status."""

    def __init__(self, code: int, message: str):
        super().__init__(message)
        self.code = code
        self.message = message


def _lib():
    return load_library()


def _check(rc: int, buf) -> None:
    if rc != _abi.ORDA_OK:
        raise OrdaError(rc, buf.value.decode())


# --------------------------------------------------------------------- types


class Mat:
    """Dense row-major f32 matrix (`Mat`, src/mat.rs:10-57)."""

    def __init__(self, rows: int, cols: int, data=None):
        if data is None:
            arr = np.zeros((rows, cols), dtype=np.float32)
        else:
            arr = np.ascontiguousarray(np.asarray(data, dtype=np.float32)).reshape(-1)
            if arr.size != rows * cols:
                raise ValueError("data length must equal rows*cols")
            arr = arr.reshape(rows, cols)
        self.a = np.ascontiguousarray(arr, dtype=np.float32)

    @classmethod
    def from_vec(cls, rows: int, cols: int, data) -> "Mat":
        return cls(rows, cols, data)

    @classmethod
    def zeros(cls, rows: int, cols: int) -> "Mat":
        return cls(rows, cols)

    @classmethod
    def from_array(cls, arr) -> "Mat":
        arr = np.asarray(arr, dtype=np.float32)
        return cls(arr.shape[0], arr.shape[1], arr)

    @property
    def rows(self) -> int:
        return self.a.shape[0]

    @property
    def cols(self) -> int:
        return self.a.shape[1]

    @property
    def data(self) -> np.ndarray:
        return self.a.reshape(-1)

    def shape(self):
        return (self.rows, self.cols)

    def row(self, r: int) -> np.ndarray:
        return self.a[r]

    def get(self, r: int, c: int) -> float:
        return float(self.a[r, c])

    def clone(self) -> "Mat":
        return Mat.from_array(self.a.copy())

    def _c(self) -> _abi.OrdaMatF32:
        return _abi.OrdaMatF32(self.a.ctypes.data_as(C.POINTER(C.c_float)), self.rows, self.cols)


class TeacherMode(enum.IntEnum):
    Tied = _abi.TEACHER_TIED
    Separate = _abi.TEACHER_SEPARATE
    Precomputed = _abi.TEACHER_PRECOMPUTED


@dataclass
class Teacher:
    """`Teacher::{Tied, Separate, Precomputed}` (src/teacher.rs:11-32)."""

    kind: TeacherMode
    hidden: Optional[Mat] = None
    weight: Optional[Mat] = None
    logits: Optional[Mat] = None

    @classmethod
    def Tied(cls, hidden: Mat) -> "Teacher":
        return cls(TeacherMode.Tied, hidden=hidden)

    @classmethod
    def Separate(cls, hidden: Mat, weight: Mat) -> "Teacher":
        return cls(TeacherMode.Separate, hidden=hidden, weight=weight)

    @classmethod
    def Precomputed(cls, logits: Mat) -> "Teacher":
        return cls(TeacherMode.Precomputed, logits=logits)

    def mode(self) -> TeacherMode:
        return self.kind

    def default_teacher_ce_weight(self) -> float:
        return float(_lib().orda_default_teacher_ce_weight(int(self.kind)))

    def _c(self) -> _abi.OrdaTeacher:
        t = _abi.OrdaTeacher()
        t.mode = int(self.kind)
        if self.hidden is not None:
            t.hidden = self.hidden._c()
        if self.weight is not None:
            t.weight = self.weight._c()
        if self.logits is not None:
            t.logits = self.logits._c()
        return t


class Reduction(enum.IntEnum):
    Mean = _abi.REDUCTION_MEAN
    Sum = _abi.REDUCTION_SUM


class Backend(enum.IntEnum):
    Auto = _abi.BACKEND_AUTO
    Cpu = _abi.BACKEND_CPU
    Cuda = _abi.BACKEND_CUDA


class Profile(enum.IntEnum):
    Balanced = _abi.PROFILE_BALANCED
    Fast = _abi.PROFILE_FAST
    Debug = _abi.PROFILE_DEBUG


@dataclass
class KernelConfig:
    """`KernelConfig` (src/config.rs:46-124)."""

    online_softmax: bool = False
    fast_math: bool = False
    quantize_grad_weight: bool = False
    stochastic_rounding: bool = False
    fp32_grad_weight_accumulation: bool = False
    max_chunks: Optional[int] = None
    max_fused_size: int = DEFAULT_MAX_FUSED_SIZE
    stochastic_seed: Optional[int] = None

    @classmethod
    def from_profile(cls, profile: Profile) -> "KernelConfig":
        c = _abi.OrdaKernelConfig()
        _lib().orda_kernel_config_from_profile(int(profile), C.byref(c))
        return cls._from_c(c)

    @classmethod
    def default(cls) -> "KernelConfig":
        return cls.from_profile(Profile.Balanced)

    def fast_math_exp(self) -> bool:
        return self.fast_math

    def fast_math_log(self) -> bool:
        return self.fast_math

    def fast_math_mul(self) -> bool:
        return self.fast_math

    def validate(self) -> None:
        buf = _abi.err_buf()
        _check(_lib().orda_kernel_config_validate(C.byref(self._c()), buf, len(buf)), buf)

    @classmethod
    def _from_c(cls, c: _abi.OrdaKernelConfig) -> "KernelConfig":
        return cls(
            online_softmax=bool(c.online_softmax),
            fast_math=bool(c.fast_math),
            quantize_grad_weight=bool(c.quantize_grad_weight),
            stochastic_rounding=bool(c.stochastic_rounding),
            fp32_grad_weight_accumulation=bool(c.fp32_grad_weight_accumulation),
            max_chunks=int(c.max_chunks) if c.has_max_chunks else None,
            max_fused_size=int(c.max_fused_size),
            stochastic_seed=int(c.stochastic_seed) if c.has_stochastic_seed else None,
        )

    def _c(self) -> _abi.OrdaKernelConfig:
        c = _abi.OrdaKernelConfig()
        c.online_softmax = int(self.online_softmax)
        c.fast_math = int(self.fast_math)
        c.quantize_grad_weight = int(self.quantize_grad_weight)
        c.stochastic_rounding = int(self.stochastic_rounding)
        c.fp32_grad_weight_accumulation = int(self.fp32_grad_weight_accumulation)
        c.has_max_chunks = int(self.max_chunks is not None)
        c.max_chunks = int(self.max_chunks or 0)
        c.max_fused_size = int(self.max_fused_size)
        c.has_stochastic_seed = int(self.stochastic_seed is not None)
        c.stochastic_seed = int(self.stochastic_seed or 0)
        return c


@dataclass(frozen=True)
class ChunkSize:
    """`ChunkSize::{Auto, Fixed(usize)}` (src/resolver.rs:10-16)."""

    fixed: Optional[int] = None

    @classmethod
    def Auto(cls) -> "ChunkSize":
        return cls(None)

    @classmethod
    def Fixed(cls, rows: int) -> "ChunkSize":
        return cls(int(rows))

    def _c(self) -> _abi.OrdaChunkSize:
        c = _abi.OrdaChunkSize()
        c.kind = _abi.CHUNK_AUTO if self.fixed is None else _abi.CHUNK_FIXED
        c.fixed_rows = 0 if self.fixed is None else self.fixed
        return c


@dataclass(frozen=True)
class ChunkPlan:
    """`ChunkPlan` (src/resolver.rs:40-45)."""

    chunk_size: int
    num_chunks: int


@dataclass
class LossOptions:
    """`LossOptions` with the defaults of src/api.rs:49-64."""

    student_ce_weight: float = 1.0
    teacher_ce_weight: Optional[float] = None
    kd_weight: float = 0.0
    temperature: float = 1.0
    ignore_index: int = -100
    label_smoothing: float = 0.0
    reduction: Reduction = Reduction.Mean
    chunk_size: ChunkSize = field(default_factory=ChunkSize.Auto)
    config: KernelConfig = field(default_factory=KernelConfig)
    backend: Backend = Backend.Auto

    def _c(self) -> _abi.OrdaLossOptions:
        o = _abi.OrdaLossOptions()
        o.student_ce_weight = self.student_ce_weight
        o.has_teacher_ce_weight = int(self.teacher_ce_weight is not None)
        o.teacher_ce_weight = float(self.teacher_ce_weight or 0.0)
        o.kd_weight = self.kd_weight
        o.temperature = self.temperature
        o.ignore_index = self.ignore_index
        o.label_smoothing = self.label_smoothing
        o.reduction = int(self.reduction)
        o.chunk_size = self.chunk_size._c()
        o.config = self.config._c()
        o.backend = int(self.backend)
        return o


@dataclass
class DistillationLossOutput:
    """`DistillationLossOutput` (src/api.rs:71-92)."""

    loss: float
    student_ce: float
    teacher_ce: float
    kl: float
    grad_student_hidden: Mat
    grad_weight: Mat
    grad_teacher_hidden: Optional[Mat]
    grad_teacher_weight: Optional[Mat]
    chunk_plan: ChunkPlan


def _labels_c(labels: Sequence[int]):
    arr = np.ascontiguousarray(np.asarray(labels, dtype=np.int64))
    return arr, arr.ctypes.data_as(C.POINTER(C.c_int64))


def _take_mat(m: _abi.OrdaMatOut) -> Optional[Mat]:
    if not m.data:
        return None
    n = m.rows * m.cols
    arr = np.ctypeslib.as_array(m.data, shape=(max(n, 1),))[:n].copy()
    return Mat(m.rows, m.cols, arr)


def distillation_loss(
    student_hidden: Mat, weight: Mat, labels: Sequence[int], teacher: Teacher, opts: Optional[LossOptions] = None
) -> DistillationLossOutput:
    """`distillation_loss` (src/api.rs:188-422) on the B200 via the C ABI."""
    opts = opts or LossOptions()
    lab, lab_p = _labels_c(labels)
    out = _abi.OrdaOutput()
    buf = _abi.err_buf()
    rc = _lib().orda_distillation_loss(
        C.byref(student_hidden._c()),
        C.byref(weight._c()),
        lab_p,
        lab.size,
        C.byref(teacher._c()),
        C.byref(opts._c()),
        C.byref(out),
        buf,
        len(buf),
    )
    _check(rc, buf)
    try:
        return DistillationLossOutput(
            loss=float(out.loss),
            student_ce=float(out.student_ce),
            teacher_ce=float(out.teacher_ce),
            kl=float(out.kl),
            grad_student_hidden=_take_mat(out.grad_student_hidden),
            grad_weight=_take_mat(out.grad_weight),
            grad_teacher_hidden=_take_mat(out.grad_teacher_hidden),
            grad_teacher_weight=_take_mat(out.grad_teacher_weight),
            chunk_plan=ChunkPlan(int(out.chunk_plan.chunk_size), int(out.chunk_plan.num_chunks)),
        )
    finally:
        _lib().orda_output_free(C.byref(out))


def validate(student_hidden: Mat, weight: Mat, labels, teacher: Teacher, opts: LossOptions):
    """`validate` (src/api.rs:104-181); returns (V, H, BT)."""
    lab, lab_p = _labels_c(labels)
    v, h, bt = C.c_size_t(), C.c_size_t(), C.c_size_t()
    buf = _abi.err_buf()
    rc = _lib().orda_validate(
        C.byref(student_hidden._c()),
        C.byref(weight._c()),
        lab_p,
        lab.size,
        C.byref(teacher._c()),
        C.byref(opts._c()),
        C.byref(v),
        C.byref(h),
        C.byref(bt),
        buf,
        len(buf),
    )
    _check(rc, buf)
    return int(v.value), int(h.value), int(bt.value)


# ------------------------------------------------------------ resolver helpers


def chunks_from_raw(raw: float) -> int:
    return int(_lib().orda_chunks_from_raw(float(raw)))


def resolve_chunk_size(bt: int, chunk_size: ChunkSize, v: Optional[int], max_chunks: Optional[int]) -> ChunkPlan:
    p = _abi.OrdaChunkPlan()
    _lib().orda_resolve_chunk_size(
        bt, chunk_size._c(), int(v is not None), int(v or 0), int(max_chunks is not None), int(max_chunks or 0),
        C.byref(p),
    )
    return ChunkPlan(int(p.chunk_size), int(p.num_chunks))


def default_max_chunks_limit(bt: int) -> int:
    return int(_lib().orda_default_max_chunks_limit(bt))


def chunk_doubling_schedule(bt: int, start: int, limit: int) -> list[int]:
    cap = 128
    arr = (C.c_size_t * cap)()
    n = int(_lib().orda_chunk_doubling_schedule(bt, start, limit, arr, cap))
    return [int(arr[i]) for i in range(min(n, cap))]


def chunk_retry(bt: int, start: int, limit: int, try_alloc) -> Optional[ChunkPlan]:
    """Walks the OOM ladder; `try_alloc(num_chunks, chunk_size) -> bool`."""

    @_abi.TRY_ALLOC_FN
    def cb(nc, cs, _user):
        return 0 if try_alloc(int(nc), int(cs)) else 1

    p = _abi.OrdaChunkPlan()
    rc = _lib().orda_chunk_retry(bt, start, limit, cb, None, C.byref(p))
    if rc != _abi.ORDA_OK:
        return None
    return ChunkPlan(int(p.chunk_size), int(p.num_chunks))


def is_available() -> bool:
    return bool(_lib().orda_is_available())


def is_power_of_two(v: int) -> bool:
    return bool(_lib().orda_is_power_of_two(v))
