"""ctypes mirror of include/orda.h and the loader of liborda_b200.so.

The structures below are field-for-field copies of the C declarations; the
loader raises if the compiled library is missing (there is no fallback).
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

PKG_ROOT = Path(__file__).resolve().parent.parent  # orda-cutile-rs_b200/
LIB_PATH = PKG_ROOT / "liborda_b200.so"

ORDA_OK = 0
ORDA_ERR_INVALID = 1
ORDA_ERR_BACKEND = 2
ORDA_ERR_CUDA = 3
ORDA_ERR_OOM = 4
ORDA_ERR_TIMEOUT = 5
ORDA_ERR_LABEL = 6

TEACHER_TIED, TEACHER_SEPARATE, TEACHER_PRECOMPUTED = 0, 1, 2
REDUCTION_MEAN, REDUCTION_SUM = 0, 1
BACKEND_AUTO, BACKEND_CPU, BACKEND_CUDA = 0, 1, 2
PROFILE_BALANCED, PROFILE_FAST, PROFILE_DEBUG = 0, 1, 2
CHUNK_AUTO, CHUNK_FIXED = 0, 1
DTYPE_BF16, DTYPE_F32 = 0, 1
NUM_PHASES = 6
PHASE_NAMES = ("logits_gemm", "rows", "dgrad_gemm", "wgrad_gemm", "quant", "prep_finalize")


class OrdaMatF32(C.Structure):
    _fields_ = [("data", C.POINTER(C.c_float)), ("rows", C.c_size_t), ("cols", C.c_size_t)]


class OrdaMatOut(C.Structure):
    _fields_ = [("data", C.POINTER(C.c_float)), ("rows", C.c_size_t), ("cols", C.c_size_t)]


class OrdaTeacher(C.Structure):
    _fields_ = [("mode", C.c_int), ("hidden", OrdaMatF32), ("weight", OrdaMatF32), ("logits", OrdaMatF32)]


class OrdaKernelConfig(C.Structure):
    _fields_ = [
        ("online_softmax", C.c_int32),
        ("fast_math", C.c_int32),
        ("quantize_grad_weight", C.c_int32),
        ("stochastic_rounding", C.c_int32),
        ("fp32_grad_weight_accumulation", C.c_int32),
        ("has_max_chunks", C.c_int32),
        ("max_chunks", C.c_size_t),
        ("max_fused_size", C.c_size_t),
        ("has_stochastic_seed", C.c_int32),
        ("stochastic_seed", C.c_uint64),
    ]


class OrdaChunkSize(C.Structure):
    _fields_ = [("kind", C.c_int), ("fixed_rows", C.c_size_t)]


class OrdaChunkPlan(C.Structure):
    _fields_ = [("chunk_size", C.c_size_t), ("num_chunks", C.c_size_t)]


class OrdaLossOptions(C.Structure):
    _fields_ = [
        ("student_ce_weight", C.c_float),
        ("has_teacher_ce_weight", C.c_int32),
        ("teacher_ce_weight", C.c_float),
        ("kd_weight", C.c_float),
        ("temperature", C.c_float),
        ("ignore_index", C.c_int64),
        ("label_smoothing", C.c_float),
        ("reduction", C.c_int),
        ("chunk_size", OrdaChunkSize),
        ("config", OrdaKernelConfig),
        ("backend", C.c_int),
    ]


class OrdaOutput(C.Structure):
    _fields_ = [
        ("loss", C.c_float),
        ("student_ce", C.c_float),
        ("teacher_ce", C.c_float),
        ("kl", C.c_float),
        ("grad_student_hidden", OrdaMatOut),
        ("grad_weight", OrdaMatOut),
        ("grad_teacher_hidden", OrdaMatOut),
        ("grad_teacher_weight", OrdaMatOut),
        ("chunk_plan", OrdaChunkPlan),
    ]


class OrdaDeviceMat(C.Structure):
    _fields_ = [
        ("data", C.c_void_p),
        ("rows", C.c_size_t),
        ("cols", C.c_size_t),
        ("ld", C.c_size_t),
        ("dtype", C.c_int),
    ]


class OrdaDeviceTeacher(C.Structure):
    _fields_ = [("mode", C.c_int), ("hidden", OrdaDeviceMat), ("weight", OrdaDeviceMat), ("logits", OrdaDeviceMat)]


class OrdaDeviceOutputs(C.Structure):
    _fields_ = [
        ("grad_student_hidden", C.c_void_p),
        ("ld_grad_student_hidden", C.c_size_t),
        ("grad_weight", C.c_void_p),
        ("ld_grad_weight", C.c_size_t),
        ("grad_teacher_hidden", C.c_void_p),
        ("ld_grad_teacher_hidden", C.c_size_t),
        ("grad_teacher_weight", C.c_void_p),
        ("ld_grad_teacher_weight", C.c_size_t),
        ("grad_weight_q", C.c_void_p),
        ("grad_weight_scale", C.c_void_p),
        ("scalars", C.c_void_p),
    ]


class OrdaFieldLayout(C.Structure):
    _fields_ = [("struct_name", C.c_char_p), ("field", C.c_char_p), ("offset", C.c_size_t), ("size", C.c_size_t)]


class OrdaShardOptions(C.Structure):
    _fields_ = [("global_non_ignore", C.c_int64), ("skip_quantize", C.c_int32),
                ("scatter_grad_weight", C.c_int32), ("int8_wire", C.c_int32), ("reserved", C.c_int32)]


VOCAB_TUPLE = 24  # ORDA_VOCAB_TUPLE


class OrdaVocabShard(C.Structure):
    _fields_ = [("v_total", C.c_int64), ("v0", C.c_int64), ("world", C.c_int32), ("include_rows", C.c_int32),
                ("scatter_grad_hidden", C.c_int32), ("pad", C.c_int32)]


class OrdaIpcHandle(C.Structure):
    _fields_ = [("bytes", C.c_ubyte * 64)]  # opaque; c_ubyte so no NUL truncation


TRY_ALLOC_FN = C.CFUNCTYPE(C.c_int, C.c_size_t, C.c_size_t, C.c_void_p)

# name -> (restype, argtypes); every entry point of include/orda.h
SIGNATURES = {
    "orda_loss_options_default": (None, [C.POINTER(OrdaLossOptions)]),
    "orda_kernel_config_from_profile": (None, [C.c_int, C.POINTER(OrdaKernelConfig)]),
    "orda_kernel_config_validate": (C.c_int, [C.POINTER(OrdaKernelConfig), C.c_char_p, C.c_size_t]),
    "orda_is_power_of_two": (C.c_int, [C.c_size_t]),
    "orda_default_teacher_ce_weight": (C.c_float, [C.c_int]),
    "orda_is_available": (C.c_int, []),
    "orda_chunks_from_raw": (C.c_size_t, [C.c_double]),
    "orda_resolve_chunk_size": (
        None,
        [C.c_size_t, OrdaChunkSize, C.c_int, C.c_size_t, C.c_int, C.c_size_t, C.POINTER(OrdaChunkPlan)],
    ),
    "orda_default_max_chunks_limit": (C.c_size_t, [C.c_size_t]),
    "orda_chunk_doubling_schedule": (
        C.c_size_t,
        [C.c_size_t, C.c_size_t, C.c_size_t, C.POINTER(C.c_size_t), C.c_size_t],
    ),
    "orda_chunk_retry": (
        C.c_int,
        [C.c_size_t, C.c_size_t, C.c_size_t, TRY_ALLOC_FN, C.c_void_p, C.POINTER(OrdaChunkPlan)],
    ),
    "orda_validate": (
        C.c_int,
        [
            C.POINTER(OrdaMatF32),
            C.POINTER(OrdaMatF32),
            C.POINTER(C.c_int64),
            C.c_size_t,
            C.POINTER(OrdaTeacher),
            C.POINTER(OrdaLossOptions),
            C.POINTER(C.c_size_t),
            C.POINTER(C.c_size_t),
            C.POINTER(C.c_size_t),
            C.c_char_p,
            C.c_size_t,
        ],
    ),
    "orda_distillation_loss": (
        C.c_int,
        [
            C.POINTER(OrdaMatF32),
            C.POINTER(OrdaMatF32),
            C.POINTER(C.c_int64),
            C.c_size_t,
            C.POINTER(OrdaTeacher),
            C.POINTER(OrdaLossOptions),
            C.POINTER(OrdaOutput),
            C.c_char_p,
            C.c_size_t,
        ],
    ),
    "orda_output_free": (None, [C.POINTER(OrdaOutput)]),
    "orda_set_host_slab_bytes": (None, [C.c_size_t]),
    "orda_last_call_bytes": (None, [C.POINTER(C.c_uint64), C.POINTER(C.c_uint64)]),
    "orda_context_set_concurrency": (None, [C.c_void_p, C.c_int]),
    "orda_abi_layout": (C.c_size_t, [C.POINTER(C.POINTER(OrdaFieldLayout))]),
    "orda_selftest_host_io": (C.c_int, [C.c_char_p, C.c_size_t]),
    "orda_selftest_exp2": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_size_t, C.c_void_p, C.c_char_p,
                                     C.c_size_t]),
    "orda_context_create": (C.c_int, [C.c_int, C.POINTER(C.c_void_p), C.c_char_p, C.c_size_t]),
    "orda_context_destroy": (None, [C.c_void_p]),
    "orda_context_check": (C.c_int, [C.c_void_p, C.c_char_p, C.c_size_t]),
    "orda_context_workspace_bytes": (C.c_size_t, [C.c_void_p]),
    "orda_context_inject_alloc_failures": (None, [C.c_void_p, C.c_int]),
    "orda_context_enable_timing": (None, [C.c_void_p, C.c_int]),
    "orda_context_phase_times": (C.c_int, [C.c_void_p, C.POINTER(C.c_double), C.POINTER(C.c_uint64)]),
    "orda_context_reset_timing": (None, [C.c_void_p]),
    "orda_context_launch_count": (C.c_uint64, [C.c_void_p]),
    "orda_vocab_forward_device": (
        C.c_int,
        [C.c_void_p, C.POINTER(OrdaDeviceMat), C.POINTER(OrdaDeviceMat), C.c_void_p, C.c_size_t,
         C.POINTER(OrdaDeviceTeacher), C.POINTER(OrdaLossOptions), C.POINTER(OrdaVocabShard), C.c_void_p, C.c_void_p,
         C.c_char_p, C.c_size_t]),
    "orda_vocab_backward_device": (
        C.c_int,
        [C.c_void_p, C.POINTER(OrdaDeviceMat), C.POINTER(OrdaDeviceMat), C.c_void_p, C.c_size_t,
         C.POINTER(OrdaDeviceTeacher), C.POINTER(OrdaLossOptions), C.POINTER(OrdaVocabShard), C.c_void_p,
         C.POINTER(OrdaDeviceOutputs), C.c_void_p, C.POINTER(OrdaChunkPlan), C.c_char_p, C.c_size_t]),
    "orda_context_slots_create": (
        C.c_int, [C.c_void_p, C.c_int, C.c_int, C.c_size_t, C.c_size_t, C.c_int, C.POINTER(OrdaIpcHandle),
                  C.c_char_p, C.c_size_t]),
    "orda_reduce_slot_set_device": (C.c_int, [C.c_void_p, C.c_int, C.c_void_p, C.c_size_t, C.c_void_p, C.c_char_p,
                                              C.c_size_t]),
    "orda_context_slots_attach": (C.c_int, [C.c_void_p, C.POINTER(OrdaIpcHandle), C.c_char_p, C.c_size_t]),
    "orda_reduce_slots_device": (
        C.c_int, [C.c_void_p, C.c_void_p, C.c_size_t, C.c_void_p, C.c_size_t, C.c_int64, C.c_int, C.c_int,
                  C.c_uint64, C.c_void_p, C.c_void_p, C.c_int, C.c_void_p, C.c_char_p, C.c_size_t]),
    "orda_context_set_l2_persisting": (C.c_int, [C.c_void_p, C.c_size_t, C.POINTER(C.c_size_t), C.c_char_p,
                                                 C.c_size_t]),
    "orda_context_selftest_bounded_wait": (C.c_int, [C.c_void_p, C.c_uint32, C.c_void_p, C.c_char_p, C.c_size_t]),
    "orda_distillation_loss_device": (
        C.c_int,
        [
            C.c_void_p,
            C.POINTER(OrdaDeviceMat),
            C.POINTER(OrdaDeviceMat),
            C.c_void_p,
            C.c_size_t,
            C.POINTER(OrdaDeviceTeacher),
            C.POINTER(OrdaLossOptions),
            C.POINTER(OrdaDeviceOutputs),
            C.POINTER(OrdaShardOptions),
            C.c_void_p,
            C.POINTER(OrdaChunkPlan),
            C.c_char_p,
            C.c_size_t,
        ],
    ),
    "orda_quantize_grad_w_device": (
        C.c_int,
        [
            C.c_void_p,
            C.c_void_p,
            C.c_size_t,
            C.c_size_t,
            C.c_size_t,
            C.c_void_p,
            C.c_size_t,
            C.c_int64,
            C.c_int,
            C.c_uint64,
            C.c_void_p,
            C.c_void_p,
            C.c_void_p,
            C.c_char_p,
            C.c_size_t,
        ],
    ),
    "orda_quantize_grad_w_device_noalloc": (
        C.c_int,
        [
            C.c_void_p,
            C.c_size_t,
            C.c_size_t,
            C.c_size_t,
            C.c_void_p,
            C.c_size_t,
            C.c_int64,
            C.c_int,
            C.c_uint64,
            C.c_void_p,
            C.c_void_p,
            C.c_void_p,
            C.c_char_p,
            C.c_size_t,
        ],
    ),
    "orda_gemm_bf16_device": (
        C.c_int,
        [
            C.c_void_p,
            C.c_void_p,
            C.c_size_t,
            C.c_int,
            C.c_void_p,
            C.c_size_t,
            C.c_int,
            C.c_void_p,
            C.c_size_t,
            C.c_size_t,
            C.c_size_t,
            C.c_size_t,
            C.c_float,
            C.c_float,
            C.c_void_p,
            C.c_char_p,
            C.c_size_t,
        ],
    ),
}

_LIB = None


def load_library(path: os.PathLike | str | None = None) -> C.CDLL:
    """Loads liborda_b200.so (built by `make` in orda-cutile-rs_b200/).

    Raises FileNotFoundError when the library has not been built: the package
    has no CPU or pure-Python fallback for the distillation path.
    """
    global _LIB
    if _LIB is not None and path is None:
        return _LIB
    p = Path(path) if path is not None else LIB_PATH
    if not p.exists():
        raise FileNotFoundError(
            f"{p} not found: build it with `make -C orda-cutile-rs_b200` (or __graft_entry__.build())"
        )
    lib = C.CDLL(str(p))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    if path is None:
        _LIB = lib
    return lib


def err_buf(n: int = 1024):
    return C.create_string_buffer(n)
