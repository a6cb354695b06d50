//! Raw bindings of the B200 library (`liborda_b200.so`, C ABI `include/orda.h`).
//!
//! `#[repr(C)]` mirrors of every struct of the header, field for field in the
//! header's order, and the `extern "C"` declarations of every entry point.
//! The repository's tests parse this file and check each struct's layout
//! against the table the compiled library reports (`orda_abi_layout`).
//! Enums of the header are C `int`s here (`c_int`); their values are the
//! `ORDA_*` constants below. The safe API is in `launch.rs`.
#![allow(non_camel_case_types, non_snake_case, dead_code)]

use std::os::raw::{c_char, c_int, c_void};

pub const ORDA_ABI_VERSION: c_int = 2;

// status codes
pub const ORDA_OK: c_int = 0;
pub const ORDA_ERR_INVALID: c_int = 1;
pub const ORDA_ERR_BACKEND: c_int = 2;
pub const ORDA_ERR_CUDA: c_int = 3;
pub const ORDA_ERR_OOM: c_int = 4;
pub const ORDA_ERR_TIMEOUT: c_int = 5;
pub const ORDA_ERR_LABEL: c_int = 6;

// OrdaTeacherMode
pub const ORDA_TEACHER_TIED: c_int = 0;
pub const ORDA_TEACHER_SEPARATE: c_int = 1;
pub const ORDA_TEACHER_PRECOMPUTED: c_int = 2;
// OrdaReduction
pub const ORDA_REDUCTION_MEAN: c_int = 0;
pub const ORDA_REDUCTION_SUM: c_int = 1;
// OrdaBackend
pub const ORDA_BACKEND_AUTO: c_int = 0;
pub const ORDA_BACKEND_CPU: c_int = 1;
pub const ORDA_BACKEND_CUDA: c_int = 2;
// OrdaProfile
pub const ORDA_PROFILE_BALANCED: c_int = 0;
pub const ORDA_PROFILE_FAST: c_int = 1;
pub const ORDA_PROFILE_DEBUG: c_int = 2;
// OrdaChunkKind
pub const ORDA_CHUNK_AUTO: c_int = 0;
pub const ORDA_CHUNK_FIXED: c_int = 1;
// OrdaDType
pub const ORDA_DTYPE_BF16: c_int = 0;
pub const ORDA_DTYPE_F32: c_int = 1;

pub const ORDA_NUM_PHASES: usize = 6;
pub const ORDA_VOCAB_TUPLE: usize = 24;
pub const ORDA_NOALLOC_MAX_V: usize = 262144;

#[repr(C)]
#[derive(Clone, Copy, Debug)]
pub struct OrdaFieldLayout {
    pub struct_name: *const c_char,
    pub field: *const c_char,
    pub offset: usize,
    pub size: usize,
}

#[repr(C)]
#[derive(Clone, Copy, Debug)]
pub struct OrdaMatF32 {
    pub data: *const f32,
    pub rows: usize,
    pub cols: usize,
}

#[repr(C)]
#[derive(Clone, Copy, Debug)]
pub struct OrdaMatOut {
    pub data: *mut f32,
    pub rows: usize,
    pub cols: usize,
}

#[repr(C)]
#[derive(Clone, Copy, Debug)]
pub struct OrdaTeacher {
    pub mode: c_int,
    pub hidden: OrdaMatF32,
    pub weight: OrdaMatF32,
    pub logits: OrdaMatF32,
}

#[repr(C)]
#[derive(Clone, Copy, Debug)]
pub struct OrdaKernelConfig {
    pub online_softmax: i32,
    pub fast_math: i32,
    pub quantize_grad_weight: i32,
    pub stochastic_rounding: i32,
    pub fp32_grad_weight_accumulation: i32,
    pub has_max_chunks: i32,
    pub max_chunks: usize,
    pub max_fused_size: usize,
    pub has_stochastic_seed: i32,
    pub stochastic_seed: u64,
}

#[repr(C)]
#[derive(Clone, Copy, Debug)]
pub struct OrdaChunkSize {
    pub kind: c_int,
    pub fixed_rows: usize,
}

#[repr(C)]
#[derive(Clone, Copy, Debug, Default)]
pub struct OrdaChunkPlan {
    pub chunk_size: usize,
    pub num_chunks: usize,
}

#[repr(C)]
#[derive(Clone, Copy, Debug)]
pub struct OrdaLossOptions {
    pub student_ce_weight: f32,
    pub has_teacher_ce_weight: i32,
    pub teacher_ce_weight: f32,
    pub kd_weight: f32,
    pub temperature: f32,
    pub ignore_index: i64,
    pub label_smoothing: f32,
    pub reduction: c_int,
    pub chunk_size: OrdaChunkSize,
    pub config: OrdaKernelConfig,
    pub backend: c_int,
}

#[repr(C)]
#[derive(Clone, Copy, Debug)]
pub struct OrdaOutput {
    pub loss: f32,
    pub student_ce: f32,
    pub teacher_ce: f32,
    pub kl: f32,
    pub grad_student_hidden: OrdaMatOut,
    pub grad_weight: OrdaMatOut,
    pub grad_teacher_hidden: OrdaMatOut,
    pub grad_teacher_weight: OrdaMatOut,
    pub chunk_plan: OrdaChunkPlan,
}

/// Opaque context (device workspace, status word, slot buffers).
#[repr(C)]
pub struct OrdaContext {
    _opaque: [u8; 0],
}

#[repr(C)]
#[derive(Clone, Copy, Debug)]
pub struct OrdaDeviceMat {
    pub data: *const c_void,
    pub rows: usize,
    pub cols: usize,
    pub ld: usize,
    pub dtype: c_int,
}

#[repr(C)]
#[derive(Clone, Copy, Debug)]
pub struct OrdaDeviceTeacher {
    pub mode: c_int,
    pub hidden: OrdaDeviceMat,
    pub weight: OrdaDeviceMat,
    pub logits: OrdaDeviceMat,
}

#[repr(C)]
#[derive(Clone, Copy, Debug)]
pub struct OrdaDeviceOutputs {
    pub grad_student_hidden: *mut f32,
    pub ld_grad_student_hidden: usize,
    pub grad_weight: *mut f32,
    pub ld_grad_weight: usize,
    pub grad_teacher_hidden: *mut f32,
    pub ld_grad_teacher_hidden: usize,
    pub grad_teacher_weight: *mut f32,
    pub ld_grad_teacher_weight: usize,
    pub grad_weight_q: *mut i8,
    pub grad_weight_scale: *mut f32,
    pub scalars: *mut f32,
}

#[repr(C)]
#[derive(Clone, Copy, Debug, Default)]
pub struct OrdaShardOptions {
    pub global_non_ignore: i64,
    pub skip_quantize: i32,
    pub scatter_grad_weight: i32,
    pub int8_wire: i32,
    pub reserved: i32,
}

#[repr(C)]
#[derive(Clone, Copy, Debug, Default)]
pub struct OrdaVocabShard {
    pub v_total: i64,
    pub v0: i64,
    pub world: i32,
    pub include_rows: i32,
    pub scatter_grad_hidden: i32,
    pub pad: i32,
}

#[repr(C)]
#[derive(Clone, Copy)]
pub struct OrdaIpcHandle {
    pub bytes: [c_char; 64],
}

pub type OrdaTryAllocFn = Option<unsafe extern "C" fn(num_chunks: usize, chunk_size: usize, user: *mut c_void) -> c_int>;

#[link(name = "orda_b200")]
extern "C" {
    pub fn orda_abi_layout(out: *mut *const OrdaFieldLayout) -> usize;

    pub fn orda_loss_options_default(out: *mut OrdaLossOptions);
    pub fn orda_kernel_config_from_profile(profile: c_int, out: *mut OrdaKernelConfig);
    pub fn orda_kernel_config_validate(cfg: *const OrdaKernelConfig, err: *mut c_char, err_len: usize) -> c_int;
    pub fn orda_is_power_of_two(value: usize) -> c_int;
    pub fn orda_default_teacher_ce_weight(mode: c_int) -> f32;
    pub fn orda_is_available() -> c_int;

    pub fn orda_chunks_from_raw(raw: f64) -> usize;
    pub fn orda_resolve_chunk_size(bt: usize, chunk_size: OrdaChunkSize, has_v: c_int, v: usize, has_max_chunks: c_int,
                                   max_chunks: usize, out: *mut OrdaChunkPlan);
    pub fn orda_default_max_chunks_limit(bt: usize) -> usize;
    pub fn orda_chunk_doubling_schedule(bt: usize, start: usize, limit: usize, out: *mut usize, out_cap: usize)
        -> usize;
    pub fn orda_chunk_retry(bt: usize, start: usize, limit: usize, try_alloc: OrdaTryAllocFn, user: *mut c_void,
                            out: *mut OrdaChunkPlan) -> c_int;
    pub fn orda_validate(student_hidden: *const OrdaMatF32, weight: *const OrdaMatF32, labels: *const i64,
                         n_labels: usize, teacher: *const OrdaTeacher, opts: *const OrdaLossOptions,
                         v_out: *mut usize, h_out: *mut usize, bt_out: *mut usize, err: *mut c_char,
                         err_len: usize) -> c_int;

    pub fn orda_distillation_loss(student_hidden: *const OrdaMatF32, weight: *const OrdaMatF32, labels: *const i64,
                                  n_labels: usize, teacher: *const OrdaTeacher, opts: *const OrdaLossOptions,
                                  out: *mut OrdaOutput, err: *mut c_char, err_len: usize) -> c_int;
    pub fn orda_output_free(out: *mut OrdaOutput);
    pub fn orda_set_host_slab_bytes(bytes: usize);
    pub fn orda_last_call_bytes(h2d: *mut u64, d2h: *mut u64);

    pub fn orda_context_create(device: c_int, out: *mut *mut OrdaContext, err: *mut c_char, err_len: usize) -> c_int;
    pub fn orda_context_destroy(ctx: *mut OrdaContext);
    pub fn orda_context_check(ctx: *mut OrdaContext, err: *mut c_char, err_len: usize) -> c_int;
    pub fn orda_context_workspace_bytes(ctx: *const OrdaContext) -> usize;
    pub fn orda_context_enable_timing(ctx: *mut OrdaContext, enable: c_int);
    pub fn orda_context_phase_times(ctx: *mut OrdaContext, ms_out: *mut f64, launches_out: *mut u64) -> c_int;
    pub fn orda_context_reset_timing(ctx: *mut OrdaContext);
    pub fn orda_context_set_concurrency(ctx: *mut OrdaContext, spare_sms: c_int);
    pub fn orda_context_launch_count(ctx: *const OrdaContext) -> u64;
    pub fn orda_context_set_l2_persisting(ctx: *mut OrdaContext, bytes: usize, granted: *mut usize,
                                          err: *mut c_char, err_len: usize) -> c_int;
    pub fn orda_context_selftest_bounded_wait(ctx: *mut OrdaContext, limit_us: u32, stream: *mut c_void,
                                              err: *mut c_char, err_len: usize) -> c_int;
    pub fn orda_context_inject_alloc_failures(ctx: *mut OrdaContext, count: c_int);
    pub fn orda_selftest_host_io(err: *mut c_char, err_len: usize) -> c_int;
    pub fn orda_selftest_exp2(x: *const f32, y_fma: *mut f32, y_sfu: *mut f32, n: usize, stream: *mut c_void,
                              err: *mut c_char, err_len: usize) -> c_int;

    pub fn orda_distillation_loss_device(ctx: *mut OrdaContext, student_hidden: *const OrdaDeviceMat,
                                         weight: *const OrdaDeviceMat, labels: *const i64, bt: usize,
                                         teacher: *const OrdaDeviceTeacher, opts: *const OrdaLossOptions,
                                         out: *const OrdaDeviceOutputs, shard: *const OrdaShardOptions,
                                         stream: *mut c_void, plan_out: *mut OrdaChunkPlan, err: *mut c_char,
                                         err_len: usize) -> c_int;
    pub fn orda_vocab_forward_device(ctx: *mut OrdaContext, student_hidden: *const OrdaDeviceMat,
                                     weight_slice: *const OrdaDeviceMat, labels: *const i64, bt: usize,
                                     teacher: *const OrdaDeviceTeacher, opts: *const OrdaLossOptions,
                                     vs: *const OrdaVocabShard, row_partials: *mut f32, stream: *mut c_void,
                                     err: *mut c_char, err_len: usize) -> c_int;
    pub fn orda_vocab_backward_device(ctx: *mut OrdaContext, student_hidden: *const OrdaDeviceMat,
                                      weight_slice: *const OrdaDeviceMat, labels: *const i64, bt: usize,
                                      teacher: *const OrdaDeviceTeacher, opts: *const OrdaLossOptions,
                                      vs: *const OrdaVocabShard, all_partials: *const f32,
                                      out: *const OrdaDeviceOutputs, stream: *mut c_void,
                                      plan_out: *mut OrdaChunkPlan, err: *mut c_char, err_len: usize) -> c_int;

    pub fn orda_context_slots_create(ctx: *mut OrdaContext, world: c_int, rank: c_int, total_rows: usize, h: usize,
                                     copies: c_int, handle_out: *mut OrdaIpcHandle, err: *mut c_char,
                                     err_len: usize) -> c_int;
    pub fn orda_context_slots_attach(ctx: *mut OrdaContext, handles: *const OrdaIpcHandle, err: *mut c_char,
                                     err_len: usize) -> c_int;
    pub fn orda_reduce_slots_device(ctx: *mut OrdaContext, grad_w_slice: *mut f32, ld: usize, labels: *const i64,
                                    n_labels: usize, ignore_index: i64, quantize: c_int, stochastic: c_int,
                                    seed: u64, q: *mut i8, scale: *mut f32, int8_wire: c_int, stream: *mut c_void,
                                    err: *mut c_char, err_len: usize) -> c_int;
    pub fn orda_reduce_slot_set_device(ctx: *mut OrdaContext, copy: c_int, out: *mut f32, ld: usize,
                                       stream: *mut c_void, err: *mut c_char, err_len: usize) -> c_int;

    pub fn orda_quantize_grad_w_device(ctx: *mut OrdaContext, grad_w: *mut f32, v: usize, h: usize, ld: usize,
                                       labels: *const i64, bt: usize, ignore_index: i64, stochastic: c_int,
                                       seed: u64, q: *mut i8, scale: *mut f32, stream: *mut c_void,
                                       err: *mut c_char, err_len: usize) -> c_int;
    pub fn orda_quantize_grad_w_device_noalloc(grad_w: *mut f32, v: usize, h: usize, ld: usize, labels: *const i64,
                                               bt: usize, ignore_index: i64, stochastic: c_int, seed: u64,
                                               q: *mut i8, scale: *mut f32, stream: *mut c_void, err: *mut c_char,
                                               err_len: usize) -> c_int;
    pub fn orda_gemm_bf16_device(ctx: *mut OrdaContext, a: *const c_void, lda: usize, a_kind: c_int,
                                 b: *const c_void, ldb: usize, b_kind: c_int, c: *mut f32, ldc: usize, m: usize,
                                 n: usize, k: usize, alpha: f32, beta: f32, stream: *mut c_void, err: *mut c_char,
                                 err_len: usize) -> c_int;
}
