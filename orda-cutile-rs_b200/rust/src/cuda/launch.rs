//! Safe wrappers over the B200 library for the crate's own types. Replaces
//! the cuTile launcher of the reference crate (src/cuda/launch.rs:51-158,
//! which covered one KL + CE chunk step) with calls that cover the whole
//! `distillation_loss` (src/api.rs:188-422) on the GPU:
//!
//! * [`distillation_loss_b200`]: host `Mat`s in, host `Mat`s out, the
//!   reference's semantics, validation messages and chunk plan;
//! * [`DeviceContext`] and [`DeviceContext::distillation_loss_device`]: bf16
//!   device tensors in, fp32 device gradients out, on the caller's stream.
use std::os::raw::{c_char, c_int, c_void};
use std::ptr;

use super::ffi::*;
use crate::api::{DistillationLossOutput, LossOptions};
use crate::config::{Backend, KernelConfig, Reduction};
use crate::mat::Mat;
use crate::resolver::{ChunkPlan, ChunkSize};
use crate::teacher::Teacher;

const ERR_LEN: usize = 1024;

fn err_string(buf: &[u8]) -> String {
    let end = buf.iter().position(|&b| b == 0).unwrap_or(buf.len());
    String::from_utf8_lossy(&buf[..end]).into_owned()
}

fn mat(m: &Mat) -> OrdaMatF32 {
    OrdaMatF32 { data: m.data.as_ptr(), rows: m.rows, cols: m.cols }
}

const NO_MAT: OrdaMatF32 = OrdaMatF32 { data: ptr::null(), rows: 0, cols: 0 };

fn teacher(t: &Teacher) -> OrdaTeacher {
    match t {
        Teacher::Tied { hidden } => {
            OrdaTeacher { mode: ORDA_TEACHER_TIED, hidden: mat(hidden), weight: NO_MAT, logits: NO_MAT }
        }
        Teacher::Separate { hidden, weight } => {
            OrdaTeacher { mode: ORDA_TEACHER_SEPARATE, hidden: mat(hidden), weight: mat(weight), logits: NO_MAT }
        }
        Teacher::Precomputed { logits } => {
            OrdaTeacher { mode: ORDA_TEACHER_PRECOMPUTED, hidden: NO_MAT, weight: NO_MAT, logits: mat(logits) }
        }
    }
}

fn kernel_config(c: &KernelConfig) -> OrdaKernelConfig {
    OrdaKernelConfig {
        online_softmax: c.online_softmax as i32,
        fast_math: c.fast_math as i32,
        quantize_grad_weight: c.quantize_grad_weight as i32,
        stochastic_rounding: c.stochastic_rounding as i32,
        fp32_grad_weight_accumulation: c.fp32_grad_weight_accumulation as i32,
        has_max_chunks: c.max_chunks.is_some() as i32,
        max_chunks: c.max_chunks.unwrap_or(0),
        max_fused_size: c.max_fused_size,
        has_stochastic_seed: c.stochastic_seed.is_some() as i32,
        stochastic_seed: c.stochastic_seed.unwrap_or(0),
    }
}

/// `LossOptions` as the C struct.
pub fn loss_options(o: &LossOptions) -> OrdaLossOptions {
    OrdaLossOptions {
        student_ce_weight: o.student_ce_weight,
        has_teacher_ce_weight: o.teacher_ce_weight.is_some() as i32,
        teacher_ce_weight: o.teacher_ce_weight.unwrap_or(0.0),
        kd_weight: o.kd_weight,
        temperature: o.temperature,
        ignore_index: o.ignore_index,
        label_smoothing: o.label_smoothing,
        reduction: match o.reduction {
            Reduction::Mean => ORDA_REDUCTION_MEAN,
            Reduction::Sum => ORDA_REDUCTION_SUM,
        },
        chunk_size: match o.chunk_size {
            ChunkSize::Auto => OrdaChunkSize { kind: ORDA_CHUNK_AUTO, fixed_rows: 0 },
            ChunkSize::Fixed(n) => OrdaChunkSize { kind: ORDA_CHUNK_FIXED, fixed_rows: n },
        },
        config: kernel_config(&o.config),
        backend: match o.backend {
            Backend::Auto => ORDA_BACKEND_AUTO,
            Backend::Cpu => ORDA_BACKEND_CPU,
            Backend::Cuda => ORDA_BACKEND_CUDA,
        },
    }
}

/// Copies a library-owned output matrix into a `Mat` (`None` when absent).
fn take(m: &OrdaMatOut) -> Option<Mat> {
    if m.data.is_null() {
        return None;
    }
    // SAFETY: the library allocated rows * cols floats at `data`; they stay
    // valid until orda_output_free.
    let v = unsafe { std::slice::from_raw_parts(m.data, m.rows * m.cols) }.to_vec();
    Some(Mat::from_vec(m.rows, m.cols, v))
}

/// `distillation_loss` (src/api.rs:188-422) on the B200: same inputs, same
/// outputs, same errors. Inputs are rounded to bf16 on the device (the
/// tensor-core operand type); all accumulation is fp32 or wider.
pub fn distillation_loss_b200(
    student_hidden: &Mat,
    weight: &Mat,
    labels: &[i64],
    teacher_: &Teacher,
    opts: &LossOptions,
) -> Result<DistillationLossOutput, String> {
    let t = teacher(teacher_);
    let o = loss_options(opts);
    let (h, w) = (mat(student_hidden), mat(weight));
    // SAFETY: OrdaOutput is plain data; the call fills it on success.
    let mut out: OrdaOutput = unsafe { std::mem::zeroed() };
    let mut err = vec![0u8; ERR_LEN];
    // SAFETY: every pointer refers to a live borrow for the whole call.
    let rc = unsafe {
        orda_distillation_loss(&h, &w, labels.as_ptr(), labels.len(), &t, &o, &mut out,
                               err.as_mut_ptr() as *mut c_char, err.len())
    };
    if rc != ORDA_OK {
        return Err(err_string(&err));
    }
    let res = DistillationLossOutput {
        loss: out.loss,
        student_ce: out.student_ce,
        teacher_ce: out.teacher_ce,
        kl: out.kl,
        grad_student_hidden: take(&out.grad_student_hidden).expect("grad_student_hidden"),
        grad_weight: take(&out.grad_weight).expect("grad_weight"),
        grad_teacher_hidden: take(&out.grad_teacher_hidden),
        grad_teacher_weight: take(&out.grad_teacher_weight),
        chunk_plan: ChunkPlan { chunk_size: out.chunk_plan.chunk_size, num_chunks: out.chunk_plan.num_chunks },
    };
    // SAFETY: returns the library's buffers to its pool.
    unsafe { orda_output_free(&mut out) };
    Ok(res)
}

/// A bf16 or fp32 device matrix (row-major, leading dimension `ld` elements).
#[derive(Clone, Copy, Debug)]
pub struct DeviceMat {
    pub data: *const c_void,
    pub rows: usize,
    pub cols: usize,
    pub ld: usize,
    pub bf16: bool,
}

impl DeviceMat {
    fn c(&self) -> OrdaDeviceMat {
        OrdaDeviceMat {
            data: self.data,
            rows: self.rows,
            cols: self.cols,
            ld: self.ld,
            dtype: if self.bf16 { ORDA_DTYPE_BF16 } else { ORDA_DTYPE_F32 },
        }
    }
}

/// The teacher of a device call.
pub enum DeviceTeacher {
    Tied { hidden: DeviceMat },
    Separate { hidden: DeviceMat, weight: DeviceMat },
    Precomputed { logits: DeviceMat },
}

/// An `OrdaContext`: device workspace, status word and slot buffers of one
/// device; use one per stream.
pub struct DeviceContext {
    raw: *mut OrdaContext,
}

impl DeviceContext {
    pub fn new(device: i32) -> Result<Self, String> {
        let mut raw: *mut OrdaContext = ptr::null_mut();
        let mut err = vec![0u8; ERR_LEN];
        // SAFETY: out-pointer to a local; err buffer of ERR_LEN bytes.
        let rc = unsafe { orda_context_create(device as c_int, &mut raw, err.as_mut_ptr() as *mut c_char, err.len()) };
        if rc != ORDA_OK {
            return Err(err_string(&err));
        }
        Ok(DeviceContext { raw })
    }

    /// Waits for the context's last stream and reports asynchronous device
    /// failures (label out of range, an expired bounded wait).
    pub fn check(&self) -> Result<(), String> {
        let mut err = vec![0u8; ERR_LEN];
        // SAFETY: live context.
        let rc = unsafe { orda_context_check(self.raw, err.as_mut_ptr() as *mut c_char, err.len()) };
        if rc != ORDA_OK {
            return Err(err_string(&err));
        }
        Ok(())
    }

    /// `orda_distillation_loss_device`: enqueues the whole loss and its
    /// gradients on `stream` (a `cudaStream_t`, null for the legacy default
    /// stream) without synchronising. `outputs` holds fp32 device pointers;
    /// its `scalars` receives loss, student CE, teacher CE and KL.
    ///
    /// # Safety
    /// Every pointer in the arguments must be a live device allocation of the
    /// described shape on the context's device until the stream reaches the
    /// end of the call.
    pub unsafe fn distillation_loss_device(
        &self,
        student_hidden: &DeviceMat,
        weight: &DeviceMat,
        labels: *const i64,
        bt: usize,
        teacher_: &DeviceTeacher,
        opts: &LossOptions,
        outputs: &OrdaDeviceOutputs,
        shard: Option<&OrdaShardOptions>,
        stream: *mut c_void,
    ) -> Result<ChunkPlan, String> {
        let none = DeviceMat { data: ptr::null(), rows: 0, cols: 0, ld: 0, bf16: true }.c();
        let t = match teacher_ {
            DeviceTeacher::Tied { hidden } => {
                OrdaDeviceTeacher { mode: ORDA_TEACHER_TIED, hidden: hidden.c(), weight: none, logits: none }
            }
            DeviceTeacher::Separate { hidden, weight } => {
                OrdaDeviceTeacher { mode: ORDA_TEACHER_SEPARATE, hidden: hidden.c(), weight: weight.c(), logits: none }
            }
            DeviceTeacher::Precomputed { logits } => {
                OrdaDeviceTeacher { mode: ORDA_TEACHER_PRECOMPUTED, hidden: none, weight: none, logits: logits.c() }
            }
        };
        let o = loss_options(opts);
        let mut plan = OrdaChunkPlan::default();
        let mut err = vec![0u8; ERR_LEN];
        let rc = orda_distillation_loss_device(
            self.raw,
            &student_hidden.c(),
            &weight.c(),
            labels,
            bt,
            &t,
            &o,
            outputs,
            shard.map_or(ptr::null(), |s| s as *const OrdaShardOptions),
            stream,
            &mut plan,
            err.as_mut_ptr() as *mut c_char,
            err.len(),
        );
        if rc != ORDA_OK {
            return Err(err_string(&err));
        }
        Ok(ChunkPlan { chunk_size: plan.chunk_size, num_chunks: plan.num_chunks })
    }

    pub fn as_raw(&self) -> *mut OrdaContext {
        self.raw
    }
}

impl Drop for DeviceContext {
    fn drop(&mut self) {
        // SAFETY: the context was created by orda_context_create and is
        // destroyed once.
        unsafe { orda_context_destroy(self.raw) };
    }
}
