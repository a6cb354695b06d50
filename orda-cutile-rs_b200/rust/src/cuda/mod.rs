//! GPU backend of the crate on NVIDIA B200 (sm_100a): replaces the cuTile
//! module of the reference crate (src/cuda/mod.rs, kl_kernel.rs,
//! ce_kernel.rs, launch.rs) with bindings to `liborda_b200.so`, whose
//! hand-written tcgen05/TMA kernels run the whole `distillation_loss`.
//!
//! The crate's public API does not change. `distillation_loss`
//! (src/api.rs:188) calls [`dispatch`] right after `validate`, in place of its
//! `match opts.backend` block (src/api.rs:197-207):
//!
//! ```ignore
//! #[cfg(feature = "cuda")]
//! if let Some(result) = crate::cuda::dispatch(student_hidden, weight, labels, teacher, opts) {
//!     return result;
//! }
//! ```
//!
//! and `is_available` (src/lib.rs:70-79) returns [`is_available`].
pub mod ffi;
pub mod launch;

use crate::api::{DistillationLossOutput, LossOptions};
use crate::config::Backend;
use crate::mat::Mat;
use crate::teacher::Teacher;

/// Whether an sm_100 (B200-class) device is present for the library.
pub fn is_available() -> bool {
    // SAFETY: no arguments; queries the CUDA runtime.
    unsafe { ffi::orda_is_available() == 1 }
}

/// Backend selection of `distillation_loss`: `Some(result)` when the B200
/// path takes the call (`Backend::Cuda`, or `Backend::Auto` with a device
/// present), `None` when the crate's CPU reference runs it (`Backend::Cpu`,
/// or `Backend::Auto` without a device). `Backend::Cuda` without a device
/// returns the library's error.
pub fn dispatch(
    student_hidden: &Mat,
    weight: &Mat,
    labels: &[i64],
    teacher: &Teacher,
    opts: &LossOptions,
) -> Option<Result<DistillationLossOutput, String>> {
    match opts.backend {
        Backend::Cuda => Some(launch::distillation_loss_b200(student_hidden, weight, labels, teacher, opts)),
        Backend::Auto if is_available() => {
            Some(launch::distillation_loss_b200(student_hidden, weight, labels, teacher, opts))
        }
        Backend::Auto | Backend::Cpu => None,
    }
}
