// abi_layout.cpp -- the memory layout of every struct of include/orda.h as
// compiled into this library (sizeof / offsetof), so that the bindings in
// other languages (the Rust #[repr(C)] mirrors, the Python ctypes mirrors)
// can be checked against the library itself rather than against a reading
// of the header.
#include <cstddef>

#include "../../include/orda.h"

namespace {

#define ORDA_STRUCT(S) {#S, "", 0, sizeof(S)}
#define ORDA_FIELD(S, F) {#S, #F, offsetof(S, F), sizeof(static_cast<S*>(nullptr)->F)}

const OrdaFieldLayout kLayout[] = {
    ORDA_STRUCT(OrdaMatF32),
    ORDA_FIELD(OrdaMatF32, data),
    ORDA_FIELD(OrdaMatF32, rows),
    ORDA_FIELD(OrdaMatF32, cols),

    ORDA_STRUCT(OrdaMatOut),
    ORDA_FIELD(OrdaMatOut, data),
    ORDA_FIELD(OrdaMatOut, rows),
    ORDA_FIELD(OrdaMatOut, cols),

    ORDA_STRUCT(OrdaTeacher),
    ORDA_FIELD(OrdaTeacher, mode),
    ORDA_FIELD(OrdaTeacher, hidden),
    ORDA_FIELD(OrdaTeacher, weight),
    ORDA_FIELD(OrdaTeacher, logits),

    ORDA_STRUCT(OrdaKernelConfig),
    ORDA_FIELD(OrdaKernelConfig, online_softmax),
    ORDA_FIELD(OrdaKernelConfig, fast_math),
    ORDA_FIELD(OrdaKernelConfig, quantize_grad_weight),
    ORDA_FIELD(OrdaKernelConfig, stochastic_rounding),
    ORDA_FIELD(OrdaKernelConfig, fp32_grad_weight_accumulation),
    ORDA_FIELD(OrdaKernelConfig, has_max_chunks),
    ORDA_FIELD(OrdaKernelConfig, max_chunks),
    ORDA_FIELD(OrdaKernelConfig, max_fused_size),
    ORDA_FIELD(OrdaKernelConfig, has_stochastic_seed),
    ORDA_FIELD(OrdaKernelConfig, stochastic_seed),

    ORDA_STRUCT(OrdaChunkSize),
    ORDA_FIELD(OrdaChunkSize, kind),
    ORDA_FIELD(OrdaChunkSize, fixed_rows),

    ORDA_STRUCT(OrdaChunkPlan),
    ORDA_FIELD(OrdaChunkPlan, chunk_size),
    ORDA_FIELD(OrdaChunkPlan, num_chunks),

    ORDA_STRUCT(OrdaLossOptions),
    ORDA_FIELD(OrdaLossOptions, student_ce_weight),
    ORDA_FIELD(OrdaLossOptions, has_teacher_ce_weight),
    ORDA_FIELD(OrdaLossOptions, teacher_ce_weight),
    ORDA_FIELD(OrdaLossOptions, kd_weight),
    ORDA_FIELD(OrdaLossOptions, temperature),
    ORDA_FIELD(OrdaLossOptions, ignore_index),
    ORDA_FIELD(OrdaLossOptions, label_smoothing),
    ORDA_FIELD(OrdaLossOptions, reduction),
    ORDA_FIELD(OrdaLossOptions, chunk_size),
    ORDA_FIELD(OrdaLossOptions, config),
    ORDA_FIELD(OrdaLossOptions, backend),

    ORDA_STRUCT(OrdaOutput),
    ORDA_FIELD(OrdaOutput, loss),
    ORDA_FIELD(OrdaOutput, student_ce),
    ORDA_FIELD(OrdaOutput, teacher_ce),
    ORDA_FIELD(OrdaOutput, kl),
    ORDA_FIELD(OrdaOutput, grad_student_hidden),
    ORDA_FIELD(OrdaOutput, grad_weight),
    ORDA_FIELD(OrdaOutput, grad_teacher_hidden),
    ORDA_FIELD(OrdaOutput, grad_teacher_weight),
    ORDA_FIELD(OrdaOutput, chunk_plan),

    ORDA_STRUCT(OrdaDeviceMat),
    ORDA_FIELD(OrdaDeviceMat, data),
    ORDA_FIELD(OrdaDeviceMat, rows),
    ORDA_FIELD(OrdaDeviceMat, cols),
    ORDA_FIELD(OrdaDeviceMat, ld),
    ORDA_FIELD(OrdaDeviceMat, dtype),

    ORDA_STRUCT(OrdaDeviceTeacher),
    ORDA_FIELD(OrdaDeviceTeacher, mode),
    ORDA_FIELD(OrdaDeviceTeacher, hidden),
    ORDA_FIELD(OrdaDeviceTeacher, weight),
    ORDA_FIELD(OrdaDeviceTeacher, logits),

    ORDA_STRUCT(OrdaDeviceOutputs),
    ORDA_FIELD(OrdaDeviceOutputs, grad_student_hidden),
    ORDA_FIELD(OrdaDeviceOutputs, ld_grad_student_hidden),
    ORDA_FIELD(OrdaDeviceOutputs, grad_weight),
    ORDA_FIELD(OrdaDeviceOutputs, ld_grad_weight),
    ORDA_FIELD(OrdaDeviceOutputs, grad_teacher_hidden),
    ORDA_FIELD(OrdaDeviceOutputs, ld_grad_teacher_hidden),
    ORDA_FIELD(OrdaDeviceOutputs, grad_teacher_weight),
    ORDA_FIELD(OrdaDeviceOutputs, ld_grad_teacher_weight),
    ORDA_FIELD(OrdaDeviceOutputs, grad_weight_q),
    ORDA_FIELD(OrdaDeviceOutputs, grad_weight_scale),
    ORDA_FIELD(OrdaDeviceOutputs, scalars),

    ORDA_STRUCT(OrdaShardOptions),
    ORDA_FIELD(OrdaShardOptions, global_non_ignore),
    ORDA_FIELD(OrdaShardOptions, skip_quantize),
    ORDA_FIELD(OrdaShardOptions, scatter_grad_weight),
    ORDA_FIELD(OrdaShardOptions, int8_wire),
    ORDA_FIELD(OrdaShardOptions, reserved),

    ORDA_STRUCT(OrdaVocabShard),
    ORDA_FIELD(OrdaVocabShard, v_total),
    ORDA_FIELD(OrdaVocabShard, v0),
    ORDA_FIELD(OrdaVocabShard, world),
    ORDA_FIELD(OrdaVocabShard, include_rows),
    ORDA_FIELD(OrdaVocabShard, scatter_grad_hidden),
    ORDA_FIELD(OrdaVocabShard, pad),

    ORDA_STRUCT(OrdaIpcHandle),
    ORDA_FIELD(OrdaIpcHandle, bytes),

    ORDA_STRUCT(OrdaFieldLayout),
    ORDA_FIELD(OrdaFieldLayout, struct_name),
    ORDA_FIELD(OrdaFieldLayout, field),
    ORDA_FIELD(OrdaFieldLayout, offset),
    ORDA_FIELD(OrdaFieldLayout, size),
};

#undef ORDA_FIELD
#undef ORDA_STRUCT

}  // namespace

extern "C" size_t orda_abi_layout(const OrdaFieldLayout** out) {
  if (out) *out = kLayout;
  return sizeof(kLayout) / sizeof(kLayout[0]);
}
