/*
 * orda.h -- C ABI of the B200 (sm_100a) ORDA distillation-loss library.
 *
 * This header is the drop-in boundary for the reference crate
 * malcolmgreaves/orda-cutile-rs. Every type and entry point below names the
 * reference item it replaces (path:line inside that crate). Plain C: no CUDA
 * or torch types appear in any signature (streams are passed as void*).
 *
 * Two families of entry points:
 *   - host-Mat entry (orda_distillation_loss): f32 host matrices in, callee
 *     allocated f32 host gradients out, exactly the semantics of
 *     `distillation_loss` (src/api.rs:188-422);
 *   - device entry (orda_distillation_loss_device): bf16 device tensors,
 *     fp32 device gradients, caller stream; the timed path.
 *
 * Status codes: 0 = Ok, non-zero = Err, with the message written to `err`
 * (the reference returns `Result<_, String>`).
 */
#ifndef ORDA_H_
#define ORDA_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define ORDA_ABI_VERSION 2

#if defined(__GNUC__)
#define ORDA_API __attribute__((visibility("default")))
#else
#define ORDA_API
#endif

enum {
  ORDA_OK = 0,
  ORDA_ERR_INVALID = 1,   /* argument validation failed (src/api.rs:104-181) */
  ORDA_ERR_BACKEND = 2,   /* backend unavailable (src/api.rs:197-207)       */
  ORDA_ERR_CUDA = 3,      /* CUDA runtime / driver error                     */
  ORDA_ERR_OOM = 4,       /* device allocation failed after the OOM ladder   */
  ORDA_ERR_TIMEOUT = 5,   /* a bounded device wait expired                   */
  ORDA_ERR_LABEL = 6      /* device-side label range check failed            */
};

/* Row-major f32 host matrix; replaces `Mat` (src/mat.rs:10-14). */
typedef struct OrdaMatF32 {
  const float* data;
  size_t rows;
  size_t cols;
} OrdaMatF32;

/* Callee-allocated f32 host matrix (output side of `Mat`). data == NULL
 * encodes `None` for the optional gradients (src/api.rs:84-89). */
typedef struct OrdaMatOut {
  float* data;
  size_t rows;
  size_t cols;
} OrdaMatOut;

/* `TeacherMode` (src/teacher.rs:37-42). */
typedef enum OrdaTeacherMode {
  ORDA_TEACHER_TIED = 0,
  ORDA_TEACHER_SEPARATE = 1,
  ORDA_TEACHER_PRECOMPUTED = 2
} OrdaTeacherMode;

/* `Teacher::{Tied{hidden}, Separate{hidden,weight}, Precomputed{logits}}`
 * (src/teacher.rs:11-32) as a tagged struct; unused members are ignored. */
typedef struct OrdaTeacher {
  OrdaTeacherMode mode;
  OrdaMatF32 hidden; /* Tied, Separate   */
  OrdaMatF32 weight; /* Separate         */
  OrdaMatF32 logits; /* Precomputed      */
} OrdaTeacher;

/* `Reduction` (src/config.rs:11-17). */
typedef enum OrdaReduction { ORDA_REDUCTION_MEAN = 0, ORDA_REDUCTION_SUM = 1 } OrdaReduction;

/* `Backend` (src/config.rs:21-31). In this library Auto and Cuda select the
 * B200 path; Cpu is rejected (the library ships no CPU path). */
typedef enum OrdaBackend { ORDA_BACKEND_AUTO = 0, ORDA_BACKEND_CPU = 1, ORDA_BACKEND_CUDA = 2 } OrdaBackend;

/* `Profile` (src/config.rs:35-42). Fast (KernelConfig.fast_math = 1) stores
 * the logits of the forward group as fp16 (saturated to the largest finite
 * value) instead of fp32, takes the label logits of the losses from an exact
 * fp32 dot product, and computes a quarter of the logits epilogue's
 * tempered-sum exp2 on the FMA pipe (range reduction and a degree-6
 * polynomial). The softmax statistics
 * still come from the fp32 GEMM accumulators, so the CE terms are as precise
 * as with Balanced; the KL cross term and the logit gradients read the fp16
 * logits. Stated tolerances against the reference: student and teacher CE
 * 1e-4 relative, KL and loss 1e-3 relative, gradients relative L2 2e-2. The
 * INT8 quantiser keeps IEEE divides in every profile (bit-exactness).
 * Balanced and Debug keep fp32 logits. */
typedef enum OrdaProfile { ORDA_PROFILE_BALANCED = 0, ORDA_PROFILE_FAST = 1, ORDA_PROFILE_DEBUG = 2 } OrdaProfile;

/* `KernelConfig` (src/config.rs:46-63). Option<T> fields carry a has_ flag. */
typedef struct OrdaKernelConfig {
  int32_t online_softmax;
  int32_t fast_math;
  int32_t quantize_grad_weight;
  int32_t stochastic_rounding;
  int32_t fp32_grad_weight_accumulation;
  int32_t has_max_chunks;
  size_t max_chunks;
  size_t max_fused_size;
  int32_t has_stochastic_seed;
  uint64_t stochastic_seed;
} OrdaKernelConfig;

/* `ChunkSize::{Auto, Fixed(usize)}` (src/resolver.rs:10-16). */
typedef enum OrdaChunkKind { ORDA_CHUNK_AUTO = 0, ORDA_CHUNK_FIXED = 1 } OrdaChunkKind;
typedef struct OrdaChunkSize {
  OrdaChunkKind kind;
  size_t fixed_rows;
} OrdaChunkSize;

/* `ChunkPlan` (src/resolver.rs:40-45). */
typedef struct OrdaChunkPlan {
  size_t chunk_size;
  size_t num_chunks;
} OrdaChunkPlan;

/* `LossOptions` (src/api.rs:25-47); `teacher_ce_weight: Option<f32>`. */
typedef struct OrdaLossOptions {
  float student_ce_weight;
  int32_t has_teacher_ce_weight;
  float teacher_ce_weight;
  float kd_weight;
  float temperature;
  int64_t ignore_index;
  float label_smoothing;
  OrdaReduction reduction;
  OrdaChunkSize chunk_size;
  OrdaKernelConfig config;
  OrdaBackend backend;
} OrdaLossOptions;

/* `DistillationLossOutput` (src/api.rs:71-92). Gradients are allocated by
 * the library (page-locked host memory from a reuse pool) and must be
 * released with orda_output_free(), never free(). */
typedef struct OrdaOutput {
  float loss;
  float student_ce;
  float teacher_ce;
  float kl;
  OrdaMatOut grad_student_hidden;
  OrdaMatOut grad_weight;
  OrdaMatOut grad_teacher_hidden; /* data == NULL: None */
  OrdaMatOut grad_teacher_weight; /* data == NULL: None */
  OrdaChunkPlan chunk_plan;
} OrdaOutput;

/* ---------------------------------------------------------------------------
 * Layout of this header's structs as compiled into the library
 * ------------------------------------------------------------------------- */

/* One entry per struct (field = "", offset 0, size = sizeof the struct)
 * followed by one per field (offsetof, sizeof), in declaration order. */
typedef struct OrdaFieldLayout {
  const char* struct_name;
  const char* field;
  size_t offset;
  size_t size;
} OrdaFieldLayout;
/* Points *out at the library's static table and returns its length. The
 * bindings in other languages (the Rust #[repr(C)] mirrors that replace the
 * reference crate's src/cuda/launch.rs, Python ctypes) are checked against
 * it; no counterpart in the reference. */
ORDA_API size_t orda_abi_layout(const OrdaFieldLayout** out);

/* ---------------------------------------------------------------------------
 * Configuration helpers (pure host logic, no device needed)
 * ------------------------------------------------------------------------- */

/* `LossOptions::default()` (src/api.rs:49-64). */
ORDA_API void orda_loss_options_default(OrdaLossOptions* out);
/* `KernelConfig::from_profile` (src/config.rs:81-93); Default = Balanced. */
ORDA_API void orda_kernel_config_from_profile(OrdaProfile profile, OrdaKernelConfig* out);
/* `KernelConfig::validate` (src/config.rs:106-119). */
ORDA_API int orda_kernel_config_validate(const OrdaKernelConfig* cfg, char* err, size_t err_len);
/* `is_power_of_two` (src/config.rs:122-124). */
ORDA_API int orda_is_power_of_two(size_t value);
/* `Teacher::default_teacher_ce_weight` (src/teacher.rs:54-59). */
ORDA_API float orda_default_teacher_ce_weight(OrdaTeacherMode mode);
/* `is_available` (src/lib.rs:70-79): 1 iff an sm_100 device is present. */
ORDA_API int orda_is_available(void);

/* `chunks_from_raw` (src/resolver.rs:28-36). */
ORDA_API size_t orda_chunks_from_raw(double raw);
/* `resolve_chunk_size` (src/resolver.rs:53-99). has_v / has_max_chunks
 * encode the Option arguments. bt must be > 0 (returns {0,0} otherwise). */
ORDA_API void orda_resolve_chunk_size(size_t bt, OrdaChunkSize chunk_size, int has_v, size_t v,
                             int has_max_chunks, size_t max_chunks, OrdaChunkPlan* out);
/* `default_max_chunks_limit` (src/resolver.rs:103-105). */
ORDA_API size_t orda_default_max_chunks_limit(size_t bt);
/* `chunk_doubling_schedule` (src/resolver.rs:114-126). Writes up to out_cap
 * entries and returns the full schedule length. */
ORDA_API size_t orda_chunk_doubling_schedule(size_t bt, size_t start, size_t limit, size_t* out, size_t out_cap);

/* OOM retry ladder around `chunk_doubling_schedule` (src/resolver.rs:107-126,
 * the upstream dispatcher's `dynamic_chunk` loop that the reference documents
 * but never wires). Calls try_alloc(num_chunks, chunk_size, user) for each
 * rung, starting at `start`; the first rung returning 0 wins and is written
 * to `out`. Returns ORDA_OK, or ORDA_ERR_OOM when every rung failed. The
 * device entry uses this with its workspace allocator. */
typedef int (*OrdaTryAllocFn)(size_t num_chunks, size_t chunk_size, void* user);
ORDA_API int orda_chunk_retry(size_t bt, size_t start, size_t limit, OrdaTryAllocFn try_alloc, void* user,
                     OrdaChunkPlan* out);

/* `validate` (src/api.rs:104-181) on host matrices. On success writes
 * (V, H, BT). Messages are identical to the reference's. */
ORDA_API int orda_validate(const OrdaMatF32* student_hidden, const OrdaMatF32* weight, const int64_t* labels,
                  size_t n_labels, const OrdaTeacher* teacher, const OrdaLossOptions* opts, size_t* v_out,
                  size_t* h_out, size_t* bt_out, char* err, size_t err_len);

/* ---------------------------------------------------------------------------
 * Host-Mat entry: `distillation_loss` (src/api.rs:188-422)
 * ------------------------------------------------------------------------- */

/* Computes loss, components and gradients on the B200 with the reference's
 * semantics. Inputs are f32 host matrices (pinned or pageable); hidden states
 * and weights are rounded to bf16 (tensor-core operand type), on the host
 * before they are copied; Precomputed teacher logits keep their fp32 values
 * (a chunk of them that holds bf16 values only is copied as bf16 and widened
 * exactly on the device). Gradients come back as library-allocated f32 host
 * matrices; free them with orda_output_free(). With quantize_grad_weight the
 * dequantised grad_W is formed on the host from the INT8 codes, scales and
 * exact target rows (the same float multiply as on the device). Runs on
 * device 0 on internal streams, synchronously, with up to 16 host worker
 * threads of its own during the call. */
ORDA_API int orda_distillation_loss(const OrdaMatF32* student_hidden, const OrdaMatF32* weight, const int64_t* labels,
                           size_t n_labels, const OrdaTeacher* teacher, const OrdaLossOptions* opts,
                           OrdaOutput* out, char* err, size_t err_len);
ORDA_API void orda_output_free(OrdaOutput* out);
/* Copy pipeline of orda_distillation_loss. The call overlaps its host<->device
 * copies with the device work: the bf16 operands are copied first, then
 * Precomputed teacher logits in row slabs of about `bytes` (whole chunks of
 * the resolver's plan) when they exceed two slabs; each slab's forward and
 * backward work runs while the next slab is copied, and grad_hidden rows are
 * copied back as they are final. Results do not depend on the slab size
 * beyond fp32 summation order of grad_W. 0 restores the default (512 MiB).
 * Process-wide; no counterpart in the reference (src/api.rs:188-422 has no
 * device copies). */
ORDA_API void orda_set_host_slab_bytes(size_t bytes);
/* Bytes the last successful orda_distillation_loss call of this process
 * copied host->device and device->host (which chunks crossed as bf16 and
 * whether grad_W came back compressed depend on the call and the host's
 * speed). Either pointer may be NULL. No counterpart in the reference. */
ORDA_API void orda_last_call_bytes(uint64_t* h2d, uint64_t* d2h);

/* ---------------------------------------------------------------------------
 * Device entry (replaces the GPU launcher src/cuda/launch.rs:51-158, which
 * covered only the KL + CE step; this covers the whole chunk loop)
 * ------------------------------------------------------------------------- */

typedef struct OrdaContext OrdaContext;

/* A context owns the device workspace (logits chunk, dlogits group, row
 * statistics) and a device status word. Use one context per stream. */
ORDA_API int orda_context_create(int device, OrdaContext** out, char* err, size_t err_len);
ORDA_API void orda_context_destroy(OrdaContext* ctx);
/* Synchronizes the context's last stream and reports asynchronous device
 * failures (label out of range, bounded-wait timeout). */
ORDA_API int orda_context_check(OrdaContext* ctx, char* err, size_t err_len);
/* Bytes of device workspace currently held by the context. */
ORDA_API size_t orda_context_workspace_bytes(const OrdaContext* ctx);
/* Phase timing: when enabled, the device entry records CUDA events around
 * each kernel phase on the stream it launches on. Phases:
 *   0 logits GEMMs (teacher + student, fused statistics epilogue)
 *   1 row kernel (losses + bf16 logit gradients)
 *   2 dgrad GEMMs   3 wgrad GEMMs   4 INT8 quantiser   5 label pass + finalize
 * orda_context_phase_times synchronizes, adds the elapsed milliseconds and
 * kernel-launch counts accumulated since the last reset into the outputs
 * (arrays of ORDA_NUM_PHASES entries) and returns ORDA_NUM_PHASES. */
#define ORDA_NUM_PHASES 6
ORDA_API void orda_context_enable_timing(OrdaContext* ctx, int enable);
ORDA_API int orda_context_phase_times(OrdaContext* ctx, double* ms_out, uint64_t* launches_out);
ORDA_API void orda_context_reset_timing(OrdaContext* ctx);
/* Concurrency of the bandwidth-bound kernels with the tensor-bound GEMMs.
 * With spare_sms > 0 (default 0: serial) the device entry runs the statistics of
 * given (Precomputed) teacher logits on a low-priority auxiliary stream while
 * the logits GEMM runs on all SMs but spare_sms, and for the last backward
 * group runs wgrad before dgrad and the INT8 round trip on that stream while
 * dgrad runs; the call still ends on the caller's stream after all of it.
 * Results do not depend on the setting. 0 makes every kernel serial on the
 * caller's stream; values are clamped to [0, 32]. Measured at c4 with 2 to 8
 * spare SMs the step got no faster: the side kernels compete with the GEMMs
 * for HBM, L2 and power. No counterpart in the reference (a single-threaded
 * CPU path). */
ORDA_API void orda_context_set_concurrency(OrdaContext* ctx, int spare_sms);
/* Total kernels this context has launched (all calls, timing on or off). */
ORDA_API uint64_t orda_context_launch_count(const OrdaContext* ctx);
/* Persisting-L2 carve-out for this context's device (cudaLimitPersistingL2CacheSize,
 * a limit of the CUDA context: it ends with the process). The GEMMs load the
 * operand that every tile re-reads (the hidden states when they take <= 64 MiB)
 * with an evict-last policy; those lines stay resident only inside this
 * carve-out, which CUDA sizes to 0 by default; after each such GEMM a small
 * kernel returns those lines to normal priority. 64 MiB cut the DRAM traffic of
 * a c4 step's GEMMs from 42 to 33 GB, but the bandwidth-bound row and INT8
 * kernels ran about 1.3 ms per step slower with the carve-out in place, so the
 * step got slower: off unless called (the carve-out is shared by every kernel
 * of the process). The request is capped at the device maximum and rounded by
 * the driver to its granularity; *granted receives the limit now in effect.
 * orda_context_destroy restores the previous limit. */
ORDA_API int orda_context_set_l2_persisting(OrdaContext* ctx, size_t bytes, size_t* granted, char* err,
                                            size_t err_len);
/* Failure-detection self-test: launches a one-warp kernel whose bounded
 * device wait (the same mechanism every kernel uses) on a barrier that nothing
 * completes gives up after limit_us microseconds (at most 1 s) and records a
 * timeout; orda_context_check then returns ORDA_ERR_TIMEOUT and the context
 * stays usable for further calls. */
ORDA_API int orda_context_selftest_bounded_wait(OrdaContext* ctx, uint32_t limit_us, void* stream, char* err,
                                                size_t err_len);
/* Test hook for the OOM ladder: the next `count` workspace allocations fail
 * as if cudaMalloc had returned cudaErrorMemoryAllocation. */
ORDA_API void orda_context_inject_alloc_failures(OrdaContext* ctx, int count);
/* Accuracy self-test of the two exp2 implementations of the kernels, on the
 * current device and `stream`: y_fma[i] = 2^x[i] computed on the FMA pipe
 * (the Fast profile's range-reduced polynomial), y_sfu[i] = the SFU's
 * ex2.approx. x, y_fma, y_sfu: device arrays of n floats. No counterpart in
 * the reference. */
ORDA_API int orda_selftest_exp2(const float* x, float* y_fma, float* y_sfu, size_t n, void* stream, char* err,
                                size_t err_len);
/* Self-test of the host-side passes of the host-Mat entry (fp32 -> bf16
 * rounding, the exact bf16 narrowing of teacher logits, the dequantisation
 * of grad_W), on the host only: every instruction-set version this CPU runs
 * (scalar, AVX2, AVX-512) against the scalar definitions, over rounding
 * ties, NaN, infinities, subnormals and misaligned outputs. Returns ORDA_OK
 * (err then names the versions checked) or ORDA_ERR_BACKEND with the first
 * difference. Needs no GPU. No counterpart in the reference. */
ORDA_API int orda_selftest_host_io(char* err, size_t err_len);

/* Element type of a device matrix. Hidden states and weights are bf16 (the
 * tensor-core operand type); Precomputed teacher logits may be bf16 or f32. */
typedef enum OrdaDType { ORDA_DTYPE_BF16 = 0, ORDA_DTYPE_F32 = 1 } OrdaDType;

/* Device matrix, row-major with leading dimension `ld` (elements).
 * Requirements: data 16-byte aligned, ld * sizeof(elem) a multiple of 16,
 * ld >= cols. */
typedef struct OrdaDeviceMat {
  const void* data;
  size_t rows;
  size_t cols;
  size_t ld;
  OrdaDType dtype;
} OrdaDeviceMat;

typedef struct OrdaDeviceTeacher {
  OrdaTeacherMode mode;
  OrdaDeviceMat hidden; /* Tied [BT,H], Separate [BT,H_t]          */
  OrdaDeviceMat weight; /* Separate [V,H_t]                         */
  OrdaDeviceMat logits; /* Precomputed [BT,V]                       */
} OrdaDeviceTeacher;

/* fp32 device outputs; leading dimensions in elements. */
typedef struct OrdaDeviceOutputs {
  float* grad_student_hidden; size_t ld_grad_student_hidden; /* [BT,H], required              */
  float* grad_weight; size_t ld_grad_weight;                 /* [V,H], required               */
  float* grad_teacher_hidden; size_t ld_grad_teacher_hidden; /* [BT,H_t] iff w_t>0, Tied|Sep  */
  float* grad_teacher_weight; size_t ld_grad_teacher_weight; /* [V,H_t] iff w_t>0, Separate   */
  int8_t* grad_weight_q;     /* optional [V,H] int8, ld = H, when quantize_grad_weight           */
  float* grad_weight_scale;  /* optional [V] per-row scales, when quantize_grad_weight           */
  float* scalars;            /* required device float[4]: loss, student_ce, teacher_ce, kl      */
} OrdaDeviceOutputs;

/* Sharding extras for data-parallel callers (rows split across ranks). */
typedef struct OrdaShardOptions {
  int64_t global_non_ignore; /* > 0: use this token count as the mean denominator */
  int32_t skip_quantize;     /* 1: leave grad_W un-quantized (quantize after the reduction) */
  int32_t scatter_grad_weight; /* 1: the wgrad GEMM writes this rank's grad_W partial straight into the
                                  owning ranks' slot buffers (orda_context_slots_*), overlapping the
                                  reduce-scatter with the GEMM; out->grad_weight is not written and may
                                  be NULL; implies skip_quantize. Finish with orda_reduce_slots_device
                                  after a cross-rank barrier. */
  int32_t int8_wire;         /* with scatter_grad_weight: send each owner its rows of this rank's partial
                                as row-wise INT8 codes + one fp32 scale per row (the quantize_rowwise_int8
                                rules of src/quant.rs:97-117) instead of fp32: 4x fewer bytes over NVLink,
                                but the reduced grad_W carries the quantisation error of every partial
                                (not bit-identical to one device; see orda_reduce_slots_device). The
                                partial is first written to a context buffer of V x H fp32. */
  int32_t reserved;          /* 0 */
} OrdaShardOptions;

/* The timed path. Enqueues everything on `stream` (a cudaStream_t; NULL =
 * legacy default stream); no host synchronization. labels is a device int64
 * array of length bt. `plan_out` (optional) receives the chunk plan used. */
ORDA_API int orda_distillation_loss_device(OrdaContext* ctx, const OrdaDeviceMat* student_hidden,
                                  const OrdaDeviceMat* weight, const int64_t* labels, size_t bt,
                                  const OrdaDeviceTeacher* teacher, const OrdaLossOptions* opts,
                                  const OrdaDeviceOutputs* out, const OrdaShardOptions* shard,
                                  void* stream, OrdaChunkPlan* plan_out, char* err, size_t err_len);

/* Vocabulary-sharded calls (tensor parallel over the output head) for the
 * largest vocabularies: rank r of `world` holds W rows [v0, v0 + V_r) of the
 * full v_total (and the same rows of a Separate teacher's W, or the same
 * columns of Precomputed teacher logits) and every rank holds all BT rows of
 * the hidden states and labels. No counterpart in the reference, which runs
 * on one device; the loss and gradients are those of `distillation_loss`
 * (src/api.rs:188-422) on the full vocabulary:
 *   1. orda_vocab_forward_device: the slice's logits GEMMs; writes one tuple
 *      of ORDA_VOCAB_TUPLE floats per row (the slice's max / sum-exp
 *      statistics of student and teacher and the label's logits when the
 *      slice holds the label column, as 12 doubles: the merge then matches
 *      the single-device one to f64 precision) to row_partials
 *      [bt][ORDA_VOCAB_TUPLE], 8-byte aligned;
 *   2. the caller all-gathers the tuples of every rank, by rank, into
 *      [world][bt][ORDA_VOCAB_TUPLE] (e.g. an NCCL all-gather);
 *   3. orda_vocab_backward_device on the same context and inputs: merges the
 *      tuples (rank order, f64), the gradient pass over the slice and the
 *      backward GEMMs. Outputs: grad_weight / grad_teacher_weight = this
 *      slice's rows [V_r, H] (complete), grad_student_hidden /
 *      grad_teacher_hidden = this rank's partial sums over its slice, and
 *      scalars = this rank's partial scalars: sum both over the ranks (e.g.
 *      an NCCL all-reduce). Exactly one rank sets include_rows = 1 (it adds
 *      the per-row CE and KL terms to its scalars). The INT8 round trip, if
 *      configured, runs on the slice (target rows = labels in the slice).
 * The slice logits of the whole batch stay in the context's workspace
 * between the two calls; nothing else may run on the context in between. */
#define ORDA_VOCAB_TUPLE 24
typedef struct OrdaVocabShard {
  int64_t v_total;      /* full vocabulary */
  int64_t v0;           /* first vocabulary row of this rank's slice */
  int32_t world;        /* ranks whose tuples phase 2 merges */
  int32_t include_rows; /* phase 2: 1 on exactly one rank */
  int32_t scatter_grad_hidden; /* phase 2: 1 = the dgrad GEMMs write this rank's grad_hidden partial of
                                  every owner's rows (owner slices as orda_context_slots_create)
                                  straight into the owners' slot buffers (orda_context_slots_create
                                  with total_rows = BT, h = H, copies = 2 when teacher hidden
                                  gradients exist, set 0 student, set 1 teacher); the grad_*_hidden
                                  outputs are then not written. After a barrier across the ranks,
                                  orda_reduce_slot_set_device gives each rank its reduced rows
                                  (a reduce-scatter of grad_hidden over rows). */
  int32_t pad;
} OrdaVocabShard;
ORDA_API int orda_vocab_forward_device(OrdaContext* ctx, const OrdaDeviceMat* student_hidden,
                                       const OrdaDeviceMat* weight_slice, const int64_t* labels, size_t bt,
                                       const OrdaDeviceTeacher* teacher, const OrdaLossOptions* opts,
                                       const OrdaVocabShard* vs, float* row_partials, void* stream, char* err,
                                       size_t err_len);
ORDA_API int orda_vocab_backward_device(OrdaContext* ctx, const OrdaDeviceMat* student_hidden,
                                        const OrdaDeviceMat* weight_slice, const int64_t* labels, size_t bt,
                                        const OrdaDeviceTeacher* teacher, const OrdaLossOptions* opts,
                                        const OrdaVocabShard* vs, const float* all_partials,
                                        const OrdaDeviceOutputs* out, void* stream, OrdaChunkPlan* plan_out,
                                        char* err, size_t err_len);

/* Fused grad_W reduce-scatter for row-sharded runs on the GPUs of one node
 * (up to 8 ranks, one process per GPU). There is no counterpart in the
 * reference, which runs on one device; for data-parallel callers that
 * split the rows across GPUs it replaces a separate NCCL reduce-scatter of
 * the fp32 grad_W.
 *   1. orda_context_slots_create: rank `rank` of `world` allocates its slot
 *      buffer for `total_rows` rows split over the owners (rank o owns rows
 *      [o*slice, min((o+1)*slice, total_rows)) with slice = ceil(total_rows /
 *      world) rounded up to 8; the last owner may hold fewer), `copies` sets
 *      of fp32 [world][slice][h] (here one set, total_rows = V), and gets its
 *      CUDA IPC handle;
 *   2. the caller all-gathers the handles; orda_context_slots_attach maps the
 *      other ranks' buffers (handles indexed by rank);
 *   3. orda_distillation_loss_device with shard->scatter_grad_weight = 1: the
 *      wgrad GEMM stores each rank's partial of grad_W rows [o*slice,
 *      (o+1)*slice) into rank o's buffer, partial index = this rank;
 *   4. after a barrier across the ranks (e.g. an NCCL all-reduce of one value
 *      on the same stream), orda_reduce_slots_device sums the `world` partials
 *      of this rank's rows in rank order into grad_w_slice [rows of this rank,
 *      h] and, if quantize, applies the INT8 round trip of
 *      orda_quantize_grad_w_device with the labels of all ranks (target rows
 *      are labels in this rank's row range; stochastic draws are indexed by
 *      the global row). int8_wire must match the scatter calls'
 *      OrdaShardOptions.int8_wire: the partials are then dequantised (q * s)
 *      before the sum; against fp32 partials the reduced rows differ by the
 *      partials' quantisation error (relative L2 about 1e-2).
 * The buffers are released by orda_context_destroy or the next create. */
typedef struct OrdaIpcHandle {
  char bytes[64];
} OrdaIpcHandle;
ORDA_API int orda_context_slots_create(OrdaContext* ctx, int world, int rank, size_t total_rows, size_t h,
                                       int copies, OrdaIpcHandle* handle_out, char* err, size_t err_len);
ORDA_API int orda_context_slots_attach(OrdaContext* ctx, const OrdaIpcHandle* handles, char* err, size_t err_len);
ORDA_API int orda_reduce_slots_device(OrdaContext* ctx, float* grad_w_slice, size_t ld, const int64_t* labels,
                                      size_t n_labels, int64_t ignore_index, int quantize, int stochastic,
                                      uint64_t seed, int8_t* q, float* scale, int int8_wire, void* stream,
                                      char* err, size_t err_len);
/* Sum, in rank order, of the `world` partials in this rank's slot set
 * `copy` into out [rows of this rank, h] (ld >= h), with no quantisation:
 * the reduce-scatter of grad_hidden of vocabulary-sharded calls. */
ORDA_API int orda_reduce_slot_set_device(OrdaContext* ctx, int copy, float* out, size_t ld, void* stream, char* err,
                                         size_t err_len);

/* INT8 row-wise grad_W quantisation on the device: `quantize_grad_w` +
 * `dequantize_grad_w(.., 1.0)` (src/quant.rs:157-202). grad_w [V,H] fp32 is
 * overwritten with the dequantized values (target rows kept exact); q and
 * scale (optional) receive the INT8 body and per-row scales. Bit-exact with
 * the reference on the same fp32 input. */
ORDA_API int orda_quantize_grad_w_device(OrdaContext* ctx, float* grad_w, size_t v, size_t h, size_t ld,
                                const int64_t* labels, size_t bt, int64_t ignore_index, int stochastic,
                                uint64_t seed, int8_t* q, float* scale, void* stream, char* err,
                                size_t err_len);

/* Allocation-free variant of orda_quantize_grad_w_device. It has no
 * counterpart in the reference crate. It exists for callers that cannot call
 * cudaMalloc (allocator hooks, out-of-memory handlers, runtimes that forbid
 * device allocations after start-up): instead of a context workspace, its
 * scratch (one flag byte per grad_W row) is a fixed device array inside the
 * library, ORDA_NOALLOC_MAX_V bytes on every GPU that loads the library.
 * Same arguments and results as orda_quantize_grad_w_device without the
 * context; runs on the current device. V above ORDA_NOALLOC_MAX_V is rejected.
 * All calls on a device share the array: calls that overlap on the GPU race,
 * so order them. Each call looks up the array's device address on the current
 * device (no caching, so a device reset leaves nothing stale); the first call
 * on a device also loads the library's device code there: make it before any
 * CUDA stream capture. */
#define ORDA_NOALLOC_MAX_V 262144
ORDA_API int orda_quantize_grad_w_device_noalloc(float* grad_w, size_t v, size_t h, size_t ld, const int64_t* labels,
                                                 size_t bt, int64_t ignore_index, int stochastic, uint64_t seed,
                                                 int8_t* q, float* scale, void* stream, char* err, size_t err_len);

/* bf16 tensor-core GEMM used by the chunk loop, exposed for unit tests:
 *   C[M,N] (fp32, ldc) = alpha * op(A) @ op(B) + (beta != 0 ? C : 0)
 * a_kind: 0 = A stored [M,K] (K contiguous), 1 = A stored [K,M] (M contiguous)
 * b_kind: 0 = B stored [N,K] (K contiguous), 1 = B stored [K,N] (N contiguous)
 * A and B are bf16 device pointers with leading dimensions lda, ldb. */
ORDA_API int orda_gemm_bf16_device(OrdaContext* ctx, const void* a, size_t lda, int a_kind, const void* b, size_t ldb,
                          int b_kind, float* c, size_t ldc, size_t m, size_t n, size_t k, float alpha,
                          float beta, void* stream, char* err, size_t err_len);

#ifdef __cplusplus
}
#endif

#endif /* ORDA_H_ */
