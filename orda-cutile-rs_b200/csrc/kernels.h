// kernels.h -- host-side launch interface of the sm_100a kernels.
#pragma once

#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

namespace orda {

// ---------------------------------------------------------------- GEMM
// One operand segment: a bf16 matrix as stored in memory, rows x cols with
// leading dimension ld (elements).
struct MatRef {
  const void* ptr = nullptr;
  long long rows = 0;
  long long cols = 0;
  long long ld = 0;
};

enum class Epi : int { Store = 0, Logits = 1 };

// Epilogue arguments. Store: out = alpha * acc (+ beta * out); rows below
// split_row go to out0, the rest to out1 (row - split_row).
// Logits: fp32 logits written to `logits` (ldl) plus per-(row, 128-column
// part) online-softmax records (see rows.cu for the record layout).
constexpr int kMaxSlotRanks = 8;  // ranks of one node that a scattered grad_W store can address

struct EpiArgs {
  // Store
  float* out0 = nullptr;
  long long ld0 = 0;
  float* out1 = nullptr;
  long long ld1 = 0;
  long long split_row = 1ll << 62;
  float alpha = 1.0f;
  const float* alpha_ptr = nullptr;  // device scalar overriding alpha
  float beta = 0.0f;
  // Logits
  void* logits = nullptr;  // fp32, or fp16 with logits_f16
  long long ldl = 0;
  float* rec_own = nullptr;   // float4 per (row, part)
  int n_parts = 0;
  float inv_t = 1.0f;
  int own_dT = 0;
  int logits_f16 = 0;  // Fast profile: logits stored as fp16 (the statistics still come from fp32)
  // Store, scattered to the owners of grad_W rows (row-sharded runs): global
  // row g belongs to rank o = g / slot_slice and lands in rank o's slot
  // buffer, at partial slot_rank, row g - o * slot_slice (fp32, ld slot_ld).
  // slot[o] is rank o's buffer (a peer mapping for o != slot_rank).
  int scatter = 0;
  int slot_rank = 0;
  long long slot_slice = 0;
  long long slot_ld = 0;
  float* slot[kMaxSlotRanks] = {};
};

struct GemmDesc {
  bool a_mn_major = false;  // A stored [K, M] instead of [M, K]
  bool b_mn_major = false;  // B stored [K, N] instead of [N, K]
  int nseg = 1;             // K segments (stacked operands along K)
  MatRef a[2];
  MatRef b[2];
  long long k_seg[2] = {0, 0};
  long long M = 0, N = 0;
  bool raster_n_fastest = false;
  Epi epi = Epi::Store;
  EpiArgs args;
  int* status = nullptr;  // device status word
  // After the GEMM, return the L2 lines of an operand it loaded evict-last to
  // normal priority (needed when a persisting-L2 carve-out is set: otherwise
  // they stay pinned and shrink L2 for the kernels that follow).
  bool demote_kept = false;
  int* launches = nullptr;  // if set, incremented by the number of kernels launched
  // SMs the persistent grid leaves free for a bandwidth-bound kernel that
  // runs concurrently on another stream (0: the grid covers every SM)
  int spare_sms = 0;
};

// Encodes the tensor maps and launches the persistent tcgen05 GEMM.
// Returns cudaSuccess or the first error.
cudaError_t gemm_launch(const GemmDesc& d, int num_sms, cudaStream_t stream, const char** why);

// ------------------------------------------------------------ row kernels
// Element type of a logits buffer the row kernels read.
enum LogitType : int { kLogitF32 = 0, kLogitBF16 = 1, kLogitF16 = 2 };

struct RowArgs {
  int n;                  // rows in this chunk
  int v;                  // vocabulary
  int n_parts;            // student record parts per row
  int n_parts_t;          // teacher record parts per row (1 after the teacher pre-pass)
  const void* logits_s;   // [n, ldl] student logits (fp32, or fp16 with logits_f16)
  int logits_f16;         // Fast profile: 16-bit student logits
  const void* teacher;    // teacher logits rows for this chunk
  long long ld_teacher;
  int teacher_dtype;      // LogitType of the teacher logits
  long long ldl;
  // Optional exact label logits (fp32) of this chunk's rows: the student's
  // (and teacher's) logit at the label column, 0 for ignored rows or labels
  // outside this rank's slice. With 16-bit logits the losses take the label
  // logit from here instead of the rounded buffer.
  const float* x_label;
  const float* t_label;
  int fast;               // Fast profile: part of the exp2 work on the FMA pipe
  const float* rec_own;   // [n] student records
  const float* rec_own_t; // [n] teacher records (from the teacher GEMM or the pre-pass)
  const int64_t* labels;  // chunk labels
  int64_t ignore_index;
  float w_s, w_t, kd, temperature, inv_t, alpha;
  int need_kl;            // kd > 0
  int teacher_ce;         // w_t > 0 (teacher CE reported)
  int teacher_grad;       // write teacher dlogits rows
  uint16_t* dlog_s;       // bf16 [n, ldd]
  uint16_t* dlog_t;       // bf16 [n, ldd] (teacher_grad)
  long long ldd;
  float* nll_s_rows;      // [n]
  float* nll_t_rows;      // [n]
  double* kl_base_rows;   // [n] lse_s^T - lse_t^T (0 for ignored rows)
  float* s_part;          // [n, nseg] KL cross-term partials sum_j p_t^T (t - x) / T
  int nseg;               // column segments of the gradient pass
  void* row_const;        // [n] x 32 B scratch: per-row constants (stats -> gradient kernel)
  int num_sms;
  // Vocabulary-sharded calls: this rank's logits cover vocabulary rows
  // [v0, v0 + v) of v_total (0 = not sharded: v_total = v, v0 = 0).
  int v_total;
  long long v0;
  float* partials_out;       // phase 1: [n][kVocabTuple] partial row statistics of the slice
  const float* partials_in;  // phase 2: [world][n][kVocabTuple] every rank's partials, by rank
  int world;
};
// Partial row statistics of one vocabulary slice, 12 doubles stored in 24
// floats: student (m, sum e^(x-m), sum e^((x-m)/T), sum x), teacher (same),
// the label's student and teacher logits and 1 when the label column lies in
// the slice (else 0), one pad.
constexpr int kVocabTuple = 24;
// Two launches: the per-row statistics kernel and the gradient kernel.
constexpr int kRowLaunches = 2;
constexpr size_t kRowConstBytes = 32;
// Columns per CTA of the gradient pass (256 threads x 8 columns x 4 steps).
constexpr int kGradSegCols = 8192;
void launch_rows(const RowArgs& a, cudaStream_t stream);
// Vocabulary-sharded phase 1: merges the slice's records of every row into
// one partial tuple (partials_out).
void launch_vocab_partials(const RowArgs& a, cudaStream_t stream);
// Vocabulary-sharded phase 2: merges every rank's tuple of each row (rank
// order), per-row losses and constants, then the slice's gradient pass.
void launch_vocab_rows(const RowArgs& a, cudaStream_t stream);

// Teacher statistics pre-pass over given teacher logits (Precomputed mode):
// one (max, sum e^(t-m), sum e^((t-m)/T), sum t) record per row. need_d1 =
// false (no teacher CE term) skips sum e^(t-m) and records 1 in its place.
// fast: half of the exp2 work on the FMA pipe (Fast profile).
void launch_teacher_stats(const void* teacher, long long ld, int is_bf16, int n, int v, float inv_t, float* rec,
                          cudaStream_t stream, bool need_d1 = true, bool fast = false);

// Exact label logits: out[i] = sum_k h[i, k] * w[labels[i] - v0, k] (fp32
// products of the bf16 inputs) for labels in [v0, v0 + v_rows), else 0
// (ignored rows and labels of other slices). One warp per row.
void launch_label_logits(const void* h, long long ldh, const void* w, long long ldw, long long k,
                         const int64_t* labels, long long n, long long v0, long long v_rows, int64_t ignore_index,
                         float* out, cudaStream_t stream);

// Label pass: counts non-ignored labels, checks the range [0, v), marks
// target rows (for the quantiser) and writes the mean scale.
void launch_label_prep(const int64_t* labels, long long bt, long long v, int64_t ignore_index, int reduction_sum,
                       long long denom_override, int* n_non_ignore, float* mean_scale, uint8_t* target_flags,
                       int* status, cudaStream_t stream);

// Final deterministic reduction of per-row losses into the four scalars:
// KL_row = (kl_base + sum over segments of s_part) * T^2. include_rows = 0
// leaves out the per-row terms (NLLs, KL base) and keeps only this rank's
// KL cross-term segments: the partial scalars of one vocabulary slice, which
// add up over the ranks when exactly one rank includes the rows.
void launch_finalize(const float* nll_s, const float* nll_t, const double* kl_base, const float* s_part, int nseg,
                     double t_sq, long long bt, const float* mean_scale, float w_s, float w_t, float kd,
                     float* scalars, cudaStream_t stream, int include_rows = 1);

// f32 -> bf16 (round to nearest even) into a padded row-major buffer.
void launch_f32_to_bf16(const float* src, long long rows, long long cols, uint16_t* dst, long long ld,
                        cudaStream_t stream);
// dst rows (fp32, ld elements apart) = the dense [rows, cols] bf16 src, exactly.
void launch_bf16_rows_to_f32(const uint16_t* src, long long rows, long long cols, float* dst, long long ld,
                             cudaStream_t stream);

// INT8 row-wise quantisation of grad_W (in place dequantised result). Row r
// of grad_w is row r + row_offset of the full matrix (the stochastic draw
// index is (r + row_offset) * h + c).
// dst[i, :] = src[idx[i], :] for i < n (fp32 rows of h elements; src ld).
// The base pointers must be 16-byte aligned for the vector path.
void launch_gather_rows(const float* src, long long ld, const int32_t* idx, long long n, long long h, float* dst,
                        cudaStream_t stream);

void launch_quant(float* grad_w, long long v, long long h, long long ld, const uint8_t* target_flags,
                  int stochastic, uint64_t seed, int8_t* q, float* scale, cudaStream_t stream,
                  long long row_offset = 0);

// Marks target rows only (used by the stand-alone quantiser entry): label t
// flags row t - row0 when that lies in [0, v).
void launch_target_flags(const int64_t* labels, long long bt, long long v, int64_t ignore_index,
                         uint8_t* target_flags, cudaStream_t stream, long long row0 = 0);

// launch_slot_reduce followed by launch_quant in one pass (the summed row
// stays in shared memory). Returns false, launching nothing, when the row
// does not fit (h % 4 != 0 or h > 12288); the caller then uses the two
// kernels.
bool launch_slot_reduce_quant(const float* slots, int world, long long slice, long long rows, long long h, float* out,
                              long long ld, const uint8_t* target_flags, int stochastic, uint64_t seed, int8_t* q,
                              float* scale, long long row_offset, cudaStream_t stream);

// out[r, :] = sum over k = 0..world-1 (in that order) of
// slots[(k * slice + r) * h + :], for r < rows <= slice (fp32).
void launch_slot_reduce(const float* slots, int world, long long slice, long long rows, long long h, float* out,
                        long long ld, cudaStream_t stream);

// INT8 wire format of the row-sharded grad_W exchange. Each owner's slot
// buffer, read as codes int8 [world][slice][h] followed (at a 256-byte
// boundary) by scales f32 [world][slice]; codes[o] / scales[o] address owner
// o's buffer (this rank's own, or a peer mapping).
struct WireSlots {
  int8_t* codes[kMaxSlotRanks] = {};
  float* scales[kMaxSlotRanks] = {};
};
// Quantises each row of this rank's local fp32 grad_W partial (v rows,
// row-wise INT8 by the quant.rs rules) into its owner's codes / scales at
// partial index slot_rank.
void launch_quant_send(const float* grad_w, long long v, long long h, long long ld, long long slice, int slot_rank,
                       int world, const WireSlots& dst, cudaStream_t stream);
// Owner side: out[r] = sum over k (rank order) of codes[k][r] * scales[k][r]
// (fp32), r < rows, then (quantize) the INT8 round trip of quant_kernel in
// the same pass. mine.codes[0] / mine.scales[0] are this rank's buffer.
// Returns false when h > 12288 (the row does not fit shared memory).
bool launch_wire_reduce(const WireSlots& mine, int world, long long slice, long long rows, long long h, float* out,
                        long long ld, const uint8_t* target_flags, int quantize, int stochastic, uint64_t seed,
                        int8_t* q, float* scale, long long row_offset, cudaStream_t stream);

// One-warp kernel whose bounded wait on a never-completed mbarrier expires
// after limit_ns and records DEV_TIMEOUT_SELFTEST in *status.
cudaError_t launch_bounded_wait_selftest(int* status, uint64_t limit_ns, cudaStream_t stream);

}  // namespace orda
