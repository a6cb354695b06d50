// rows.cu -- bandwidth-bound row kernels of the distillation loss.
//
// Record layout (float4 per record): m = max x, d1 = sum e^(x-m),
// dT = sum e^((x-m)/T), sx = sum x. The logits GEMM epilogue writes one
// record per (row, 128-column part) of the student (and of the teacher for
// Tied/Separate); teacher_stats_kernel writes one record per row for given
// (Precomputed) teacher logits.
//
// Per chunk:
//   row_stats_kernel  merges a row's records (f64), evaluates the row's NLLs
//                     (src/reference/cross_entropy.rs:32-57, label smoothing
//                     included) and the lse terms of the KL, writes the row's
//                     constants;
//   row_grad_kernel   one pass over the row writing the bf16 logit gradients
//                       dlogit_s = w_s((p - a/V) - [j==y](1-a)) + kd T (p_s^T - p_t^T)
//                       dlogit_t = w_t((p_t - a/V) - [j==y](1-a))
//                     (the merged CE + KL gradient of src/api.rs:303-344) and,
//                     from the p_t^T it already evaluates, the KL cross term
//                     sum_j p_t^T (t - x)/T per 8192-column segment, so that
//                     KL = cross + lse_s^T - lse_t^T (src/reference/kl.rs:66-127)
//                     without another pass; finalize adds the segments in a
//                     fixed order (deterministic).
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>

#include "bf16_bits.h"
#include "kernels.h"
#include "ptx.cuh"

namespace orda {

namespace {

constexpr float LOG2E_F = 1.4426950408889634f;
constexpr int ROW_THREADS = 256;
constexpr int GRAD_THREADS = 256;
constexpr int GRAD_STEPS = kGradSegCols / (GRAD_THREADS * 8);  // 4

// e^x as 2^(x * log2 e) with the PTX ex2.approx.ftz.f32 instruction; its
// ~2^-22 relative error is far below the bf16 rounding of the gradient.
__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

struct Acc {
  double m, d1, dT, sx;
};

__device__ __forceinline__ Acc load_rec(const float* rec, long long idx) {
  const float4 r = reinterpret_cast<const float4*>(rec)[idx];
  return Acc{r.x, r.y, r.z, r.w};
}

__device__ __forceinline__ uint32_t pack_bf16x2(float a, float b) {
  const __nv_bfloat16 ha = __float2bfloat16_rn(a), hb = __float2bfloat16_rn(b);
  return static_cast<uint32_t>(__bfloat16_as_ushort(ha)) | (static_cast<uint32_t>(__bfloat16_as_ushort(hb)) << 16);
}

__device__ __forceinline__ float bf16_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }
__device__ __forceinline__ float f16_lo(uint32_t w) {
  return __half2float(__ushort_as_half(static_cast<unsigned short>(w & 0xFFFFu)));
}
__device__ __forceinline__ float f16_hi(uint32_t w) {
  return __half2float(__ushort_as_half(static_cast<unsigned short>(w >> 16)));
}

// One logit of a buffer of LogitType `dtype`.
__device__ __forceinline__ float logit_at(const void* base, int dtype, long long idx) {
  if (dtype == kLogitBF16)
    return __uint_as_float(static_cast<uint32_t>(static_cast<const uint16_t*>(base)[idx]) << 16);
  if (dtype == kLogitF16) return __half2float(static_cast<const __half*>(base)[idx]);
  return static_cast<const float*>(base)[idx];
}

// ------------------------------------------------------ block reductions
// Results are returned to every thread; the order of additions is fixed, so
// the sums are deterministic.
__device__ __forceinline__ double block_max(double v, double* sh) {
  for (int off = 16; off > 0; off >>= 1) v = fmax(v, __shfl_xor_sync(0xffffffffu, v, off));
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) sh[w] = v;
  __syncthreads();
  v = sh[0];
  for (int k = 1; k < static_cast<int>(blockDim.x >> 5); ++k) v = fmax(v, sh[k]);
  return v;
}

template <int N>
__device__ __forceinline__ void block_sum(double (&v)[N], double* sh) {
#pragma unroll
  for (int q = 0; q < N; ++q)
    for (int off = 16; off > 0; off >>= 1) v[q] += __shfl_xor_sync(0xffffffffu, v[q], off);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31, nw = blockDim.x >> 5;
  __syncthreads();
  if (l == 0)
#pragma unroll
    for (int q = 0; q < N; ++q) sh[q * 32 + w] = v[q];
  __syncthreads();
#pragma unroll
  for (int q = 0; q < N; ++q) {
    double t = 0.0;
    for (int k = 0; k < nw; ++k) t += sh[q * 32 + k];
    v[q] = t;
  }
}

constexpr int kMaxPartsPerThread = 4;

// Merges the records of one row in two passes (block max, then one rescale
// per record and plain sums) in double precision.
__device__ Acc merge_row(const float* rec, long long row, int P, double inv_t, double* sh) {
  Acc loc[kMaxPartsPerThread];
  double mx = -INFINITY;
#pragma unroll
  for (int k = 0; k < kMaxPartsPerThread; ++k) {
    const int p = threadIdx.x + k * blockDim.x;
    loc[k] = p < P ? load_rec(rec, row * P + p) : Acc{-INFINITY, 0.0, 0.0, 0.0};
    mx = fmax(mx, loc[k].m);
  }
  for (int p = threadIdx.x + kMaxPartsPerThread * blockDim.x; p < P; p += blockDim.x)
    mx = fmax(mx, static_cast<double>(rec[(row * P + p) * 4]));
  const double M = block_max(mx, sh);
  double sums[3] = {0.0, 0.0, 0.0};  // d1, dT, sx
#pragma unroll
  for (int k = 0; k < kMaxPartsPerThread; ++k) {
    if (loc[k].m != -INFINITY) {
      sums[0] += loc[k].d1 * exp(loc[k].m - M);
      sums[1] += loc[k].dT * exp((loc[k].m - M) * inv_t);
    }
    sums[2] += loc[k].sx;
  }
  for (int p = threadIdx.x + kMaxPartsPerThread * blockDim.x; p < P; p += blockDim.x) {
    const Acc r = load_rec(rec, row * P + p);
    sums[0] += r.d1 * exp(r.m - M);
    sums[1] += r.dT * exp((r.m - M) * inv_t);
    sums[2] += r.sx;
  }
  block_sum(sums, sh);
  return Acc{M, sums[0], sums[1], sums[2]};
}

// Per-row constants handed from the statistics kernel to the gradient kernel
// (lse terms pre-multiplied by log2(e) for exp2).
struct RowConst {
  float c_s1, c_sT, c_tT, c_t1;
  int y;
  int ignored;
  int pad0, pad1;
};

__device__ __forceinline__ int vocab_total(const RowArgs& a) { return a.v_total > 0 ? a.v_total : a.v; }

// Row i's label: ignored (ignore_index or out of [0, V): range errors are
// reported by the label pass) or its global column.
__device__ __forceinline__ bool row_label(const RowArgs& a, int i, long long& y) {
  const int64_t y64 = a.labels[i];
  y = static_cast<long long>(y64);
  return y64 == a.ignore_index || y64 < 0 || y64 >= vocab_total(a);
}

__device__ __forceinline__ double teacher_value(const RowArgs& a, long long i, long long col) {
  return static_cast<double>(logit_at(a.teacher, a.teacher_dtype, i * a.ld_teacher + col));
}

// Per-row losses and constants of row i from its merged statistics (own:
// student, ts: teacher) and the student / teacher logits at the label
// (x_y, t_y; unused for ignored rows). y_local is the label's column in this
// rank's logits, or -1 when another rank holds it. Smoothing uses the full
// vocabulary (alpha / V_total).
__device__ void finish_row(const RowArgs& a, int i, const Acc& own, const Acc& ts, bool ignored, double x_y,
                           double t_y, int y_local) {
  const double inv_t = static_cast<double>(a.inv_t);
  const double alpha = static_cast<double>(a.alpha);
  const double vd = static_cast<double>(vocab_total(a));

  const double lse_s1 = own.m + log(own.d1);
  double nll_s = 0.0;
  if (!ignored) nll_s = alpha > 0.0 ? lse_s1 - (1.0 - alpha) * x_y - (alpha / vd) * own.sx : lse_s1 - x_y;
  a.nll_s_rows[i] = static_cast<float>(nll_s);

  double lse_sT = 0.0, lse_tT = 0.0;
  if (a.need_kl) {
    lse_sT = own.m * inv_t + log(own.dT);
    lse_tT = ts.m * inv_t + log(ts.dT);
  }
  a.kl_base_rows[i] = (a.need_kl && !ignored) ? lse_sT - lse_tT : 0.0;

  double lse_t1 = 0.0;
  if (a.teacher_ce) {
    lse_t1 = ts.m + log(ts.d1);
    double nll_t = 0.0;
    if (!ignored) nll_t = alpha > 0.0 ? lse_t1 - (1.0 - alpha) * t_y - (alpha / vd) * ts.sx : lse_t1 - t_y;
    a.nll_t_rows[i] = static_cast<float>(nll_t);
  } else {
    a.nll_t_rows[i] = 0.0f;
  }

  RowConst rc;
  rc.c_s1 = static_cast<float>(lse_s1 * static_cast<double>(LOG2E_F));
  rc.c_sT = static_cast<float>(lse_sT * static_cast<double>(LOG2E_F));
  rc.c_tT = static_cast<float>(lse_tT * static_cast<double>(LOG2E_F));
  rc.c_t1 = static_cast<float>(lse_t1 * static_cast<double>(LOG2E_F));
  rc.y = ignored ? 0 : y_local;
  rc.ignored = ignored;
  rc.pad0 = rc.pad1 = 0;
  reinterpret_cast<RowConst*>(a.row_const)[i] = rc;
}

// ---- one CTA per row: merge records, per-row losses, constants.
__global__ void __launch_bounds__(ROW_THREADS) row_stats_kernel(const RowArgs a) {
  __shared__ double sh[3 * 32];
  const int i = blockIdx.x;
  const double inv_t = static_cast<double>(a.inv_t);
  const bool want_t = a.need_kl || a.teacher_ce;

  const Acc own = merge_row(a.rec_own, i, a.n_parts, inv_t, sh);
  const Acc ts = want_t ? merge_row(a.rec_own_t, i, a.n_parts_t, inv_t, sh) : Acc{0.0, 1.0, 1.0, 0.0};
  if (threadIdx.x != 0) return;
  long long y;
  const bool ignored = row_label(a, i, y);
  double x_y = 0.0, t_y = 0.0;
  if (!ignored) {
    x_y = a.x_label ? static_cast<double>(a.x_label[i])
                    : static_cast<double>(logit_at(a.logits_s, a.logits_f16 ? kLogitF16 : kLogitF32,
                                                   static_cast<long long>(i) * a.ldl + y));
    if (a.teacher_ce) t_y = a.t_label ? static_cast<double>(a.t_label[i]) : teacher_value(a, i, y);
  }
  finish_row(a, i, own, ts, ignored, x_y, t_y, static_cast<int>(y));
}

// ---- vocabulary-sharded phase 1, one CTA per row: the slice's statistics
// of the row as one tuple, with the label's logits if the slice holds it.
__global__ void __launch_bounds__(ROW_THREADS) vocab_partials_kernel(const RowArgs a) {
  __shared__ double sh[3 * 32];
  const int i = blockIdx.x;
  const double inv_t = static_cast<double>(a.inv_t);
  const bool want_t = a.need_kl || a.teacher_ce;
  const Acc own = merge_row(a.rec_own, i, a.n_parts, inv_t, sh);
  const Acc ts = want_t ? merge_row(a.rec_own_t, i, a.n_parts_t, inv_t, sh) : Acc{0.0, 1.0, 1.0, 0.0};
  if (threadIdx.x != 0) return;
  long long y;
  const bool ignored = row_label(a, i, y);
  const long long yl = y - a.v0;
  double x_y = 0.0, t_y = 0.0, has_y = 0.0;
  if (!ignored && yl >= 0 && yl < a.v) {
    x_y = a.x_label ? a.x_label[i]
                    : logit_at(a.logits_s, a.logits_f16 ? kLogitF16 : kLogitF32, static_cast<long long>(i) * a.ldl + yl);
    if (a.teacher_ce) t_y = a.t_label ? static_cast<double>(a.t_label[i]) : teacher_value(a, i, yl);
    has_y = 1.0;
  }
  // f64, so that the merge of the slices matches the single-device merge of
  // the same records to f64 precision (an f32 tuple moves the row's lse by
  // an f32 rounding, which flips the bf16 rounding of some logit gradients)
  double2* out = reinterpret_cast<double2*>(a.partials_out + static_cast<long long>(i) * kVocabTuple);
  out[0] = make_double2(own.m, own.d1);
  out[1] = make_double2(own.dT, own.sx);
  out[2] = make_double2(ts.m, ts.d1);
  out[3] = make_double2(ts.dT, ts.sx);
  out[4] = make_double2(x_y, t_y);
  out[5] = make_double2(has_y, 0.0);
}

// ---- vocabulary-sharded phase 2, one thread per row: merges the ranks'
// tuples in rank order (f64), then the same per-row losses and constants as
// row_stats_kernel with the label column made local to this rank's slice.
__global__ void __launch_bounds__(128) vocab_merge_kernel(const RowArgs a) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= a.n) return;
  const double inv_t = static_cast<double>(a.inv_t);
  // tuples of kVocabTuple floats per row, read as 12 doubles
  const long long stride = static_cast<long long>(a.n) * kVocabTuple / 2;
  const double* base = reinterpret_cast<const double*>(a.partials_in) + static_cast<long long>(i) * kVocabTuple / 2;
  double ms = -INFINITY, mt = -INFINITY;
  for (int r = 0; r < a.world; ++r) {
    ms = fmax(ms, base[r * stride + 0]);
    mt = fmax(mt, base[r * stride + 4]);
  }
  Acc own{ms, 0.0, 0.0, 0.0}, ts{mt, 0.0, 0.0, 0.0};
  double x_y = 0.0, t_y = 0.0;
  for (int r = 0; r < a.world; ++r) {
    const double* q = base + r * stride;
    const double m_r = q[0], mt_r = q[4];
    own.d1 += q[1] * exp(m_r - ms);
    own.dT += q[2] * exp((m_r - ms) * inv_t);
    own.sx += q[3];
    if (a.need_kl || a.teacher_ce) {
      ts.d1 += q[5] * exp(mt_r - mt);
      ts.dT += q[6] * exp((mt_r - mt) * inv_t);
      ts.sx += q[7];
    }
    if (q[10] != 0.0) {
      x_y = q[8];
      t_y = q[9];
    }
  }
  if (!(a.need_kl || a.teacher_ce)) ts = Acc{0.0, 1.0, 1.0, 0.0};
  long long y;
  const bool ignored = row_label(a, i, y);
  const long long yl = y - a.v0;
  finish_row(a, i, own, ts, ignored, x_y, t_y, (yl >= 0 && yl < a.v) ? static_cast<int>(yl) : -1);
}

// Scalars shared by every element of the gradient pass.
struct GradScalars {
  float ws, wt, kdT, eps, ws_tgt, wt_tgt, l1, lT, inv_t;
};

// One element: the student (and teacher) logit gradient and the KL cross
// term p_t^T (t - x) / T.
// All exp2 on the SFU: with about 20 other instructions per element this
// kernel keeps the SFU and the issue slots about equally busy, and the FMA
// polynomial (about 10 issue slots per exp2) would make it issue-bound.
template <bool KL, bool TGRAD>
__device__ __forceinline__ void grad_elem(const GradScalars& g, const RowConst& c, int j, float x, float t, float& gs,
                                          float& gt, float& cross) {
  float s = g.ws * (fast_exp2(fmaf(x, g.l1, -c.c_s1)) - g.eps);
  if (KL) {
    const float pt = fast_exp2(fmaf(t, g.lT, -c.c_tT));
    s += g.kdT * (fast_exp2(fmaf(x, g.lT, -c.c_sT)) - pt);
    cross = fmaf(pt, (t - x) * g.inv_t, cross);
  }
  if (j == c.y) s -= g.ws_tgt;
  float u = 0.0f;
  if (TGRAD) {
    u = g.wt * (fast_exp2(fmaf(t, g.l1, -c.c_t1)) - g.eps);
    if (j == c.y) u -= g.wt_tgt;
  }
  gs = s;
  gt = u;
}

// Eight consecutive logits of a buffer of LogitType `dtype` (16-byte aligned
// for the 16-bit types, 32-byte for fp32).
__device__ __forceinline__ void load_teacher8(const void* teacher, int dtype, long long off, float (&t)[8]) {
  if (dtype == kLogitBF16) {
    const uint4 q = __ldg(reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(teacher) + off));
    t[0] = bf16_lo(q.x);
    t[1] = bf16_hi(q.x);
    t[2] = bf16_lo(q.y);
    t[3] = bf16_hi(q.y);
    t[4] = bf16_lo(q.z);
    t[5] = bf16_hi(q.z);
    t[6] = bf16_lo(q.w);
    t[7] = bf16_hi(q.w);
  } else if (dtype == kLogitF16) {
    const uint4 q = __ldg(reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(teacher) + off));
    t[0] = f16_lo(q.x);
    t[1] = f16_hi(q.x);
    t[2] = f16_lo(q.y);
    t[3] = f16_hi(q.y);
    t[4] = f16_lo(q.z);
    t[5] = f16_hi(q.z);
    t[6] = f16_lo(q.w);
    t[7] = f16_hi(q.w);
  } else {
    const float* tp = static_cast<const float*>(teacher) + off;
    const float4 t0 = __ldg(reinterpret_cast<const float4*>(tp));
    const float4 t1 = __ldg(reinterpret_cast<const float4*>(tp + 4));
    t[0] = t0.x; t[1] = t0.y; t[2] = t0.z; t[3] = t0.w;
    t[4] = t1.x; t[5] = t1.y; t[6] = t1.z; t[7] = t1.w;
  }
}

// Block sum of one float, deterministic; result valid in thread 0.
__device__ __forceinline__ float block_sum_f(float v, float* sh) {
  for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) sh[w] = v;
  __syncthreads();
  float t = 0.0f;
  if (threadIdx.x == 0)
    for (int k = 0; k < static_cast<int>(blockDim.x >> 5); ++k) t += sh[k];
  return t;
}

// ---- grid (row, segment): gradients of one 8192-column segment of one row
// (rows on grid x, which has no 65535 limit).
// VEC: V % 8 == 0 and 16-byte aligned rows (8 columns per thread step).
// FAST (Fast profile): fp16 student logits (half the bytes of the pass).
template <bool VEC, bool KL, bool TGRAD, bool FAST>
__global__ void __launch_bounds__(GRAD_THREADS) row_grad_kernel(const RowArgs a, const GradScalars g) {
  __shared__ float sh[GRAD_THREADS / 32];
  const int seg = blockIdx.y;
  const long long row = blockIdx.x;
  const RowConst c = reinterpret_cast<const RowConst*>(a.row_const)[row];
  const float* xs = FAST ? nullptr : static_cast<const float*>(a.logits_s) + row * a.ldl;
  const __half* xh = FAST ? static_cast<const __half*>(a.logits_s) + row * a.ldl : nullptr;
  uint16_t* gs_row = a.dlog_s + row * a.ldd;
  uint16_t* gt_row = TGRAD ? a.dlog_t + row * a.ldd : nullptr;
  const bool need_t = KL || TGRAD;
  const int V = a.v;
  const int c0 = seg * kGradSegCols;
  const int c1 = min(V, c0 + kGradSegCols);
  float cross = 0.0f;
  if (c.ignored) {
    // ignored row: zero gradients, no KL contribution
    if (VEC) {
      for (int j0 = c0 + threadIdx.x * 8; j0 < c1; j0 += GRAD_THREADS * 8) {
        *reinterpret_cast<uint4*>(gs_row + j0) = make_uint4(0, 0, 0, 0);
        if (TGRAD) *reinterpret_cast<uint4*>(gt_row + j0) = make_uint4(0, 0, 0, 0);
      }
    } else {
      for (int j = c0 + threadIdx.x; j < c1; j += GRAD_THREADS) {
        gs_row[j] = 0;
        if (TGRAD) gt_row[j] = 0;
      }
    }
  } else if (VEC) {
#pragma unroll
    for (int step = 0; step < GRAD_STEPS; ++step) {
      const int j0 = c0 + (step * GRAD_THREADS + threadIdx.x) * 8;
      if (j0 < c1) {
        float x[8];
        if (FAST) {
          const uint4 q = __ldg(reinterpret_cast<const uint4*>(xh + j0));
          x[0] = f16_lo(q.x); x[1] = f16_hi(q.x); x[2] = f16_lo(q.y); x[3] = f16_hi(q.y);
          x[4] = f16_lo(q.z); x[5] = f16_hi(q.z); x[6] = f16_lo(q.w); x[7] = f16_hi(q.w);
        } else {
          const float4 x0 = __ldg(reinterpret_cast<const float4*>(xs + j0));
          const float4 x1 = __ldg(reinterpret_cast<const float4*>(xs + j0 + 4));
          x[0] = x0.x; x[1] = x0.y; x[2] = x0.z; x[3] = x0.w;
          x[4] = x1.x; x[5] = x1.y; x[6] = x1.z; x[7] = x1.w;
        }
        float t[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        if (need_t) load_teacher8(a.teacher, a.teacher_dtype, row * a.ld_teacher + j0, t);
        float gsv[8], gtv[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) grad_elem<KL, TGRAD>(g, c, j0 + k, x[k], t[k], gsv[k], gtv[k], cross);
        *reinterpret_cast<uint4*>(gs_row + j0) = make_uint4(pack_bf16x2(gsv[0], gsv[1]), pack_bf16x2(gsv[2], gsv[3]),
                                                            pack_bf16x2(gsv[4], gsv[5]), pack_bf16x2(gsv[6], gsv[7]));
        if (TGRAD)
          *reinterpret_cast<uint4*>(gt_row + j0) =
              make_uint4(pack_bf16x2(gtv[0], gtv[1]), pack_bf16x2(gtv[2], gtv[3]), pack_bf16x2(gtv[4], gtv[5]),
                         pack_bf16x2(gtv[6], gtv[7]));
      }
    }
  } else {
    for (int j = c0 + threadIdx.x; j < c1; j += GRAD_THREADS) {
      float t = 0.0f;
      if (need_t) t = logit_at(a.teacher, a.teacher_dtype, row * a.ld_teacher + j);
      const float x = FAST ? __half2float(xh[j]) : xs[j];
      float gs, gt;
      grad_elem<KL, TGRAD>(g, c, j, x, t, gs, gt, cross);
      gs_row[j] = __bfloat16_as_ushort(__float2bfloat16_rn(gs));
      if (TGRAD) gt_row[j] = __bfloat16_as_ushort(__float2bfloat16_rn(gt));
    }
  }
  if (KL) {
    const float tot = block_sum_f(cross, sh);
    if (threadIdx.x == 0) a.s_part[row * a.nseg + seg] = tot;
  }
}

__device__ __forceinline__ float teacher_at(const void* teacher, int is_bf16, long long idx) {
  return is_bf16 ? __uint_as_float(static_cast<uint32_t>(static_cast<const uint16_t*>(teacher)[idx]) << 16)
                 : static_cast<const float*>(teacher)[idx];
}

// ---- teacher statistics pre-pass over given teacher logits: one CTA per
// row; every thread keeps four independent 16-byte loads in flight. The
// sums cost one exp2 each per element on the SFU, which bounds this kernel
// before HBM does: NEED_D1 = false (no teacher CE term) skips sum e^(t-m)
// and records d1 = 1.
// The exp2 work stays on the SFU in every profile (FAST is unused): with one
// exp2 and about six other instructions per element, moving any of it to the
// ten-instruction FMA polynomial costs more issue slots than it frees. BF16:
// the teacher logits are bf16 (else fp32).
template <bool NEED_D1, bool FAST, bool BF16>
__global__ void __launch_bounds__(ROW_THREADS, 3) teacher_stats_kernel(const void* teacher, long long ld, int is_bf16,
                                                                       int v, float inv_t, float* rec) {
  __shared__ double sh[3 * 32];
  const long long row = blockIdx.x;
  const bool vec = (v % 8 == 0) && ((ld * (is_bf16 ? 2 : 4)) % 16 == 0) &&
                   ((reinterpret_cast<uintptr_t>(teacher) & 15) == 0);
  const float lt = LOG2E_F * inv_t;
  float m = -INFINITY, d1 = 0.f, dT = 0.f, sx = 0.f;
  if (vec) {
    // U vectors of 8 per thread per iteration; the next iteration's raw
    // 16-byte words are loaded before the current ones are reduced, so the
    // loads of two iterations are in flight (the reduction would otherwise
    // leave the memory pipe idle between iterations)
    constexpr int U = 4;
    constexpr int STEP = ROW_THREADS * 8 * U;
    constexpr int NW = BF16 ? 1 : 2;  // 16-byte words per vector of 8
    const uint4* src = reinterpret_cast<const uint4*>(static_cast<const uint8_t*>(teacher) +
                                                      row * ld * (BF16 ? 2 : 4));
    auto fetch = [&](int base, uint4 (&r)[U][NW]) {
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int j0 = base + u * ROW_THREADS * 8;
        if (j0 < v) {
#pragma unroll
          for (int q = 0; q < NW; ++q) r[u][q] = __ldg(src + static_cast<long long>(j0) * NW / 8 + q);
        }
      }
    };
    uint4 cur[U][NW], nxt[U][NW];
    fetch(threadIdx.x * 8, cur);
    for (int base = threadIdx.x * 8; base < v; base += STEP) {
      if (base + STEP < v) fetch(base + STEP, nxt);
      float t[U][8];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        if (base + u * ROW_THREADS * 8 < v) {
          const uint4 a = cur[u][0];
          if constexpr (BF16) {
            t[u][0] = bf16_lo(a.x); t[u][1] = bf16_hi(a.x); t[u][2] = bf16_lo(a.y); t[u][3] = bf16_hi(a.y);
            t[u][4] = bf16_lo(a.z); t[u][5] = bf16_hi(a.z); t[u][6] = bf16_lo(a.w); t[u][7] = bf16_hi(a.w);
          } else {
            const uint4 b = cur[u][NW - 1];
            t[u][0] = __uint_as_float(a.x); t[u][1] = __uint_as_float(a.y);
            t[u][2] = __uint_as_float(a.z); t[u][3] = __uint_as_float(a.w);
            t[u][4] = __uint_as_float(b.x); t[u][5] = __uint_as_float(b.y);
            t[u][6] = __uint_as_float(b.z); t[u][7] = __uint_as_float(b.w);
          }
        } else {
#pragma unroll
          for (int k = 0; k < 8; ++k) t[u][k] = -INFINITY;
        }
      }
      float vm = -INFINITY;
#pragma unroll
      for (int u = 0; u < U; ++u)
#pragma unroll
        for (int k = 0; k < 8; ++k) vm = fmaxf(vm, t[u][k]);
      if (vm > m) {
        const float dm = m - vm;  // -inf on the first block: factors 0
        if (NEED_D1) d1 *= fast_exp2(dm * LOG2E_F);
        dT *= fast_exp2(dm * lt);
        m = vm;
      }
#pragma unroll
      for (int u = 0; u < U; ++u)
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          if (t[u][k] != -INFINITY) {
            const float x = t[u][k] - m;
            if (NEED_D1) d1 += fast_exp2(x * LOG2E_F);
            dT += fast_exp2(x * lt);
            sx += t[u][k];
          }
        }
#pragma unroll
      for (int u = 0; u < U; ++u)
#pragma unroll
        for (int q = 0; q < NW; ++q) cur[u][q] = nxt[u][q];
    }
  } else {
    for (int j = threadIdx.x; j < v; j += ROW_THREADS) m = fmaxf(m, teacher_at(teacher, is_bf16, row * ld + j));
    for (int j = threadIdx.x; j < v; j += ROW_THREADS) {
      const float t = teacher_at(teacher, is_bf16, row * ld + j);
      if (NEED_D1) d1 += fast_exp2((t - m) * LOG2E_F);
      dT += fast_exp2((t - m) * lt);
      sx += t;
    }
  }
  const double M = block_max(static_cast<double>(m), sh);
  const double f1 = m == -INFINITY ? 0.0 : exp(static_cast<double>(m) - M);
  const double fT = m == -INFINITY ? 0.0 : exp((static_cast<double>(m) - M) * static_cast<double>(inv_t));
  double sums[3] = {static_cast<double>(d1) * f1, static_cast<double>(dT) * fT, static_cast<double>(sx)};
  block_sum(sums, sh);
  if (threadIdx.x == 0)
    reinterpret_cast<float4*>(rec)[row] = make_float4(static_cast<float>(M), NEED_D1 ? static_cast<float>(sums[0]) : 1.0f,
                                                      static_cast<float>(sums[1]), static_cast<float>(sums[2]));
}

// ------------------------------------------------------------ label pass
__global__ void __launch_bounds__(1024) label_prep_kernel(const int64_t* labels, long long bt, long long v,
                                                          int64_t ignore_index, int reduction_sum,
                                                          long long denom_override, int* n_non_ignore,
                                                          float* mean_scale, uint8_t* target_flags, int* status) {
  __shared__ long long sh[32];
  long long cnt = 0;
  bool bad = false;
  for (long long r = threadIdx.x; r < bt; r += blockDim.x) {
    const int64_t t = labels[r];
    if (t != ignore_index) {
      ++cnt;
      if (t < 0 || t >= v) bad = true;
      else if (target_flags) target_flags[t] = 1;
    }
  }
  if (bad) atomicCAS(status, DEV_OK, DEV_LABEL_RANGE);
  for (int off = 16; off > 0; off >>= 1) cnt += __shfl_down_sync(0xffffffffu, cnt, off);
  if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = cnt;
  __syncthreads();
  if (threadIdx.x < 32) {
    cnt = threadIdx.x < (blockDim.x >> 5) ? sh[threadIdx.x] : 0;
    for (int off = 16; off > 0; off >>= 1) cnt += __shfl_down_sync(0xffffffffu, cnt, off);
    if (threadIdx.x == 0) {
      *n_non_ignore = static_cast<int>(cnt);
      long long n = denom_override > 0 ? denom_override : cnt;
      long long denom = reduction_sum ? 1 : (n > 1 ? n : 1);
      // `1.0f32 / denom as f32` (src/api.rs:230)
      *mean_scale = 1.0f / static_cast<float>(denom);
    }
  }
}

__global__ void target_flags_kernel(const int64_t* labels, long long bt, long long v, int64_t ignore_index,
                                    uint8_t* flags, long long row0) {
  for (long long r = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; r < bt;
       r += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int64_t t = labels[r];
    if (t == ignore_index) continue;
    const long long u = static_cast<long long>(t) - row0;
    if (u >= 0 && u < v) flags[u] = 1;
  }
}

// ------------------------------------------------------------- finalize
__global__ void __launch_bounds__(1024) finalize_kernel(const float* nll_s, const float* nll_t,
                                                        const double* kl_base, const float* s_part, int nseg,
                                                        double t_sq, long long bt, const float* mean_scale,
                                                        float w_s, float w_t, float kd, float* scalars,
                                                        int include_rows) {
  __shared__ double sh[3][32];
  double s0 = 0.0, s1 = 0.0, s2 = 0.0;
  for (long long r = threadIdx.x; r < bt; r += blockDim.x) {
    if (include_rows) {
      s0 += static_cast<double>(nll_s[r]);
      s1 += static_cast<double>(nll_t[r]);
    }
    if (nseg > 0) {
      // ignored rows have kl_base 0 and no cross-term segments
      double cross = 0.0;
      for (int k = 0; k < nseg; ++k) cross += static_cast<double>(s_part[r * nseg + k]);
      s2 += ((include_rows ? kl_base[r] : 0.0) + cross) * t_sq;
    }
  }
  for (int off = 16; off > 0; off >>= 1) {
    s0 += __shfl_down_sync(0xffffffffu, s0, off);
    s1 += __shfl_down_sync(0xffffffffu, s1, off);
    s2 += __shfl_down_sync(0xffffffffu, s2, off);
  }
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) {
    sh[0][w] = s0;
    sh[1][w] = s1;
    sh[2][w] = s2;
  }
  __syncthreads();
  if (w == 0) {
    const int nw = blockDim.x >> 5;
    s0 = l < nw ? sh[0][l] : 0.0;
    s1 = l < nw ? sh[1][l] : 0.0;
    s2 = l < nw ? sh[2][l] : 0.0;
    for (int off = 16; off > 0; off >>= 1) {
      s0 += __shfl_down_sync(0xffffffffu, s0, off);
      s1 += __shfl_down_sync(0xffffffffu, s1, off);
      s2 += __shfl_down_sync(0xffffffffu, s2, off);
    }
    if (l == 0) {
      // loss assembly as src/api.rs:401-405
      const double ms = static_cast<double>(*mean_scale);
      scalars[1] = static_cast<float>(s0 * ms);
      scalars[2] = static_cast<float>(s1 * ms);
      scalars[3] = static_cast<float>(s2 * ms);
      scalars[0] = static_cast<float>((static_cast<double>(w_s) * s0 + static_cast<double>(w_t) * s1 +
                                       static_cast<double>(kd) * s2) * ms);
    }
  }
}

// ------------------------------------------------------------ conversion
__global__ void f32_to_bf16_kernel(const float* src, long long rows, long long cols, uint16_t* dst, long long ld) {
  const long long total = rows * cols;
  for (long long idx = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; idx < total;
       idx += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long r = idx / cols, c = idx - r * cols;
    dst[r * ld + c] = f32_bits_to_bf16(__float_as_uint(src[idx]));
  }
}

// dst rows (fp32, ld elements apart) = the dense [rows, cols] bf16 src,
// exactly (a bf16 value is the high half of its fp32).
__global__ void bf16_rows_to_f32_kernel(const uint16_t* src, long long rows, long long cols, float* dst,
                                        long long ld) {
  const long long total = rows * cols;
  for (long long idx = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; idx < total;
       idx += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long r = idx / cols, c = idx - r * cols;
    dst[r * ld + c] = __uint_as_float(static_cast<uint32_t>(src[idx]) << 16);
  }
}

template <bool VEC, bool FAST>
void launch_grad(const RowArgs& a, const GradScalars& g, cudaStream_t stream) {
  const dim3 grid(static_cast<unsigned>(a.n), static_cast<unsigned>((a.v + kGradSegCols - 1) / kGradSegCols));
  const bool kl = a.need_kl != 0, tg = a.teacher_grad != 0;
  if (kl && tg) row_grad_kernel<VEC, true, true, FAST><<<grid, GRAD_THREADS, 0, stream>>>(a, g);
  else if (kl) row_grad_kernel<VEC, true, false, FAST><<<grid, GRAD_THREADS, 0, stream>>>(a, g);
  else if (tg) row_grad_kernel<VEC, false, true, FAST><<<grid, GRAD_THREADS, 0, stream>>>(a, g);
  else row_grad_kernel<VEC, false, false, FAST><<<grid, GRAD_THREADS, 0, stream>>>(a, g);
}

// ---- exact label logits: one warp per row, fp32 dot product of the bf16
// hidden row and the label's weight row (16-byte loads when aligned)
__global__ void __launch_bounds__(256) label_logit_kernel(const uint16_t* h, long long ldh, const uint16_t* w,
                                                          long long ldw, long long k, const int64_t* labels,
                                                          long long n, long long v0, long long v_rows,
                                                          int64_t ignore_index, float* out) {
  const long long i = blockIdx.x * 8ll + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (i >= n) return;
  const int64_t y = labels[i];
  const long long yl = static_cast<long long>(y) - v0;
  if (y == ignore_index || yl < 0 || yl >= v_rows) {
    if (lane == 0) out[i] = 0.0f;
    return;
  }
  const uint16_t* hr = h + i * ldh;
  const uint16_t* wr = w + yl * ldw;
  float acc = 0.0f;
  const bool vec = ((reinterpret_cast<uintptr_t>(hr) | reinterpret_cast<uintptr_t>(wr)) & 15) == 0;
  // 16-byte loads over the whole groups of 8 columns, then the tail
  const long long kv = vec ? (k / 8) * 8 : 0;
  for (long long c = lane * 8; c < kv; c += 256) {
    const uint4 p = __ldg(reinterpret_cast<const uint4*>(hr + c));
    const uint4 q = __ldg(reinterpret_cast<const uint4*>(wr + c));
    acc = fmaf(bf16_lo(p.x), bf16_lo(q.x), acc);
    acc = fmaf(bf16_hi(p.x), bf16_hi(q.x), acc);
    acc = fmaf(bf16_lo(p.y), bf16_lo(q.y), acc);
    acc = fmaf(bf16_hi(p.y), bf16_hi(q.y), acc);
    acc = fmaf(bf16_lo(p.z), bf16_lo(q.z), acc);
    acc = fmaf(bf16_hi(p.z), bf16_hi(q.z), acc);
    acc = fmaf(bf16_lo(p.w), bf16_lo(q.w), acc);
    acc = fmaf(bf16_hi(p.w), bf16_hi(q.w), acc);
  }
  for (long long j = kv + lane; j < k; j += 32)
    acc = fmaf(__uint_as_float(static_cast<uint32_t>(hr[j]) << 16), __uint_as_float(static_cast<uint32_t>(wr[j]) << 16),
               acc);
  for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
  if (lane == 0) out[i] = acc;
}

void launch_row_grad(const RowArgs& a, cudaStream_t stream);

}  // namespace

void launch_rows(const RowArgs& a, cudaStream_t stream) {
  if (a.n <= 0) return;
  row_stats_kernel<<<a.n, ROW_THREADS, 0, stream>>>(a);
  launch_row_grad(a, stream);
}

void launch_vocab_partials(const RowArgs& a, cudaStream_t stream) {
  if (a.n <= 0) return;
  vocab_partials_kernel<<<a.n, ROW_THREADS, 0, stream>>>(a);
}

void launch_vocab_rows(const RowArgs& a, cudaStream_t stream) {
  if (a.n <= 0) return;
  vocab_merge_kernel<<<(a.n + 127) / 128, 128, 0, stream>>>(a);
  launch_row_grad(a, stream);
}

namespace {

void launch_row_grad(const RowArgs& a, cudaStream_t stream) {
  GradScalars g;
  g.ws = a.w_s;
  g.wt = a.w_t;
  g.kdT = a.need_kl ? a.kd * a.temperature : 0.0f;
  const double alpha = static_cast<double>(a.alpha);
  g.eps = static_cast<float>(alpha / static_cast<double>(a.v_total > 0 ? a.v_total : a.v));
  const float one_minus_a = static_cast<float>(1.0 - alpha);
  g.ws_tgt = a.w_s * one_minus_a;
  g.wt_tgt = a.w_t * one_minus_a;
  g.l1 = LOG2E_F;
  g.lT = LOG2E_F * a.inv_t;
  g.inv_t = a.inv_t;
  const long long tsz = a.teacher_dtype == kLogitF32 ? 4 : 2;
  const bool teacher_ok = !(a.need_kl || a.teacher_grad) ||
                          (((a.ld_teacher * tsz) % 16 == 0) && ((reinterpret_cast<uintptr_t>(a.teacher) & 15) == 0));
  const long long lsz = a.logits_f16 ? 2 : 4;
  const bool vec = (a.v % 8 == 0) && ((a.ldl * lsz) % 16 == 0) && (a.ldd % 8 == 0) && teacher_ok &&
                   ((reinterpret_cast<uintptr_t>(a.logits_s) & 15) == 0);
  if (a.logits_f16) {
    if (vec) launch_grad<true, true>(a, g, stream);
    else launch_grad<false, true>(a, g, stream);
  } else {
    if (vec) launch_grad<true, false>(a, g, stream);
    else launch_grad<false, false>(a, g, stream);
  }
}

}  // namespace

void launch_teacher_stats(const void* teacher, long long ld, int is_bf16, int n, int v, float inv_t, float* rec,
                          cudaStream_t stream, bool need_d1, bool fast) {
  if (n <= 0) return;
  (void)fast;  // the Fast profile keeps this kernel's arithmetic (see teacher_stats_kernel)
  auto go = [&](auto kern) { kern<<<n, ROW_THREADS, 0, stream>>>(teacher, ld, is_bf16, v, inv_t, rec); };
  if (need_d1 && is_bf16) go(teacher_stats_kernel<true, false, true>);
  else if (need_d1) go(teacher_stats_kernel<true, false, false>);
  else if (is_bf16) go(teacher_stats_kernel<false, false, true>);
  else go(teacher_stats_kernel<false, false, false>);
}

void launch_label_logits(const void* h, long long ldh, const void* w, long long ldw, long long k,
                         const int64_t* labels, long long n, long long v0, long long v_rows, int64_t ignore_index,
                         float* out, cudaStream_t stream) {
  if (n <= 0) return;
  label_logit_kernel<<<static_cast<unsigned>((n + 7) / 8), 256, 0, stream>>>(
      static_cast<const uint16_t*>(h), ldh, static_cast<const uint16_t*>(w), ldw, k, labels, n, v0, v_rows,
      ignore_index, out);
}

void launch_label_prep(const int64_t* labels, long long bt, long long v, int64_t ignore_index, int reduction_sum,
                       long long denom_override, int* n_non_ignore, float* mean_scale, uint8_t* target_flags,
                       int* status, cudaStream_t stream) {
  label_prep_kernel<<<1, 1024, 0, stream>>>(labels, bt, v, ignore_index, reduction_sum, denom_override,
                                            n_non_ignore, mean_scale, target_flags, status);
}

void launch_target_flags(const int64_t* labels, long long bt, long long v, int64_t ignore_index,
                         uint8_t* target_flags, cudaStream_t stream, long long row0) {
  if (bt <= 0) return;
  const int blocks = static_cast<int>((bt + 255) / 256 < 1024 ? (bt + 255) / 256 : 1024);
  target_flags_kernel<<<blocks, 256, 0, stream>>>(labels, bt, v, ignore_index, target_flags, row0);
}

void launch_finalize(const float* nll_s, const float* nll_t, const double* kl_base, const float* s_part, int nseg,
                     double t_sq, long long bt, const float* mean_scale, float w_s, float w_t, float kd,
                     float* scalars, cudaStream_t stream, int include_rows) {
  finalize_kernel<<<1, 1024, 0, stream>>>(nll_s, nll_t, kl_base, s_part, nseg, t_sq, bt, mean_scale, w_s, w_t, kd,
                                          scalars, include_rows);
}

void launch_f32_to_bf16(const float* src, long long rows, long long cols, uint16_t* dst, long long ld,
                        cudaStream_t stream) {
  const long long total = rows * cols;
  if (total <= 0) return;
  long long blocks = (total + 255) / 256;
  if (blocks > 148 * 32) blocks = 148 * 32;
  f32_to_bf16_kernel<<<static_cast<int>(blocks), 256, 0, stream>>>(src, rows, cols, dst, ld);
}

void launch_bf16_rows_to_f32(const uint16_t* src, long long rows, long long cols, float* dst, long long ld,
                             cudaStream_t stream) {
  const long long total = rows * cols;
  if (total <= 0) return;
  long long blocks = (total + 255) / 256;
  if (blocks > 148 * 32) blocks = 148 * 32;
  bf16_rows_to_f32_kernel<<<static_cast<int>(blocks), 256, 0, stream>>>(src, rows, cols, dst, ld);
}

}  // namespace orda
