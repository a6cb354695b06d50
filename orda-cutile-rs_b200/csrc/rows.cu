// rows.cu -- bandwidth-bound row kernels of the distillation loss.
//
// Record layout written by the logits GEMM epilogue (gemm_sm100.cu), one
// record per (row, 128-column part):
//   own  (float4): m = max x, d1 = sum exp(x - m), dT = sum exp((x - m)/T),
//                  sx = sum x
//   pair (2 x float4, teacher values of the same row/columns):
//                  m_t, d1_t, dT_t, S = sum exp((t - m_t)/T) * (t - x)/T | sx_t
// The row kernel merges the records in double precision, evaluates the
// per-row NLL and KL exactly as the reference defines them
// (src/reference/cross_entropy.rs:20-74, src/reference/kl.rs:66-127), and
// streams the row once to write the merged logit gradient
//   dlogit_s = w_s*((p - a/V) - [j==y](1-a)) + kd*T*(p_s^T - p_t^T)
//   dlogit_t = w_t*((p_t - a/V) - [j==y](1-a))
// in bf16 (the operand type of the backward GEMMs), as src/api.rs:301-344
// does on the CPU.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>

#include "kernels.h"
#include "ptx.cuh"

namespace orda {

namespace {

constexpr float LOG2E_F = 1.4426950408889634f;
constexpr int ROW_THREADS = 256;

struct Acc {
  double m, d1, dT, s, sx;
};

__device__ __forceinline__ Acc acc_empty() { return Acc{-INFINITY, 0.0, 0.0, 0.0, 0.0}; }

// Merge of two online-softmax partial states (d1 scales with exp(dm), dT and
// S with exp(dm / T), sx adds).
__device__ __forceinline__ Acc acc_merge(const Acc& a, const Acc& b, double inv_t) {
  if (a.m == -INFINITY) return Acc{b.m, b.d1, b.dT, b.s, a.sx + b.sx};
  if (b.m == -INFINITY) return Acc{a.m, a.d1, a.dT, a.s, a.sx + b.sx};
  const double m = a.m > b.m ? a.m : b.m;
  const double fa1 = exp(a.m - m), fb1 = exp(b.m - m);
  const double faT = exp((a.m - m) * inv_t), fbT = exp((b.m - m) * inv_t);
  return Acc{m, a.d1 * fa1 + b.d1 * fb1, a.dT * faT + b.dT * fbT, a.s * faT + b.s * fbT, a.sx + b.sx};
}

__device__ __forceinline__ Acc acc_shfl_down(const Acc& a, int off) {
  Acc r;
  r.m = __shfl_down_sync(0xffffffffu, a.m, off);
  r.d1 = __shfl_down_sync(0xffffffffu, a.d1, off);
  r.dT = __shfl_down_sync(0xffffffffu, a.dT, off);
  r.s = __shfl_down_sync(0xffffffffu, a.s, off);
  r.sx = __shfl_down_sync(0xffffffffu, a.sx, off);
  return r;
}

// Block-wide merge; result valid in thread 0.
__device__ Acc block_merge(Acc a, double inv_t, Acc* sh) {
  for (int off = 16; off > 0; off >>= 1) a = acc_merge(a, acc_shfl_down(a, off), inv_t);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) sh[w] = a;
  __syncthreads();
  if (w == 0) {
    a = l < (blockDim.x >> 5) ? sh[l] : acc_empty();
    for (int off = 16; off > 0; off >>= 1) a = acc_merge(a, acc_shfl_down(a, off), inv_t);
  }
  __syncthreads();
  return a;
}

__device__ __forceinline__ Acc load_own(const float* rec, long long idx) {
  const float4 r = reinterpret_cast<const float4*>(rec)[idx];
  return Acc{r.x, r.y, r.z, 0.0, r.w};
}
__device__ __forceinline__ Acc load_pair(const float* rec, long long idx) {
  const float4 r0 = reinterpret_cast<const float4*>(rec)[idx * 2];
  const float4 r1 = reinterpret_cast<const float4*>(rec)[idx * 2 + 1];
  return Acc{r0.x, r0.y, r0.z, r0.w, r1.x};
}

__device__ __forceinline__ uint32_t pack_bf16x2(float a, float b) {
  const __nv_bfloat16 ha = __float2bfloat16_rn(a), hb = __float2bfloat16_rn(b);
  return static_cast<uint32_t>(__bfloat16_as_ushort(ha)) | (static_cast<uint32_t>(__bfloat16_as_ushort(hb)) << 16);
}

// Per-row constants handed from the statistics kernel to the gradient
// kernel (lse terms pre-multiplied by log2(e) for exp2).
struct RowConst {
  float c_s1, c_sT, c_tT, c_t1;
  int y;
  int ignored;
  int pad0, pad1;
};

// ---- kernel 1: merge the records of one row, evaluate its losses, write
// its constants. One CTA per row.
__global__ void __launch_bounds__(ROW_THREADS) row_stats_kernel(const RowArgs a) {
  __shared__ Acc sh[ROW_THREADS / 32];
  const int i = blockIdx.x;
  const int P = a.n_parts;
  const double inv_t = static_cast<double>(a.inv_t);
  const bool want_pair = a.need_kl || (a.teacher_ce && !a.teacher_ce_from_own);
  const bool want_tow = a.teacher_ce && a.teacher_ce_from_own;

  Acc own = acc_empty(), pr = acc_empty(), tow = acc_empty();
  for (int p = threadIdx.x; p < P; p += blockDim.x) {
    own = acc_merge(own, load_own(a.rec_own, static_cast<long long>(i) * P + p), inv_t);
    if (want_pair) pr = acc_merge(pr, load_pair(a.rec_pair, static_cast<long long>(i) * P + p), inv_t);
    if (want_tow) tow = acc_merge(tow, load_own(a.rec_own_t, static_cast<long long>(i) * P + p), inv_t);
  }
  own = block_merge(own, inv_t, sh);
  if (want_pair) pr = block_merge(pr, inv_t, sh);
  if (want_tow) tow = block_merge(tow, inv_t, sh);
  if (threadIdx.x != 0) return;

  const int64_t y64 = a.labels[i];
  int ignored = y64 == a.ignore_index;
  if (!ignored && (y64 < 0 || y64 >= a.v)) ignored = 1;  // range errors are reported by the label pass
  const int y = ignored ? 0 : static_cast<int>(y64);
  const double alpha = static_cast<double>(a.alpha);
  const double vd = static_cast<double>(a.v);
  const float* xs = a.logits_s + static_cast<long long>(i) * a.ldl;

  const double lse_s1 = own.m + log(own.d1);
  double nll_s = 0.0;
  if (!ignored) {
    const double x_y = static_cast<double>(xs[y]);
    nll_s = alpha > 0.0 ? lse_s1 - (1.0 - alpha) * x_y - (alpha / vd) * own.sx : lse_s1 - x_y;
  }
  a.nll_s_rows[i] = static_cast<float>(nll_s);

  double lse_sT = 0.0, lse_tT = 0.0;
  if (a.need_kl) {
    lse_sT = own.m * inv_t + log(own.dT);
    lse_tT = pr.m * inv_t + log(pr.dT);
    // KL = sum p_t (log p_t - log p_s) = S / d_t + lse_s^T - lse_t^T
    const double kl = pr.s / pr.dT + lse_sT - lse_tT;
    const double t_sq = static_cast<double>(a.temperature * a.temperature);
    a.kl_rows[i] = ignored ? 0.0 : kl * t_sq;
  } else {
    a.kl_rows[i] = 0.0;
  }

  double lse_t1 = 0.0;
  if (a.teacher_ce) {
    const Acc& ts = a.teacher_ce_from_own ? tow : pr;
    lse_t1 = ts.m + log(ts.d1);
    double nll_t = 0.0;
    if (!ignored) {
      double t_y;
      if (a.teacher_is_bf16) {
        const uint16_t b = static_cast<const uint16_t*>(a.teacher)[static_cast<long long>(i) * a.ld_teacher + y];
        t_y = static_cast<double>(__uint_as_float(static_cast<uint32_t>(b) << 16));
      } else {
        t_y = static_cast<double>(static_cast<const float*>(a.teacher)[static_cast<long long>(i) * a.ld_teacher + y]);
      }
      nll_t = alpha > 0.0 ? lse_t1 - (1.0 - alpha) * t_y - (alpha / vd) * ts.sx : lse_t1 - t_y;
    }
    a.nll_t_rows[i] = static_cast<float>(nll_t);
  } else {
    a.nll_t_rows[i] = 0.0f;
  }

  RowConst rc;
  rc.c_s1 = static_cast<float>(lse_s1 * static_cast<double>(LOG2E_F));
  rc.c_sT = static_cast<float>(lse_sT * static_cast<double>(LOG2E_F));
  rc.c_tT = static_cast<float>(lse_tT * static_cast<double>(LOG2E_F));
  rc.c_t1 = static_cast<float>(lse_t1 * static_cast<double>(LOG2E_F));
  rc.y = y;
  rc.ignored = ignored;
  rc.pad0 = rc.pad1 = 0;
  reinterpret_cast<RowConst*>(a.row_const)[i] = rc;
}

// Scalars shared by every element of the gradient pass.
struct GradScalars {
  float ws, wt, kdT, eps, ws_tgt, wt_tgt, l1, lT;
};

__device__ __forceinline__ void grad_elem(const GradScalars& g, const RowConst& c, bool want_kl, bool want_t,
                                          int j, float x, float t, float& gs, float& gt) {
  float s = g.ws * (exp2f(fmaf(x, g.l1, -c.c_s1)) - g.eps);
  if (want_kl) s += g.kdT * (exp2f(fmaf(x, g.lT, -c.c_sT)) - exp2f(fmaf(t, g.lT, -c.c_tT)));
  if (j == c.y) s -= g.ws_tgt;
  float u = 0.0f;
  if (want_t) {
    u = g.wt * (exp2f(fmaf(t, g.l1, -c.c_t1)) - g.eps);
    if (j == c.y) u -= g.wt_tgt;
  }
  if (c.ignored) {
    s = 0.0f;
    u = 0.0f;
  }
  gs = s;
  gt = u;
}

__device__ __forceinline__ void load_teacher8(const RowArgs& a, long long row, int j0, float (&t)[8]) {
  if (a.teacher_is_bf16) {
    const uint4 q = __ldg(reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(a.teacher) +
                                                         row * a.ld_teacher + j0));
    t[0] = __uint_as_float(q.x << 16);
    t[1] = __uint_as_float(q.x & 0xFFFF0000u);
    t[2] = __uint_as_float(q.y << 16);
    t[3] = __uint_as_float(q.y & 0xFFFF0000u);
    t[4] = __uint_as_float(q.z << 16);
    t[5] = __uint_as_float(q.z & 0xFFFF0000u);
    t[6] = __uint_as_float(q.w << 16);
    t[7] = __uint_as_float(q.w & 0xFFFF0000u);
  } else {
    const float* tp = static_cast<const float*>(a.teacher) + row * a.ld_teacher + j0;
    const float4 t0 = __ldg(reinterpret_cast<const float4*>(tp));
    const float4 t1 = __ldg(reinterpret_cast<const float4*>(tp + 4));
    t[0] = t0.x; t[1] = t0.y; t[2] = t0.z; t[3] = t0.w;
    t[4] = t1.x; t[5] = t1.y; t[6] = t1.z; t[7] = t1.w;
  }
}

// ---- kernel 2: flat elementwise pass over the chunk's [n, V] logits,
// 8 columns per thread per step (32 B fp32 student, 16/32 B teacher in;
// 16 B bf16 gradient out per row kind), grid-stride so every SM stays busy.
// Requires V % 8 == 0 and 16-byte aligned rows (checked by the launcher).
__global__ void __launch_bounds__(256) row_grad_kernel_vec(const RowArgs a, const GradScalars g) {
  const long long vecs_per_row = a.v / 8;
  const long long total = static_cast<long long>(a.n) * vecs_per_row;
  const bool want_kl = a.need_kl != 0;
  const bool want_t = a.teacher_grad != 0;
  const bool need_teacher = want_kl || want_t;
  const RowConst* rcs = reinterpret_cast<const RowConst*>(a.row_const);
  for (long long idx = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; idx < total;
       idx += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long row = idx / vecs_per_row;
    const int j0 = static_cast<int>(idx - row * vecs_per_row) * 8;
    const RowConst c = rcs[row];
    const float* xs = a.logits_s + row * a.ldl + j0;
    const float4 x0 = __ldg(reinterpret_cast<const float4*>(xs));
    const float4 x1 = __ldg(reinterpret_cast<const float4*>(xs + 4));
    const float x[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
    float t[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    if (need_teacher) load_teacher8(a, row, j0, t);
    float gs[8], gt[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) grad_elem(g, c, want_kl, want_t, j0 + k, x[k], t[k], gs[k], gt[k]);
    uint4 o;
    o.x = pack_bf16x2(gs[0], gs[1]);
    o.y = pack_bf16x2(gs[2], gs[3]);
    o.z = pack_bf16x2(gs[4], gs[5]);
    o.w = pack_bf16x2(gs[6], gs[7]);
    *reinterpret_cast<uint4*>(a.dlog_s + row * a.ldd + j0) = o;
    if (want_t) {
      o.x = pack_bf16x2(gt[0], gt[1]);
      o.y = pack_bf16x2(gt[2], gt[3]);
      o.z = pack_bf16x2(gt[4], gt[5]);
      o.w = pack_bf16x2(gt[6], gt[7]);
      *reinterpret_cast<uint4*>(a.dlog_t + row * a.ldd + j0) = o;
    }
  }
}

// Scalar fallback for vocabularies that are not a multiple of 8.
__global__ void __launch_bounds__(256) row_grad_kernel_scalar(const RowArgs a, const GradScalars g) {
  const long long total = static_cast<long long>(a.n) * a.v;
  const bool want_kl = a.need_kl != 0;
  const bool want_t = a.teacher_grad != 0;
  const bool need_teacher = want_kl || want_t;
  const RowConst* rcs = reinterpret_cast<const RowConst*>(a.row_const);
  for (long long idx = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; idx < total;
       idx += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long row = idx / a.v;
    const int j = static_cast<int>(idx - row * a.v);
    const RowConst c = rcs[row];
    const float x = a.logits_s[row * a.ldl + j];
    float t = 0.0f;
    if (need_teacher) {
      if (a.teacher_is_bf16) {
        const uint16_t b = static_cast<const uint16_t*>(a.teacher)[row * a.ld_teacher + j];
        t = __uint_as_float(static_cast<uint32_t>(b) << 16);
      } else {
        t = static_cast<const float*>(a.teacher)[row * a.ld_teacher + j];
      }
    }
    float gs, gt;
    grad_elem(g, c, want_kl, want_t, j, x, t, gs, gt);
    a.dlog_s[row * a.ldd + j] = __bfloat16_as_ushort(__float2bfloat16_rn(gs));
    if (want_t) a.dlog_t[row * a.ldd + j] = __bfloat16_as_ushort(__float2bfloat16_rn(gt));
  }
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
                                    uint8_t* flags) {
  for (long long r = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; r < bt;
       r += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int64_t t = labels[r];
    if (t != ignore_index && t >= 0 && t < v) flags[t] = 1;
  }
}

// ------------------------------------------------------------- finalize
__global__ void __launch_bounds__(1024) finalize_kernel(const float* nll_s, const float* nll_t,
                                                        const double* kl_rows, long long bt,
                                                        const float* mean_scale, float w_s, float w_t, float kd,
                                                        float* scalars) {
  __shared__ double sh[3][32];
  double s0 = 0.0, s1 = 0.0, s2 = 0.0;
  for (long long r = threadIdx.x; r < bt; r += blockDim.x) {
    s0 += static_cast<double>(nll_s[r]);
    s1 += static_cast<double>(nll_t[r]);
    s2 += kl_rows[r];
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
    dst[r * ld + c] = __bfloat16_as_ushort(__float2bfloat16_rn(src[idx]));
  }
}

}  // namespace

void launch_rows(const RowArgs& a, cudaStream_t stream) {
  if (a.n <= 0) return;
  row_stats_kernel<<<a.n, ROW_THREADS, 0, stream>>>(a);
  GradScalars g;
  g.ws = a.w_s;
  g.wt = a.w_t;
  g.kdT = a.need_kl ? a.kd * a.temperature : 0.0f;
  const double alpha = static_cast<double>(a.alpha);
  g.eps = static_cast<float>(alpha / static_cast<double>(a.v));
  const float one_minus_a = static_cast<float>(1.0 - alpha);
  g.ws_tgt = a.w_s * one_minus_a;
  g.wt_tgt = a.w_t * one_minus_a;
  g.l1 = LOG2E_F;
  g.lT = LOG2E_F * a.inv_t;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const long long tsz = a.teacher_is_bf16 ? 2 : 4;
  const bool vec = (a.v % 8 == 0) && (a.ldl % 4 == 0) && (a.ldd % 8 == 0) &&
                   ((a.ld_teacher * tsz) % 16 == 0) && ((reinterpret_cast<uintptr_t>(a.teacher) & 15) == 0) &&
                   ((reinterpret_cast<uintptr_t>(a.logits_s) & 15) == 0);
  const long long work = vec ? static_cast<long long>(a.n) * (a.v / 8) : static_cast<long long>(a.n) * a.v;
  long long blocks = (work + 255) / 256;
  const long long cap = static_cast<long long>(sms) * 8;
  if (blocks > cap) blocks = cap;
  if (vec) row_grad_kernel_vec<<<static_cast<int>(blocks), 256, 0, stream>>>(a, g);
  else row_grad_kernel_scalar<<<static_cast<int>(blocks), 256, 0, stream>>>(a, g);
}

void launch_label_prep(const int64_t* labels, long long bt, long long v, int64_t ignore_index, int reduction_sum,
                       long long denom_override, int* n_non_ignore, float* mean_scale, uint8_t* target_flags,
                       int* status, cudaStream_t stream) {
  label_prep_kernel<<<1, 1024, 0, stream>>>(labels, bt, v, ignore_index, reduction_sum, denom_override,
                                            n_non_ignore, mean_scale, target_flags, status);
}

void launch_target_flags(const int64_t* labels, long long bt, long long v, int64_t ignore_index,
                         uint8_t* target_flags, cudaStream_t stream) {
  if (bt <= 0) return;
  const int blocks = static_cast<int>((bt + 255) / 256 < 1024 ? (bt + 255) / 256 : 1024);
  target_flags_kernel<<<blocks, 256, 0, stream>>>(labels, bt, v, ignore_index, target_flags);
}

void launch_finalize(const float* nll_s, const float* nll_t, const double* kl_rows, long long bt,
                     const float* mean_scale, float w_s, float w_t, float kd, float* scalars, cudaStream_t stream) {
  finalize_kernel<<<1, 1024, 0, stream>>>(nll_s, nll_t, kl_rows, bt, mean_scale, w_s, w_t, kd, scalars);
}

void launch_f32_to_bf16(const float* src, long long rows, long long cols, uint16_t* dst, long long ld,
                        cudaStream_t stream) {
  const long long total = rows * cols;
  if (total <= 0) return;
  long long blocks = (total + 255) / 256;
  if (blocks > 148 * 32) blocks = 148 * 32;
  f32_to_bf16_kernel<<<static_cast<int>(blocks), 256, 0, stream>>>(src, rows, cols, dst, ld);
}

}  // namespace orda
