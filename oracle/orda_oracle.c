/*
 * orda_oracle.c -- CPU restatement of the reference crate's CPU path.
 *
 * TEST INFRASTRUCTURE ONLY. This file is the parity oracle for the B200
 * library: only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline
 * legs load it, and only as the checker or as the timed CPU baseline. The
 * product library (liborda_b200.so) never links or calls it.
 *
 * Reference: malcolmgreaves/orda-cutile-rs (Rust). Rust is not available in
 * this build environment, so the crate cannot be compiled; this restatement
 * follows its loop order and precision exactly:
 *   - f32 sequential dot products, no FMA contraction (Rust does not contract;
 *     build with -ffp-contract=off -fno-fast-math),
 *   - f64 softmax/log-softmax math with f32 results,
 *   - f64 accumulation of per-row / per-chunk sums, f32 mean scale.
 * Each function cites the reference file:line it follows.
 *
 * Parity pinning: the reference ships no stored output files. This oracle is
 * pinned by the reference's own known-answer tests and identities, restated
 * in tests/test_oracle_*.py (mat known answers, resolver integers, KL/CE
 * identities, round-half-even table, quantiser bounds, finite-difference
 * gradient checks of tests/end_to_end.rs).
 *
 * Parallel variant: every `nthreads` argument > 1 enables an OpenMP split
 * that keeps the accumulation order of every output element identical to the
 * sequential loops (parallel only over independent output elements or rows;
 * all cross-row sums stay sequential), so results are bit-identical for any
 * thread count.
 */
#include <float.h>
#include <math.h>
#include <stdarg.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

#include "../include/orda.h"

#define EXPORT __attribute__((visibility("default")))

/* ------------------------------------------------------------------------ */
/* small helpers                                                             */
/* ------------------------------------------------------------------------ */

static void set_err(char* err, size_t len, const char* fmt, ...) {
  if (!err || len == 0) return;
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(err, len, fmt, ap);
  va_end(ap);
}

/* Rust `Display` for f32: shortest digits that round-trip, never exponent
 * notation, "NaN"/"inf"/"-inf" for non-finite values. */
EXPORT void oref_format_f32(float x, char* out, size_t len) {
  if (isnan(x)) { snprintf(out, len, "NaN"); return; }
  if (isinf(x)) { snprintf(out, len, x > 0 ? "inf" : "-inf"); return; }
  char buf[64];
  int prec;
  for (prec = 1; prec <= 9; ++prec) {
    snprintf(buf, sizeof buf, "%.*e", prec - 1, (double)x);
    if (strtof(buf, NULL) == x) break;
  }
  /* buf = [-]d.ddde[+-]XX ; rebuild in fixed notation */
  const char* p = buf;
  int neg = 0;
  if (*p == '-') { neg = 1; ++p; }
  char digits[32];
  int nd = 0;
  while (*p && *p != 'e') {
    if (*p >= '0' && *p <= '9') digits[nd++] = *p;
    ++p;
  }
  int exp10 = atoi(p + 1);
  /* strip trailing zeros of the mantissa */
  while (nd > 1 && digits[nd - 1] == '0') --nd;
  char res[128];
  int r = 0;
  if (neg) res[r++] = '-';
  if (nd == 1 && digits[0] == '0') { /* zero */
    res[r++] = '0';
  } else if (exp10 >= 0) {
    /* integer part: digits[0..exp10], zero padded; fraction: the rest */
    for (int i = 0; i <= exp10; ++i) res[r++] = i < nd ? digits[i] : '0';
    if (nd > exp10 + 1) {
      res[r++] = '.';
      for (int i = exp10 + 1; i < nd; ++i) res[r++] = digits[i];
    }
  } else {
    res[r++] = '0';
    res[r++] = '.';
    for (int i = 0; i < -exp10 - 1; ++i) res[r++] = '0';
    for (int i = 0; i < nd; ++i) res[r++] = digits[i];
  }
  res[r] = 0;
  snprintf(out, len, "%s", res);
}

static int nthreads_eff(int n) { return n < 1 ? 1 : n; }

/* ------------------------------------------------------------------------ */
/* mat.rs                                                                    */
/* ------------------------------------------------------------------------ */

/* `matmul_nt` src/mat.rs:63-80: out[i][j] = sum_p a[i][p]*b[j][p], f32 acc. */
EXPORT void oref_matmul_nt(const float* a, const float* b, float* out, size_t m, size_t k, size_t n,
                           int nthreads) {
  long long total = (long long)m * (long long)n;
#pragma omp parallel for schedule(static) num_threads(nthreads_eff(nthreads)) if (nthreads > 1)
  for (long long idx = 0; idx < total; ++idx) {
    size_t i = (size_t)(idx / (long long)n), j = (size_t)(idx % (long long)n);
    const float* arow = a + i * k;
    const float* brow = b + j * k;
    float acc = 0.0f;
    for (size_t p = 0; p < k; ++p) acc += arow[p] * brow[p];
    out[i * n + j] = acc;
  }
}

/* `matmul_nn` src/mat.rs:86-105: out = a@b, skipping exact zeros of a. */
EXPORT void oref_matmul_nn(const float* a, const float* b, float* out, size_t m, size_t k, size_t n,
                           int nthreads) {
  memset(out, 0, sizeof(float) * m * n);
  const size_t JB = 256;
  size_t njb = (n + JB - 1) / JB;
  long long total = (long long)m * (long long)njb;
#pragma omp parallel for schedule(static) num_threads(nthreads_eff(nthreads)) if (nthreads > 1)
  for (long long idx = 0; idx < total; ++idx) {
    size_t i = (size_t)(idx / (long long)njb), jb = (size_t)(idx % (long long)njb);
    size_t j0 = jb * JB, j1 = j0 + JB < n ? j0 + JB : n;
    const float* arow = a + i * k;
    float* orow = out + i * n;
    for (size_t p = 0; p < k; ++p) {
      float aip = arow[p];
      if (aip == 0.0f) continue;
      const float* brow = b + p * n;
      for (size_t j = j0; j < j1; ++j) orow[j] += aip * brow[j];
    }
  }
}

/* `matmul_tn` src/mat.rs:111-130: out = a^T@b with a [k,m], b [k,n]. */
EXPORT void oref_matmul_tn(const float* a, const float* b, float* out, size_t k, size_t m, size_t n,
                           int nthreads) {
  memset(out, 0, sizeof(float) * m * n);
#pragma omp parallel for schedule(static) num_threads(nthreads_eff(nthreads)) if (nthreads > 1)
  for (long long ii = 0; ii < (long long)m; ++ii) {
    size_t i = (size_t)ii;
    float* orow = out + i * n;
    for (size_t p = 0; p < k; ++p) {
      float aip = a[p * m + i];
      if (aip == 0.0f) continue;
      const float* brow = b + p * n;
      for (size_t j = 0; j < n; ++j) orow[j] += aip * brow[j];
    }
  }
}

/* `add_assign` src/mat.rs:133-138. */
static void add_assign(float* dst, const float* src, size_t count, int nthreads) {
#pragma omp parallel for schedule(static) num_threads(nthreads_eff(nthreads)) if (nthreads > 1)
  for (long long i = 0; i < (long long)count; ++i) dst[i] += src[i];
}

/* `scale_assign` src/mat.rs:141-145. */
static void scale_assign(float* m, size_t count, float s, int nthreads) {
#pragma omp parallel for schedule(static) num_threads(nthreads_eff(nthreads)) if (nthreads > 1)
  for (long long i = 0; i < (long long)count; ++i) m[i] *= s;
}

/* ------------------------------------------------------------------------ */
/* reference/kl.rs                                                           */
/* ------------------------------------------------------------------------ */

/* `softmax_logsoftmax` src/reference/kl.rs:20-41 (f64). */
EXPORT void oref_softmax_logsoftmax(const float* x, size_t n, double inv_t, double* p, double* log_p) {
  double m = -INFINITY;
  for (size_t i = 0; i < n; ++i) {
    double z = (double)x[i] * inv_t;
    if (z > m) m = z;
  }
  double d = 0.0;
  for (size_t i = 0; i < n; ++i) d += exp(((double)x[i] * inv_t) - m);
  double log_d = log(d);
  for (size_t i = 0; i < n; ++i) {
    double zc = ((double)x[i] * inv_t) - m;
    p[i] = exp(zc) / d;
    log_p[i] = zc - log_d;
  }
}

/* `forward_kl_row` src/reference/kl.rs:45-54 (unscaled). */
EXPORT double oref_forward_kl_row(const float* s, const float* t, size_t n, double temperature) {
  double inv_t = 1.0 / temperature;
  double* buf = (double*)malloc(sizeof(double) * 4 * n);
  double *ps = buf, *lps = buf + n, *pt = buf + 2 * n, *lpt = buf + 3 * n;
  oref_softmax_logsoftmax(s, n, inv_t, ps, lps);
  oref_softmax_logsoftmax(t, n, inv_t, pt, lpt);
  double kl = 0.0;
  for (size_t j = 0; j < n; ++j) kl += pt[j] * (lpt[j] - lps[j]);
  free(buf);
  return kl;
}

/* `kl_chunk` src/reference/kl.rs:66-127. logits [2*n_rows, v]; grad (nullable)
 * [n_rows, v]. Returns the chunk sum of KL*T^2 cast to f32. */
EXPORT float oref_kl_chunk(const float* logits, size_t v, const int64_t* targets, size_t n_rows, float kl_weight,
                           float temperature, int64_t ignore_index, float grad_denom, float* grad,
                           int nthreads) {
  double inv_t = 1.0 / (double)temperature;
  double grad_scale = (double)(kl_weight * temperature / grad_denom);
  double t_sq = (double)(temperature * temperature);
  double* kl_rows = (double*)malloc(sizeof(double) * (n_rows ? n_rows : 1));
#pragma omp parallel num_threads(nthreads_eff(nthreads)) if (nthreads > 1)
  {
    double* buf = (double*)malloc(sizeof(double) * 4 * (v ? v : 1));
    double *ps = buf, *lps = buf + v, *pt = buf + 2 * v, *lpt = buf + 3 * v;
#pragma omp for schedule(static)
    for (long long ii = 0; ii < (long long)n_rows; ++ii) {
      size_t i = (size_t)ii;
      int ignored = targets[i] == ignore_index;
      const float* s = logits + i * v;
      const float* t = logits + (n_rows + i) * v;
      oref_softmax_logsoftmax(s, v, inv_t, ps, lps);
      oref_softmax_logsoftmax(t, v, inv_t, pt, lpt);
      double kl_row = 0.0;
      for (size_t j = 0; j < v; ++j) kl_row += pt[j] * (lpt[j] - lps[j]);
      if (ignored) kl_row = 0.0;
      kl_rows[i] = kl_row;
      if (grad) {
        float* grow = grad + i * v;
        if (ignored) {
          for (size_t j = 0; j < v; ++j) grow[j] = 0.0f;
        } else {
          for (size_t j = 0; j < v; ++j) grow[j] = (float)(grad_scale * (ps[j] - pt[j]));
        }
      }
    }
    free(buf);
  }
  double kl_accum = 0.0;
  for (size_t i = 0; i < n_rows; ++i) kl_accum += kl_rows[i] * t_sq;
  free(kl_rows);
  return (float)kl_accum;
}

/* ------------------------------------------------------------------------ */
/* reference/cross_entropy.rs                                                */
/* ------------------------------------------------------------------------ */

/* `ce_fwdbwd_row` src/reference/cross_entropy.rs:20-74. Returns the f32 NLL
 * and writes the f32 gradient row (may alias x: x is fully read first). */
EXPORT float oref_ce_fwdbwd_row(const float* x, size_t v, int64_t y, int64_t ignore_index,
                                float label_smoothing, float scale, float* grad) {
  int ignored = y == ignore_index;
  double alpha = (double)label_smoothing;
  double m = -INFINITY;
  for (size_t i = 0; i < v; ++i)
    if ((double)x[i] > m) m = (double)x[i];
  double d = 0.0, sum_x = 0.0;
  for (size_t i = 0; i < v; ++i) {
    d += exp((double)x[i] - m);
    if (alpha > 0.0) sum_x += (double)x[i];
  }
  double lse = m + log(d);
  size_t y_safe = ignored ? 0 : (size_t)y;
  double logit_tgt = (double)x[y_safe];
  double nll = alpha > 0.0 ? lse - (1.0 - alpha) * logit_tgt - (alpha / (double)v) * sum_x : lse - logit_tgt;
  if (ignored) nll = 0.0;
  double eff_scale = ignored ? 0.0 : (double)scale;
  double eps = alpha / (double)v;
  if (eff_scale != 0.0) {
    /* compute into a temporary so grad may alias x */
    float* tmp = (float*)malloc(sizeof(float) * (v ? v : 1));
    for (size_t j = 0; j < v; ++j) {
      double p = exp((double)x[j] - m) / d;
      double prob = alpha > 0.0 ? p - eps : p;
      if (j == y_safe) prob -= 1.0 - alpha;
      tmp[j] = (float)(prob * eff_scale);
    }
    memcpy(grad, tmp, sizeof(float) * v);
    free(tmp);
  } else {
    for (size_t j = 0; j < v; ++j) grad[j] = 0.0f;
  }
  return (float)nll;
}

/* ------------------------------------------------------------------------ */
/* resolver.rs                                                               */
/* ------------------------------------------------------------------------ */

/* `chunks_from_raw` src/resolver.rs:28-36. */
EXPORT size_t oref_chunks_from_raw(double raw) {
  if (raw < 1.5) return 1;
  double e = floor(log2(raw / 1.5));
  long long ei;
  if (isnan(e)) ei = 0;
  else if (e >= 9.2e18) ei = INT64_MAX;
  else if (e <= -9.2e18) ei = INT64_MIN;
  else ei = (long long)e;
  long long sh = (ei >= INT64_MAX - 1) ? 60 : ei + 1;
  if (sh < 0) sh = 0;
  if (sh > 60) sh = 60;
  return (size_t)1 << sh;
}

static size_t min_sz(size_t a, size_t b) { return a < b ? a : b; }
static size_t max_sz(size_t a, size_t b) { return a > b ? a : b; }
static size_t ceil_div(size_t a, size_t b) { return (a + b - 1) / b; }

/* `resolve_chunk_size` src/resolver.rs:53-99. */
EXPORT void oref_resolve_chunk_size(size_t bt, int fixed, size_t fixed_rows, int has_v, size_t v,
                                    int has_max_chunks, size_t max_chunks, OrdaChunkPlan* out) {
  if (bt == 0) { out->chunk_size = 0; out->num_chunks = 0; return; }
  if (fixed) {
    size_t cs = max_sz(min_sz(fixed_rows, bt), 1);
    out->chunk_size = cs;
    out->num_chunks = ceil_div(bt, cs);
    return;
  }
  if (!has_v) { out->chunk_size = bt; out->num_chunks = 1; return; }
  size_t max_useful = max_sz(bt / 512, 1);
  size_t mc = has_max_chunks ? max_chunks : 2 * max_useful;
  double vr = (double)v / 32768.0;
  double raw_pressure = ((double)bt / 1024.0) * (vr * vr);
  double raw_bt_floor = (double)bt / 4096.0;
  double raw = fmax(raw_pressure, raw_bt_floor);
  size_t nc = oref_chunks_from_raw(raw);
  nc = min_sz(nc, mc);
  nc = min_sz(nc, max_useful);
  nc = min_sz(nc, bt);
  nc = max_sz(nc, 1);
  out->chunk_size = ceil_div(bt, nc);
  out->num_chunks = nc;
}

/* `default_max_chunks_limit` src/resolver.rs:103-105. */
EXPORT size_t oref_default_max_chunks_limit(size_t bt) { return 2 * max_sz(bt / 512, 1); }

/* `chunk_doubling_schedule` src/resolver.rs:114-126. */
EXPORT size_t oref_chunk_doubling_schedule(size_t bt, size_t start, size_t limit, size_t* out, size_t cap) {
  size_t lim = min_sz(max_sz(limit, 1), bt);
  size_t n = start < 1 ? 1 : (start > lim ? lim : start);
  size_t len = 0;
  if (len < cap) out[len] = n;
  ++len;
  while (n < bt && n < lim) {
    n = min_sz(min_sz(n * 2, bt), lim);
    if (len < cap) out[len] = n;
    ++len;
    if (n >= bt || n >= lim) break;
  }
  return len;
}

/* ------------------------------------------------------------------------ */
/* quant.rs                                                                  */
/* ------------------------------------------------------------------------ */

#define GOLDEN 0x9E3779B97F4A7C15ULL

/* `Rng` src/quant.rs:18-44 (SplitMix64). */
typedef struct { uint64_t state; } ORng;
static void rng_new(ORng* r, uint64_t seed) { r->state = seed + GOLDEN; }
static uint64_t rng_next_u64(ORng* r) {
  r->state += GOLDEN;
  uint64_t z = r->state;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
  return z ^ (z >> 31);
}
static float rng_next_f32(ORng* r) {
  return ((float)(rng_next_u64(r) >> 40)) * (1.0f / (float)(1u << 24));
}
EXPORT void oref_rng_f32_stream(uint64_t seed, float* out, size_t n) {
  ORng r;
  rng_new(&r, seed);
  for (size_t i = 0; i < n; ++i) out[i] = rng_next_f32(&r);
}

/* `round_half_even` src/quant.rs:48-63. */
EXPORT float oref_round_half_even(float x) {
  float f = floorf(x);
  float diff = x - f;
  if (diff < 0.5f) return f;
  if (diff > 0.5f) return f + 1.0f;
  long long fi = (long long)f;
  return (fi % 2 == 0) ? f : f + 1.0f;
}

/* Rust `f32::clamp(-127,127)` then `as i8` (saturating; NaN -> 0). */
static int8_t to_i8(float v) {
  if (isnan(v)) return 0;
  if (v < -127.0f) v = -127.0f;
  if (v > 127.0f) v = 127.0f;
  return (int8_t)v;
}

/* `row_scale` src/quant.rs:91-94. */
static float row_scale(const float* row, size_t cols) {
  float amax = 0.0f;
  for (size_t c = 0; c < cols; ++c) amax = fmaxf(amax, fabsf(row[c]));
  return fmaxf(amax, 1e-12f) / 127.0f;
}

/* `quantize_rowwise_int8` src/quant.rs:97-117. */
EXPORT void oref_quantize_rowwise_int8(const float* m, size_t rows, size_t cols, int8_t* q, float* scale,
                                       int nthreads) {
#pragma omp parallel for schedule(static) num_threads(nthreads_eff(nthreads)) if (nthreads > 1)
  for (long long rr = 0; rr < (long long)rows; ++rr) {
    size_t r = (size_t)rr;
    const float* row = m + r * cols;
    float s = row_scale(row, cols);
    scale[r] = s;
    for (size_t c = 0; c < cols; ++c) q[r * cols + c] = to_i8(oref_round_half_even(row[c] / s));
  }
}

/* `quantize_rowwise_int8_stochastic` src/quant.rs:120-144 (one sequential
 * RNG stream over the whole matrix in row-major order). */
EXPORT void oref_quantize_rowwise_int8_stochastic(const float* m, size_t rows, size_t cols, uint64_t seed,
                                                  int8_t* q, float* scale) {
  ORng rng;
  rng_new(&rng, seed);
  for (size_t r = 0; r < rows; ++r) {
    const float* row = m + r * cols;
    float s = row_scale(row, cols);
    scale[r] = s;
    for (size_t c = 0; c < cols; ++c) {
      float scaled = row[c] / s;
      float floor_v = floorf(scaled);
      float frac = scaled - floor_v;
      float bump = frac > rng_next_f32(&rng) ? 1.0f : 0.0f;
      q[r * cols + c] = to_i8(floor_v + bump);
    }
  }
}

static int cmp_size(const void* a, const void* b) {
  size_t x = *(const size_t*)a, y = *(const size_t*)b;
  return x < y ? -1 : (x > y ? 1 : 0);
}

/* unique, sorted target ids as in `quantize_grad_w` src/quant.rs:164-171.
 * Returns the count; ids written to out (capacity n_labels). */
EXPORT size_t oref_unique_targets(const int64_t* target, size_t n, int64_t ignore_index, size_t rows,
                                  size_t* out) {
  size_t k = 0;
  for (size_t i = 0; i < n; ++i) {
    int64_t t = target[i];
    if (t != ignore_index && t >= 0 && (uint64_t)t < rows) out[k++] = (size_t)t;
  }
  qsort(out, k, sizeof(size_t), cmp_size);
  size_t u = 0;
  for (size_t i = 0; i < k; ++i)
    if (u == 0 || out[u - 1] != out[i]) out[u++] = out[i];
  return u;
}

/* `quantize_grad_w` + `dequantize_grad_w(.., grad_output)` src/quant.rs:157-202.
 * q / scale receive the INT8 body; deq [rows, cols] the reconstructed grad_W. */
EXPORT void oref_quantize_grad_w(const float* grad_w, size_t rows, size_t cols, const int64_t* target,
                                 size_t n_target, int64_t ignore_index, int stochastic, uint64_t seed,
                                 float grad_output, int8_t* q, float* scale, float* deq, int nthreads) {
  size_t* uniq = (size_t*)malloc(sizeof(size_t) * (n_target ? n_target : 1));
  size_t nu = oref_unique_targets(target, n_target, ignore_index, rows, uniq);
  float* target_rows = (float*)malloc(sizeof(float) * (nu * cols > 0 ? nu * cols : 1));
  for (size_t i = 0; i < nu; ++i) memcpy(target_rows + i * cols, grad_w + uniq[i] * cols, sizeof(float) * cols);
  if (stochastic) oref_quantize_rowwise_int8_stochastic(grad_w, rows, cols, seed, q, scale);
  else oref_quantize_rowwise_int8(grad_w, rows, cols, q, scale, nthreads);
  /* `QuantRows::dequantize` src/quant.rs:77-87 */
#pragma omp parallel for schedule(static) num_threads(nthreads_eff(nthreads)) if (nthreads > 1)
  for (long long rr = 0; rr < (long long)rows; ++rr) {
    size_t r = (size_t)rr;
    float s = scale[r];
    for (size_t c = 0; c < cols; ++c) deq[r * cols + c] = (float)q[r * cols + c] * s;
  }
  for (size_t i = 0; i < nu; ++i) memcpy(deq + uniq[i] * cols, target_rows + i * cols, sizeof(float) * cols);
  scale_assign(deq, rows * cols, grad_output, nthreads);
  free(target_rows);
  free(uniq);
}

/* ------------------------------------------------------------------------ */
/* config.rs / teacher.rs / api.rs                                           */
/* ------------------------------------------------------------------------ */

/* `is_power_of_two` src/config.rs:122-124. */
EXPORT int oref_is_power_of_two(size_t v) { return v > 0 && (v & (v - 1)) == 0; }

/* `KernelConfig::from_profile` src/config.rs:81-93. */
EXPORT void oref_kernel_config_from_profile(int profile, OrdaKernelConfig* c) {
  memset(c, 0, sizeof *c);
  c->fast_math = profile == ORDA_PROFILE_FAST;
  c->max_fused_size = 65536 / 2; /* DEFAULT_MAX_FUSED_SIZE src/config.rs:66 */
}

/* `LossOptions::default` src/api.rs:49-64. */
EXPORT void oref_loss_options_default(OrdaLossOptions* o) {
  memset(o, 0, sizeof *o);
  o->student_ce_weight = 1.0f;
  o->has_teacher_ce_weight = 0;
  o->kd_weight = 0.0f;
  o->temperature = 1.0f;
  o->ignore_index = -100;
  o->label_smoothing = 0.0f;
  o->reduction = ORDA_REDUCTION_MEAN;
  o->chunk_size.kind = ORDA_CHUNK_AUTO;
  oref_kernel_config_from_profile(ORDA_PROFILE_BALANCED, &o->config);
  o->backend = ORDA_BACKEND_AUTO;
}

/* `KernelConfig::validate` src/config.rs:106-119. */
EXPORT int oref_kernel_config_validate(const OrdaKernelConfig* c, char* err, size_t len) {
  if (c->max_fused_size < 1 || !oref_is_power_of_two(c->max_fused_size)) {
    set_err(err, len, "max_fused_size must be a power of two >= 1, got %zu", c->max_fused_size);
    return ORDA_ERR_INVALID;
  }
  if (c->has_max_chunks && c->max_chunks < 1) {
    set_err(err, len, "max_chunks must be >= 1, got %zu", c->max_chunks);
    return ORDA_ERR_INVALID;
  }
  return ORDA_OK;
}

/* `default_teacher_ce_weight` src/teacher.rs:54-59. */
EXPORT float oref_default_teacher_ce_weight(int mode) { return mode == ORDA_TEACHER_TIED ? 1.0f : 0.0f; }

/* `validate` src/api.rs:104-181. */
EXPORT int oref_validate(const OrdaMatF32* sh, const OrdaMatF32* w, const int64_t* labels, size_t n_labels,
                         const OrdaTeacher* t, const OrdaLossOptions* o, size_t* v_out, size_t* h_out,
                         size_t* bt_out, char* err, size_t len) {
  int rc = oref_kernel_config_validate(&o->config, err, len);
  if (rc) return rc;
  size_t bt = sh->rows, h = sh->cols;
  if (bt == 0) { set_err(err, len, "student_hidden has 0 rows (BT must be > 0)"); return ORDA_ERR_INVALID; }
  if (w->cols != h) {
    set_err(err, len, "weight must have shape (V, %zu), got (%zu, %zu)", h, w->rows, w->cols);
    return ORDA_ERR_INVALID;
  }
  size_t v = w->rows;
  if (n_labels != bt) {
    set_err(err, len, "labels must have length BT=%zu, got %zu", bt, n_labels);
    return ORDA_ERR_INVALID;
  }
  for (size_t i = 0; i < n_labels; ++i) {
    int64_t lab = labels[i];
    if (lab != o->ignore_index && (lab < 0 || (uint64_t)lab >= v)) {
      set_err(err, len, "label %lld out of range [0, %zu) and != ignore_index %lld", (long long)lab, v,
              (long long)o->ignore_index);
      return ORDA_ERR_INVALID;
    }
  }
  char fb[64];
  if (!(o->label_smoothing >= 0.0f && o->label_smoothing <= 1.0f)) {
    oref_format_f32(o->label_smoothing, fb, sizeof fb);
    set_err(err, len, "label_smoothing must be in [0,1], got %s", fb);
    return ORDA_ERR_INVALID;
  }
  if (o->kd_weight < 0.0f) {
    oref_format_f32(o->kd_weight, fb, sizeof fb);
    set_err(err, len, "kd_weight must be >= 0, got %s", fb);
    return ORDA_ERR_INVALID;
  }
  if (o->temperature <= 0.0f) {
    oref_format_f32(o->temperature, fb, sizeof fb);
    set_err(err, len, "temperature must be > 0, got %s", fb);
    return ORDA_ERR_INVALID;
  }
  switch (t->mode) {
    case ORDA_TEACHER_TIED:
      if (t->hidden.rows != bt || t->hidden.cols != h) {
        set_err(err, len, "Tied teacher hidden must be (%zu, %zu), got (%zu, %zu)", bt, h, t->hidden.rows,
                t->hidden.cols);
        return ORDA_ERR_INVALID;
      }
      break;
    case ORDA_TEACHER_SEPARATE: {
      if (t->hidden.rows != bt) {
        set_err(err, len, "Separate teacher hidden must have BT=%zu rows", bt);
        return ORDA_ERR_INVALID;
      }
      size_t ht = t->hidden.cols;
      if (t->weight.rows != v || t->weight.cols != ht) {
        set_err(err, len, "Separate teacher weight must be (%zu, %zu), got (%zu, %zu)", v, ht, t->weight.rows,
                t->weight.cols);
        return ORDA_ERR_INVALID;
      }
      break;
    }
    case ORDA_TEACHER_PRECOMPUTED:
      if (t->logits.rows != bt || t->logits.cols != v) {
        set_err(err, len, "Precomputed teacher logits must be (%zu, %zu), got (%zu, %zu)", bt, v,
                t->logits.rows, t->logits.cols);
        return ORDA_ERR_INVALID;
      }
      break;
    default:
      set_err(err, len, "unknown teacher mode %d", (int)t->mode);
      return ORDA_ERR_INVALID;
  }
  *v_out = v;
  *h_out = h;
  *bt_out = bt;
  return ORDA_OK;
}

/* `distillation_loss` src/api.rs:188-422 (CPU path). The oracle runs the
 * reference's CPU loop for Backend::Auto / Backend::Cpu; Backend::Cuda gives
 * the reference's own error (src/api.rs:198-205).
 *
 * scalars[4] = {loss, student_ce, teacher_ce, kl}. grad_h_t / grad_w_t may be
 * NULL; *has_gh_t / *has_gw_t report whether the reference returns Some.
 * raw_grad_w (nullable) receives grad_W after the deferred mean and before the
 * optional INT8 round trip. */
EXPORT int oref_distillation_loss(const OrdaMatF32* student_hidden, const OrdaMatF32* weight,
                                  const int64_t* labels, size_t n_labels, const OrdaTeacher* teacher,
                                  const OrdaLossOptions* opts, int nthreads, float* scalars, float* grad_h_s,
                                  float* grad_w, float* grad_h_t, float* grad_w_t, int* has_gh_t,
                                  int* has_gw_t, float* raw_grad_w, OrdaChunkPlan* plan_out, char* err,
                                  size_t err_len) {
  size_t v, h, bt;
  int rc = oref_validate(student_hidden, weight, labels, n_labels, teacher, opts, &v, &h, &bt, err, err_len);
  if (rc) return rc;
  if (opts->backend == ORDA_BACKEND_CUDA) {
    set_err(err, err_len,
            "Backend::Cuda requires building with --features cuda on an NVIDIA sm_80+ GPU with CUDA 13.3. "
            "This build has no GPU backend. See docs/BLOCKERS.md.");
    return ORDA_ERR_BACKEND;
  }
  int mode = teacher->mode;
  float w_s = opts->student_ce_weight;
  float w_t = opts->has_teacher_ce_weight ? opts->teacher_ce_weight : oref_default_teacher_ce_weight(mode);
  if (w_t < 0.0f) {
    char fb[64];
    oref_format_f32(w_t, fb, sizeof fb);
    set_err(err, err_len, "teacher_ce_weight must be >= 0, got %s", fb);
    return ORDA_ERR_INVALID;
  }
  float kd = opts->kd_weight, temperature = opts->temperature, ls = opts->label_smoothing;
  int64_t ignore = opts->ignore_index;
  int need_teacher = kd > 0.0f || w_t > 0.0f;
  size_t n_non_ignore = 0;
  for (size_t i = 0; i < bt; ++i) n_non_ignore += labels[i] != ignore;
  size_t denom = opts->reduction == ORDA_REDUCTION_MEAN ? max_sz(n_non_ignore, 1) : 1;
  float mean_scale = 1.0f / (float)denom;

  OrdaChunkPlan plan;
  oref_resolve_chunk_size(bt, opts->chunk_size.kind == ORDA_CHUNK_FIXED, opts->chunk_size.fixed_rows, 1, v,
                          opts->config.has_max_chunks, opts->config.max_chunks, &plan);
  size_t ht_dim = mode == ORDA_TEACHER_SEPARATE ? teacher->hidden.cols : h;
  int gh_t = w_t > 0.0f && (mode == ORDA_TEACHER_TIED || mode == ORDA_TEACHER_SEPARATE);
  int gw_t = w_t > 0.0f && mode == ORDA_TEACHER_SEPARATE;
  if (has_gh_t) *has_gh_t = gh_t;
  if (has_gw_t) *has_gw_t = gw_t;
  if (gh_t && !grad_h_t) { set_err(err, err_len, "oracle: grad_h_t buffer required"); return ORDA_ERR_INVALID; }
  if (gw_t && !grad_w_t) { set_err(err, err_len, "oracle: grad_w_t buffer required"); return ORDA_ERR_INVALID; }

  memset(grad_h_s, 0, sizeof(float) * bt * h);
  memset(grad_w, 0, sizeof(float) * v * h);
  if (gh_t) memset(grad_h_t, 0, sizeof(float) * bt * ht_dim);
  if (gw_t) memset(grad_w_t, 0, sizeof(float) * v * ht_dim);

  double sum_nll_s = 0.0, sum_nll_t = 0.0, kl_accum = 0.0;
  size_t cs = plan.chunk_size;
  size_t maxw = h > ht_dim ? h : ht_dim;
  float* logits_chunk = (float*)malloc(sizeof(float) * 2 * cs * v);
  float* grad_kl = (float*)malloc(sizeof(float) * cs * v);
  float* tmp_h = (float*)malloc(sizeof(float) * cs * maxw);
  float* tmp_w = (float*)malloc(sizeof(float) * v * maxw);
  float* nll_rows = (float*)malloc(sizeof(float) * cs);
  if (!logits_chunk || !grad_kl || !tmp_h || !tmp_w || !nll_rows) {
    free(logits_chunk); free(grad_kl); free(tmp_h); free(tmp_w); free(nll_rows);
    set_err(err, err_len, "oracle: host allocation failed");
    return ORDA_ERR_OOM;
  }

  for (size_t c = 0; c < plan.num_chunks; ++c) {
    size_t start = c * cs;
    if (start >= bt) break;
    size_t end = min_sz(start + cs, bt), n = end - start;
    const float* h_s_chunk = student_hidden->data + start * h;
    /* logits_s = matmul_nt(h_s_chunk, W) straight into the chunk buffer */
    oref_matmul_nt(h_s_chunk, weight->data, logits_chunk, n, h, v, nthreads);
    const float* h_t_chunk = NULL;
    if (need_teacher) {
      float* lt = logits_chunk + n * v;
      if (mode == ORDA_TEACHER_TIED) {
        h_t_chunk = teacher->hidden.data + start * h;
        oref_matmul_nt(h_t_chunk, weight->data, lt, n, h, v, nthreads);
      } else if (mode == ORDA_TEACHER_SEPARATE) {
        h_t_chunk = teacher->hidden.data + start * ht_dim;
        oref_matmul_nt(h_t_chunk, teacher->weight.data, lt, n, ht_dim, v, nthreads);
      } else {
        memcpy(lt, teacher->logits.data + start * v, sizeof(float) * n * v);
      }
    }
    int have_kl = 0;
    if (kd > 0.0f) {
      float kl_sum_chunk = oref_kl_chunk(logits_chunk, v, labels + start, n, kd, temperature, ignore, 1.0f,
                                         grad_kl, nthreads);
      kl_accum += (double)kl_sum_chunk;
      have_kl = 1;
    }
    /* CE student rows, in place (src/api.rs:319-323) */
#pragma omp parallel for schedule(static) num_threads(nthreads_eff(nthreads)) if (nthreads > 1)
    for (long long rr = 0; rr < (long long)n; ++rr) {
      size_t r = (size_t)rr;
      nll_rows[r] = oref_ce_fwdbwd_row(logits_chunk + r * v, v, labels[start + r], ignore, ls, w_s,
                                       logits_chunk + r * v);
    }
    for (size_t r = 0; r < n; ++r) sum_nll_s += (double)nll_rows[r];
    if (w_t > 0.0f) { /* src/api.rs:326-333 */
#pragma omp parallel for schedule(static) num_threads(nthreads_eff(nthreads)) if (nthreads > 1)
      for (long long rr = 0; rr < (long long)n; ++rr) {
        size_t r = (size_t)rr;
        nll_rows[r] = oref_ce_fwdbwd_row(logits_chunk + (n + r) * v, v, labels[start + r], ignore, ls, w_t,
                                         logits_chunk + (n + r) * v);
      }
      for (size_t r = 0; r < n; ++r) sum_nll_t += (double)nll_rows[r];
    }
    if (have_kl) add_assign(logits_chunk, grad_kl, n * v, nthreads); /* src/api.rs:336-344 */

    /* GEMM backward (src/api.rs:347-377) */
    const float* sgr = logits_chunk;
    oref_matmul_nn(sgr, weight->data, tmp_h, n, v, h, nthreads);
    memcpy(grad_h_s + start * h, tmp_h, sizeof(float) * n * h);
    oref_matmul_tn(sgr, h_s_chunk, tmp_w, n, v, h, nthreads);
    add_assign(grad_w, tmp_w, v * h, nthreads);
    if (w_t > 0.0f) {
      const float* tgr = logits_chunk + n * v;
      if (mode == ORDA_TEACHER_TIED) {
        oref_matmul_nn(tgr, weight->data, tmp_h, n, v, h, nthreads);
        memcpy(grad_h_t + start * ht_dim, tmp_h, sizeof(float) * n * ht_dim);
        oref_matmul_tn(tgr, h_t_chunk, tmp_w, n, v, h, nthreads);
        add_assign(grad_w, tmp_w, v * h, nthreads);
      } else if (mode == ORDA_TEACHER_SEPARATE) {
        oref_matmul_nn(tgr, teacher->weight.data, tmp_h, n, v, ht_dim, nthreads);
        memcpy(grad_h_t + start * ht_dim, tmp_h, sizeof(float) * n * ht_dim);
        oref_matmul_tn(tgr, h_t_chunk, tmp_w, n, v, ht_dim, nthreads);
        add_assign(grad_w_t, tmp_w, v * ht_dim, nthreads);
      }
    }
  }
  free(logits_chunk); free(grad_kl); free(tmp_h); free(tmp_w); free(nll_rows);

  /* deferred mean (src/api.rs:381-388) */
  scale_assign(grad_h_s, bt * h, mean_scale, nthreads);
  scale_assign(grad_w, v * h, mean_scale, nthreads);
  if (gh_t) scale_assign(grad_h_t, bt * ht_dim, mean_scale, nthreads);
  if (gw_t) scale_assign(grad_w_t, v * ht_dim, mean_scale, nthreads);
  if (raw_grad_w) memcpy(raw_grad_w, grad_w, sizeof(float) * v * h);

  /* optional INT8 round trip (src/api.rs:391-399) */
  if (opts->config.quantize_grad_weight) {
    int8_t* q = (int8_t*)malloc(v * h);
    float* sc = (float*)malloc(sizeof(float) * v);
    float* deq = (float*)malloc(sizeof(float) * v * h);
    uint64_t seed = opts->config.has_stochastic_seed ? opts->config.stochastic_seed : 0;
    oref_quantize_grad_w(grad_w, v, h, labels, bt, ignore, opts->config.stochastic_rounding, seed, 1.0f, q, sc,
                         deq, nthreads);
    memcpy(grad_w, deq, sizeof(float) * v * h);
    free(q); free(sc); free(deq);
  }

  double ms = (double)mean_scale;
  scalars[1] = (float)(sum_nll_s * ms);
  scalars[2] = (float)(sum_nll_t * ms);
  scalars[3] = (float)(kl_accum * ms);
  scalars[0] = (float)(((double)w_s * sum_nll_s + (double)w_t * sum_nll_t + (double)kd * kl_accum) * ms);
  if (plan_out) *plan_out = plan;
  return ORDA_OK;
}

/* ------------------------------------------------------------------------ */
/* f64 forward oracle (src/api.rs:424-584)                                   */
/* ------------------------------------------------------------------------ */

/* `logits_row_f64` src/api.rs:427-438. */
static void logits_row_f64(const float* h_row, size_t hd, const float* w, size_t wrows, double* out) {
  for (size_t vr = 0; vr < wrows; ++vr) {
    const float* wr = w + vr * hd;
    double acc = 0.0;
    for (size_t k = 0; k < hd; ++k) acc += (double)h_row[k] * (double)wr[k];
    out[vr] = acc;
  }
}

/* `nll_f64` src/api.rs:441-462. */
static double nll_f64(const double* logits, size_t v, int64_t y, int64_t ignore_index, double ls) {
  if (y == ignore_index) return 0.0;
  double m = -INFINITY;
  for (size_t i = 0; i < v; ++i) m = fmax(m, logits[i]);
  double d = 0.0, sum_x = 0.0;
  for (size_t i = 0; i < v; ++i) {
    d += exp(logits[i] - m);
    if (ls > 0.0) sum_x += logits[i];
  }
  double lse = m + log(d);
  double tgt = logits[(size_t)y];
  return ls > 0.0 ? lse - (1.0 - ls) * tgt - (ls / (double)v) * sum_x : lse - tgt;
}

/* `kl_f64` src/api.rs:465-485. */
static double kl_f64(const double* s, const double* t, size_t v, double temperature) {
  double inv_t = 1.0 / temperature;
  double ms = -INFINITY, mt = -INFINITY;
  for (size_t j = 0; j < v; ++j) { ms = fmax(ms, s[j] * inv_t); mt = fmax(mt, t[j] * inv_t); }
  double ds = 0.0, dt = 0.0;
  for (size_t j = 0; j < v; ++j) ds += exp(s[j] * inv_t - ms);
  for (size_t j = 0; j < v; ++j) dt += exp(t[j] * inv_t - mt);
  double lds = log(ds), ldt = log(dt);
  double kl = 0.0;
  for (size_t j = 0; j < v; ++j) {
    double pt = exp(t[j] * inv_t - mt) / dt;
    double lpt = (t[j] * inv_t - mt) - ldt;
    double lps = (s[j] * inv_t - ms) - lds;
    kl += pt * (lpt - lps);
  }
  return kl;
}

/* `forward_loss_f64` src/api.rs:511-572. kl_teacher_logits (nullable) is the
 * detached teacher distribution [BT, V]. */
EXPORT int oref_forward_loss_f64(const OrdaMatF32* student_hidden, const OrdaMatF32* weight,
                                 const int64_t* labels, size_t n_labels, const OrdaTeacher* teacher,
                                 const OrdaLossOptions* opts, const float* kl_teacher_logits, double* out,
                                 char* err, size_t err_len) {
  size_t v, h, bt;
  int rc = oref_validate(student_hidden, weight, labels, n_labels, teacher, opts, &v, &h, &bt, err, err_len);
  if (rc) return rc;
  if (opts->backend == ORDA_BACKEND_CUDA) {
    set_err(err, err_len, "Backend::Cuda is unavailable in this build (see docs/BLOCKERS.md)");
    return ORDA_ERR_BACKEND;
  }
  double w_s = (double)opts->student_ce_weight;
  double w_t = (double)(opts->has_teacher_ce_weight ? opts->teacher_ce_weight
                                                     : oref_default_teacher_ce_weight(teacher->mode));
  double kd = (double)opts->kd_weight, temperature = (double)opts->temperature;
  double ls = (double)opts->label_smoothing;
  int64_t ignore = opts->ignore_index;
  double t_sq = temperature * temperature;
  size_t n_non_ignore = 0;
  for (size_t i = 0; i < bt; ++i) n_non_ignore += labels[i] != ignore;
  double denom = opts->reduction == ORDA_REDUCTION_MEAN ? (double)max_sz(n_non_ignore, 1) : 1.0;
  double *ls_row = (double*)malloc(sizeof(double) * v), *lt_row = (double*)malloc(sizeof(double) * v),
         *kt_row = (double*)malloc(sizeof(double) * v);
  double sum_nll_s = 0.0, sum_nll_t = 0.0, sum_kl = 0.0;
  for (size_t r = 0; r < bt; ++r) {
    logits_row_f64(student_hidden->data + r * h, h, weight->data, v, ls_row);
    sum_nll_s += nll_f64(ls_row, v, labels[r], ignore, ls);
    int need_teacher = kd > 0.0 || w_t > 0.0;
    if (need_teacher) {
      if (teacher->mode == ORDA_TEACHER_TIED) {
        logits_row_f64(teacher->hidden.data + r * h, h, weight->data, v, lt_row);
      } else if (teacher->mode == ORDA_TEACHER_SEPARATE) {
        size_t ht = teacher->hidden.cols;
        logits_row_f64(teacher->hidden.data + r * ht, ht, teacher->weight.data, v, lt_row);
      } else {
        for (size_t j = 0; j < v; ++j) lt_row[j] = (double)teacher->logits.data[r * v + j];
      }
      if (w_t > 0.0) sum_nll_t += nll_f64(lt_row, v, labels[r], ignore, ls);
      if (kd > 0.0 && labels[r] != ignore) {
        const double* kt = lt_row;
        if (kl_teacher_logits) {
          for (size_t j = 0; j < v; ++j) kt_row[j] = (double)kl_teacher_logits[r * v + j];
          kt = kt_row;
        }
        sum_kl += kl_f64(ls_row, kt, v, temperature) * t_sq;
      }
    }
  }
  free(ls_row); free(lt_row); free(kt_row);
  *out = (w_s * sum_nll_s + w_t * sum_nll_t + kd * sum_kl) / denom;
  return ORDA_OK;
}

/* `teacher_logits` src/api.rs:490-496. out [BT, V]. */
EXPORT void oref_teacher_logits(const OrdaTeacher* teacher, const OrdaMatF32* weight, float* out, int nthreads) {
  if (teacher->mode == ORDA_TEACHER_TIED)
    oref_matmul_nt(teacher->hidden.data, weight->data, out, teacher->hidden.rows, teacher->hidden.cols,
                   weight->rows, nthreads);
  else if (teacher->mode == ORDA_TEACHER_SEPARATE)
    oref_matmul_nt(teacher->hidden.data, teacher->weight.data, out, teacher->hidden.rows, teacher->hidden.cols,
                   teacher->weight.rows, nthreads);
  else
    memcpy(out, teacher->logits.data, sizeof(float) * teacher->logits.rows * teacher->logits.cols);
}

/* ------------------------------------------------------------------------ */
/* test data helpers                                                         */
/* ------------------------------------------------------------------------ */

/* `fill` of tests/end_to_end.rs:14-27 and src/main.rs:11-24 (LCG, f32). */
EXPORT void oref_lcg_fill(float* out, size_t n, uint64_t seed, float scale) {
  uint64_t s = seed * 2862933555777941757ULL + 3037000493ULL;
  for (size_t i = 0; i < n; ++i) {
    s = s * 6364136223846793005ULL + 1442695040888963407ULL;
    float u = ((float)(s >> 33)) / ((float)(1ULL << 31));
    out[i] = (u * 2.0f - 1.0f) * scale;
  }
}

EXPORT int oref_max_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}
