// host_logic.cpp -- pure host logic of the C ABI: option defaults, config
// validation, the chunk resolver and OOM ladder, argument validation with the
// reference's exact error messages. No device code; callable without a GPU.
#include <algorithm>
#include <charconv>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include "../../include/orda.h"
#include "host_logic.h"

namespace orda {

void set_error(char* err, size_t len, const char* fmt, ...) {
  if (!err || len == 0) return;
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(err, len, fmt, ap);
  va_end(ap);
}

// Rust `Display` of an f32: shortest round-trip digits, fixed notation.
std::string fmt_f32(float x) {
  if (std::isnan(x)) return "NaN";
  if (std::isinf(x)) return x > 0 ? "inf" : "-inf";
  char buf[128];
  auto res = std::to_chars(buf, buf + sizeof buf, x, std::chars_format::fixed);
  return std::string(buf, res.ptr);
}

size_t ceil_div(size_t a, size_t b) { return (a + b - 1) / b; }

size_t chunks_from_raw(double raw) {
  if (raw < 1.5) return 1;
  const double e = std::floor(std::log2(raw / 1.5));
  long long ei;
  if (std::isnan(e)) ei = 0;
  else if (e >= 9.2e18) ei = 60;
  else if (e <= -9.2e18) ei = -1;
  else ei = static_cast<long long>(e);
  long long sh = ei + 1;
  sh = std::clamp(sh, 0ll, 60ll);
  return size_t{1} << sh;
}

OrdaChunkPlan resolve_chunk_size(size_t bt, const OrdaChunkSize& cs, bool has_v, size_t v, bool has_mc,
                                 size_t max_chunks) {
  OrdaChunkPlan p{0, 0};
  if (bt == 0) return p;
  if (cs.kind == ORDA_CHUNK_FIXED) {
    const size_t c = std::max<size_t>(std::min(cs.fixed_rows, bt), 1);
    p.chunk_size = c;
    p.num_chunks = ceil_div(bt, c);
    return p;
  }
  if (!has_v) {
    p.chunk_size = bt;
    p.num_chunks = 1;
    return p;
  }
  const size_t max_useful = std::max<size_t>(bt / 512, 1);
  const size_t mc = has_mc ? max_chunks : 2 * max_useful;
  const double vr = static_cast<double>(v) / 32768.0;
  const double raw_pressure = (static_cast<double>(bt) / 1024.0) * (vr * vr);
  const double raw_bt_floor = static_cast<double>(bt) / 4096.0;
  const double raw = std::fmax(raw_pressure, raw_bt_floor);
  size_t nc = chunks_from_raw(raw);
  nc = std::min(nc, mc);
  nc = std::min(nc, max_useful);
  nc = std::min(nc, bt);
  nc = std::max<size_t>(nc, 1);
  p.chunk_size = ceil_div(bt, nc);
  p.num_chunks = nc;
  return p;
}

size_t default_max_chunks_limit(size_t bt) { return 2 * std::max<size_t>(bt / 512, 1); }

std::vector<size_t> chunk_doubling_schedule(size_t bt, size_t start, size_t limit) {
  const size_t lim = std::min(std::max<size_t>(limit, 1), bt);
  size_t n = std::clamp<size_t>(start, 1, std::max<size_t>(lim, 1));
  std::vector<size_t> out{n};
  while (n < bt && n < lim) {
    n = std::min(std::min(n * 2, bt), lim);
    out.push_back(n);
    if (n >= bt || n >= lim) break;
  }
  return out;
}

int kernel_config_validate(const OrdaKernelConfig& c, char* err, size_t len) {
  if (c.max_fused_size < 1 || !((c.max_fused_size & (c.max_fused_size - 1)) == 0)) {
    set_error(err, len, "max_fused_size must be a power of two >= 1, got %zu", c.max_fused_size);
    return ORDA_ERR_INVALID;
  }
  if (c.has_max_chunks && c.max_chunks < 1) {
    set_error(err, len, "max_chunks must be >= 1, got %zu", c.max_chunks);
    return ORDA_ERR_INVALID;
  }
  return ORDA_OK;
}

int validate_shapes(const Shape2& sh, const Shape2& w, size_t n_labels, OrdaTeacherMode mode, const Shape2& t_hidden,
                    const Shape2& t_weight, const Shape2& t_logits, const OrdaLossOptions& o, size_t* v_out,
                    size_t* h_out, size_t* bt_out, char* err, size_t len) {
  if (int rc = kernel_config_validate(o.config, err, len)) return rc;
  const size_t bt = sh.rows, h = sh.cols;
  if (bt == 0) {
    set_error(err, len, "student_hidden has 0 rows (BT must be > 0)");
    return ORDA_ERR_INVALID;
  }
  if (w.cols != h) {
    set_error(err, len, "weight must have shape (V, %zu), got (%zu, %zu)", h, w.rows, w.cols);
    return ORDA_ERR_INVALID;
  }
  const size_t v = w.rows;
  if (n_labels != bt) {
    set_error(err, len, "labels must have length BT=%zu, got %zu", bt, n_labels);
    return ORDA_ERR_INVALID;
  }
  if (v_out) *v_out = v;
  if (h_out) *h_out = h;
  if (bt_out) *bt_out = bt;
  (void)mode;
  (void)t_hidden;
  (void)t_weight;
  (void)t_logits;
  return ORDA_OK;
}

int validate_scalars_and_teacher(size_t bt, size_t h, size_t v, OrdaTeacherMode mode, const Shape2& t_hidden,
                                 const Shape2& t_weight, const Shape2& t_logits, const OrdaLossOptions& o,
                                 char* err, size_t len) {
  if (!(o.label_smoothing >= 0.0f && o.label_smoothing <= 1.0f)) {
    set_error(err, len, "label_smoothing must be in [0,1], got %s", fmt_f32(o.label_smoothing).c_str());
    return ORDA_ERR_INVALID;
  }
  if (o.kd_weight < 0.0f) {
    set_error(err, len, "kd_weight must be >= 0, got %s", fmt_f32(o.kd_weight).c_str());
    return ORDA_ERR_INVALID;
  }
  if (o.temperature <= 0.0f) {
    set_error(err, len, "temperature must be > 0, got %s", fmt_f32(o.temperature).c_str());
    return ORDA_ERR_INVALID;
  }
  switch (mode) {
    case ORDA_TEACHER_TIED:
      if (t_hidden.rows != bt || t_hidden.cols != h) {
        set_error(err, len, "Tied teacher hidden must be (%zu, %zu), got (%zu, %zu)", bt, h, t_hidden.rows,
                  t_hidden.cols);
        return ORDA_ERR_INVALID;
      }
      break;
    case ORDA_TEACHER_SEPARATE: {
      if (t_hidden.rows != bt) {
        set_error(err, len, "Separate teacher hidden must have BT=%zu rows", bt);
        return ORDA_ERR_INVALID;
      }
      const size_t ht = t_hidden.cols;
      if (t_weight.rows != v || t_weight.cols != ht) {
        set_error(err, len, "Separate teacher weight must be (%zu, %zu), got (%zu, %zu)", v, ht, t_weight.rows,
                  t_weight.cols);
        return ORDA_ERR_INVALID;
      }
      break;
    }
    case ORDA_TEACHER_PRECOMPUTED:
      if (t_logits.rows != bt || t_logits.cols != v) {
        set_error(err, len, "Precomputed teacher logits must be (%zu, %zu), got (%zu, %zu)", bt, v, t_logits.rows,
                  t_logits.cols);
        return ORDA_ERR_INVALID;
      }
      break;
    default:
      set_error(err, len, "unknown teacher mode %d", static_cast<int>(mode));
      return ORDA_ERR_INVALID;
  }
  return ORDA_OK;
}

int validate_labels(const int64_t* labels, size_t n, size_t v, int64_t ignore, char* err, size_t len) {
  for (size_t i = 0; i < n; ++i) {
    const int64_t t = labels[i];
    if (t != ignore && (t < 0 || static_cast<uint64_t>(t) >= v)) {
      set_error(err, len, "label %lld out of range [0, %zu) and != ignore_index %lld", static_cast<long long>(t), v,
                static_cast<long long>(ignore));
      return ORDA_ERR_INVALID;
    }
  }
  return ORDA_OK;
}

}  // namespace orda

using namespace orda;

extern "C" {

void orda_kernel_config_from_profile(OrdaProfile profile, OrdaKernelConfig* out) {
  std::memset(out, 0, sizeof *out);
  out->fast_math = profile == ORDA_PROFILE_FAST ? 1 : 0;
  out->max_fused_size = 65536 / 2;  // DEFAULT_MAX_FUSED_SIZE (src/config.rs:66)
}

void orda_loss_options_default(OrdaLossOptions* o) {
  std::memset(o, 0, sizeof *o);
  o->student_ce_weight = 1.0f;
  o->has_teacher_ce_weight = 0;
  o->teacher_ce_weight = 0.0f;
  o->kd_weight = 0.0f;
  o->temperature = 1.0f;
  o->ignore_index = -100;
  o->label_smoothing = 0.0f;
  o->reduction = ORDA_REDUCTION_MEAN;
  o->chunk_size.kind = ORDA_CHUNK_AUTO;
  o->chunk_size.fixed_rows = 0;
  orda_kernel_config_from_profile(ORDA_PROFILE_BALANCED, &o->config);
  o->backend = ORDA_BACKEND_AUTO;
}

int orda_kernel_config_validate(const OrdaKernelConfig* cfg, char* err, size_t err_len) {
  return kernel_config_validate(*cfg, err, err_len);
}

int orda_is_power_of_two(size_t value) { return value > 0 && (value & (value - 1)) == 0; }

float orda_default_teacher_ce_weight(OrdaTeacherMode mode) { return mode == ORDA_TEACHER_TIED ? 1.0f : 0.0f; }

size_t orda_chunks_from_raw(double raw) { return chunks_from_raw(raw); }

void orda_resolve_chunk_size(size_t bt, OrdaChunkSize chunk_size, int has_v, size_t v, int has_max_chunks,
                             size_t max_chunks, OrdaChunkPlan* out) {
  *out = resolve_chunk_size(bt, chunk_size, has_v != 0, v, has_max_chunks != 0, max_chunks);
}

size_t orda_default_max_chunks_limit(size_t bt) { return default_max_chunks_limit(bt); }

size_t orda_chunk_doubling_schedule(size_t bt, size_t start, size_t limit, size_t* out, size_t out_cap) {
  if (bt == 0) return 0;
  const std::vector<size_t> s = chunk_doubling_schedule(bt, start, limit);
  for (size_t i = 0; i < s.size() && i < out_cap; ++i) out[i] = s[i];
  return s.size();
}

int orda_chunk_retry(size_t bt, size_t start, size_t limit, OrdaTryAllocFn try_alloc, void* user, OrdaChunkPlan* out) {
  if (bt == 0 || !try_alloc) return ORDA_ERR_INVALID;
  for (size_t nc : chunk_doubling_schedule(bt, start, limit)) {
    const size_t cs = ceil_div(bt, nc);
    if (try_alloc(nc, cs, user) == 0) {
      if (out) {
        out->chunk_size = cs;
        out->num_chunks = nc;
      }
      return ORDA_OK;
    }
  }
  return ORDA_ERR_OOM;
}

int orda_validate(const OrdaMatF32* student_hidden, const OrdaMatF32* weight, const int64_t* labels, size_t n_labels,
                  const OrdaTeacher* teacher, const OrdaLossOptions* opts, size_t* v_out, size_t* h_out,
                  size_t* bt_out, char* err, size_t err_len) {
  const Shape2 sh{student_hidden->rows, student_hidden->cols}, w{weight->rows, weight->cols};
  const Shape2 th{teacher->hidden.rows, teacher->hidden.cols}, tw{teacher->weight.rows, teacher->weight.cols},
      tl{teacher->logits.rows, teacher->logits.cols};
  size_t v = 0, h = 0, bt = 0;
  if (int rc = validate_shapes(sh, w, n_labels, teacher->mode, th, tw, tl, *opts, &v, &h, &bt, err, err_len))
    return rc;
  if (int rc = validate_labels(labels, n_labels, v, opts->ignore_index, err, err_len)) return rc;
  if (int rc = validate_scalars_and_teacher(bt, h, v, teacher->mode, th, tw, tl, *opts, err, err_len)) return rc;
  if (v_out) *v_out = v;
  if (h_out) *h_out = h;
  if (bt_out) *bt_out = bt;
  return ORDA_OK;
}

}  // extern "C"
