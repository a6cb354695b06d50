// host_logic.h -- shared host helpers of the C ABI implementation.
#pragma once

#include <cstddef>
#include <cstdint>
#include <string>
#include <vector>

#include "../../include/orda.h"

namespace orda {

struct Shape2 {
  size_t rows = 0, cols = 0;
};

void set_error(char* err, size_t len, const char* fmt, ...) __attribute__((format(printf, 3, 4)));
std::string fmt_f32(float x);
size_t ceil_div(size_t a, size_t b);
size_t chunks_from_raw(double raw);
OrdaChunkPlan resolve_chunk_size(size_t bt, const OrdaChunkSize& cs, bool has_v, size_t v, bool has_mc,
                                 size_t max_chunks);
size_t default_max_chunks_limit(size_t bt);
std::vector<size_t> chunk_doubling_schedule(size_t bt, size_t start, size_t limit);
int kernel_config_validate(const OrdaKernelConfig& c, char* err, size_t len);

// `validate` (src/api.rs:104-181) split in the reference's order: config,
// BT, weight shape, label count | label range | smoothing, kd, T, teacher.
int validate_shapes(const Shape2& sh, const Shape2& w, size_t n_labels, OrdaTeacherMode mode, const Shape2& t_hidden,
                    const Shape2& t_weight, const Shape2& t_logits, const OrdaLossOptions& o, size_t* v_out,
                    size_t* h_out, size_t* bt_out, char* err, size_t len);
int validate_labels(const int64_t* labels, size_t n, size_t v, int64_t ignore, char* err, size_t len);
int validate_scalars_and_teacher(size_t bt, size_t h, size_t v, OrdaTeacherMode mode, const Shape2& t_hidden,
                                 const Shape2& t_weight, const Shape2& t_logits, const OrdaLossOptions& o, char* err,
                                 size_t len);

}  // namespace orda
