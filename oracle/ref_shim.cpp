// TEST INFRASTRUCTURE ONLY: extern "C" wrappers around the reference's own host code, compiled from the reference
// tree by oracle/Makefile into oracle/_ref/libartlite_ref.so (never committed, never linked by the product).
// They let the tests check the C restatement (oracle/oracle.c) and the CUDA path against the reference's compiled
// moe_route / moe_plan (csrc/artlite/moe_host.h:13-22) and dequant_rows (csrc/artlite/dequant.h:16).
// artlite::Error becomes a negative status; its message is kept for artlite_ref_last_error().
#include <cstdint>
#include <cstring>
#include <string>

#include "artlite/dequant.h"
#include "artlite/error.h"
#include "artlite/moe_host.h"

namespace {
thread_local std::string g_err;

template <class F>
int guarded(F&& f) {
  try {
    f();
    return 0;
  } catch (const artlite::Error& e) {
    g_err = e.what();
    return -1;
  } catch (const std::exception& e) {
    g_err = e.what();
    return -2;
  }
}
}  // namespace

extern "C" {

const char* artlite_ref_last_error(void) { return g_err.c_str(); }

int artlite_ref_moe_route(const float* logits, int64_t n, int64_t row, int per_col, int64_t pitch, int E, int k,
                          int sigmoid, int32_t* ids, float* weights) {
  return guarded([&] { artlite::moe_route(logits, n, row, per_col, pitch, E, k, sigmoid != 0, ids, weights); });
}

int artlite_ref_moe_plan(const int32_t* ids, int64_t n, int k, int E, int cols, int cap, int chunk, int32_t* experts,
                         int32_t* counts, int32_t* sizes, int32_t* rows, int64_t* pos) {
  return guarded([&] { artlite::moe_plan(ids, n, k, E, cols, cap, chunk, experts, counts, sizes, rows, pos); });
}

int artlite_ref_dequant_rows(const char* qtype, const uint8_t* raw, int64_t n, int64_t row_bytes, int64_t cols,
                             float* out) {
  return guarded([&] { artlite::dequant_rows(qtype, raw, size_t(n), size_t(row_bytes), size_t(cols), out); });
}

}  // extern "C"
