// Shared host/device helpers of libartlite_moe_cuda.so: status handling, device buffers, pointer classification.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdarg>
#include <cstdio>
#include <string>

#include "../../include/artlite_moe.h"

namespace artlite {

// The thread's last error message (artlite_moe_last_error).
void set_error(const char* fmt, ...);
std::string& last_error();

struct Status {
  int code = ARTLITE_OK;
  bool ok() const { return code == ARTLITE_OK; }
};

#define AL_CUDA(call)                                                                              \
  do {                                                                                             \
    cudaError_t e_ = (call);                                                                       \
    if (e_ != cudaSuccess) {                                                                       \
      ::artlite::set_error("%s:%d %s: %s", __FILE__, __LINE__, #call, cudaGetErrorString(e_));     \
      return ARTLITE_ECUDA;                                                                        \
    }                                                                                              \
  } while (0)

#define AL_CHECK(cond, code, ...)        \
  do {                                   \
    if (!(cond)) {                       \
      ::artlite::set_error(__VA_ARGS__); \
      return (code);                     \
    }                                    \
  } while (0)

// after a kernel launch: its launch error, and the launch counted
#define AL_LAUNCHED()                  \
  do {                                 \
    AL_CUDA(cudaGetLastError());       \
    ::artlite::count_launch();         \
  } while (0)

#define AL_TRY(expr)               \
  do {                             \
    int rc_ = (expr);              \
    if (rc_ != ARTLITE_OK) return rc_; \
  } while (0)

// Whether p is device-accessible memory of the current device (device or managed); false for host memory.
bool is_device_ptr(const void* p);

// A growable device buffer (cudaMalloc'd on the device current at its first use).
struct DevBuf {
  void* ptr = nullptr;
  size_t bytes = 0;
  int reserve(size_t n);  // at least n bytes (contents lost on growth)
  void release();
  template <class T>
  T* as() const { return static_cast<T*>(ptr); }
  ~DevBuf() { release(); }
};

// Device-side status word written by kernels that find a bad input (never __trap): code, and up to 3 details.
struct DevStatus {
  int32_t code;   // 0 ok, else ARTLITE_E* (negative)
  int32_t a, b, c;
};

__device__ __forceinline__ void report(DevStatus* st, int32_t code, int32_t a, int32_t b = 0, int32_t c = 0) {
  if (atomicCAS(&st->code, 0, code) == 0) {
    st->a = a;
    st->b = b;
    st->c = c;
  }
}

constexpr int kNumSMs = 148;  // B200

// kernels launched by this library (counted at each launch site)
int64_t launch_count();
void count_launch(int n = 1);

inline int64_t cdiv(int64_t a, int64_t b) { return (a + b - 1) / b; }
__host__ __device__ __forceinline__ int64_t min64(int64_t a, int64_t b) { return a < b ? a : b; }

}  // namespace artlite
