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

// Programmatic dependent launch: a kernel launched by launch_pdl may begin while the kernel before it on the stream is
// still running, and must call griddep_wait() before it reads anything an earlier kernel wrote (the wait returns once
// the earlier grids have completed and their memory is visible; without a programmatic predecessor it returns at
// once). griddep_launch() lets the next such kernel begin launching.
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

bool pdl_enabled();  // ARTLITE_PDL=0 turns programmatic launches into ordinary ones

template <class... KArgs, class... Args>
int launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, Args... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  AL_CUDA(cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...));
  count_launch();
  return ARTLITE_OK;
}
__host__ __device__ __forceinline__ int64_t min64(int64_t a, int64_t b) { return a < b ? a : b; }

// exclusive scan of one value per thread over a block of up to 1024 threads; returns the block total in *total
template <class T>
__device__ T block_exclusive_scan(T v, T* smem, T* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
  T incl = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const T n = __shfl_up_sync(0xFFFFFFFFu, incl, o);
    if (lane >= o) incl += n;
  }
  if (lane == 31) smem[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    T s = lane < nw ? smem[lane] : T(0);
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const T n = __shfl_up_sync(0xFFFFFFFFu, s, o);
      if (lane >= o) s += n;
    }
    if (lane < nw) smem[lane] = s;  // inclusive per warp
  }
  __syncthreads();
  const T base = warp ? smem[warp - 1] : T(0);
  *total = smem[nw - 1];
  __syncthreads();
  return base + incl - v;
}

}  // namespace artlite
