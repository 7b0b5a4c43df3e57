// The router logits, logits (T x E fp32) = x (T x H) . W_r^T (W_r: E x H, the GGUF's blk.L.ffn_gate_inp.weight), in
// fp32 on the CUDA cores: the reference computes them to fp32 quality (moe/gemm.py:47-61, BFP16 hi + lo planes,
// tests/moe/test_prefill.py:88-92 checks 5e-5), and top-k ids are only as stable as the logits. An optional per-expert
// bias (E fp32) is added to every token's logits. A 64 x 64 output tile
// per CTA, K in steps of 32 staged in shared memory (transposed, padded), 4 x 4 outputs per thread.
#include <cuda_bf16.h>

#include "common.cuh"
#include "kernels.cuh"

namespace artlite {

namespace {
constexpr int BM = 64, BN = 64, BK = 32;

__device__ __forceinline__ float ld(const void* p, int dtype, int64_t i) {
  if (dtype == ARTLITE_BF16) return __uint_as_float((uint32_t)reinterpret_cast<const uint16_t*>(p)[i] << 16);
  return reinterpret_cast<const float*>(p)[i];
}
}  // namespace

__global__ void __launch_bounds__(256) router_kernel(const void* x, int x_dtype, const void* w, int w_dtype,
                                                     const float* bias, int64_t T, int H, int E, float* logits) {
  __shared__ float xs[BK][BM + 4];
  __shared__ float ws[BK][BN + 4];
  const int64_t m0 = (int64_t)blockIdx.x * BM;
  const int n0 = blockIdx.y * BN;
  const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
  float acc[4][4] = {};
  for (int k0 = 0; k0 < H; k0 += BK) {
    for (int i = threadIdx.x; i < BM * BK; i += 256) {
      const int r = i / BK, c = i % BK;
      const int64_t m = m0 + r;
      xs[c][r] = (m < T && k0 + c < H) ? ld(x, x_dtype, m * H + k0 + c) : 0.0f;
      const int n = n0 + r;
      ws[c][r] = (n < E && k0 + c < H) ? ld(w, w_dtype, (int64_t)n * H + k0 + c) : 0.0f;
    }
    __syncthreads();
#pragma unroll 8
    for (int c = 0; c < BK; c++) {
      float a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; i++) a[i] = xs[c][ty + 16 * i], b[i] = ws[c][tx + 16 * i];
#pragma unroll
      for (int i = 0; i < 4; i++)
#pragma unroll
        for (int j = 0; j < 4; j++) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; i++) {
    const int64_t m = m0 + ty + 16 * i;
    if (m >= T) continue;
#pragma unroll
    for (int j = 0; j < 4; j++) {
      const int n = n0 + tx + 16 * j;
      if (n < E) logits[m * E + n] = bias ? acc[i][j] + bias[n] : acc[i][j];
    }
  }
}

int launch_router(const void* x, int x_dtype, const void* w, int w_dtype, const float* bias, int64_t T, int H, int E,
                  float* logits, cudaStream_t st) {
  if (T == 0) return ARTLITE_OK;
  dim3 grid((unsigned)cdiv(T, BM), (unsigned)cdiv(E, BN));
  router_kernel<<<grid, 256, 0, st>>>(x, x_dtype, w, w_dtype, bias, T, H, E, logits);
  AL_LAUNCHED();
  return ARTLITE_OK;
}

}  // namespace artlite
