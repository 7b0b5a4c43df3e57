// The router logits, logits (T x E fp32) = x (T x H) . W_r^T (W_r: E x H, the GGUF's blk.L.ffn_gate_inp.weight), in
// fp32 on the CUDA cores: the reference computes them to fp32 quality (moe/gemm.py:47-61, BFP16 hi + lo planes,
// tests/moe/test_prefill.py:88-92 checks 5e-5), and top-k ids are only as stable as the logits. An optional per-expert
// bias (E fp32) is added to every token's logits. A 64 x 64 output tile
// per CTA, K in steps of 32 staged in shared memory (transposed, padded), 4 x 4 outputs per thread.
#include <cuda_bf16.h>

#include <algorithm>

#include "common.cuh"
#include "kernels.cuh"
#include "norm.cuh"

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


// ---------------------------------------------------------------- decode-sized batches
//
// A warp per (token, expert) logit over the whole grid: each lane reads 4 consecutive columns of the W row and of the
// token row per 128-column stripe with 16-byte loads (all of a 1024-column chunk's loads in flight at once), fp32 FMAs,
// a warp reduction in fixed order, + bias. Where the tiled kernels give one CTA to a small batch, this spreads the
// E x H weight read over every SM.
namespace {
__device__ __forceinline__ void load4(const void* p, int dtype, int64_t i, float (&v)[4]) {
  if (dtype == ARTLITE_BF16) {
    const uint2 u = *reinterpret_cast<const uint2*>(reinterpret_cast<const uint16_t*>(p) + i);
    v[0] = __uint_as_float(u.x << 16), v[1] = __uint_as_float(u.x & 0xFFFF0000u);
    v[2] = __uint_as_float(u.y << 16), v[3] = __uint_as_float(u.y & 0xFFFF0000u);
  } else {
    const float4 f = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(p) + i);
    v[0] = f.x, v[1] = f.y, v[2] = f.z, v[3] = f.w;
  }
}
}  // namespace

__global__ void __launch_bounds__(256) router_small_kernel(const void* x, int x_dtype, const void* w, int w_dtype,
                                                           const float* bias, int64_t T, int H, int E, float* logits) {
  griddep_wait();
  griddep_launch();
  const int lane = threadIdx.x & 31;
  const int64_t units = T * E;
  for (int64_t u = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; u < units;
       u += ((int64_t)gridDim.x * blockDim.x) >> 5) {
    const int64_t t = u / E;
    const int e = (int)(u - t * E);
    float acc = 0.0f;
    for (int c0 = 0; c0 < H; c0 += 1024) {
      float wv[8][4], xv[8][4];
#pragma unroll
      for (int i = 0; i < 8; i++) {
        const int c = c0 + 4 * lane + 128 * i;
        if (c < H) {
          load4(w, w_dtype, (int64_t)e * H + c, wv[i]);
          load4(x, x_dtype, t * H + c, xv[i]);
        } else {
#pragma unroll
          for (int j = 0; j < 4; j++) wv[i][j] = xv[i][j] = 0.0f;
        }
      }
#pragma unroll
      for (int i = 0; i < 8; i++)
#pragma unroll
        for (int j = 0; j < 4; j++) acc = fmaf(wv[i][j], xv[i][j], acc);
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) acc += __shfl_xor_sync(0xFFFFFFFFu, acc, o);
    if (lane == 0) logits[t * E + e] = bias ? acc + bias[e] : acc;
  }
}

// 8 consecutive values (p + i is 8-aligned): two 16-byte loads of fp32 or one of bf16
__device__ __forceinline__ void load8(const void* p, int dtype, int64_t i, float (&v)[8]) {
  if (dtype == ARTLITE_BF16) {
    const uint4 u = __ldg(reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(p) + i));
    const uint32_t q[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int j = 0; j < 4; j++) v[2 * j] = __uint_as_float(q[j] << 16), v[2 * j + 1] = __uint_as_float(q[j] & 0xFFFF0000u);
  } else {
    const float4 a = __ldg(reinterpret_cast<const float4*>(reinterpret_cast<const float*>(p) + i));
    const float4 b = __ldg(reinterpret_cast<const float4*>(reinterpret_cast<const float*>(p) + i) + 1);
    v[0] = a.x, v[1] = a.y, v[2] = a.z, v[3] = a.w, v[4] = b.x, v[5] = b.y, v[6] = b.z, v[7] = b.w;
  }
}

// The same for H % 256 == 0 and T <= 16: a CTA per expert, its 8 warps splitting H (each lane 8 consecutive values of every
// 256-wide slice its warp owns), tokens in chunks of 8. The router row is read once per CTA and every expert's CTA
// runs at once, so a one-token batch's 1 MB of router weights is read by E SMs in one round of loads; the warps'
// partial sums meet in shared memory and add in a fixed order, + bias.
__device__ __forceinline__ void router_cta_expert(const void* x, int x_dtype, const void* w, int w_dtype,
                                                  const float* bias, int64_t T, int H, int E, float* logits, int e,
                                                  float (*part)[8]) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int64_t t0 = 0; t0 < T; t0 += 8) {
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int c = warp * 256 + lane * 8; c < H; c += 8 * 256) {
      float wv[8];
      load8(w, w_dtype, (int64_t)e * H + c, wv);
#pragma unroll
      for (int i = 0; i < 8; i++) {
        if (t0 + i < T) {
          float xv[8];
          nrm::ld8p(x, x_dtype, (t0 + i) * H + c, xv);  // (global rows, or the CTA's normed rows in shared memory)
#pragma unroll
          for (int j = 0; j < 8; j++) acc[i] = fmaf(wv[j], xv[j], acc[i]);
        }
      }
    }
#pragma unroll
    for (int i = 0; i < 8; i++)
#pragma unroll
      for (int o = 16; o; o >>= 1) acc[i] += __shfl_xor_sync(0xFFFFFFFFu, acc[i], o);
    if (lane == 0)
#pragma unroll
      for (int i = 0; i < 8; i++) part[warp][i] = acc[i];
    __syncthreads();
    if (threadIdx.x < 8 && t0 + threadIdx.x < T) {
      const int i = threadIdx.x;
      const float v = ((part[0][i] + part[1][i]) + (part[2][i] + part[3][i])) +
                      ((part[4][i] + part[5][i]) + (part[6][i] + part[7][i]));
      logits[(t0 + i) * E + e] = bias ? v + bias[e] : v;
    }
    __syncthreads();
  }
}

// With the layer's input norm (norm.x_in set): every CTA norms the batch's raw rows into its own shared memory
// (norm.cuh norm_rows_cta: the T rows are a few KB each, so the copy per CTA is cheaper than any wait for another
// CTA) and reads them from there; CTA b < T also stores normed row b to x for the kernels that follow
__global__ void __launch_bounds__(256) router_cta_kernel(const void* x, int x_dtype, const void* w, int w_dtype,
                                                         const float* bias, int64_t T, int H, int E, float* logits,
                                                         NormFuse norm) {
  extern __shared__ __align__(16) uint8_t xsm[];
  __shared__ float part[8][8];
  griddep_wait();
  griddep_launch();
  const void* xr = x;
  if (norm.x_in) {
    const int64_t rb = (int64_t)H * (w_dtype == ARTLITE_F32 ? 4 : 2);  // (H % 256 == 0: a multiple of 16 bytes)
    if (threadIdx.x == 0 && blockIdx.x < E)  // the expert's router row into L2 while the rows are normed
      asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(static_cast<const uint8_t*>(w) + blockIdx.x * rb),
                   "r"((uint32_t)rb) : "memory");
    nrm::norm_rows_cta(norm.x_in, x_dtype, norm.w, norm.w_dtype, norm.eps, H, (int)T, xsm,
                       blockIdx.x < T ? (int)blockIdx.x : -1, const_cast<void*>(x));
    xr = xsm;
  }
  for (int e = blockIdx.x; e < E; e += gridDim.x) router_cta_expert(xr, x_dtype, w, w_dtype, bias, T, H, E, logits, e, part);
}

bool router_small_ok(int64_t T, int H) { return T <= kRouterSmallTokens && H % 4 == 0; }
constexpr int kNormSmem = 128 * 1024;
bool router_small_norms(int64_t T, int H, int x_dtype) {
  return T <= nrm::kRowsCta && H % 256 == 0 && T * H * (x_dtype == ARTLITE_BF16 ? 2 : 4) <= kNormSmem;
}

int launch_router_small(const void* x, int x_dtype, const void* w, int w_dtype, const float* bias, int64_t T, int H,
                        int E, float* logits, cudaStream_t st, const NormFuse* norm) {
  AL_CHECK(router_small_ok(T, H), ARTLITE_EINVAL, "router_small: T %lld H %d", (long long)T, H);
  AL_CHECK(!norm || router_small_norms(T, H, x_dtype), ARTLITE_EINVAL, "router_small: no fused norm at T %lld H %d",
           (long long)T, H);
  if (T == 0) return ARTLITE_OK;
  if (H % 256 == 0 && T <= 16) {
    const size_t smem = norm ? (size_t)T * H * (x_dtype == ARTLITE_BF16 ? 2 : 4) : 0;
    if (smem > 48 * 1024)
      AL_CUDA(cudaFuncSetAttribute(router_cta_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kNormSmem));
    return launch_pdl(router_cta_kernel, dim3((unsigned)E), dim3(256), smem, st, x, x_dtype, w, w_dtype, bias, T, H, E,
                      logits, norm ? *norm : NormFuse{});
  }
  const int64_t warps = T * E;
  const unsigned grid = (unsigned)std::min<int64_t>(cdiv(warps, 8), (int64_t)kNumSMs * 8);
  return launch_pdl(router_small_kernel, dim3(grid), dim3(256), 0, st, x, x_dtype, w, w_dtype, bias, T, H, E, logits);
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
