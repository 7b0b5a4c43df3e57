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


// ---------------------------------------------------------------- decode-sized batches
//
// Two experts per CTA, each expert's row split over four warps in 128-column stripes (each lane: 4 consecutive columns
// per stripe, 16-byte loads of W and x straight from global memory), 16 tokens per CTA; per warp a reduce-scatter of
// the 16 token sums across its lanes, then the four stripes' partial sums meet in shared memory. Grid (E / 2, T / 16):
// every W row is read once per 16 tokens by many CTAs at once, where the tiled kernels give one CTA to a small batch.
constexpr int kRsTok = 16;

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
  __shared__ float red[8][kRsTok];
  griddep_wait();
  griddep_launch();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int e = blockIdx.x * 2 + (warp >> 2), part = warp & 3;
  const int64_t t0 = (int64_t)blockIdx.y * kRsTok;
  const int nt = (int)min64(kRsTok, T - t0);
  float acc[kRsTok];
#pragma unroll
  for (int n = 0; n < kRsTok; n++) acc[n] = 0.0f;
  if (e < E) {
#pragma unroll 4
    for (int c = part * 128 + lane * 4; c < H; c += 512) {
      float wv[4];
      load4(w, w_dtype, (int64_t)e * H + c, wv);
#pragma unroll
      for (int n = 0; n < kRsTok; n++) {
        if (n < nt) {
          float xv[4];
          load4(x, x_dtype, (t0 + n) * H + c, xv);
          acc[n] = fmaf(wv[0], xv[0], acc[n]);
          acc[n] = fmaf(wv[1], xv[1], acc[n]);
          acc[n] = fmaf(wv[2], xv[2], acc[n]);
          acc[n] = fmaf(wv[3], xv[3], acc[n]);
        }
      }
    }
  }
  // reduce-scatter over the lanes: afterwards lanes 2j and 2j + 1 hold token j's sum
#pragma unroll
  for (int h = 8, o = 16; h >= 1; h >>= 1, o >>= 1) {
    const bool up = lane & o;
#pragma unroll
    for (int j = 0; j < h; j++) {
      const float send = up ? acc[j] : acc[j + h];
      const float keep = up ? acc[j + h] : acc[j];
      acc[j] = keep + __shfl_xor_sync(0xFFFFFFFFu, send, o);
    }
  }
  acc[0] += __shfl_xor_sync(0xFFFFFFFFu, acc[0], 1);
  if (!(lane & 1)) red[warp][lane >> 1] = acc[0];
  __syncthreads();
  if (threadIdx.x < 2 * kRsTok) {
    const int ex = blockIdx.x * 2 + (threadIdx.x >> 4), n = threadIdx.x & 15;
    const int wb = (threadIdx.x >> 4) * 4;
    if (ex < E && n < nt) {
      float v = (red[wb][n] + red[wb + 1][n]) + (red[wb + 2][n] + red[wb + 3][n]);
      if (bias) v += bias[ex];
      logits[(t0 + n) * E + ex] = v;
    }
  }
}

bool router_small_ok(int64_t T, int H) { return T <= kRouterSmallTokens && H % 4 == 0; }

int launch_router_small(const void* x, int x_dtype, const void* w, int w_dtype, const float* bias, int64_t T, int H,
                        int E, float* logits, cudaStream_t st) {
  AL_CHECK(router_small_ok(T, H), ARTLITE_EINVAL, "router_small: T %lld H %d", (long long)T, H);
  if (T == 0) return ARTLITE_OK;
  return launch_pdl(router_small_kernel, dim3((unsigned)cdiv(E, 2), (unsigned)cdiv(T, kRsTok)), dim3(256), 0, st, x,
                    x_dtype, w, w_dtype, bias, T, H, E, logits);
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
