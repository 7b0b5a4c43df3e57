// The weighted combine (CombineOperator, src/artlite/moe/gather.py:11-17,295-384): per token t,
// out_t = sum_i w[t, i] y[slot[t k + i]] with an fp32 accumulator in slot order i = 0 .. k - 1 (deterministic), one
// rounding to the output type; and the dispatch-order gather of the token rows for the grouped GEMM.
#include <cuda_bf16.h>

#include <algorithm>

#include "common.cuh"
#include "kernels.cuh"
#include "norm.cuh"

namespace artlite {

namespace {

__device__ __forceinline__ void load8(const void* base, int dtype, int64_t i, float* v) {
  if (dtype == ARTLITE_BF16) {
    const uint4 u = *reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(base) + i);
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int j = 0; j < 4; j++) {
      v[2 * j] = __uint_as_float(w[j] << 16);
      v[2 * j + 1] = __uint_as_float(w[j] & 0xFFFF0000u);
    }
  } else {
    const float4* p = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(base) + i);
    const float4 a = p[0], b = p[1];
    v[0] = a.x, v[1] = a.y, v[2] = a.z, v[3] = a.w, v[4] = b.x, v[5] = b.y, v[6] = b.z, v[7] = b.w;
  }
}

__device__ __forceinline__ void store8(void* base, int dtype, int64_t i, const float* v) {
  if (dtype == ARTLITE_BF16) {
    uint32_t w[4];
#pragma unroll
    for (int j = 0; j < 4; j++) {
      const __nv_bfloat162 h = __floats2bfloat162_rn(v[2 * j], v[2 * j + 1]);
      w[j] = *reinterpret_cast<const uint32_t*>(&h);
    }
    *reinterpret_cast<uint4*>(reinterpret_cast<uint16_t*>(base) + i) = make_uint4(w[0], w[1], w[2], w[3]);
  } else {
    float4* p = reinterpret_cast<float4*>(reinterpret_cast<float*>(base) + i);
    p[0] = make_float4(v[0], v[1], v[2], v[3]);
    p[1] = make_float4(v[4], v[5], v[6], v[7]);
  }
}

}  // namespace

// one CTA per token row, 8 values per thread (H % 8 == 0)
// kGrouped: four pairs' loads in flight at once (decode-sized batches, where latency dominates; it takes more
// registers, which costs a large batch its occupancy: the per-pair loop there)
// the residual's row t, columns c .. c + 7, added last to the fp32 sum (res null: nothing)
__device__ __forceinline__ void add_res(const void* res, int dtype, int64_t i, float (&acc)[8]) {
  if (!res) return;
  float v[8];
  load8(res, dtype, i, v);
#pragma unroll
  for (int j = 0; j < 8; j++) acc[j] = __fadd_rn(acc[j], v[j]);
}

template <bool kGrouped>
__global__ void __launch_bounds__(256) combine_kernel(const void* y, int y_dtype, const int32_t* slot, const float* w,
                                                      int64_t T, int k, int H, void* out, int out_dtype, CombineOwn own,
                                                      CombineShared sh, const void* res) {
  griddep_wait();
  griddep_launch();
  const int64_t t = blockIdx.x;
  for (int c = threadIdx.x * 8; c < H; c += blockDim.x * 8) {
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    if (!kGrouped) {
      for (int i = 0; i < k; i++) {
        const float wi = w[t * k + i];
        const int64_t sl = slot[t * k + i];
        float v[8];
        if (own.own && sl >= own.own_lo && sl < own.own_hi)
          load8(own.own, y_dtype, (sl - own.own_lo) * H + c, v);
        else
          load8(y, y_dtype, sl * H + c, v);
#pragma unroll
        for (int j = 0; j < 8; j++) acc[j] = fmaf(wi, v[j], acc[j]);
      }
    }
    for (int i0 = 0; kGrouped && i0 < k; i0 += 4) {  // (four pairs' loads in flight at once; the sum keeps the pair order)
      float wi[4], v[4][8];
      int64_t sl[4];
#pragma unroll
      for (int u = 0; u < 4; u++)
        if (i0 + u < k) wi[u] = w[t * k + i0 + u], sl[u] = slot[t * k + i0 + u];
#pragma unroll
      for (int u = 0; u < 4; u++) {
        if (i0 + u < k) {
          if (own.own && sl[u] >= own.own_lo && sl[u] < own.own_hi)
            load8(own.own, y_dtype, (sl[u] - own.own_lo) * H + c, v[u]);
          else
            load8(y, y_dtype, sl[u] * H + c, v[u]);
        }
      }
#pragma unroll
      for (int u = 0; u < 4; u++)
        if (i0 + u < k)
#pragma unroll
          for (int j = 0; j < 8; j++) acc[j] = fmaf(wi[u], v[u][j], acc[j]);
    }
    if (sh.y) {  // the shared expert's gated term, last in the sum
      const float si = sh.s[t];
      float v[8];
      load8(sh.y, sh.y_dtype, t * H + c, v);
#pragma unroll
      for (int j = 0; j < 8; j++) acc[j] = fmaf(si, v[j], acc[j]);
    }
    add_res(res, out_dtype, t * H + c, acc);
    store8(out, out_dtype, t * H + c, acc);
  }
}

int launch_combine(const void* y, int y_dtype, const int32_t* slot, const float* w, int64_t T, int k, int H, void* out,
                   int out_dtype, cudaStream_t st, CombineOwn own, CombineShared sh, const void* res) {
  AL_CHECK(H % 8 == 0, ARTLITE_EUNSUPPORTED, "combine: H %d (a multiple of 8)", H);
  if (T == 0) return ARTLITE_OK;
  if (T <= 64)
    return launch_pdl(combine_kernel<true>, dim3((unsigned)T), dim3(256), 0, st, y, y_dtype, slot, w, T, k, H, out,
                      out_dtype, own, sh, res);
  return launch_pdl(combine_kernel<false>, dim3((unsigned)T), dim3(256), 0, st, y, y_dtype, slot, w, T, k, H, out,
                    out_dtype, own, sh, res);
}

// the layer's input norm as its own pass (norm.cuh): four rows a CTA (their loads, sums and reductions interleaved),
// one instance per (x, w) dtype pair (a fixed pair takes fewer registers: 4 CTAs an SM instead of 3)
template <int XD, int WD>
__global__ void __launch_bounds__(256) norm_kernel(const void* x, const void* w, double eps, int64_t T, int H,
                                                   void* out) {
  griddep_wait();
  griddep_launch();
  const int64_t r0 = (int64_t)blockIdx.x * 4;
  nrm::norm_rows<4>(x, XD, w, WD, eps, H, r0, (int)min64(4, T - r0), out);
}

int launch_norm(const void* x, int x_dtype, const void* w, int w_dtype, double eps, int64_t T, int H, void* out,
                cudaStream_t st) {
  AL_CHECK(H % 8 == 0, ARTLITE_EUNSUPPORTED, "norm: H %d (a multiple of 8)", H);
  AL_CHECK(w_dtype == ARTLITE_F32 || w_dtype == ARTLITE_BF16, ARTLITE_EINVAL, "norm: weight type %d", w_dtype);
  if (T == 0) return ARTLITE_OK;
  const dim3 grid((unsigned)cdiv(T, 4));
  const bool xb = x_dtype == ARTLITE_BF16, wb = w_dtype == ARTLITE_BF16;
  if (xb && !wb) return launch_pdl(norm_kernel<ARTLITE_BF16, ARTLITE_F32>, grid, dim3(256), 0, st, x, w, eps, T, H, out);
  if (xb && wb) return launch_pdl(norm_kernel<ARTLITE_BF16, ARTLITE_BF16>, grid, dim3(256), 0, st, x, w, eps, T, H, out);
  if (wb) return launch_pdl(norm_kernel<ARTLITE_F32, ARTLITE_BF16>, grid, dim3(256), 0, st, x, w, eps, T, H, out);
  return launch_pdl(norm_kernel<ARTLITE_F32, ARTLITE_F32>, grid, dim3(256), 0, st, x, w, eps, T, H, out);
}

// a grid-stride loop over 16-byte chunks of the output rows (8 values each): row i of xp = token perm[i] / k of x
__global__ void __launch_bounds__(256) gather_kernel(const void* x, int x_dtype, const int32_t* perm, int64_t P, int k,
                                                     int H, uint16_t* xp, uint16_t* own_dst, int64_t own_lo,
                                                     int64_t own_hi) {
  const int per_row = H >> 3;
  const int64_t n = P * per_row;
  for (int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; c < n; c += (int64_t)gridDim.x * blockDim.x) {
    const int64_t i = c / per_row;
    const int col = (int)(c - i * per_row) * 8;
    const int64_t t = perm[i] / k;
    uint16_t* dst = (own_dst && i >= own_lo && i < own_hi) ? own_dst + (i - own_lo) * H : xp + i * H;
    if (x_dtype == ARTLITE_BF16) {
      *reinterpret_cast<uint4*>(dst + col) =
          __ldg(reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(x) + t * H + col));
    } else {
      float v[8];
      load8(x, ARTLITE_F32, t * H + col, v);
      store8(dst, ARTLITE_BF16, col, v);
    }
  }
}

int launch_gather(const void* x, int x_dtype, const int32_t* perm, int64_t P, int k, int H, uint16_t* xp,
                  cudaStream_t st, uint16_t* own_dst, int64_t own_lo, int64_t own_hi) {
  AL_CHECK(H % 8 == 0, ARTLITE_EUNSUPPORTED, "gather: H %d (a multiple of 8)", H);
  if (P == 0) return ARTLITE_OK;
  const int64_t chunks = P * (H / 8);
  const unsigned grid = (unsigned)std::min<int64_t>(cdiv(chunks, 256), (int64_t)kNumSMs * 16);
  gather_kernel<<<grid, 256, 0, st>>>(x, x_dtype, perm, P, k, H, xp, own_dst, own_lo, own_hi);
  AL_LAUNCHED();
  return ARTLITE_OK;
}

// a warp per token: s[t] = sigmoid(x_t . g), fp32 products and a fixed-order fp32 sum (ref.shared_expert's
// sigmoid(x @ gate_inp), tests/moe/ref.py:55-60, np_ops.sigmoid = 1 / (1 + exp(-z)))
__global__ void __launch_bounds__(256) shared_gate_kernel(const void* x, int x_dtype, const void* g, int g_dtype,
                                                          int64_t T, int H, float* s, int64_t* off) {
  griddep_wait();
  griddep_launch();
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    off[0] = 0;
    off[1] = T;
    reinterpret_cast<int32_t*>(off + 2)[0] = (int32_t)T;
  }
  const int lane = threadIdx.x & 31;
  const int64_t t = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  if (t >= T) return;
  float acc = 0.0f;
  if (g) {
    for (int c = lane * 8; c < H; c += 256) {
      float a[8], b[8];
      load8(x, x_dtype, t * H + c, a);
      load8(g, g_dtype, c, b);
#pragma unroll
      for (int j = 0; j < 8; j++) acc = fmaf(a[j], b[j], acc);
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) acc += __shfl_xor_sync(0xFFFFFFFFu, acc, o);
  }
  if (lane == 0) s[t] = g ? __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-acc))) : 1.0f;
}

int launch_shared_gate(const void* x, int x_dtype, const void* g, int g_dtype, int64_t T, int H, float* s,
                       int64_t* off, cudaStream_t st) {
  AL_CHECK(H % 8 == 0, ARTLITE_EUNSUPPORTED, "shared gate: H %d (a multiple of 8)", H);
  if (T == 0) return ARTLITE_OK;
  return launch_pdl(shared_gate_kernel, dim3((unsigned)cdiv(T, 8)), dim3(256), 0, st, x, x_dtype, g, g_dtype, T, H, s,
                    off);
}

}  // namespace artlite
