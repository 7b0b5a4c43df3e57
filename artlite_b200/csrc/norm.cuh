// The block's optional input norm, RMSNorm as the reference's float32 numpy (tests/np_ops.py:27-32): the mean of the
// squares in float64, x over sqrt(mean + eps) in float64 rounded to float32, times w in float32, stored in x's dtype.
// norm_rows norms up to G rows with one CTA of 256 threads (H % 8 == 0) in one summation order (below), so every
// kernel that norms rows gives the same bits: the norm kernel (four rows a CTA), the fused decode kernel's first phase
// (CTA b norms rows b, b + G, .., publishes them with norm_publish, one count a row, and every CTA waits for all of
// them with norm_wait, bounded: after about two seconds it reports ARTLITE_ETIMEOUT through the status word and
// returns false), and norm_rows_cta, with which every CTA of the small-batch router norms all of a batch's rows (up
// to 16) into its own shared memory, so that no CTA waits for another.
#pragma once

#include <cuda_bf16.h>

#include "common.cuh"

namespace artlite {
namespace nrm {

constexpr long long kWaitCycles = 4000000000LL;  // about 2 s

// 8 consecutive values (element i is 8-aligned); coherent loads: a row may have been written earlier in the launch
__device__ __forceinline__ void ld8(const void* p, int dtype, int64_t i, float (&v)[8]) {
  if (dtype == ARTLITE_BF16) {
    const uint4 u = __ldcg(reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(p) + i));
    const uint32_t q[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int j = 0; j < 4; j++) v[2 * j] = __uint_as_float(q[j] << 16), v[2 * j + 1] = __uint_as_float(q[j] & 0xFFFF0000u);
  } else {
    const float4 a = __ldcg(reinterpret_cast<const float4*>(reinterpret_cast<const float*>(p) + i));
    const float4 b = __ldcg(reinterpret_cast<const float4*>(reinterpret_cast<const float*>(p) + i) + 1);
    v[0] = a.x, v[1] = a.y, v[2] = a.z, v[3] = a.w, v[4] = b.x, v[5] = b.y, v[6] = b.z, v[7] = b.w;
  }
}

// the same through a generic pointer (shared memory, or global rows written before the launch)
__device__ __forceinline__ void ld8p(const void* p, int dtype, int64_t i, float (&v)[8]) {
  if (dtype == ARTLITE_BF16) {
    const uint4 u = *reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(p) + i);
    const uint32_t q[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int j = 0; j < 4; j++) v[2 * j] = __uint_as_float(q[j] << 16), v[2 * j + 1] = __uint_as_float(q[j] & 0xFFFF0000u);
  } else {
    const float4 a = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(p) + i);
    const float4 b = *(reinterpret_cast<const float4*>(reinterpret_cast<const float*>(p) + i) + 1);
    v[0] = a.x, v[1] = a.y, v[2] = a.z, v[3] = a.w, v[4] = b.x, v[5] = b.y, v[6] = b.z, v[7] = b.w;
  }
}

__device__ __forceinline__ void st8(void* p, int dtype, int64_t i, const float (&v)[8]) {
  if (dtype == ARTLITE_BF16) {
    uint32_t w[4];
#pragma unroll
    for (int j = 0; j < 4; j++) {
      const __nv_bfloat162 h = __floats2bfloat162_rn(v[2 * j], v[2 * j + 1]);
      w[j] = *reinterpret_cast<const uint32_t*>(&h);
    }
    *reinterpret_cast<uint4*>(reinterpret_cast<uint16_t*>(p) + i) = make_uint4(w[0], w[1], w[2], w[3]);
  } else {
    float4* q = reinterpret_cast<float4*>(reinterpret_cast<float*>(p) + i);
    q[0] = make_float4(v[0], v[1], v[2], v[3]);
    q[1] = make_float4(v[4], v[5], v[6], v[7]);
  }
}

// float(v / d) as the float64 division rounded to float32, from r = 1 / d (float64, correctly rounded; d positive,
// normal and finite): q0 = v r, then two corrections q += (v - q d) r, each remainder by one fused multiply-add. The
// first leaves q within one unit in the last place of v / d; from such a q and a correctly rounded reciprocal, one
// correction gives the correctly rounded quotient (Markstein's theorem), so q2 is the division's float64 result bit for
// bit, and its rounding to float32 the reference's. No overflow or underflow is reachable: v is a float, d lies in
// [2^-149, 2^128]. For v = +-0 the corrections lose the zero's sign: q0 keeps it.
__host__ __device__ __forceinline__ float div_to_f32(double v, double d, double r) {
  const double q0 = v * r;
  const double q1 = fma(fma(-q0, d, v), r, q0);
  const double q2 = fma(fma(-q1, d, v), r, q1);
  return (float)(q2 != 0.0 ? q2 : q0);
}

// rows r0 .. r0 + n - 1 (n <= G) of x normed into the same rows of out (and row `mine` also into out2, if set), by
// one CTA of 256 threads, each row with norm_row's arithmetic: thread i sums the squares of its 8-value chunks
// (columns 8i + 2048k) in column order, a warp's shuffle tree adds its lanes, then the 8 warps' sums in warp order;
// the G rows' loads, sums and trees interleave, and thread t finishes row t (sqrt, 1 / d). x: generic pointer (global
// rows written before the launch, or shared memory); out may be x (in place).
template <int G>
__device__ __forceinline__ void norm_rows(const void* x, int x_dtype, const void* w, int w_dtype, double eps, int H,
                                          int64_t r0, int n, void* out, void* out2 = nullptr, int64_t mine = -1) {
  __shared__ double part[8][G];
  __shared__ double dr[G][2];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  double s[G];
#pragma unroll
  for (int t = 0; t < G; t++) s[t] = 0.0;
  for (int c = threadIdx.x * 8; c < H; c += 256 * 8) {
#pragma unroll
    for (int t = 0; t < G; t++) {
      if (t < n) {
        float v[8];
        ld8p(x, x_dtype, (r0 + t) * H + c, v);
#pragma unroll
        for (int j = 0; j < 8; j++) s[t] = fma((double)v[j], (double)v[j], s[t]);
      }
    }
  }
#pragma unroll
  for (int t = 0; t < G; t++) {
    if (t < n) {
#pragma unroll
      for (int o = 16; o; o >>= 1) s[t] += __shfl_xor_sync(0xFFFFFFFFu, s[t], o);
      if (lane == 0) part[warp][t] = s[t];
    }
  }
  __syncthreads();
  if (threadIdx.x < n) {
    double tot = 0.0;
    for (int i = 0; i < 8; i++) tot += part[i][threadIdx.x];
    const double den = sqrt(tot / H + eps);
    dr[threadIdx.x][0] = den;
    dr[threadIdx.x][1] = 1.0 / den;  // (a row whose d is not positive, normal and finite: r = 0 marks the division)
    if (!(den >= 0x1p-1022 && den <= 0x1.fffffffffffffp+1023)) dr[threadIdx.x][1] = 0.0;
  }
  __syncthreads();
  for (int c = threadIdx.x * 8; c < H; c += 256 * 8) {
    float g[8];
    ld8(w, w_dtype, c, g);
#pragma unroll
    for (int t = 0; t < G; t++) {
      if (t < n) {
        const double d = dr[t][0], r = dr[t][1];
        float v[8];
        ld8p(x, x_dtype, (r0 + t) * H + c, v);
        if (r != 0.0) {
#pragma unroll
          for (int j = 0; j < 8; j++) v[j] = __fmul_rn(div_to_f32(v[j], d, r), g[j]);
        } else {
#pragma unroll
          for (int j = 0; j < 8; j++) v[j] = __fmul_rn((float)((double)v[j] / d), g[j]);
        }
        st8(out, x_dtype, (r0 + t) * H + c, v);
        if (out2 && r0 + t == mine) st8(out2, x_dtype, (r0 + t) * H + c, v);
      }
    }
  }
  __syncthreads();  // (part and dr are reused by the next call)
}

// rows 0 .. T - 1 (T <= kRowsCta) of x normed by one CTA of 256 threads into its shared memory xs (T x H of x_dtype,
// 16-byte aligned): the raw rows copied in, then normed in place four at a time; the CTA also stores its row `mine`
// (0 <= mine < T; else none) to out
constexpr int kRowsCta = 16;
__device__ __forceinline__ void norm_rows_cta(const void* x, int x_dtype, const void* w, int w_dtype, double eps,
                                              int H, int T, void* xs, int mine, void* out) {
  const int n16 = T * H * (x_dtype == ARTLITE_BF16 ? 2 : 4) / 16;
  for (int i = threadIdx.x; i < n16; i += blockDim.x)
    reinterpret_cast<uint4*>(xs)[i] = __ldcg(reinterpret_cast<const uint4*>(x) + i);
  __syncthreads();
  for (int r0 = 0; r0 < T; r0 += 4) norm_rows<4>(xs, x_dtype, w, w_dtype, eps, H, r0, min(4, T - r0), xs, out, mine);
}

// the CTA's normed rows published: every thread's stores ordered before one count per row (rows may be 0)
__device__ __forceinline__ void norm_publish(unsigned* cnt, unsigned rows) {
  __syncthreads();
  if (threadIdx.x == 0 && rows) {
    __threadfence();
    atomicAdd(cnt, rows);
  }
}

// every CTA: wait until want rows are published; false if the wait ran out (reported: where, this CTA)
__device__ __forceinline__ bool norm_wait(const unsigned* cnt, unsigned want, DevStatus* st, int where) {
  __shared__ int ok;
  if (threadIdx.x == 0) {
    ok = 1;
    const long long t0 = clock64();
    for (;;) {
      unsigned v;
      asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(cnt) : "memory");
      if (v >= want) break;
      if (clock64() - t0 > kWaitCycles) {
        report(st, ARTLITE_ETIMEOUT, where, (int)blockIdx.x);
        ok = 0;
        break;
      }
      __nanosleep(32);
    }
    __threadfence();
  }
  __syncthreads();
  return ok != 0;
}

}  // namespace nrm
}  // namespace artlite
