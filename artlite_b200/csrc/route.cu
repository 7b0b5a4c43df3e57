// Routing: one warp per token, top-k by rounds of a warp arg-max over 64-bit ordered keys, softmax / sigmoid weights
// over the k in double, normalised in numpy's pairwise order.
//
// Semantics follow artlite::moe_route (csrc/artlite/moe_host.cpp:85-113 route_rows_scalar, :138-214
// route_rows_avx512, :216-239 route_rows / moe_route):
//   key(l, x) = (bits(l + 0) flipped to an unsigned order) << 32 | ~x  (ties to the lower id, -0 == +0, :95-96);
//   e_j = e^(l_j - l_0) in double; on the reference's vector-path shapes (k <= 16, per_col % 16 == 0, E <= 512) rows
//   with k == 8, softmax and no NaN take its degree-12 Taylor exp_nonpos (:115-130, restated below from that
//   source), every other row exp() (the reference's std::exp); sigmoid: 1 / (1 + e^-l) with the sum clamped at 2^-14;
//   the sum in numpy's pairwise order (row_sum, :64-79); w_j = float(e_j / sum).
// The GPU's float add returns a canonical NaN where x86's keeps the operand's sign and payload, so the key is built
// from the bits directly: -0 -> +0, a NaN quietened with its sign kept (what addss(l, 0) gives).
#include "common.cuh"
#include "kernels.cuh"

namespace artlite {

__device__ __forceinline__ uint32_t route_bits(float l) {
  uint32_t u = __float_as_uint(l);
  if (u == 0x80000000u) return 0u;
  if ((u & 0x7F800000u) == 0x7F800000u && (u & 0x007FFFFFu)) u |= 0x00400000u;
  return u;
}

__device__ __forceinline__ uint64_t route_key(float l, int x) {
  const uint32_t u = route_bits(l);
  return (uint64_t)(u ^ ((u >> 31) ? 0xFFFFFFFFu : 0x80000000u)) << 32 | (uint32_t)(~(uint32_t)x);
}

// the logit a key was made from (for a NaN: a NaN, whose weights are NaN either way)
__device__ __forceinline__ float key_logit(uint64_t key) {
  const uint32_t o = (uint32_t)(key >> 32);
  return __uint_as_float((o & 0x80000000u) ? (o ^ 0x80000000u) : ~o);
}

// e^x for x <= 0 by the reference's method (moe_host.cpp:115-130): x = n ln 2 + r (ln 2 in two parts), a degree-12
// Taylor polynomial of r by Horner with fused multiply-adds, times 2^n; x clamped at -708.
__device__ __forceinline__ double exp_nonpos(double x) {
  const double log2e = 1.4426950408889634, ln2hi = 6.93147180369123816490e-01, ln2lo = 1.90821492927058770002e-10;
  x = x > -708.0 ? x : -708.0;
  const double n = rint(x * log2e);
  const double r = fma(-n, ln2lo, fma(-n, ln2hi, x));
  double p = 1.0 / 479001600;
  p = fma(p, r, 1.0 / 39916800);
  p = fma(p, r, 1.0 / 3628800);
  p = fma(p, r, 1.0 / 362880);
  p = fma(p, r, 1.0 / 40320);
  p = fma(p, r, 1.0 / 5040);
  p = fma(p, r, 1.0 / 720);
  p = fma(p, r, 1.0 / 120);
  p = fma(p, r, 1.0 / 24);
  p = fma(p, r, 1.0 / 6);
  p = fma(p, r, 1.0 / 2);
  p = fma(p, r, 1.0);
  p = fma(p, r, 1.0);
  return p * __longlong_as_double((long long)((int64_t)n + 1023) << 52);
}

template <int J>
__global__ void __launch_bounds__(256) route_kernel(RouteArgs a) {
  const int lane = threadIdx.x & 31;
  const int64_t t = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (t >= a.n) return;
  const float* p = a.logits + t * a.row;
  uint64_t key[J];
  bool nan = false;
#pragma unroll
  for (int j = 0; j < J; j++) {
    const int x = lane + 32 * j;
    key[j] = 0;  // below every real key (~x != 0)
    if (x < a.E) {
      const float l = __ldg(p + (int64_t)(x / a.per_col) * a.pitch + x % a.per_col);
      nan |= l != l;
      key[j] = route_key(l, x);
    }
  }
  nan = __any_sync(0xFFFFFFFFu, nan);
  uint64_t mine = 0;  // lane r < k: the r-th largest key
  for (int r = 0; r < a.k; r++) {
    uint64_t m = 0;
    int mj = 0;
#pragma unroll
    for (int j = 0; j < J; j++)
      if (key[j] > m) m = key[j], mj = j;
    uint64_t wm = m;
#pragma unroll
    for (int off = 16; off; off >>= 1) {
      const uint64_t o = __shfl_xor_sync(0xFFFFFFFFu, wm, off);
      wm = o > wm ? o : wm;
    }
    if (m == wm) {  // the owner (keys are unique)
#pragma unroll
      for (int j = 0; j < J; j++)
        if (j == mj) key[j] = 0;
    }
    if (lane == r) mine = wm;
  }
  const double l0 = (double)key_logit(__shfl_sync(0xFFFFFFFFu, mine, 0));
  const bool taylor = a.vector_shape && !nan && a.k == 8 && !a.sigmoid;
  double e = 0.0;
  if (lane < a.k) {
    const double l = (double)key_logit(mine);
    e = a.sigmoid ? 1.0 / (1.0 + exp(-l)) : (taylor ? exp_nonpos(l - l0) : exp(l - l0));
  }
  // numpy's pairwise order for a row of k <= 32 (moe_host.cpp:64-79)
  double s = 0.0, r0 = 0, r1 = 0, r2 = 0, r3 = 0, r4 = 0, r5 = 0, r6 = 0, r7 = 0;
  const int full = a.k < 8 ? 0 : (a.k / 8) * 8;
#pragma unroll
  for (int i = 0; i < 32; i++) {
    if (i >= a.k) break;
    const double ei = __shfl_sync(0xFFFFFFFFu, e, i);
    if (i < full) {
      switch (i & 7) {
        case 0: r0 = i < 8 ? ei : r0 + ei; break;
        case 1: r1 = i < 8 ? ei : r1 + ei; break;
        case 2: r2 = i < 8 ? ei : r2 + ei; break;
        case 3: r3 = i < 8 ? ei : r3 + ei; break;
        case 4: r4 = i < 8 ? ei : r4 + ei; break;
        case 5: r5 = i < 8 ? ei : r5 + ei; break;
        case 6: r6 = i < 8 ? ei : r6 + ei; break;
        default: r7 = i < 8 ? ei : r7 + ei; break;
      }
      if (i == full - 1) s = ((r0 + r1) + (r2 + r3)) + ((r4 + r5) + (r6 + r7));
    } else {
      s += ei;
    }
  }
  if (a.sigmoid && s < 6.103515625e-5) s = 6.103515625e-5;  // std::max(s, 2^-14): a NaN stays
  if (lane < a.k) {
    a.ids[t * a.k + lane] = (int32_t)(~(uint32_t)mine);
    a.w[t * a.k + lane] = (float)(e / s);
  }
}

int launch_route(const RouteArgs& a, cudaStream_t st) {
  if (a.n == 0) return ARTLITE_OK;
  const int warps = 8;
  const unsigned grid = (unsigned)cdiv(a.n, warps);
  const int J = (a.E + 31) / 32;
  if (J <= 1) route_kernel<1><<<grid, warps * 32, 0, st>>>(a);
  else if (J <= 2) route_kernel<2><<<grid, warps * 32, 0, st>>>(a);
  else if (J <= 4) route_kernel<4><<<grid, warps * 32, 0, st>>>(a);
  else if (J <= 8) route_kernel<8><<<grid, warps * 32, 0, st>>>(a);
  else if (J <= 16) route_kernel<16><<<grid, warps * 32, 0, st>>>(a);
  else route_kernel<32><<<grid, warps * 32, 0, st>>>(a);
  AL_LAUNCHED();
  return ARTLITE_OK;
}

int check_route_args(int64_t n, int per_col, int E, int k) {
  // the reference's own check (moe_host.cpp:228), then this build's limits
  AL_CHECK(per_col > 0 && k >= 1 && k <= E && E % per_col == 0, ARTLITE_EINVAL, "moe_route: k %d of E %d (%d per column)",
           k, E, per_col);
  AL_CHECK(E <= 1024 && k <= 32, ARTLITE_EUNSUPPORTED, "moe_route: E %d k %d (this build: E <= 1024, k <= 32)", E, k);
  AL_CHECK(n >= 0, ARTLITE_EINVAL, "moe_route: n %lld", (long long)n);
  return ARTLITE_OK;
}

}  // namespace artlite
