// The routing of one token row by one warp (route.cu's kernel and the fused decode-batch kernel of dispatch.cu).
// Semantics: see route.cu.
#pragma once

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

// e^x for x <= 0 by the reference's method (moe_host.cpp:75-90): x = n ln 2 + r (ln 2 in two parts), a degree-12
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

// one token's row by one warp (t < a.n; every lane calls)
template <int J>
__device__ __forceinline__ void route_row(const RouteArgs& a, int64_t t, int lane) {
  const float* p = a.logits + t * a.row;
  const bool flat = a.per_col >= a.E;  // (one column: the logit of x at p[x], no division)
  uint64_t key[J];
  bool nan = false;
#pragma unroll
  for (int j = 0; j < J; j++) {
    const int x = lane + 32 * j;
    key[j] = 0;  // below every real key (~x != 0)
    if (x < a.E) {
      const float l = __ldcg(flat ? p + x : p + (int64_t)(x / a.per_col) * a.pitch + x % a.per_col);
      nan |= l != l;
      key[j] = route_key(l, x);
    }
  }
  nan = __any_sync(0xFFFFFFFFu, nan);
  // lane r < k: the r-th largest key. A round's warp maximum of the 64-bit keys by two 32-bit reductions: the largest
  // high word, then the largest low word among the lanes whose best key has it (keys are unique: one owner)
  uint64_t mine = 0;
  for (int r = 0; r < a.k; r++) {
    uint64_t m = 0;
    int mj = 0;
#pragma unroll
    for (int j = 0; j < J; j++)
      if (key[j] > m) m = key[j], mj = j;
    const uint32_t hi = (uint32_t)(m >> 32), whi = __reduce_max_sync(0xFFFFFFFFu, hi);
    const uint32_t wlo = __reduce_max_sync(0xFFFFFFFFu, hi == whi ? (uint32_t)m : 0u);
    const uint64_t wm = (uint64_t)whi << 32 | wlo;
    if (m == wm) {  // the owner
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
  // numpy's pairwise order for a row of k <= 32 (moe_host.cpp:24-39)
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

// The routing and dispatch of a decode-sized batch by one CTA of NT threads (r.ids is a.ids; n k <= kSmallPairs pairs,
// E <= kSmallExperts, NT >= E): every token routed into shared memory (a warp a row), the ids and weights copied out
// for the caller, then the histogram, the scan and the stable rank of the pairs exactly as the dispatch kernels do for
// a single block, and both expert GEMVs' unit scans. sm: dynamic shared memory of
// 4 ((NT / 32 + 2) E + 1) + 8 E + 8 P bytes. Called by dispatch.cu's route_dispatch_small.
template <int J, int NT>
__device__ __forceinline__ void route_dispatch_cta(RouteArgs r, const DispatchArgs& a, int mult2, int32_t* unit_off2,
                                                   int32_t* sm) {
  __shared__ int64_t s64[32];
  __shared__ int32_t s32[32];
  constexpr int NW = NT / 32;
  int32_t* wc = sm;                 // [NW][E] per-warp counts of the current round
  int32_t* run = sm + NW * a.E;     // [E] placed so far
  int32_t* cnt = run + a.E;         // [E] histogram
  int64_t* off = reinterpret_cast<int64_t*>(cnt + a.E + (a.E & 1));  // [E] offsets
  int32_t* ids_s = reinterpret_cast<int32_t*>(off + a.E);             // [P] the routed ids
  float* w_s = reinterpret_cast<float*>(ids_s + a.P);                 // [P] and weights
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  {
    RouteArgs rl = r;
    rl.ids = ids_s;
    rl.w = w_s;
    for (int64_t t = warp; t < r.n; t += NW) route_row<J>(rl, t, lane);
  }
  for (int i = threadIdx.x; i < (NW + 2) * a.E; i += NT) sm[i] = 0;
  __syncthreads();  // (the rows' ids are visible to the block)
  for (int64_t p = threadIdx.x; p < a.P; p += NT) {
    const int32_t x = ids_s[p];
    r.ids[p] = x;
    r.w[p] = w_s[p];
    if (x < 0 || x >= a.E)
      report(a.status, ARTLITE_EDEVICE, x, a.E, 1);
    else
      atomicAdd(&cnt[x], 1);
  }
  __syncthreads();
  const int e = threadIdx.x;
  const int32_t c = e < a.E ? cnt[e] : 0;
  int64_t tot64;
  const int64_t o = block_exclusive_scan<int64_t>(c, s64, &tot64);
  if (e < a.E) {
    off[e] = o;
    a.offsets[e] = o;
    a.counts[e] = c;
  }
  if (e == 0) a.offsets[a.E] = tot64;
  for (int which = 0; which < 2; which++) {
    const int mult = which ? mult2 : a.unit_mult;
    int32_t* uo = which ? unit_off2 : a.unit_off;
    if (!uo) continue;
    const int32_t u = e < a.E ? (c + a.unit_rows - 1) / a.unit_rows * mult : 0;
    int32_t tot;
    const int32_t v = block_exclusive_scan<int32_t>(u, s32, &tot);
    if (e < a.E) uo[e] = v;
    if (e == 0) uo[a.E] = tot;
  }
  __syncthreads();
  const unsigned lt = (1u << lane) - 1u;
  for (int64_t r0 = 0; r0 < a.P; r0 += NT) {
    const int64_t p = r0 + threadIdx.x;
    int32_t x = p < a.P ? ids_s[p] : -1;
    const bool valid = x >= 0 && x < a.E;
    if (!valid) x = -1 - lane;
    const unsigned peers = __match_any_sync(0xFFFFFFFFu, x);
    const int rank = __popc(peers & lt);
    const bool leader = rank == 0;
    if (valid && leader) wc[warp * a.E + x] = __popc(peers);
    __syncthreads();
    if (valid) {
      int32_t pre = run[x];
      for (int w = 0; w < warp; w++) pre += wc[w * a.E + x];
      const int64_t dest = off[x] + pre + rank;
      a.perm[dest] = (int32_t)p;
      a.slot[p] = (int32_t)dest;
    }
    __syncthreads();
    if (valid && leader) {
      atomicAdd(&run[x], __popc(peers));
      wc[warp * a.E + x] = 0;
    }
    __syncthreads();
  }
}


}  // namespace artlite
