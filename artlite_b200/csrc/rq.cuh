// The register-decoding expert GEMV (Q4_0, Q8_0, Q4_K): device code shared by the GEMV kernels (gemv.cu) and the
// fused decode kernel (decode.cu).
#pragma once

#include <cuda_fp16.h>

#include "common.cuh"
#include "kernels.cuh"

namespace artlite {

__device__ __forceinline__ float rq_silu(float g) { return __fdiv_rn(g, __fadd_rn(1.0f, expf(-g))); }

// // A lane owns (weight row, 256-value segment): the segment's raw bytes (144 B; 272 B for Q8_0) come straight from HBM
// in 16-byte loads into registers (a row's segments are contiguous across its lanes). The dot products run on the
// quantised values, the block scales applied once per 32-value group, since the reference's dequantised weight is affine
// in the quantised value q (gguf_model.py:278-330):
//   Q4_0  w = d (q - 8),   Q4_K  w = (d sc) q - (dmin m),   Q8_0  w = d q,
// so a group's sum_j w_j x_j = A S' - B X with S' = sum_j (1/2 + q_j / 256) x_j, X = sum_j x_j and A = 256 d, B = 136 d
// (Q4_K: A = 256 d sc, B = 128 d sc + dmin m); Q8_0: d sum_j q_j x_j with q_j exact. 1/2 + q/256 is one byte permute
// (q into bits 16..23 under the exponent byte 0x3F), then one packed fp32 FMA per two weights and token; X comes with
// the staging of x (per token and group). These are exact-weight dot products up to fp32 rounding, in another order
// than the reference's fp32 sums (the relative difference stays near 1e-6).
// Gate and up rows interleave in a warp: R gate rows, then the same R up rows, each row's segments on consecutive lanes;
// a row's partial sums meet by shuffles and the up sum moves to its gate lane for silu(g) u.

namespace rq {

__device__ __forceinline__ uint4 ldg_stream(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}
__device__ __forceinline__ uint32_t byte_at(const uint32_t* w, int b) { return (w[b >> 2] >> ((b & 3) * 8)) & 0xFFu; }
__device__ __forceinline__ float half_at(const uint32_t* w, int b) {  // b even
  const uint32_t v = (b & 2) ? (w[b >> 2] >> 16) : (w[b >> 2] & 0xFFFFu);
  return __half2float(__ushort_as_half((unsigned short)v));
}
// 4 words from byte offset o (even)
__device__ __forceinline__ void words16(const uint32_t* w, int o, uint32_t (&q)[4]) {
#pragma unroll
  for (int k = 0; k < 4; k++)
    q[k] = (o & 2) ? __funnelshift_r(w[(o >> 2) + k], w[(o >> 2) + k + 1], 16) : w[(o >> 2) + k];
}
// byte b of u (< 128) as the float 1/2 + q / 256
__device__ __forceinline__ float q_half(uint32_t u, int b) {
  return __uint_as_float(__byte_perm(u, 0x3F000000u, 0x7044u | (b << 8)));
}
// byte b of u as the float 2^23 + q
__device__ __forceinline__ float q_magic(uint32_t u, int b) { return __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7440u | b)); }
__device__ __forceinline__ uint64_t pack(float a, float b) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ uint64_t add2(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t fma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}
__device__ __forceinline__ float hsum2(uint64_t v) {
  float a, b;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v));
  return a + b;
}

template <int QT>
struct Seg {  // a 256-value segment
  static constexpr int bytes = QT == ARTLITE_Q8_0 ? 272 : 144;
  static constexpr int v16 = bytes / 16;
  static constexpr int words = v16 * 4;
};

constexpr int kSegStride = 260;  // floats per staged 256-value x segment (4 of padding: the lanes of a row read
                                 // their segments' float4s conflict-free)
constexpr int kWarps = 8;

// Token-group sizes the kernel is compiled for (a group of nt <= 8 pairs runs the smallest that holds it).
__host__ __device__ constexpr int nt_bucket(int nt) { return nt <= 1 ? 1 : nt <= 2 ? 2 : nt <= 4 ? 4 : 8; }

// The dot products of one lane's segment with NTC staged tokens: y[n] (n < NTC) for this segment.
template <int QT, int NTC>
__device__ __forceinline__ void segment_dot(const uint32_t (&w)[Seg<QT>::words], const float* xseg, int xtok,
                                            const float* xg, int gtok, float (&y)[NTC]) {
#pragma unroll
  for (int n = 0; n < NTC; n++) y[n] = 0.0f;
  float d = 0.0f, dmin = 0.0f;
  if constexpr (QT == ARTLITE_Q4_K) {
    d = half_at(w, 0);
    dmin = half_at(w, 2);
  }
#pragma unroll
  for (int g = 0; g < 8; g++) {
    uint32_t qw[8];
    float A, B = 0.0f;
    if constexpr (QT == ARTLITE_Q4_0) {
      uint32_t q[4];
      words16(w, 18 * g + 2, q);
#pragma unroll
      for (int k = 0; k < 4; k++) qw[k] = q[k] & 0x0F0F0F0Fu, qw[k + 4] = (q[k] >> 4) & 0x0F0F0F0Fu;
      const float dd = half_at(w, 18 * g);
      A = 256.0f * dd;
      B = 136.0f * dd;
    } else if constexpr (QT == ARTLITE_Q8_0) {
      uint32_t lo[4], hi[4];
      words16(w, 34 * g + 2, lo);
      words16(w, 34 * g + 18, hi);
#pragma unroll
      for (int k = 0; k < 4; k++) qw[k] = lo[k] ^ 0x80808080u, qw[k + 4] = hi[k] ^ 0x80808080u;
      A = half_at(w, 34 * g);
    } else {
      const int wb = 4 + 8 * (g >> 1);
#pragma unroll
      for (int k = 0; k < 8; k++) qw[k] = ((g & 1) ? (w[wb + k] >> 4) : w[wb + k]) & 0x0F0F0F0Fu;
      int sc, mn;
      if (g < 4) {
        sc = byte_at(w, 4 + g) & 63;
        mn = byte_at(w, 8 + g) & 63;
      } else {
        sc = (byte_at(w, 8 + g) & 15) | (byte_at(w, g) >> 6) << 4;
        mn = (byte_at(w, 8 + g) >> 4) | (byte_at(w, 4 + g) >> 6) << 4;
      }
      const float dsc = __fmul_rn(d, (float)sc), dmn = __fmul_rn(dmin, (float)mn);
      A = 256.0f * dsc;
      B = __fmaf_rn(128.0f, dsc, dmn);
    }
    constexpr bool kTwo = NTC <= 2;  // (two chains per token when there are few tokens)
    uint64_t s0[NTC], s1[kTwo ? NTC : 1];
#pragma unroll
    for (int n = 0; n < NTC; n++) {
      s0[n] = 0;
      if constexpr (kTwo) s1[n] = 0;
    }
#pragma unroll
    for (int k = 0; k < 8; k++) {
      uint64_t v01, v23;
      if constexpr (QT == ARTLITE_Q8_0) {
        const uint64_t off = pack(-8388736.0f, -8388736.0f);  // -(2^23 + 128)
        v01 = add2(pack(q_magic(qw[k], 0), q_magic(qw[k], 1)), off);
        v23 = add2(pack(q_magic(qw[k], 2), q_magic(qw[k], 3)), off);
      } else {
        v01 = pack(q_half(qw[k], 0), q_half(qw[k], 1));
        v23 = pack(q_half(qw[k], 2), q_half(qw[k], 3));
      }
#pragma unroll
      for (int n = 0; n < NTC; n++) {
        const float4 xv = *reinterpret_cast<const float4*>(xseg + n * xtok + 32 * g + 4 * k);
        s0[n] = fma2(v01, pack(xv.x, xv.y), s0[n]);
        if constexpr (kTwo)
          s1[n] = fma2(v23, pack(xv.z, xv.w), s1[n]);
        else
          s0[n] = fma2(v23, pack(xv.z, xv.w), s0[n]);
      }
    }
#pragma unroll
    for (int n = 0; n < NTC; n++) {
      float sg = hsum2(s0[n]);
      if constexpr (kTwo) sg += hsum2(s1[n]);
      if constexpr (QT == ARTLITE_Q8_0)
        y[n] = fmaf(A, sg, y[n]);
      else
        y[n] = fmaf(A, sg, fmaf(-B, xg[n * gtok + g], y[n]));
    }
  }
}

}  // namespace rq


namespace rq {

// Stage token group tg of expert e for the items that follow: x rows (GU: the tokens perm[d] / k; down: rows d of x)
// as fp32 into xs [NT][segs][kSegStride], zero past nt, and the per-(token, group) sums into xg [NT][K / 32]. Every
// thread of the CTA calls it; the caller synchronises before and after. x is read through L2 (it may have been
// written by other CTAs of the same kernel).
template <bool GU>
__device__ __forceinline__ void stage(const ExpertGemvArgs& a, const int64_t* offs, const int32_t* perm, int e, int tg,
                                      float* xs, float* xg, int64_t* d0_out, int* nt_out) {
  constexpr int NT = kGemvTokens;
  const int segs = a.K >> 8, G = a.K >> 5;
  const int64_t d0 = offs[e] + (int64_t)tg * NT;
  const int nt = (int)min64(NT, offs[e + 1] - d0);
  *d0_out = d0;
  *nt_out = nt;
  const int per_tok = a.K >> 3;
  for (int c8 = threadIdx.x; c8 < NT * per_tok; c8 += blockDim.x) {
    const int n = c8 / per_tok, k = (c8 - n * per_tok) * 8;
    float v[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    if (n < nt) {
      const int64_t src = (GU ? (int64_t)(perm[d0 + n] / a.k) : d0 + n) * a.K + k;
      if (a.x_dtype == ARTLITE_BF16) {
        const uint4 u = __ldcg(reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(a.x) + src));
        const uint32_t q[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int j = 0; j < 4; j++) v[2 * j] = __uint_as_float(q[j] << 16), v[2 * j + 1] = __uint_as_float(q[j] & 0xFFFF0000u);
      } else {
        const float4* f = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(a.x) + src);
        const float4 f0 = __ldcg(f), f1 = __ldcg(f + 1);
        v[0] = f0.x, v[1] = f0.y, v[2] = f0.z, v[3] = f0.w, v[4] = f1.x, v[5] = f1.y, v[6] = f1.z, v[7] = f1.w;
      }
    }
    float4* dst = reinterpret_cast<float4*>(xs + (n * segs + (k >> 8)) * kSegStride + (k & 255));
    dst[0] = make_float4(v[0], v[1], v[2], v[3]);
    dst[1] = make_float4(v[4], v[5], v[6], v[7]);
    float part = ((v[0] + v[1]) + (v[2] + v[3])) + ((v[4] + v[5]) + (v[6] + v[7]));
    part += __shfl_xor_sync(0xFFFFFFFFu, part, 1);
    part += __shfl_xor_sync(0xFFFFFFFFu, part, 2);
    if ((c8 & 3) == 0) xg[n * G + (k >> 5)] = part;
  }
}

// shared-memory floats stage() needs
__host__ __device__ constexpr size_t stage_floats(int K) { return (size_t)kGemvTokens * ((K / 256) * kSegStride + K / 32); }

// Items [i0, i1) of a GEMV (uo: the items' scan per expert, E + 1 entries; offs / perm: the dispatch), rows per warp R.
// Every thread of the CTA calls it (it synchronises around each staging).
template <int QT, bool GU>
__device__ __forceinline__ void run_items(const ExpertGemvArgs& a, int R, const int32_t* uo, const int64_t* offs,
                                          const int32_t* perm, float* xs, int i0, int i1) {
  constexpr int NT = kGemvTokens;
  const int segs = a.K >> 8, G = a.K >> 5;
  float* xg = xs + NT * segs * kSegStride;
  const int rows_item = R * kWarps, ntile = (a.N + rows_item - 1) / rows_item;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int slot = lane / segs, seg = lane - slot * segs;
  const int nslot = GU ? 2 * R : R;
  const bool mat = GU && slot >= R;
  const int r = mat ? slot - R : slot;
  const float* xseg = xs + seg * kSegStride;
  const float* xgs = xg + seg * 8;
  int cur_e = -1, cur_tg = -1, nt = 0;
  int64_t d0 = 0;
  for (int i = i0; i < i1; i++) {
    int lo = 0, hi = a.E;
    while (hi - lo > 1) {
      const int mid = (lo + hi) >> 1;
      if (uo[mid] <= i) lo = mid; else hi = mid;
    }
    const int li = i - uo[lo], tg = li / ntile, rt = li - tg * ntile;
    const int row = rt * rows_item + warp * R + r;
    const bool valid = slot < nslot && row < a.N;
    uint32_t w[Seg<QT>::words];
    if (valid) {  // (issued before the staging below: their latency overlaps it)
      const int64_t we = a.wexp ? a.wexp[lo] : lo;  // (the row group's weight expert)
      const uint8_t* p = (mat ? a.w1 : a.w0) + (we * a.N + row) * a.row_bytes + (int64_t)seg * Seg<QT>::bytes;
#pragma unroll
      for (int v = 0; v < Seg<QT>::v16; v++) {
        const uint4 u = ldg_stream(p + 16 * v);
        w[4 * v] = u.x, w[4 * v + 1] = u.y, w[4 * v + 2] = u.z, w[4 * v + 3] = u.w;
      }
    }
    if (lo != cur_e || tg != cur_tg) {
      __syncthreads();
      cur_e = lo;
      cur_tg = tg;
      stage<GU>(a, offs, perm, lo, tg, xs, xg, &d0, &nt);
      __syncthreads();
    }
    const int ntb = nt_bucket(nt);
#define RQ_BODY(NTC)                                                                                      \
    {                                                                                                     \
      float y[NTC];                                                                                       \
      if (valid) segment_dot<QT, NTC>(w, xseg, segs * kSegStride, xgs, G, y);                             \
      else {                                                                                              \
        _Pragma("unroll") for (int n = 0; n < NTC; n++) y[n] = 0.0f;                                      \
      }                                                                                                   \
      _Pragma("unroll") for (int n = 0; n < NTC; n++) {                                                   \
        float s = y[n];                                                                                   \
        for (int o = 1; o < segs; o <<= 1) {                                                              \
          const float t = __shfl_down_sync(0xFFFFFFFFu, s, o);                                            \
          if (seg + o < segs) s += t;                                                                     \
        }                                                                                                 \
        float u = 0.0f;                                                                                   \
        if (GU) u = __shfl_sync(0xFFFFFFFFu, s, (lane + R * segs) & 31);                                  \
        if (valid && !mat && seg == 0 && n < nt)                                                          \
          a.out[(d0 + n) * a.N + row] = GU ? __fmul_rn(rq_silu(s), u) : s;                                \
      }                                                                                                   \
    }
    if (ntb == 1) RQ_BODY(1)
    else if (ntb == 2) RQ_BODY(2)
    else if (ntb == 4) RQ_BODY(4)
    else RQ_BODY(8)
#undef RQ_BODY
  }
}

}  // namespace rq

// rows per warp of the register-decoding GEMV (0: the type or shape goes to the staged kernel)
int gemv_rq_rows_per_warp(int qtype, int K, bool gu);

}  // namespace artlite
