// GGUF block decoding on the device, fp32 and exact: the reference's fp32 operations in their order
// (csrc/artlite/dequant.cpp:21-140, itself built with -ffp-contract=off), written with the _rn intrinsics so that
// nvcc contracts nothing into an FMA. Every product here has at most 21 significant bits, so the values are exact.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "../../include/artlite_moe.h"

namespace artlite {

__device__ __forceinline__ float f16_at(const uint8_t* p) {
  const unsigned short h = (unsigned short)(p[0] | (p[1] << 8));
  return __half2float(__ushort_as_half(h));
}

// Q4_0 (dequant.cpp:40-47): 18 B per 32, w = (q - 8) d; values 0..15 the low nibbles of bytes 2..17, 16..31 the high
__device__ __forceinline__ void dq_q4_0(const uint8_t* b, float* o) {
  const float d = f16_at(b);
#pragma unroll
  for (int j = 0; j < 16; j++) {
    const int c = b[2 + j];
    o[j] = __fmul_rn(__fsub_rn((float)(c & 15), 8.0f), d);
    o[j + 16] = __fmul_rn(__fsub_rn((float)(c >> 4), 8.0f), d);
  }
}

// Q4_1 (dequant.cpp:49-56): 20 B per 32, w = d q + m
__device__ __forceinline__ void dq_q4_1(const uint8_t* b, float* o) {
  const float d = f16_at(b), m = f16_at(b + 2);
#pragma unroll
  for (int j = 0; j < 16; j++) {
    const int c = b[4 + j];
    o[j] = __fadd_rn(__fmul_rn(d, (float)(c & 15)), m);
    o[j + 16] = __fadd_rn(__fmul_rn(d, (float)(c >> 4)), m);
  }
}

// Q8_0 (dequant.cpp:58-62): 34 B per 32, w = d q, q int8
__device__ __forceinline__ void dq_q8_0(const uint8_t* b, float* o) {
  const float d = f16_at(b);
#pragma unroll
  for (int j = 0; j < 32; j++) o[j] = __fmul_rn(d, (float)(int8_t)b[2 + j]);
}

// Q4_K / Q5_K scale and min of 32-group g (dequant.cpp:70-73): six bits each, packed in 12 bytes at b + 4
__device__ __forceinline__ void k_scale_min(const uint8_t* b, int g, int* sc, int* mn) {
  const uint8_t *lo = b + 4, *hi = b + 8, *top = b + 12;
  if (g < 4) {
    *sc = lo[g] & 63;
    *mn = hi[g] & 63;
  } else {
    *sc = (top[g - 4] & 15) | (lo[g - 4] >> 6) << 4;
    *mn = (top[g - 4] >> 4) | (hi[g - 4] >> 6) << 4;
  }
}

// Q4_K / Q5_K 32-group g of a 256 super-block (dequant.cpp:64-81): w = q (d sc_g) - dmin mn_g
template <bool Q5>
__device__ __forceinline__ void dq_k45_group(const uint8_t* b, int g, float* o) {
  const float d = f16_at(b), dmin = f16_at(b + 2);
  int sc, mn;
  k_scale_min(b, g, &sc, &mn);
  const float dsc = __fmul_rn(d, (float)sc), dmn = __fmul_rn(dmin, (float)mn);
  const uint8_t* qs = b + (Q5 ? 48 : 16) + 32 * (g >> 1);
  const uint8_t* qh = b + 16;
#pragma unroll
  for (int l = 0; l < 32; l++) {
    int q = (g & 1) ? (qs[l] >> 4) : (qs[l] & 15);
    if (Q5) q |= ((qh[l] >> g) & 1) << 4;
    o[l] = __fsub_rn(__fmul_rn((float)q, dsc), dmn);
  }
}

// Q6_K 32-group g (dequant.cpp:83-101): w = (q - 32) (sc_j d), sc per 16
__device__ __forceinline__ void dq_q6_k_group(const uint8_t* b, int g, float* o) {
  const int h = g >> 2, jj = g & 3;
  const uint8_t* c = b + 64 * h + 32 * (jj & 1);
  const uint8_t* e = b + 128 + 32 * h;
  const int8_t* sc = reinterpret_cast<const int8_t*>(b + 192);
  const float d = f16_at(b + 208);
  const int sh = jj < 2 ? 0 : 4;
  const float s0 = __fmul_rn((float)sc[8 * h + 2 * jj], d), s1 = __fmul_rn((float)sc[8 * h + 2 * jj + 1], d);
#pragma unroll
  for (int l = 0; l < 32; l++) {
    const int q = (((c[l] >> sh) & 15) | ((e[l] >> (2 * jj)) & 3) << 4) - 32;
    o[l] = __fmul_rn((float)q, l < 16 ? s0 : s1);
  }
}

// Q3_K 16-value sub-block s (dequant.cpp:103-117): 110 B per 256 = hmask[32], qs[64], 12 scale bytes, d (fp16 at
// 108). Its 6-bit scale (stored + 32): low nibble of byte s (s < 8) or high nibble of byte s - 8, top crumb from byte
// 8 + s % 4 at bit 2 (s / 4). Value 16 s + l = 128 n + 32 j + i: q = crumb j of qs[32 n + i] | bit (4 n + j) of
// hmask[i] << 2, w = (d (scale - 32)) (q - 4)
__device__ __forceinline__ void dq_q3_k_sub(const uint8_t* b, int s, float* o) {
  const uint8_t* sc = b + 96;
  const int low = s < 8 ? sc[s] & 15 : sc[s - 8] >> 4, top = (sc[8 + (s & 3)] >> (2 * (s >> 2))) & 3;
  const float a = __fmul_rn(f16_at(b + 108), (float)((low | top << 4) - 32));
  const int n = s >> 3, j = (s >> 1) & 3, i0 = 16 * (s & 1);
#pragma unroll
  for (int l = 0; l < 16; l++) {
    const int q = ((b[32 + 32 * n + i0 + l] >> (2 * j)) & 3) | ((b[i0 + l] >> (4 * n + j)) & 1) << 2;
    o[l] = __fmul_rn(a, __fsub_rn((float)q, 4.0f));
  }
}

// the IQ4_NL / IQ4_XS code values (dequant.cpp:119, ggml's non-linear 4-bit grid), as a byte lookup
__device__ __forceinline__ float iq4_value(int q) {
  constexpr int8_t v[16] = {-127, -104, -83, -65, -49, -35, -22, -10, 1, 13, 25, 38, 53, 69, 89, 113};
  return (float)v[q];
}

// IQ4_NL (dequant.cpp:121-126): 18 B per 32, Q4_0's layout, w = d grid[q]
__device__ __forceinline__ void dq_iq4_nl(const uint8_t* b, float* o) {
  const float d = f16_at(b);
#pragma unroll
  for (int j = 0; j < 16; j++) {
    const int c = b[2 + j];
    o[j] = __fmul_rn(d, iq4_value(c & 15));
    o[j + 16] = __fmul_rn(d, iq4_value(c >> 4));
  }
}

// IQ4_XS 32-group g (dequant.cpp:128-140): 136 B per 256 = d, a u16 of high scale crumbs, 4 bytes of low scale
// nibbles, 8 x 16 code bytes; ls = nibble (g % 2) of byte 4 + g / 2 | crumb g of the u16 << 4, w = (d (ls - 32)) grid[q]
__device__ __forceinline__ void dq_iq4_xs_group(const uint8_t* b, int g, float* o) {
  const int hi = b[2] | b[3] << 8;
  const int ls = ((b[4 + (g >> 1)] >> (4 * (g & 1))) & 15) | ((hi >> (2 * g)) & 3) << 4;
  const float dl = __fmul_rn(f16_at(b), (float)(ls - 32));
  const uint8_t* q = b + 8 + 16 * g;
#pragma unroll
  for (int j = 0; j < 16; j++) {
    o[j] = __fmul_rn(dl, iq4_value(q[j] & 15));
    o[j + 16] = __fmul_rn(dl, iq4_value(q[j] >> 4));
  }
}

// values and bytes per block of a GGUF type (0: not read by this build)
__host__ __device__ constexpr int q_per(int qt) {
  return qt == ARTLITE_Q4_0 || qt == ARTLITE_Q4_1 || qt == ARTLITE_Q8_0 || qt == ARTLITE_IQ4_NL ? 32
         : (qt == ARTLITE_Q3_K || qt == ARTLITE_Q4_K || qt == ARTLITE_Q5_K || qt == ARTLITE_Q6_K || qt == ARTLITE_IQ4_XS)
             ? 256
         : (qt == ARTLITE_F32 || qt == ARTLITE_F16 || qt == ARTLITE_BF16) ? 1
                                                                          : 0;
}
__host__ __device__ constexpr int q_bytes(int qt) {
  return qt == ARTLITE_Q4_0 ? 18 : qt == ARTLITE_Q4_1 ? 20 : qt == ARTLITE_Q8_0 ? 34 : qt == ARTLITE_Q4_K ? 144
         : qt == ARTLITE_Q5_K ? 176 : qt == ARTLITE_Q6_K ? 210 : qt == ARTLITE_Q3_K ? 110 : qt == ARTLITE_IQ4_NL ? 18
         : qt == ARTLITE_IQ4_XS ? 136 : qt == ARTLITE_F32 ? 4
         : (qt == ARTLITE_F16 || qt == ARTLITE_BF16) ? 2 : 0;
}

// 32 consecutive values of a row, starting at value 32 g (g: the row's 32-group), decoded from the row's raw bytes
template <int QT>
__device__ __forceinline__ void dq_group(const uint8_t* row, int g, float* o) {
  if constexpr (QT == ARTLITE_Q4_0) {
    dq_q4_0(row + 18 * g, o);
  } else if constexpr (QT == ARTLITE_Q4_1) {
    dq_q4_1(row + 20 * g, o);
  } else if constexpr (QT == ARTLITE_Q8_0) {
    dq_q8_0(row + 34 * g, o);
  } else if constexpr (QT == ARTLITE_Q4_K) {
    dq_k45_group<false>(row + 144 * (g >> 3), g & 7, o);
  } else if constexpr (QT == ARTLITE_Q5_K) {
    dq_k45_group<true>(row + 176 * (g >> 3), g & 7, o);
  } else if constexpr (QT == ARTLITE_Q6_K) {
    dq_q6_k_group(row + 210 * (g >> 3), g & 7, o);
  } else if constexpr (QT == ARTLITE_Q3_K) {
    dq_q3_k_sub(row + 110 * (g >> 3), 2 * (g & 7), o);
    dq_q3_k_sub(row + 110 * (g >> 3), 2 * (g & 7) + 1, o + 16);
  } else if constexpr (QT == ARTLITE_IQ4_NL) {
    dq_iq4_nl(row + 18 * g, o);
  } else if constexpr (QT == ARTLITE_IQ4_XS) {
    dq_iq4_xs_group(row + 136 * (g >> 3), g & 7, o);
  } else if constexpr (QT == ARTLITE_F32) {
#pragma unroll
    for (int j = 0; j < 32; j++) o[j] = reinterpret_cast<const float*>(row)[32 * g + j];
  } else if constexpr (QT == ARTLITE_F16) {
#pragma unroll
    for (int j = 0; j < 32; j++) o[j] = f16_at(row + 2 * (32 * g + j));
  } else {  // BF16
#pragma unroll
    for (int j = 0; j < 32; j++) {
      const uint8_t* p = row + 2 * (32 * g + j);
      o[j] = __uint_as_float((uint32_t)(p[0] | (p[1] << 8)) << 16);
    }
  }
}

}  // namespace artlite
