// The streaming tensor-core decode GEMV for Q4_K weights and bf16 activations: device code of the fused decode kernel
// (decode.cu).
//
// Work: items (expert, group of 8 pairs, tile of rows), split over the CTAs; a CTA walks its items' 256-value
// super-block columns as steps. Each step's weights arrive in one of three shared-memory stages by TMA (one 2D tile per
// matrix: 64 gate and 64 up rows, or 128 down rows, one 144-byte super-block wide; completion counted on the stage's
// mbarrier), two steps in flight while one is computed. The 8 token slots' x for the column (pre-arranged as bf16 in
// the mma fragment order, with per-group sums) come from global memory (L2) with plain loads issued before the wait.
//
// The product: mma.sync m16n8k16 (bf16 x bf16 -> fp32), a warp per 16-row tile (and matrix), the 8 token slots as the
// n side. Lane (g = lane / 4, t = lane % 4) takes bytes 8t .. 8t + 7 of each 32-byte quant chunk of rows g and g + 8
// (chunk c: group 2c in the low nibbles, group 2c + 1 in the high ones) straight into A fragments by one LOP3 per two
// values, (q | 0x4300) = the bf16 value 128 + q exactly; within a 32-value group the k order is permuted (lane t's
// eight values fill its k slots 2t, 2t + 1, 2t + 8, 2t + 9 of two k16 steps) and x is arranged in the same order, so
// the dot products are unchanged. A group's scales apply after its two mma steps:
//   sum_j w_j x_j = (d sc) S - (128 d sc + dmin m) X,   S = sum_j (128 + q_j) x_j,   X = sum_j x_j,
// the reference's dequantised weight being w = (d sc) q - (dmin m) (gguf_model.py:278-330). Products are exact, the
// sums differ from the reference's fp32 order by rounding; x is the bf16 activation (for the down projection, h rounded
// to bf16, as on the tcgen05 path).
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "common.cuh"
#include "kernels.cuh"

namespace artlite {
namespace ms {

constexpr int kThreads = 256;
constexpr int kStages = 3;
constexpr int kRows = 128;                     // raw rows per step (gate 64 + up 64, or 128 down rows)
constexpr int kStageBytes = kRows * 144;       // 18432 (a multiple of 128: TMA destinations)
constexpr int kOutBytes = 3 * 64 * 8 * 4;      // gate / up tile outputs of an item (gu), and h
constexpr int kTabBytes = 8 * 16 * 8 * 8;      // per warp: 16 rows x 8 groups x {A, B}
constexpr long long kWaitCycles = 4000000000LL;  // about 2 s

__host__ __device__ constexpr size_t smem_bytes() { return (size_t)kStages * kStageBytes + kOutBytes + kTabBytes + 64; }

// the activations in fragment order: for token row r and 32-value group grp, xq[(r * G + grp) * 4 + t] = the words
// {x[8t], x[8t+2]}, {x[8t+1], x[8t+3]}, {x[8t+4], x[8t+6]}, {x[8t+5], x[8t+7]} of the group (bf16 pairs), and
// xs[r * G + grp] = the sum of the group's 32 bf16 values (fp32, fixed order)
__device__ __forceinline__ uint4 arrange(const float (&v)[8]) {
  uint32_t b[8];
#pragma unroll
  for (int j = 0; j < 8; j++) b[j] = __float_as_uint(v[j]) >> 16;  // (v are bf16 values)
  return make_uint4(b[0] | b[2] << 16, b[1] | b[3] << 16, b[4] | b[6] << 16, b[5] | b[7] << 16);
}

__device__ __forceinline__ uint32_t su32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t* b, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(su32(b)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect(uint64_t* b, unsigned bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(su32(b)), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_test(uint64_t* b, unsigned parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(su32(b)), "r"(parity)
      : "memory");
  return ok != 0;
}
// bounded wait for the phase of the given parity; false (reported) when it ran out
__device__ __forceinline__ bool mbar_wait(uint64_t* b, unsigned parity, DevStatus* st) {
  if (mbar_test(b, parity)) return true;
  const long long t0 = clock64();
  while (!mbar_test(b, parity))
    if (clock64() - t0 > kWaitCycles) {
      report(st, ARTLITE_ETIMEOUT, 20, (int)blockIdx.x);
      return false;
    }
  return true;
}
__device__ __forceinline__ void tma_load(void* dst, const CUtensorMap* map, uint64_t* b, int x, int y) {
  asm volatile("cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::
                   "r"(su32(dst)),
               "l"(map), "r"(su32(b)), "r"(x), "r"(y)
               : "memory");
}

__device__ __forceinline__ void mma_bf16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t nib2(uint32_t w) { return (w & 0x000F000Fu) | 0x43004300u; }
__device__ __forceinline__ float silu(float g) { return __fdiv_rn(g, __fadd_rn(1.0f, expf(-g))); }

struct Gemv {
  const CUtensorMap *m0, *m1;  // gate / up rows (gu: boxes of 64 rows) or down rows (128), raw Q4_K, E x N rows
  int K, N, E, k;          // K = 256 SB; N % rows_item == 0
  const uint4* xq;         // x in fragment order: token rows (gu) or pair rows (down), G = K / 32 groups per row
  const float* xs;         // their group sums
  // outputs: gu -> hq / hs (pair rows, fragment order, G_out = N / 32 groups); down -> y (pair rows, fp32, N wide)
  uint4* hq;
  float* hs;
  float* y;
};

struct Pipe {  // the CTA's stages: full (the copies landed: one arrival + bytes) and empty (every warp is done: 8
               // arrivals) mbarriers, and the parity each thread waits for next (bit i: stage i)
  uint64_t *full, *empty;
  unsigned full_parity, empty_parity;
  int* failed;   // (shared) set once a wait ran out: no more copies are started, no more results written
};

struct Step {
  int e, rt, sb, nt;
  int64_t d0;
};

template <bool GU>
__device__ __forceinline__ Step step_of(const Gemv& a, int s, int i0, const int32_t* uo, const int64_t* offs) {
  const int SB = a.K >> 8;
  const int rows_item = GU ? 64 : 128, ntile = a.N / rows_item;
  const int item = i0 + s / SB;
  int lo = 0, hi = a.E;
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (uo[mid] <= item) lo = mid; else hi = mid;
  }
  const int li = item - uo[lo], tg = li / ntile;
  Step st;
  st.e = lo;
  st.rt = li - tg * ntile;
  st.sb = s - (s / SB) * SB;
  st.d0 = offs[lo] + (int64_t)tg * kGemvTokens;
  st.nt = (int)min64(kGemvTokens, offs[lo + 1] - st.d0);
  return st;
}

// the TMA copies of a step into stage buffer buf (thread 0, after announcing kStageBytes)
template <bool GU>
__device__ __forceinline__ void issue(const Gemv& a, const Step& st, uint8_t* buf, uint64_t* bar) {
  const int y = st.e * a.N + st.rt * (GU ? 64 : 128);
  tma_load(buf, a.m0, bar, st.sb * 72, y);
  if (GU) tma_load(buf + 64 * 144, a.m1, bar, st.sb * 72, y);
}

// x of a step for this lane: the B fragments of token slot g for the column's 8 groups, and the group sums of slots
// 2t, 2t + 1 (slots past nt read slot 0's row: their products are discarded)
struct XFrag {
  uint4 b[8];
  float4 s[2][2];
};

template <bool GU>
__device__ __forceinline__ void load_x(const Gemv& a, const Step& st, const int32_t* perm, int lane, XFrag& x) {
  const int g = lane >> 2, t = lane & 3;
  const int G = a.K >> 5;
  auto row_of = [&](int n) -> int64_t {
    n = n < st.nt ? n : 0;
    return GU ? (int64_t)(perm[st.d0 + n] / a.k) : st.d0 + n;
  };
  const uint4* xr = a.xq + (row_of(g) * G + st.sb * 8) * 4 + t;
#pragma unroll
  for (int j = 0; j < 8; j++) x.b[j] = __ldcg(xr + 4 * j);
#pragma unroll
  for (int i = 0; i < 2; i++) {
    const float4* sr = reinterpret_cast<const float4*>(a.xs + row_of(2 * t + i) * G + st.sb * 8);
    x.s[i][0] = __ldcg(sr);
    x.s[i][1] = __ldcg(sr + 1);
  }
}

// this warp's 16-row tile x one super-block column: accumulates y (rows g, g + 8 x tokens 2t, 2t + 1)
__device__ __forceinline__ float f4at(const float4 (&v)[2], int j) {
  const float4 q = v[j >> 2];
  return (j & 3) == 0 ? q.x : (j & 3) == 1 ? q.y : (j & 3) == 2 ? q.z : q.w;
}

__device__ __forceinline__ void tile_sb(const uint8_t* rows, const XFrag& x, float* tab, int lane, float (&y)[4]) {
  const int g = lane >> 2, t = lane & 3;
  // scales of rows (g, g + 8) x groups (2t, 2t + 1) into the warp's table. The twelve scale bytes q0 .. q11 hold the
  // six-bit scale / min of group j < 4 in q[j] / q[j + 4] (low six bits) and of j >= 4 in the nibbles of q[j + 4] with
  // the top two bits of q[j - 4] / q[j]: as packed bytes, sc(0..3) = w1 & 0x3F.., sc(4..7) = (w3 & 0x0F..) |
  // ((w1 & 0xC0..) >> 2), mn(0..3) = w2 & 0x3F.., mn(4..7) = ((w3 >> 4) & 0x0F..) | ((w2 & 0xC0..) >> 2).
#pragma unroll
  for (int i = 0; i < 2; i++) {
    const uint4 h = *reinterpret_cast<const uint4*>(rows + (g + 8 * i) * 144);
    const float d = __half2float(__ushort_as_half((unsigned short)(h.x & 0xFFFFu)));
    const float dmin = __half2float(__ushort_as_half((unsigned short)(h.x >> 16)));
    const uint32_t sc_w = t < 2 ? (h.y & 0x3F3F3F3Fu) : ((h.w & 0x0F0F0F0Fu) | ((h.y & 0xC0C0C0C0u) >> 2));
    const uint32_t mn_w = t < 2 ? (h.z & 0x3F3F3F3Fu) : (((h.w >> 4) & 0x0F0F0F0Fu) | ((h.z & 0xC0C0C0C0u) >> 2));
    const int sh = 16 * (t & 1);
#pragma unroll
    for (int jj = 0; jj < 2; jj++) {
      const float sc = (float)((sc_w >> (sh + 8 * jj)) & 0xFFu), mn = (float)((mn_w >> (sh + 8 * jj)) & 0xFFu);
      const float dsc = __fmul_rn(d, sc), dmn = __fmul_rn(dmin, mn);
      reinterpret_cast<float2*>(tab)[(g + 8 * i) * 8 + 2 * t + jj] = make_float2(dsc, __fmaf_rn(128.0f, dsc, dmn));
    }
  }
  __syncwarp();
#pragma unroll
  for (int c = 0; c < 4; c++) {
    const uint2 q0 = *reinterpret_cast<const uint2*>(rows + g * 144 + 16 + 32 * c + 8 * t);
    const uint2 q1 = *reinterpret_cast<const uint2*>(rows + (g + 8) * 144 + 16 + 32 * c + 8 * t);
#pragma unroll
    for (int p = 0; p < 2; p++) {
      const int j = 2 * c + p, sh = 4 * p;
      const uint4 bx = x.b[j];
      const float x0 = f4at(x.s[0], j), x1 = f4at(x.s[1], j);
      uint32_t a0[4], a1[4];
      a0[0] = nib2(q0.x >> sh), a0[1] = nib2(q1.x >> sh), a0[2] = nib2(q0.x >> (sh + 8)), a0[3] = nib2(q1.x >> (sh + 8));
      a1[0] = nib2(q0.y >> sh), a1[1] = nib2(q1.y >> sh), a1[2] = nib2(q0.y >> (sh + 8)), a1[3] = nib2(q1.y >> (sh + 8));
      float acc[4] = {0, 0, 0, 0};
      mma_bf16(acc, a0, bx.x, bx.y);
      mma_bf16(acc, a1, bx.z, bx.w);
      const float2 s0 = reinterpret_cast<const float2*>(tab)[g * 8 + j];
      const float2 s8 = reinterpret_cast<const float2*>(tab)[(g + 8) * 8 + j];
      y[0] = fmaf(s0.x, acc[0], fmaf(-s0.y, x0, y[0]));
      y[1] = fmaf(s0.x, acc[1], fmaf(-s0.y, x1, y[1]));
      y[2] = fmaf(s8.x, acc[2], fmaf(-s8.y, x0, y[2]));
      y[3] = fmaf(s8.x, acc[3], fmaf(-s8.y, x1, y[3]));
    }
  }
  __syncwarp();
}

// Items [i0, i1) of one GEMV (gu: 64 output rows an item, gate and up; down: 128 rows). Every thread of the CTA calls
// it; smem (128-byte aligned): the stages, the output tile, the per-warp tables (smem_bytes()). x must be complete in
// global memory (a grid barrier before). Thread 0 starts the copies: a stage is refilled once its empty barrier shows
// every warp done with it; the warps otherwise run ahead of one another by up to the stages in flight.
template <bool GU>
__device__ __forceinline__ void run(const Gemv& a, const int32_t* uo, const int64_t* offs, const int32_t* perm,
                                   uint8_t* smem, Pipe& pp, int i0, int i1, DevStatus* status) {
  static_assert(kThreads == 256, "8 warps");
  const int SB = a.K >> 8;
  const int S = (i1 - i0) * SB;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  float* out = reinterpret_cast<float*>(smem + kStages * kStageBytes);  // [2][64][8]
  float* tab = reinterpret_cast<float*>(smem + kStages * kStageBytes + kOutBytes) + warp * 16 * 8 * 2;
  if (S <= 0) return;
  if ((su32(smem) & 127u) != 0) {  // (TMA destinations: never issued to a misaligned stage)
    if (threadIdx.x == 0) {
      report(status, ARTLITE_EUNSUPPORTED, 128, 0, 0);
      *pp.failed = 1;
    }
    __syncthreads();
    return;
  }
  const bool producer = threadIdx.x == 0;
  // prologue: steps 0 .. kStages - 1 (the stages are free: the previous user waited for every copy it started)
  int issued = 0;
  if (producer && !*pp.failed)
    for (int s = 0; s < kStages && s < S; s++) {
      mbar_expect(&pp.full[s], kStageBytes);
      issue<GU>(a, step_of<GU>(a, s, i0, uo, offs), smem + s * kStageBytes, &pp.full[s]);
      issued = s + 1;
    }
  float y[4] = {0, 0, 0, 0};
  const int tile = GU ? warp >> 1 : warp, mat = GU ? warp & 1 : 0;
  int waited = 0;  // (producer: steps whose copies are known complete)
  for (int s = 0; s < S; s++) {
    const int b = s % kStages;
    const Step st = step_of<GU>(a, s, i0, uo, offs);
    uint8_t* buf = smem + b * kStageBytes;
    XFrag xf;
    load_x<GU>(a, st, perm, lane, xf);
    bool ok = !*(volatile int*)pp.failed;
    if (ok) {
      ok = mbar_wait(&pp.full[b], (pp.full_parity >> b) & 1u, status);
      if (!ok) *(volatile int*)pp.failed = 1;
    }
    pp.full_parity ^= 1u << b;
    ok = __all_sync(0xFFFFFFFFu, ok);
    if (producer && ok) waited = s + 1;
    if (ok) tile_sb(buf + (mat * 64 + tile * 16) * 144, xf, tab, lane, y);
    __syncwarp();
    if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(su32(&pp.empty[b])) : "memory");
    if (st.sb == SB - 1) {  // the item's last column: its outputs (every warp meets here)
      const int g = lane >> 2, t = lane & 3;
      const bool good = !*(volatile int*)pp.failed;
      if (GU) {
        float* o = out + mat * 64 * 8;
        o[(tile * 16 + g) * 8 + 2 * t] = y[0];
        o[(tile * 16 + g) * 8 + 2 * t + 1] = y[1];
        o[(tile * 16 + g + 8) * 8 + 2 * t] = y[2];
        o[(tile * 16 + g + 8) * 8 + 2 * t + 1] = y[3];
        __syncthreads();
        float* hb = out + 2 * 64 * 8;  // [8 tokens][64 rows]: h rounded to bf16
        for (int v = threadIdx.x; v < 64 * 8; v += kThreads) {
          const int r = v >> 3, n = v & 7;
          hb[n * 64 + r] = __bfloat162float(__float2bfloat16_rn(__fmul_rn(silu(out[r * 8 + n]), out[64 * 8 + r * 8 + n])));
        }
        __syncthreads();
        if (threadIdx.x < 64) {  // (n, group of 32 rows, t): 8 h values in fragment order, and the group sum
          const int n = threadIdx.x >> 3, grp = (threadIdx.x >> 2) & 1, tq = threadIdx.x & 3;
          const float4 h0 = *reinterpret_cast<const float4*>(hb + n * 64 + grp * 32 + 8 * tq);
          const float4 h1 = *reinterpret_cast<const float4*>(hb + n * 64 + grp * 32 + 8 * tq + 4);
          const float v[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
          float part = ((v[0] + v[1]) + (v[2] + v[3])) + ((v[4] + v[5]) + (v[6] + v[7]));
          part += __shfl_xor_sync(0xFFFFFFFFu, part, 1);
          part += __shfl_xor_sync(0xFFFFFFFFu, part, 2);
          if (n < st.nt && good) {
            const int Go = a.N >> 5;
            const int64_t pr = st.d0 + n;
            const int og = st.rt * 2 + grp;
            a.hq[(pr * Go + og) * 4 + tq] = arrange(v);
            if (tq == 0) a.hs[pr * Go + og] = part;
          }
        }
        __syncthreads();  // (out is free again)
      } else if (good) {
        const int64_t row = (int64_t)st.rt * 128 + tile * 16 + g;
        if (2 * t < st.nt) {
          a.y[(st.d0 + 2 * t) * a.N + row] = y[0];
          a.y[(st.d0 + 2 * t) * a.N + row + 8] = y[2];
        }
        if (2 * t + 1 < st.nt) {
          a.y[(st.d0 + 2 * t + 1) * a.N + row] = y[1];
          a.y[(st.d0 + 2 * t + 1) * a.N + row + 8] = y[3];
        }
      }
      y[0] = y[1] = y[2] = y[3] = 0.0f;
    }
    // the producer refills this stage with step s + kStages once every warp is done with it
    if (producer) {
      const int s2 = s + kStages;
      bool free_ok = true;
      if (s < issued) {  // (its empty phase for step s completes when all 8 warps arrived)
        free_ok = !*(volatile int*)pp.failed && mbar_wait(&pp.empty[b], (pp.empty_parity >> b) & 1u, status);
        pp.empty_parity ^= 1u << b;
        if (!free_ok) *(volatile int*)pp.failed = 1;
      }
      if (s2 < S && free_ok && !*(volatile int*)pp.failed) {
        mbar_expect(&pp.full[b], kStageBytes);
        issue<GU>(a, step_of<GU>(a, s2, i0, uo, offs), buf, &pp.full[b]);
        issued = s2 + 1;
      }
    }
  }
  // after a failure: wait (bounded) for the copies already started, so that none lands in a stage after this
  if (producer)
    for (int s = waited; s < issued; s++) {
      const int b = s % kStages;
      if (!mbar_test(&pp.full[b], (pp.full_parity >> b) & 1u)) mbar_wait(&pp.full[b], (pp.full_parity >> b) & 1u, status);
    }
  __syncthreads();
}

}  // namespace ms
}  // namespace artlite
