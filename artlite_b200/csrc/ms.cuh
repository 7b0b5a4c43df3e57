// The streaming tensor-core decode GEMV for Q4_K weights and bf16 activations: device code of the fused decode kernel
// (decode.cu).
//
// Work: items (expert, group of 8 pairs, tile of rows), split over the CTAs; a CTA walks its items' 256-value
// super-block columns as steps. Each step arrives in one of three shared-memory stages, its completion counted on the
// stage's mbarrier: the weights by TMA (one 2D tile per matrix: 64 gate and 64 up rows, or 128 down rows, one 144-byte
// super-block wide) and the 8 token slots' x for the column (pre-arranged as bf16 in the mma fragment order, with
// per-group sums) by the refilling warp's cp.async (16 bytes a lane, their completion arriving on the same mbarrier),
// so that no warp waits on a global load inside a step and the CTA reads x once, not once per warp. Two steps are in
// flight while one is computed; the last warp done with a stage refills it.
//
// The product: mma.sync m16n8k16 (bf16 x bf16 -> fp32), a warp per 16-row tile, the 8 token slots as the n side. For
// gate / up the tile's rows 0-7 are 8 gate rows and rows 8-15 the same 8 up rows, so that a lane holds gate and up of
// one output row and applies silu(gate) x up in registers. Lane (g = lane / 4, t = lane % 4) takes bytes 8t .. 8t + 7
// of each 32-byte quant chunk of its two rows (chunk c: group 2c in the low nibbles, group 2c + 1 in the high ones)
// straight into A fragments by one LOP3 per two values, (q | 0x4300) = the bf16 value 128 + q exactly; within a
// 32-value group the k order is permuted (lane t's eight values fill its k slots 2t, 2t + 1, 2t + 8, 2t + 9 of two k16
// steps) and x is arranged in the same order, so the dot products are unchanged. A group's scales apply after its two
// mma steps:
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
constexpr int kWBytes = kRows * 144;           // 18432: the step's weights
constexpr int kXRow = 528;                     // a token slot's x in the stage: 512 bytes + 16 of padding (banks)
constexpr int kXOff = kWBytes;                 // 8 slots x kXRow
constexpr int kSOff = kXOff + 8 * kXRow;       // 8 slots x 8 group sums (32 bytes)
constexpr int kStageBytes = kSOff + 8 * 32;    // 22912 (a multiple of 128: TMA destinations)
constexpr unsigned kFullArrivals = 33;         // a stage's full barrier: the refiller's expect_tx + 32 lanes' cp.async
constexpr int kOutBytes = 2 * 64 * 8 * 4;      // h of an item (gu), [8 tokens][64 rows], two buffers
constexpr int kTabRow = 9;                     // a row's {A, B} pairs: 8 groups + 1 of padding (banks)
constexpr int kTabBytes = 8 * 16 * kTabRow * 8;  // per warp: 16 rows x 8 groups x {A, B}
static_assert(kStageBytes % 128 == 0, "stages start 128-byte aligned");
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

// 16 bytes global -> shared (L2 only), asynchronous
__device__ __forceinline__ void cp16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(su32(dst)), "l"(src) : "memory");
}
// one arrival on b once this thread's earlier cp.async copies have landed (counted in the barrier's init count)
__device__ __forceinline__ void cp_arrive(uint64_t* b) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(su32(b)) : "memory");
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
  int natural;  // gu: h in the mma's natural k order (for a Q6_K down kernel), else this tile's order
};

struct Pipe {  // the CTA's stages: full mbarriers (the copies landed: one arrival + bytes) and the parity each thread
               // waits for next (bit i: stage i); per stage a count of the warps done with its current step (shared)
  uint64_t* full;
  unsigned full_parity;
  int* done;     // [kStages]: the warp that makes it 8 resets it and refills the stage
  int* issued;   // (shared) steps whose copies were started in the current run
  int* failed;   // (shared) set once a wait ran out: no more copies are started, no more results written
};

// an item: expert e, row tile rt, its pairs [d0, d0 + nt) in dispatch order (nt <= 8)
struct Item {
  int e, rt, nt;
  int64_t d0;
};

// the item's fields; e is a hint at or below its expert (items ascend, so a forward scan finds it)
template <bool GU>
__device__ __forceinline__ Item item_at(const Gemv& a, int item, int& e, const int32_t* uo, const int64_t* offs) {
  while (uo[e + 1] <= item) e++;
  const int ntile = a.N / (GU ? 64 : 128);
  const int li = item - uo[e], tg = li / ntile;
  Item it;
  it.e = e;
  it.rt = li - tg * ntile;
  it.d0 = offs[e] + (int64_t)tg * kGemvTokens;
  it.nt = (int)min64(kGemvTokens, offs[e + 1] - it.d0);
  return it;
}

// the expert of item i0 (binary search over the item offsets)
__device__ __forceinline__ int expert_of(int item, int E, const int32_t* uo) {
  int lo = 0, hi = E;
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (uo[mid] <= item) lo = mid; else hi = mid;
  }
  return lo;
}

// the copies of step (it, sb) into stage buffer buf, completing on bar; a whole warp calls it: lane 0 announces the
// weight bytes and starts the weight tiles (TMA), every lane copies 16 bytes of each token slot's 512 bytes of x and
// lanes 0-15 the slots' 32 bytes of group sums, then arrives once its copies land (slots past nt copy slot 0's row:
// their products are discarded)
template <bool GU>
__device__ __forceinline__ void refill(const Gemv& a, const Item& it, int sb, const int32_t* perm, uint8_t* buf,
                                       uint64_t* bar, int lane) {
  if (lane == 0) {
    const int y = it.e * a.N + it.rt * (GU ? 64 : 128);
    mbar_expect(bar, kWBytes);
    tma_load(buf, a.m0, bar, sb * 72, y);
    if (GU) tma_load(buf + 64 * 144, a.m1, bar, sb * 72, y);
  }
  const int G = a.K >> 5;
  const int n = lane & 7;
  const int64_t d = it.d0 + (n < it.nt ? n : 0);
  const int64_t my_row = GU ? (int64_t)(perm[d] / a.k) : d;  // (slot lane & 7's x row)
#pragma unroll
  for (int i = 0; i < 8; i++) {
    const int64_t row = __shfl_sync(0xFFFFFFFFu, my_row, i);
    cp16(buf + kXOff + i * kXRow + lane * 16, a.xq + (row * G + sb * 8) * 4 + lane);
  }
  const int64_t srow = __shfl_sync(0xFFFFFFFFu, my_row, (lane >> 1) & 7);
  if (lane < 16) cp16(buf + kSOff + (lane >> 1) * 32 + (lane & 1) * 16, a.xs + srow * G + sb * 8 + (lane & 1) * 4);
  cp_arrive(bar);
}

// x of a step for this lane, from the stage: the B fragments of token slot g for the column's 8 groups, and the group
// sums of slots 2t, 2t + 1
struct XFrag {
  uint4 b[8];
  float4 s[2][2];
};

__device__ __forceinline__ void load_x(const uint8_t* buf, int lane, XFrag& x) {
  const int g = lane >> 2, t = lane & 3;
  const uint4* xr = reinterpret_cast<const uint4*>(buf + kXOff + g * kXRow) + t;
#pragma unroll
  for (int j = 0; j < 8; j++) x.b[j] = xr[4 * j];
#pragma unroll
  for (int i = 0; i < 2; i++) {
    const float4* sr = reinterpret_cast<const float4*>(buf + kSOff + (2 * t + i) * 32);
    x.s[i][0] = sr[0];
    x.s[i][1] = sr[1];
  }
}

// the physical row (of 8) that tile row g reads: rows 0-3 of the tile from the even rows, 4-7 from the odd ones, so
// that each half-warp's 8-byte loads of a 144-byte-stride tile fall on 32 distinct banks
__device__ __forceinline__ int prow(int g) { return ((g & 3) << 1) | (g >> 2); }

// this warp's 16-row tile x one super-block column: tile rows 0-7 at lo, 8-15 at hi (144-byte rows, tile row g reading
// physical row prow(g)); accumulates y (tile rows g, g + 8 x tokens 2t, 2t + 1)
__device__ __forceinline__ float f4at(const float4 (&v)[2], int j) {
  const float4 q = v[j >> 2];
  return (j & 3) == 0 ? q.x : (j & 3) == 1 ? q.y : (j & 3) == 2 ? q.z : q.w;
}

__device__ __forceinline__ void tile_sb(const uint8_t* lo, const uint8_t* hi, const XFrag& x, float* tab, int lane,
                                        float (&y)[4]) {
  const int g = lane >> 2, t = lane & 3;
  const uint8_t* r0 = lo + prow(g) * 144;
  const uint8_t* r1 = hi + prow(g) * 144;
  // scales of rows (g, g + 8) x groups (2t, 2t + 1) into the warp's table. The twelve scale bytes q0 .. q11 hold the
  // six-bit scale / min of group j < 4 in q[j] / q[j + 4] (low six bits) and of j >= 4 in the nibbles of q[j + 4] with
  // the top two bits of q[j - 4] / q[j]: as packed bytes, sc(0..3) = w1 & 0x3F.., sc(4..7) = (w3 & 0x0F..) |
  // ((w1 & 0xC0..) >> 2), mn(0..3) = w2 & 0x3F.., mn(4..7) = ((w3 >> 4) & 0x0F..) | ((w2 & 0xC0..) >> 2).
#pragma unroll
  for (int i = 0; i < 2; i++) {
    const uint4 h = *reinterpret_cast<const uint4*>(i ? r1 : r0);
    const float d = __half2float(__ushort_as_half((unsigned short)(h.x & 0xFFFFu)));
    const float dmin = __half2float(__ushort_as_half((unsigned short)(h.x >> 16)));
    const uint32_t sc_w = t < 2 ? (h.y & 0x3F3F3F3Fu) : ((h.w & 0x0F0F0F0Fu) | ((h.y & 0xC0C0C0C0u) >> 2));
    const uint32_t mn_w = t < 2 ? (h.z & 0x3F3F3F3Fu) : (((h.w >> 4) & 0x0F0F0F0Fu) | ((h.z & 0xC0C0C0C0u) >> 2));
    const int sh = 16 * (t & 1);
#pragma unroll
    for (int jj = 0; jj < 2; jj++) {
      const float sc = (float)((sc_w >> (sh + 8 * jj)) & 0xFFu), mn = (float)((mn_w >> (sh + 8 * jj)) & 0xFFu);
      const float dsc = __fmul_rn(d, sc), dmn = __fmul_rn(dmin, mn);
      reinterpret_cast<float2*>(tab)[(g + 8 * i) * kTabRow + 2 * t + jj] = make_float2(dsc, __fmaf_rn(128.0f, dsc, dmn));
    }
  }
  __syncwarp();
#pragma unroll
  for (int c = 0; c < 4; c++) {
    const uint2 q0 = *reinterpret_cast<const uint2*>(r0 + 16 + 32 * c + 8 * t);
    const uint2 q1 = *reinterpret_cast<const uint2*>(r1 + 16 + 32 * c + 8 * t);
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
      const float2 s0 = reinterpret_cast<const float2*>(tab)[g * kTabRow + j];
      const float2 s8 = reinterpret_cast<const float2*>(tab)[(g + 8) * kTabRow + j];
      y[0] = fmaf(s0.x, acc[0], fmaf(-s0.y, x0, y[0]));
      y[1] = fmaf(s0.x, acc[1], fmaf(-s0.y, x1, y[1]));
      y[2] = fmaf(s8.x, acc[2], fmaf(-s8.y, x0, y[2]));
      y[3] = fmaf(s8.x, acc[3], fmaf(-s8.y, x1, y[3]));
    }
  }
  __syncwarp();
}

// Items [i0, i1) of one GEMV (gu: 64 output rows an item, gate and up; down: 128 rows). Every thread of the CTA calls
// it; smem (128-byte aligned): the stages, the h buffers, the per-warp tables (smem_bytes()). x must be complete in
// global memory (a grid barrier before). Thread 0 starts the first copies; afterwards the last warp to finish with a
// stage refills it with the step kStages ahead (no waiting producer: the copy starts the moment the stage is free, and
// no warp both computes and waits for the others); the warps otherwise run ahead of one another by up to the stages in
// flight.
template <bool GU>
__device__ __forceinline__ void run(const Gemv& a, const int32_t* uo, const int64_t* offs, const int32_t* perm,
                                   uint8_t* smem, Pipe& pp, int i0, int i1, DevStatus* status) {
  static_assert(kThreads == 256, "8 warps");
  const int SB = a.K >> 8;
  const int S = (i1 - i0) * SB;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  float* out = reinterpret_cast<float*>(smem + kStages * kStageBytes);  // [2][8 tokens][64 rows]
  float* tab = reinterpret_cast<float*>(smem + kStages * kStageBytes + kOutBytes) + warp * 16 * kTabRow * 2;
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
  int e_run = expert_of(i0, a.E, uo);  // (the compute side's expert hint)
  int e_fill = e_run;                  // (this warp's hint for the refills it issues)
  // prologue (warp 0): steps 0 .. kStages - 1 (the stages are free: the previous user waited for every copy it started)
  if (warp == 0) {
    const bool go = !*(volatile int*)pp.failed;
    int n = 0;
    if (go)
      for (int s = 0; s < kStages && s < S; s++, n++)
        refill<GU>(a, item_at<GU>(a, i0 + s / SB, e_fill, uo, offs), s % SB, perm, smem + s * kStageBytes, &pp.full[s],
                   lane);
    if (lane == 0) *(volatile int*)pp.issued = n;
  }
  float y[4] = {0, 0, 0, 0};
  // gu: this warp's 8 output rows (gate rows at the stage's first 64, up rows at the next 64); down: its 16 rows
  const int r_lo = GU ? warp * 8 : warp * 16, r_hi = GU ? 64 + warp * 8 : warp * 16 + 8;
  int waited = 0;  // (producer: steps whose copies are known complete)
  Item it = item_at<GU>(a, i0, e_run, uo, offs);
  int sb = 0, li = 0;  // (column of the current item, items done)
  for (int s = 0; s < S; s++) {
    const int b = s % kStages;
    uint8_t* buf = smem + b * kStageBytes;
    bool ok = !*(volatile int*)pp.failed;
    if (ok) {
      ok = mbar_wait(&pp.full[b], (pp.full_parity >> b) & 1u, status);
      if (!ok) *(volatile int*)pp.failed = 1;
    }
    pp.full_parity ^= 1u << b;
    ok = __all_sync(0xFFFFFFFFu, ok);
    if (producer && ok) waited = s + 1;
    if (ok) {
      XFrag xf;
      load_x(buf, lane, xf);
      tile_sb(buf + r_lo * 144, buf + r_hi * 144, xf, tab, lane, y);
    }
    __syncwarp();
    // done with stage b: the eighth warp to get here refills it with step s + kStages (the count is reset before the
    // copy starts; no warp counts on stage b again before that copy has landed)
    int last = 0;
    if (lane == 0) {
      __threadfence_block();
      last = atomicAdd(&pp.done[b], 1) == kThreads / 32 - 1;
      if (last) atomicExch(&pp.done[b], 0);
    }
    const int s2 = s + kStages;
    if (__shfl_sync(0xFFFFFFFFu, last, 0) && s2 < S && !*(volatile int*)pp.failed) {
      const int q = s2 / SB;
      refill<GU>(a, item_at<GU>(a, i0 + q, e_fill, uo, offs), s2 - q * SB, perm, buf, &pp.full[b], lane);
      if (lane == 0) atomicMax(pp.issued, s2 + 1);
    }
    if (++sb == SB) {  // the item's last column: its outputs
      const int g = lane >> 2, t = lane & 3;
      const bool good = !*(volatile int*)pp.failed;
      if (GU) {  // h = silu(gate) x up, rounded to bf16, into this item's buffer [8 tokens][64 rows]
        float* hb = out + (li & 1) * 64 * 8;
        const int r = warp * 8 + prow(g);
        hb[(2 * t) * 64 + r] = __bfloat162float(__float2bfloat16_rn(__fmul_rn(silu(y[0]), y[2])));
        hb[(2 * t + 1) * 64 + r] = __bfloat162float(__float2bfloat16_rn(__fmul_rn(silu(y[1]), y[3])));
        __syncthreads();  // (the other buffer: free since the previous item's barrier)
        if (threadIdx.x < 64) {  // (n, group of 32 rows, t): 8 h values in fragment order, and the group sum
          const int n = threadIdx.x >> 3, grp = (threadIdx.x >> 2) & 1, tq = threadIdx.x & 3;
          const float* hg = hb + n * 64 + grp * 32;
          float v[8];
          if (a.natural) {  // values 2 tq, 2 tq + 1, 2 tq + 8, 2 tq + 9 and the same + 16, as bf16 pairs in that order
#pragma unroll
            for (int j = 0; j < 4; j++) v[2 * j] = hg[2 * tq + 8 * j], v[2 * j + 1] = hg[2 * tq + 8 * j + 1];
          } else {
            const float4 h0 = *reinterpret_cast<const float4*>(hg + 8 * tq);
            const float4 h1 = *reinterpret_cast<const float4*>(hg + 8 * tq + 4);
            v[0] = h0.x, v[1] = h0.y, v[2] = h0.z, v[3] = h0.w, v[4] = h1.x, v[5] = h1.y, v[6] = h1.z, v[7] = h1.w;
          }
          float part = ((v[0] + v[1]) + (v[2] + v[3])) + ((v[4] + v[5]) + (v[6] + v[7]));
          part += __shfl_xor_sync(0xFFFFFFFFu, part, 1);
          part += __shfl_xor_sync(0xFFFFFFFFu, part, 2);
          if (n < it.nt && good) {
            const int Go = a.N >> 5;
            const int64_t pr = it.d0 + n;
            const int og = it.rt * 2 + grp;
            uint4 o;
            if (a.natural) {
              uint32_t b[8];
#pragma unroll
              for (int j = 0; j < 8; j++) b[j] = __float_as_uint(v[j]) >> 16;  // (v are bf16 values)
              o = make_uint4(b[0] | b[1] << 16, b[2] | b[3] << 16, b[4] | b[5] << 16, b[6] | b[7] << 16);
            } else {
              o = arrange(v);
            }
            a.hq[(pr * Go + og) * 4 + tq] = o;
            if (tq == 0) a.hs[pr * Go + og] = part;
          }
        }
      } else if (good) {
        const int64_t row = (int64_t)it.rt * 128 + warp * 16 + prow(g);
        if (2 * t < it.nt) {
          a.y[(it.d0 + 2 * t) * a.N + row] = y[0];
          a.y[(it.d0 + 2 * t) * a.N + row + 8] = y[2];
        }
        if (2 * t + 1 < it.nt) {
          a.y[(it.d0 + 2 * t + 1) * a.N + row] = y[1];
          a.y[(it.d0 + 2 * t + 1) * a.N + row + 8] = y[3];
        }
      }
      y[0] = y[1] = y[2] = y[3] = 0.0f;
      sb = 0;
      li++;
      if (i0 + li < i1) it = item_at<GU>(a, i0 + li, e_run, uo, offs);
    }
  }
  // after a failure: wait (bounded) for the copies already started, so that none lands in a stage after this
  __syncthreads();
  const int issued = *(volatile int*)pp.issued;
  if (producer)
    for (int s = waited; s < issued; s++) {
      const int b = s % kStages;
      if (!mbar_test(&pp.full[b], (pp.full_parity >> b) & 1u)) mbar_wait(&pp.full[b], (pp.full_parity >> b) & 1u, status);
    }
  __syncthreads();
}

}  // namespace ms
}  // namespace artlite
