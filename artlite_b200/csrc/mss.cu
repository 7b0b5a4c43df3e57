// The small-batch tensor-core expert GEMVs for Q4_K weights and bf16 activations (decode batches below the fused
// kernel's 8 tokens, and any GEMV-path forward whose weights have the maps): the mma tile of the fused decode kernel
// (ms.cuh) with work units sized for a grid that a handful of tokens leaves mostly idle.
//
// Items: gate / up (expert, group of <= 8 pairs, 32 output rows); down (expert, group, 128 output rows), one CTA an
// item at a time. A thread starts the item's weights with one 2D TMA box per 256-value super-block column (32 gate
// and 32 up rows, or 128 down rows, 144 bytes wide; shared-memory layout [column][row][144 B], the fused kernel's,
// whose tile loads are free of bank conflicts), the CTA stages the pairs' x meanwhile (gate / up: the tokens' bf16
// rows rearranged into the mma fragment order with per-group sums; down: the fragment-order h rows the gate / up
// kernel wrote). The products: mma.sync m16n8k16 with the Q4_K nibbles as bf16 128 + q and the group scales applied
// after each group (ms.cuh). Gate / up: four 16-row tiles (8 gate rows and the same 8 up rows each), each tile's
// columns split over two warps whose sums meet in shared memory in a fixed order; silu(gate) x up rounded to bf16 into
// h (fragment order + group sums, as the down kernel and the fused kernel read it). Down: 8 warps x 16 rows over all
// columns, fp32 rows out. The next item's weights are requested as soon as every warp is done with the current ones.
// Every wait is bounded: on expiry the CTA reports ARTLITE_ETIMEOUT, waits (bounded) for its copies in flight and
// leaves.
//
// Q6_K downs (Q4_K_M files: Q4_K gate / up, Q6_K down; the reference's q6_k, dequant.cpp:83-101) take their own down
// kernel. An item's 128 raw rows are one contiguous range (rows of 210 B a super-block need not be 16-byte pitched,
// but 128 of them are 26,880 B a column, a multiple of 16), so one bulk copy brings the whole item. The gate / up kernel
// then writes h in the natural k order of the mma (lane t of a 32-value group holding values 2t, 2t + 1, 2t + 8, 2t + 9
// and the same + 16), so that each m16n8k16 step covers exactly one 16-value Q6_K scale group: the A values are
// bf16(q - 32) (exact: (q | 0x4300) is 128 + q, minus 160 in bf16), and each step's sum is scaled once, d sc_j,
// before it joins the row's fp32 sum.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>

#include "block.cuh"
#include "common.cuh"
#include "kernels.cuh"
#include "ms.cuh"

namespace artlite {
namespace {

constexpr int kThreads = 256;
constexpr int kGuRows = 32;   // output rows a gate / up item
constexpr int kDnRows = 128;  // output rows a down item
constexpr int kMaxSB = 8;     // gate / up columns (H <= 2048)
constexpr int kMaxSBd = 4;    // down columns (F <= 1024)

struct MssArgs {
  CUtensorMap m0, m1;  // gu: gate / up rows, boxes of 32 rows; down: down rows, boxes of 128 rows (72 u16 wide)
  int K, N, E, k;      // K = 256 SB; N % rows_item == 0
  const void* x;       // gu: token rows (bf16), row perm[d] / k; down: unused
  const uint4* hq;     // down: the h rows in fragment order (pair rows, K / 32 groups)
  const float* hs;     // down: their group sums
  uint4* hq_out;       // gu: h out (pair rows, N / 32 groups)
  float* hs_out;
  float* y;            // down: fp32 rows (pair rows x N)
  const int32_t* uo;   // items per expert: exclusive scan, E + 1
  const int64_t* offsets;
  const int32_t* perm;
  int slots;           // token slots staged (min(8, the most pairs an expert can get))
  DevStatus* status;
  int natural;         // gu: h in the mma's natural k order (for a Q6_K down), else the Q4_K tile's order
  const uint8_t* raw;  // Q6_K down: the raw rows, rb bytes a row
  int64_t rb;
};

// shared memory: weights | x slots | group sums | per-warp partial sums | h tile | scale tables | mbarrier | the item
// scan and the dispatch offsets (E + 1 each: the items are found in shared memory, not by dependent L2 loads)
struct Layout {
  int w_bytes, x_stride, x_off, s_off, red_off, hb_off, tab_off, bar_off, off_off, uo_off, total;
};

__host__ __device__ inline Layout layout(bool gu, int SB, int slots, int E) {
  Layout l;
  l.w_bytes = gu ? 2 * SB * kGuRows * 144 : SB * kDnRows * 144;
  l.x_stride = SB * 512 + 16;  // (a slot's row, padded so that the 8 slots' fragment loads fall on distinct banks)
  l.x_off = (l.w_bytes + 127) & ~127;
  l.s_off = l.x_off + slots * l.x_stride;
  l.red_off = (l.s_off + slots * SB * 8 * 4 + 15) & ~15;
  l.hb_off = l.red_off + 8 * 32 * 4 * 4;
  l.tab_off = l.hb_off + 8 * kGuRows * 4;
  l.bar_off = l.tab_off + 8 * 16 * ms::kTabRow * 8;
  l.off_off = l.bar_off + 16;
  l.uo_off = l.off_off + 8 * (E + 1);
  l.total = l.uo_off + 4 * (E + 1);
  return l;
}

struct ItemS {
  int e, rt, nt;
  int64_t d0;
};

// item i from the shared copies of the item scan (uo) and the dispatch offsets (offs)
__device__ __forceinline__ ItemS item_of(const MssArgs& a, const int32_t* uo, const int64_t* offs, int i,
                                         int rows_item) {
  int lo = 0, hi = a.E;
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (uo[mid] <= i) lo = mid; else hi = mid;
  }
  const int ntile = a.N / rows_item;
  const int li = i - uo[lo], tg = li / ntile;
  ItemS it;
  it.e = lo;
  it.rt = li - tg * ntile;
  it.d0 = offs[lo] + (int64_t)tg * kGemvTokens;
  it.nt = (int)min64(kGemvTokens, offs[lo + 1] - it.d0);
  return it;
}

// the item's weights: one box per column into [column][row][144 B] (one thread)
template <bool GU>
__device__ __forceinline__ void request(const MssArgs& a, const ItemS& it, int SB, uint8_t* w, uint64_t* bar) {
  const int rows = GU ? kGuRows : kDnRows;
  const int y = it.e * a.N + it.rt * rows;
  ms::mbar_expect(bar, (unsigned)((GU ? 2 : 1) * SB * rows * 144));
  for (int c = 0; c < SB; c++) {
    ms::tma_load(w + c * rows * 144, &a.m0, bar, c * 72, y);
    if (GU) ms::tma_load(w + (SB + c) * rows * 144, &a.m1, bar, c * 72, y);
  }
}

// lane (g, t)'s x fragments of column c: slot g's 8 groups, and the group sums of slots 2t, 2t + 1 (slots at or past
// nt hold stale values, slots past the staged ones read slot 0: their products land in discarded output columns)
__device__ __forceinline__ void load_xs(const uint8_t* xs, const float* ss, int x_stride, int SB, int slots, int c,
                                        int lane, ms::XFrag& x) {
  const int g = lane >> 2, t = lane & 3;
  const uint4* xr = reinterpret_cast<const uint4*>(xs + (g < slots ? g : 0) * x_stride) + c * 32 + t;
#pragma unroll
  for (int j = 0; j < 8; j++) x.b[j] = xr[4 * j];
#pragma unroll
  for (int i = 0; i < 2; i++) {
    const int sl = 2 * t + i < slots ? 2 * t + i : 0;
    const float4* sr = reinterpret_cast<const float4*>(ss + (sl * SB + c) * 8);
    x.s[i][0] = sr[0];
    x.s[i][1] = sr[1];
  }
}

template <bool GU>
__global__ void __launch_bounds__(kThreads, 2) mss_kernel(const __grid_constant__ MssArgs a) {
  extern __shared__ __align__(128) uint8_t sm[];
  griddep_wait();
  griddep_launch();
  const int SB = a.K >> 8, G = a.K >> 5;
  const int slots = a.slots;
  const Layout L = layout(GU, SB, slots, a.E);
  uint8_t* w = sm;
  uint8_t* xs = sm + L.x_off;
  float* ss = reinterpret_cast<float*>(sm + L.s_off);
  float* red = reinterpret_cast<float*>(sm + L.red_off);
  float* hb = reinterpret_cast<float*>(sm + L.hb_off);
  uint64_t* bar = reinterpret_cast<uint64_t*>(sm + L.bar_off);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  float* tab = reinterpret_cast<float*>(sm + L.tab_off) + warp * 16 * ms::kTabRow * 2;
  const int rows_item = GU ? kGuRows : kDnRows;
  if ((ms::su32(sm) & 127u) != 0) {  // (TMA destinations: never issued to a misaligned buffer)
    if (threadIdx.x == 0) report(a.status, ARTLITE_EUNSUPPORTED, 128, 0, 0);
    return;
  }
  int64_t* offs = reinterpret_cast<int64_t*>(sm + L.off_off);
  int32_t* uo = reinterpret_cast<int32_t*>(sm + L.uo_off);
  for (int e = threadIdx.x; e <= a.E; e += kThreads) {  // (one round of independent loads)
    uo[e] = __ldcg(a.uo + e);
    offs[e] = __ldcg(a.offsets + e);
  }
  if (threadIdx.x == 0) ms::mbar_init(bar, 1);
  __syncthreads();
  const int total = uo[a.E];
  int i = blockIdx.x;
  if (i >= total) return;
  unsigned parity = 0;
  bool pending = false;  // (thread 0: a request not yet waited for)
  ItemS it = item_of(a, uo, offs, i, rows_item);
  if (threadIdx.x == 0) request<GU>(a, it, SB, w, bar), pending = true;
  for (; i < total; i += gridDim.x) {
    // x of the item's pairs, in fragment order with group sums (an item never has more pairs than the staged slots:
    // a token routes to distinct experts; more is reported, and the excess pairs are left out)
    if (it.nt > slots && threadIdx.x == 0) report(a.status, ARTLITE_EDEVICE, it.nt, slots, 3);
    const int ns = it.nt < slots ? it.nt : slots;
    if (GU) {
      for (int u = threadIdx.x; u < ns * G * 4; u += kThreads) {  // (4 | kThreads: a group's 4 threads share a warp)
        const int t = u & 3, grp = (u >> 2) % G, n = (u >> 2) / G;
        const int64_t tok = a.perm[it.d0 + n] / a.k;
        const uint4 q = __ldg(reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(a.x) + tok * a.K + grp * 32 + 8 * t));
        const uint32_t qw[4] = {q.x, q.y, q.z, q.w};
        float v[8];
#pragma unroll
        for (int j = 0; j < 4; j++) v[2 * j] = __uint_as_float(qw[j] << 16), v[2 * j + 1] = __uint_as_float(qw[j] & 0xFFFF0000u);
        reinterpret_cast<uint4*>(xs + n * L.x_stride)[grp * 4 + t] = ms::arrange(v);
        float part = ((v[0] + v[1]) + (v[2] + v[3])) + ((v[4] + v[5]) + (v[6] + v[7]));
        part += __shfl_xor_sync(0xFFFFFFFFu, part, 1);
        part += __shfl_xor_sync(0xFFFFFFFFu, part, 2);
        if (t == 0) ss[n * G + grp] = part;
      }
    } else {
      for (int u = threadIdx.x; u < ns * G * 4; u += kThreads) {
        const int n = u / (G * 4), r = u - n * G * 4;
        reinterpret_cast<uint4*>(xs + n * L.x_stride)[r] = __ldcg(a.hq + (it.d0 + n) * G * 4 + r);
      }
      for (int u = threadIdx.x; u < ns * G; u += kThreads) {
        const int n = u / G, r = u - n * G;
        ss[n * G + r] = __ldcg(a.hs + (it.d0 + n) * G + r);
      }
    }
    __syncthreads();
    const bool ok = __syncthreads_and(ms::mbar_wait(bar, parity, a.status));
    if (!ok) break;  // (thread 0 waits below, bounded, for the copies still in flight: parity names their phase)
    parity ^= 1u;
    if (threadIdx.x == 0) pending = false;
    float y[4] = {0, 0, 0, 0};
    if (GU) {  // warp: tile warp & 3 (8 gate rows and the same 8 up rows), columns [h SB / 2, (h + 1) SB / 2)
      const int tile = warp & 3, half = warp >> 2;
      for (int c = half * (SB >> 1); c < (half + 1) * (SB >> 1); c++) {
        ms::XFrag xf;
        load_xs(xs, ss, L.x_stride, SB, slots, c, lane, xf);
        ms::tile_sb(w + (c * kGuRows + tile * 8) * 144, w + ((SB + c) * kGuRows + tile * 8) * 144, xf, tab, lane, y);
      }
      if (half) {
#pragma unroll
        for (int j = 0; j < 4; j++) red[(tile * 32 + lane) * 4 + j] = y[j];
      }
    } else {  // warp: rows 16 warp .. 16 warp + 15, every column
      for (int c = 0; c < SB; c++) {
        ms::XFrag xf;
        load_xs(xs, ss, L.x_stride, SB, slots, c, lane, xf);
        ms::tile_sb(w + (c * kDnRows + warp * 16) * 144, w + (c * kDnRows + warp * 16 + 8) * 144, xf, tab, lane, y);
      }
    }
    __syncthreads();  // (every warp is done with the weights and x of this item)
    const ItemS cur = it;
    const int nxt = i + gridDim.x;
    if (nxt < total) {
      it = item_of(a, uo, offs, nxt, rows_item);
      if (threadIdx.x == 0) request<GU>(a, it, SB, w, bar), pending = true;
    }
    const int g = lane >> 2, t = lane & 3;
    if (GU) {
      if (warp < 4) {  // the two halves in order, then h = silu(gate) x up rounded to bf16 into [token][32 rows]
#pragma unroll
        for (int j = 0; j < 4; j++) y[j] += red[(warp * 32 + lane) * 4 + j];
        const int r = warp * 8 + ms::prow(g);
        hb[(2 * t) * kGuRows + r] = __bfloat162float(__float2bfloat16_rn(__fmul_rn(ms::silu(y[0]), y[2])));
        hb[(2 * t + 1) * kGuRows + r] = __bfloat162float(__float2bfloat16_rn(__fmul_rn(ms::silu(y[1]), y[3])));
      }
      __syncthreads();
      if (threadIdx.x < 32) {  // (token n, 8-row quarter tq): 8 h values in fragment order, and the group sum
        const int n = threadIdx.x >> 2, tq = threadIdx.x & 3;
        const float* hn = hb + n * kGuRows;
        float v[8];
        if (a.natural) {  // values 2 tq, 2 tq + 1, 2 tq + 8, 2 tq + 9, and the same + 16
#pragma unroll
          for (int j = 0; j < 4; j++) v[2 * j] = hn[2 * tq + 8 * j], v[2 * j + 1] = hn[2 * tq + 8 * j + 1];
        } else {
          const float4 h0 = *reinterpret_cast<const float4*>(hn + 8 * tq);
          const float4 h1 = *reinterpret_cast<const float4*>(hn + 8 * tq + 4);
          v[0] = h0.x, v[1] = h0.y, v[2] = h0.z, v[3] = h0.w, v[4] = h1.x, v[5] = h1.y, v[6] = h1.z, v[7] = h1.w;
        }
        float part = ((v[0] + v[1]) + (v[2] + v[3])) + ((v[4] + v[5]) + (v[6] + v[7]));
        part += __shfl_xor_sync(0xFFFFFFFFu, part, 1);
        part += __shfl_xor_sync(0xFFFFFFFFu, part, 2);
        if (n < cur.nt && n < slots) {
          const int Go = a.N >> 5;
          const int64_t pr = cur.d0 + n;
          uint4 o;
          if (a.natural) {  // (bf16 pairs in k order: the B registers of the group's two steps)
            uint32_t b[8];
#pragma unroll
            for (int j = 0; j < 8; j++) b[j] = __float_as_uint(v[j]) >> 16;
            o = make_uint4(b[0] | b[1] << 16, b[2] | b[3] << 16, b[4] | b[5] << 16, b[6] | b[7] << 16);
          } else {
            o = ms::arrange(v);
          }
          a.hq_out[(pr * Go + cur.rt) * 4 + tq] = o;
          if (tq == 0) a.hs_out[pr * Go + cur.rt] = part;
        }
      }
    } else {
      const int64_t row = (int64_t)cur.rt * kDnRows + warp * 16 + ms::prow(g);
#pragma unroll
      for (int q = 0; q < 2; q++) {
        const int n = 2 * t + q;
        if (n < cur.nt && n < slots) {
          a.y[(cur.d0 + n) * a.N + row] = y[q];
          a.y[(cur.d0 + n) * a.N + row + 8] = y[2 + q];
        }
      }
    }
    __syncthreads();  // (x slots, sums and the h tile are free again)
  }
  if (threadIdx.x == 0 && pending && !ms::mbar_test(bar, parity)) ms::mbar_wait(bar, parity, a.status);
}

// ---------------------------------------------------------------- Q6_K downs

// shared memory of the Q6_K down kernel: the item's raw rows (128 x rb, 16-byte aligned) | x slots | mbarrier | the
// item scan and the dispatch offsets
struct Layout6 {
  int w_bytes, x_stride, x_off, bar_off, off_off, uo_off, total;
};
__host__ __device__ inline Layout6 layout6(int64_t rb, int SB, int slots, int E) {
  Layout6 l;
  l.w_bytes = (int)(kDnRows * rb);
  l.x_stride = SB * 512 + 16;
  l.x_off = (l.w_bytes + 127) & ~127;
  l.bar_off = l.x_off + slots * l.x_stride;
  l.off_off = l.bar_off + 16;
  l.uo_off = l.off_off + 8 * (E + 1);
  l.total = l.uo_off + 4 * (E + 1);
  return l;
}

__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   ms::su32(dst)),
               "l"(src), "r"(bytes), "r"(ms::su32(bar))
               : "memory");
}

// the two bytes at p (2-byte aligned) spread into the low bytes of the two 16-bit halves
__device__ __forceinline__ uint32_t spread2(const uint8_t* p) {
  return __byte_perm((uint32_t)*reinterpret_cast<const uint16_t*>(p), 0u, 0x4140u);
}

// One warp's 16 rows (rows g and g + 8 of lane (g, t) at r0 / r1, rb bytes a row) x one super-block column c of
// the staged x (natural k order): y (rows g, g + 8 x tokens 2t, 2t + 1) += sum over the 16 scale groups j of
// d sc_j (sum_k (q_k - 32) x_k). Group j = 16-value half (j & 1) of 32-group j / 2 = (h, jj): 128 h + 32 jj + l
// (dequant.cpp:83-101): q = (nibble jj / 2 of ql[64 h + 32 (jj & 1) + l] | crumb jj of qh[32 h + l] << 4).
__device__ __forceinline__ void tile6_sb(const uint8_t* r0, const uint8_t* r1, const uint8_t* xs, int x_stride,
                                         int slots, int c, int lane, float (&y)[4]) {
  const int g = lane >> 2, t = lane & 3;
  const uint8_t* b0 = r0 + 210 * c;
  const uint8_t* b1 = r1 + 210 * c;
  const float d0 = __half2float(__ushort_as_half(*reinterpret_cast<const uint16_t*>(b0 + 208)));
  const float d1 = __half2float(__ushort_as_half(*reinterpret_cast<const uint16_t*>(b1 + 208)));
  const uint4* xr = reinterpret_cast<const uint4*>(xs + (g < slots ? g : 0) * x_stride) + c * 32 + t;
  const __nv_bfloat162 m160 = __floats2bfloat162_rn(-160.0f, -160.0f);
#pragma unroll
  for (int h = 0; h < 2; h++) {
    uint4 bx[4];  // (this lane's x of the four 32-groups (h, jj): both steps each)
#pragma unroll
    for (int jj = 0; jj < 4; jj++) bx[jj] = xr[4 * (4 * h + jj)];
#pragma unroll
    for (int half = 0; half < 2; half++) {
      const int l = 16 * half + 2 * t;
      uint32_t a[4][4];  // [jj][register]: a qh pair serves the four crumbs, a ql pair both nibbles
#pragma unroll
      for (int r = 0; r < 4; r++) {  // (a0: row g, k 2t; a1: row g + 8, k 2t; a2: row g, k 2t + 8; a3: row g + 8)
        const uint8_t* b = (r & 1) ? b1 : b0;
        const int k8 = (r >> 1) * 8;
        const uint32_t qh = spread2(b + 128 + 32 * h + l + k8);
#pragma unroll
        for (int p = 0; p < 2; p++) {
          const uint32_t ql = spread2(b + 64 * h + 32 * p + l + k8);
#pragma unroll
          for (int hi = 0; hi < 2; hi++) {
            const int jj = p + 2 * hi;
            const uint32_t nib = ((hi ? ql >> 4 : ql) & 0x000F000Fu) | 0x43004300u;
            const uint32_t crumb = jj == 0 ? qh << 4 : jj == 1 ? qh << 2 : jj == 2 ? qh : qh >> 2;
            const uint32_t v = (crumb & 0x00300030u) | nib;  // bf16 128 + q
            __nv_bfloat162 w = __hadd2(*reinterpret_cast<const __nv_bfloat162*>(&v), m160);  // q - 32, exact
            a[jj][r] = *reinterpret_cast<const uint32_t*>(&w);
          }
        }
      }
#pragma unroll
      for (int jj = 0; jj < 4; jj++) {
        float acc[4] = {0, 0, 0, 0};
        ms::mma_bf16(acc, a[jj], half ? bx[jj].z : bx[jj].x, half ? bx[jj].w : bx[jj].y);
        const int j = 2 * (4 * h + jj) + half;  // (the scale index: 16-value group j of the super-block)
        const float s0 = __fmul_rn(d0, (float)(int8_t)b0[192 + j]), s1 = __fmul_rn(d1, (float)(int8_t)b1[192 + j]);
        y[0] = fmaf(s0, acc[0], y[0]);
        y[1] = fmaf(s0, acc[1], y[1]);
        y[2] = fmaf(s1, acc[2], y[2]);
        y[3] = fmaf(s1, acc[3], y[3]);
      }
    }
  }
}

__global__ void __launch_bounds__(kThreads, 2) mss_q6_down_kernel(const __grid_constant__ MssArgs a) {
  extern __shared__ __align__(128) uint8_t sm[];
  griddep_wait();
  griddep_launch();
  const int SB = a.K >> 8, G = a.K >> 5;
  const int slots = a.slots;
  const Layout6 L = layout6(a.rb, SB, slots, a.E);
  uint8_t* w = sm;
  uint8_t* xs = sm + L.x_off;
  uint64_t* bar = reinterpret_cast<uint64_t*>(sm + L.bar_off);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if ((ms::su32(sm) & 127u) != 0) {  // (bulk-copy destinations: never issued to a misaligned buffer)
    if (threadIdx.x == 0) report(a.status, ARTLITE_EUNSUPPORTED, 128, 0, 0);
    return;
  }
  int64_t* offs = reinterpret_cast<int64_t*>(sm + L.off_off);
  int32_t* uo = reinterpret_cast<int32_t*>(sm + L.uo_off);
  for (int e = threadIdx.x; e <= a.E; e += kThreads) {
    uo[e] = __ldcg(a.uo + e);
    offs[e] = __ldcg(a.offsets + e);
  }
  if (threadIdx.x == 0) ms::mbar_init(bar, 1);
  __syncthreads();
  const int total = uo[a.E];
  const uint32_t item_bytes = (uint32_t)(kDnRows * a.rb);
  int i = blockIdx.x;
  if (i >= total) return;
  unsigned parity = 0;
  bool pending = false;
  auto request = [&](const ItemS& it) {  // (one thread) the item's 128 rows: one contiguous range
    ms::mbar_expect(bar, item_bytes);
    bulk_load(w, a.raw + ((int64_t)it.e * a.N + (int64_t)it.rt * kDnRows) * a.rb, item_bytes, bar);
  };
  ItemS it = item_of(a, uo, offs, i, kDnRows);
  if (threadIdx.x == 0) request(it), pending = true;
  for (; i < total; i += gridDim.x) {
    if (it.nt > slots && threadIdx.x == 0) report(a.status, ARTLITE_EDEVICE, it.nt, slots, 3);
    const int ns = it.nt < slots ? it.nt : slots;
    for (int u = threadIdx.x; u < ns * G * 4; u += kThreads) {
      const int n = u / (G * 4), r = u - n * G * 4;
      reinterpret_cast<uint4*>(xs + n * L.x_stride)[r] = __ldcg(a.hq + (it.d0 + n) * G * 4 + r);
    }
    __syncthreads();
    const bool ok = __syncthreads_and(ms::mbar_wait(bar, parity, a.status));
    if (!ok) break;
    parity ^= 1u;
    if (threadIdx.x == 0) pending = false;
    float y[4] = {0, 0, 0, 0};
    const int g = lane >> 2, t = lane & 3;
    const uint8_t* r0 = w + (warp * 16 + g) * a.rb;
    const uint8_t* r1 = r0 + 8 * a.rb;
    for (int c = 0; c < SB; c++) tile6_sb(r0, r1, xs, L.x_stride, slots, c, lane, y);
    __syncthreads();  // (every warp is done with the weights and x of this item)
    const ItemS cur = it;
    const int nxt = i + gridDim.x;
    if (nxt < total) {
      it = item_of(a, uo, offs, nxt, kDnRows);
      if (threadIdx.x == 0) request(it), pending = true;
    }
    const int64_t row = (int64_t)cur.rt * kDnRows + warp * 16 + g;
#pragma unroll
    for (int q = 0; q < 2; q++) {
      const int n = 2 * t + q;
      if (n < cur.nt && n < slots) {
        a.y[(cur.d0 + n) * a.N + row] = y[q];
        a.y[(cur.d0 + n) * a.N + row + 8] = y[2 + q];
      }
    }
    __syncthreads();  // (the x slots are free again)
  }
  if (threadIdx.x == 0 && pending && !ms::mbar_test(bar, parity)) ms::mbar_wait(bar, parity, a.status);
}

}  // namespace

bool mss_ok(int qtype, int down_qtype, int x_dtype, int H, int F, bool has_maps) {
  return has_maps && qtype == ARTLITE_Q4_K && (down_qtype == ARTLITE_Q4_K || down_qtype == ARTLITE_Q6_K) &&
         x_dtype == ARTLITE_BF16 && H % 512 == 0 && H / 256 <= kMaxSB && F % 256 == 0 && F / 256 <= kMaxSBd &&
         F % kGuRows == 0 && H % kDnRows == 0;
}
int mss_mult_gu(int F) { return F / kGuRows; }
int mss_mult_dn(int H) { return H / kDnRows; }

int launch_mss(const MssLaunch& s, bool gu, cudaStream_t st) {
  AL_CHECK(s.slots >= 1 && s.slots <= kGemvTokens, ARTLITE_EINVAL, "small gemv: %d token slots", s.slots);
  int dev = 0, sms = 0;
  AL_CUDA(cudaGetDevice(&dev));
  AL_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  MssArgs a{};
  AL_CHECK(gu ? s.gate_map && s.up_map : s.down_map || s.down_qtype == ARTLITE_Q6_K, ARTLITE_EINVAL,
           "small gemv: no tensor map for the %s rows", gu ? "gate / up" : "down");
  if (gu) a.m0 = *s.gate_map, a.m1 = *s.up_map;
  else if (s.down_map) a.m0 = *s.down_map;  // (a Q6_K down has none: its rows are bulk-copied)
  a.K = gu ? s.H : s.F;
  a.N = gu ? s.F : s.H;
  a.E = s.E;
  a.k = s.k;
  a.x = s.x;
  a.hq = s.hq;
  a.hs = s.hs;
  a.hq_out = s.hq;
  a.hs_out = s.hs;
  a.y = s.y;
  a.uo = gu ? s.unit_gu : s.unit_dn;
  a.offsets = s.offsets;
  a.perm = s.perm;
  a.slots = s.slots;
  a.status = s.status;
  a.natural = s.down_qtype == ARTLITE_Q6_K;
  if (!gu && s.down_qtype == ARTLITE_Q6_K) {  // (the Q6_K down kernel: whole items by one bulk copy)
    a.raw = s.down_raw;
    a.rb = s.rb_dn;
    AL_CHECK(a.rb == (int64_t)(a.K / 256) * 210 && ((uintptr_t)a.raw % 16) == 0, ARTLITE_EINVAL,
             "small gemv: Q6_K rows of %lld bytes", (long long)a.rb);
    const Layout6 l6 = layout6(a.rb, a.K >> 8, s.slots, s.E);
    const size_t smem6 = (size_t)l6.total;
    AL_CUDA(cudaFuncSetAttribute(mss_q6_down_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem6));
    int per_sm6 = 0;
    AL_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm6, mss_q6_down_kernel, kThreads, smem6));
    AL_CHECK(per_sm6 >= 1, ARTLITE_EUNSUPPORTED, "small gemv: %zu B of shared memory", smem6);
    return launch_pdl(mss_q6_down_kernel, dim3((unsigned)(per_sm6 * sms)), dim3(kThreads), smem6, st, a);
  }
  const Layout l = layout(gu, a.K >> 8, s.slots, s.E);
  const size_t smem = (size_t)l.total;
  auto kern = gu ? mss_kernel<true> : mss_kernel<false>;
  AL_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  int per_sm = 0;
  AL_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kThreads, smem));
  AL_CHECK(per_sm >= 1, ARTLITE_EUNSUPPORTED, "small gemv: %zu B of shared memory", smem);
  return launch_pdl(kern, dim3((unsigned)(per_sm * sms)), dim3(kThreads), smem, st, a);
}

}  // namespace artlite
