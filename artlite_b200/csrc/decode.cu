// The fused decode-batch forward: one cooperative kernel per layer for small batches on the GEMV path (8 <= T, or
// 16 <= T where the small-batch tensor-core GEMVs of mss.cu apply; T k <= 512 pairs, E <= 256, Q4_0 / Q8_0 / Q4_K
// weights, and Q4_K gate / up with Q6_K downs; a Q4_K shared expert rides along as one more expert). It runs the same
// steps as the separate kernels of a forward, in phases separated by grid barriers (for Q4_K layers without a shared
// expert, by default, the kernel ends after phase 3 and the small-batch down kernel of mss.cu and the combine follow
// as two more launches: faster than phases 4-5 here, and the only way for Q6_K downs):
//   0. with the layer's input norm: CTA b norms rows b, b + G, .. of the raw input into x (norm.cuh, the norm kernel's
//      arithmetic), one count a row; every CTA waits for all T rows (bounded), so no norm launch precedes the kernel;
//   1. router logits (router.cu's semantics: fp32 products, fp32 sums, + bias): register-blocked 4 tokens x 4 experts
//      a warp over a quarter of H (router_tiles), or a warp per (token, expert) for other shapes; for Q4_K also the
//      tokens' x in the streaming GEMV's fragment order (ms.cuh);
//   2. routing (route.cuh, the reference's moe_route): when T <= 8 every CTA routes all tokens for its own copy (no
//      barrier), else CTA c routes tokens 8c .. 8c + 7 and a barrier follows; then every CTA builds the dispatch of the
//      T k pairs in its shared memory (histogram, scan, stable rank: the order dispatch.cu gives, the same in every
//      CTA) and CTA 0 writes ids / weights / offsets / counts / perm / slot for the caller;
//   3. gate/up: Q4_K the streaming tensor-core GEMV (ms.cuh) -> h as bf16 in fragment order; Q4_0 / Q8_0 the
//      register-decoding GEMV (rq.cuh) -> h (fp32); both in dispatch order, items spread over the grid;
//   4. down: the same -> y rows (fp32);
//   5. combine (combine.cu's semantics): out[t] = sum_i w[t, i] y[slot[t k + i]] in slot order, one rounding.
// A cooperative launch guarantees that every CTA is resident (or the launch fails). Each barrier waits at most about
// two seconds; then it reports ARTLITE_ETIMEOUT through the status word and the kernel returns.
#include <cuda_bf16.h>

#include <algorithm>

#include "block.cuh"
#include "common.cuh"
#include "kernels.cuh"
#include "route.cuh"
#include "ms.cuh"
#include "norm.cuh"
#include "rq.cuh"

namespace artlite {

namespace {

constexpr int kThreads = rq::kWarps * 32;
constexpr int kMaxPairs = 512, kMaxExperts = 256;
constexpr long long kBarrierCycles = 4000000000LL;  // about 2 s

struct GridBar {
  unsigned count, gen;
  unsigned norm_cnt;  // rows normed in this launch (phase 0; zeroed by CTA 0 after barrier 1)
  unsigned pad[13];
  int tb_done[kMaxPairs / 4];  // per block of 4 tokens: router units finished (the last one routes the tokens)
};

__device__ __forceinline__ unsigned ld_acquire(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// every CTA of the grid arrives; false if the wait ran out (reported)
__device__ __forceinline__ bool grid_sync(GridBar* b, DevStatus* st, int where) {
  __shared__ int ok;
  __syncthreads();
  if (threadIdx.x == 0) {
    ok = 1;
    const unsigned g = ld_acquire(&b->gen);
    __threadfence();
    if (atomicAdd(&b->count, 1u) + 1 == gridDim.x) {
      atomicExch(&b->count, 0u);
      __threadfence();
      atomicAdd(&b->gen, 1u);
    } else {
      const long long t0 = clock64();
      while (ld_acquire(&b->gen) == g) {
        if (clock64() - t0 > kBarrierCycles) {
          report(st, ARTLITE_ETIMEOUT, where, (int)blockIdx.x);
          ok = 0;
          break;
        }
        __nanosleep(64);
      }
    }
    __threadfence();
  }
  __syncthreads();
  return ok != 0;
}

static_assert(sizeof(GridBar) <= 1024, "the handle reserves 1 KiB for the grid barrier and the token-block counts");

struct DecodeArgs {
  const void* x;
  int x_dtype;
  int T, H, E, K, F;
  const void* router;
  int router_dtype;
  const float* bias;
  int gating, vector_shape;
  const uint8_t *gate, *up, *down;
  int64_t rb_gu, rb_dn;
  int R_gu, R_dn, mult_gu, mult_dn;  // (Q4_K: R_* unused)
  size_t stage_bytes;
  uint4 *xq, *hq;  // Q4_K: the tokens' x and h in fragment order, with their group sums
  float *xs, *hs;
  CUtensorMap mg, mu, md;  // Q4_K: the raw rows' tensor maps (Layer::dm_*)
  float* logits;
  int32_t* ids;
  float* w;
  int64_t* offsets;
  int32_t *counts, *perm, *slot;
  float *h, *y;
  const void* res;  // rows added last to the output (the residual of a layer with a norm), or null
  // a layer's input norm (x_in set): phase 0 norms the raw rows x_in into x (norm.cuh), CTA b rows b, b + G, ..
  const void* x_in;
  const void* norm_w;
  int norm_dtype;
  double norm_eps;
  // the shared expert (Q4_K, ref.shared_expert): its raw rows' maps, width, gate vector (fp32, or null: ungated), its
  // h rows (fragment order) and sums, its output rows (fp32, T x H), the per-token gates, 0 .. T - 1
  bool shared;
  CUtensorMap smg, smu, smd;
  int Fs;
  const float* sgate;
  uint4* shq;
  float *shs, *shy, *sh_s;
  const int32_t* iota;
  // gu_only: the kernel ends after gate / up, h written in the mma's natural k order (natural) for the small-batch
  // Q6_K down kernel that follows (Q4_K_M layers), and CTA 0 writes the down items' scan to unit_dn
  int gu_only, natural;
  int32_t* unit_dn;
  void* out;
  GridBar* bar;
  DevStatus* status;
};

__device__ __forceinline__ void load4(const void* p, int dtype, int64_t i, float (&v)[4]) {
  if (dtype == ARTLITE_BF16) {
    const uint2 u = __ldcg(reinterpret_cast<const uint2*>(reinterpret_cast<const uint16_t*>(p) + i));
    v[0] = __uint_as_float(u.x << 16), v[1] = __uint_as_float(u.x & 0xFFFF0000u);
    v[2] = __uint_as_float(u.y << 16), v[3] = __uint_as_float(u.y & 0xFFFF0000u);
  } else {
    const float4 f = __ldcg(reinterpret_cast<const float4*>(reinterpret_cast<const float*>(p) + i));
    v[0] = f.x, v[1] = f.y, v[2] = f.z, v[3] = f.w;
  }
}

// phase 1: one warp's logit (token t, expert e)
__device__ __forceinline__ void router_unit(const DecodeArgs& a, int t, int e, int lane) {
  float acc = 0.0f;
  for (int c0 = 0; c0 < a.H; c0 += 1024) {
    float wv[8][4], xv[8][4];
#pragma unroll
    for (int i = 0; i < 8; i++) {
      const int c = c0 + 4 * lane + 128 * i;
      if (c < a.H) {
        load4(a.router, a.router_dtype, (int64_t)e * a.H + c, wv[i]);
        load4(a.x, a.x_dtype, (int64_t)t * a.H + c, xv[i]);
      } else {
#pragma unroll
        for (int j = 0; j < 4; j++) wv[i][j] = xv[i][j] = 0.0f;
      }
    }
#pragma unroll
    for (int i = 0; i < 8; i++)
#pragma unroll
      for (int j = 0; j < 4; j++) acc = fmaf(wv[i][j], xv[i][j], acc);
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) acc += __shfl_xor_sync(0xFFFFFFFFu, acc, o);
  if (lane == 0) a.logits[(int64_t)t * a.E + e] = a.bias ? acc + a.bias[e] : acc;
}

// phase 1 when H % 512 == 0 and E % 4 == 0: register-blocked logits. A CTA takes two (4 tokens x 4 experts) blocks, a
// warp one block over a quarter of H (each lane 4 consecutive values of every 128), so that a router row and an x row
// are read 4 times less often than a warp per logit reads them; the quarters' sums meet in shared memory (part: 128
// floats) and add in a fixed order, + bias
template <int J>
__device__ __forceinline__ void router_tiles(const DecodeArgs& a, float* part, int warp, int lane) {
  __shared__ int route_tb[2];
  const int TB = (a.T + 3) >> 2, EB = a.E >> 2, units = TB * EB;
  const int kq = a.H >> 2;
  for (int u0 = blockIdx.x * 2; u0 < units; u0 += gridDim.x * 2) {  // (the same trip count for the whole CTA)
    const int u = u0 + (warp >> 2), kp = warp & 3;
    float acc[4][4];
#pragma unroll
    for (int i = 0; i < 4; i++)
#pragma unroll
      for (int j = 0; j < 4; j++) acc[i][j] = 0.0f;
    if (u < units) {
      const int t0 = (u / EB) * 4, e0 = (u - (u / EB) * EB) * 4;
#pragma unroll 2
      for (int c = kp * kq + lane * 4; c < (kp + 1) * kq; c += 128) {
        float wv[4][4], xv[4][4];
#pragma unroll
        for (int i = 0; i < 4; i++) load4(a.router, a.router_dtype, (int64_t)(e0 + i) * a.H + c, wv[i]);
#pragma unroll
        for (int i = 0; i < 4; i++) {
          if (t0 + i < a.T) {
            load4(a.x, a.x_dtype, (int64_t)(t0 + i) * a.H + c, xv[i]);
          } else {
#pragma unroll
            for (int j = 0; j < 4; j++) xv[i][j] = 0.0f;
          }
        }
#pragma unroll
        for (int ti = 0; ti < 4; ti++)
#pragma unroll
          for (int ei = 0; ei < 4; ei++)
#pragma unroll
            for (int j = 0; j < 4; j++) acc[ti][ei] = fmaf(wv[ei][j], xv[ti][j], acc[ti][ei]);
      }
    }
#pragma unroll
    for (int ti = 0; ti < 4; ti++)
#pragma unroll
      for (int ei = 0; ei < 4; ei++)
#pragma unroll
        for (int o = 16; o; o >>= 1) acc[ti][ei] += __shfl_xor_sync(0xFFFFFFFFu, acc[ti][ei], o);
    if (lane == 0)
#pragma unroll
      for (int ti = 0; ti < 4; ti++)
#pragma unroll
        for (int ei = 0; ei < 4; ei++) part[warp * 16 + ti * 4 + ei] = acc[ti][ei];
    __syncthreads();
    if (threadIdx.x < 32) {
      const int uu = threadIdx.x >> 4, q = threadIdx.x & 15, u2 = u0 + uu;
      if (u2 < units) {
        const int t = (u2 / EB) * 4 + (q >> 2), e = (u2 - (u2 / EB) * EB) * 4 + (q & 3);
        if (t < a.T) {
          const float* pp = part + uu * 64 + q;
          const float v = (pp[0] + pp[16]) + (pp[32] + pp[48]);
          a.logits[(int64_t)t * a.E + e] = a.bias ? v + a.bias[e] : v;
        }
      }
      __threadfence();
    }
    // a token block is routed by the CTA that writes its last logits: the logits published (fence), one count a unit;
    // the CTA whose count completes the block's E / 4 units routes its tokens (a warp each) and resets the count
    if (a.T > rq::kWarps) {
      __syncthreads();
      if (threadIdx.x < 2) {
        const int u2 = u0 + threadIdx.x;
        int tb = -1;
        if (u2 < units) {
          __threadfence();
          if (atomicAdd(&a.bar->tb_done[u2 / EB], 1) == EB - 1) {
            __threadfence();
            tb = u2 / EB;
            a.bar->tb_done[tb] = 0;
          }
        }
        route_tb[threadIdx.x] = tb;
      }
      __syncthreads();
      const int tb = route_tb[warp >> 2], t = tb * 4 + (warp & 3);
      if (tb >= 0 && t < a.T) {
        RouteArgs r{a.logits, a.T, a.E, a.E, 0, a.E, a.K, a.gating, a.vector_shape, a.ids, a.w};
        route_row<J>(r, t, lane);
      }
    }
    __syncthreads();
  }
}

template <int QG, int QD, int J>
__global__ void __launch_bounds__(kThreads, 2) decode_kernel(const __grid_constant__ DecodeArgs a) {
  extern __shared__ __align__(128) float sm[];
  __shared__ int64_t s64[32];
  __shared__ int32_t s32[32];
  __shared__ int32_t sh_uo[2];  // (the shared expert's item offsets and pair offsets: one expert of T pairs)
  __shared__ int64_t sh_off[2];
  const int P = a.T * a.K, E = a.E;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  // shared memory: x staging | ids | w | perm | slot | cnt | run | wc | offs | uo_gu | uo_dn
  float* xs = sm;
  int32_t* ids_s = reinterpret_cast<int32_t*>(reinterpret_cast<uint8_t*>(sm) + a.stage_bytes);
  float* w_s = reinterpret_cast<float*>(ids_s + kMaxPairs);
  int32_t* perm_s = reinterpret_cast<int32_t*>(w_s + kMaxPairs);
  int32_t* slot_s = perm_s + kMaxPairs;
  int32_t* cnt = slot_s + kMaxPairs;
  int32_t* run = cnt + kMaxExperts;
  int32_t* wc = run + kMaxExperts;                                     // [8][E]
  int64_t* offs = reinterpret_cast<int64_t*>(wc + rq::kWarps * kMaxExperts);  // [E + 1]
  int32_t* uo_gu = reinterpret_cast<int32_t*>(offs + kMaxExperts + 1);
  int32_t* uo_dn = uo_gu + kMaxExperts + 1;

  // the router rows and the tokens' x, prefetched into L2 at once by every CTA (its share, one bulk prefetch each):
  // the router phase's loads are then L2 hits instead of a few rounds of DRAM latency
  if (threadIdx.x == 0) {
    const int64_t rbytes = (int64_t)a.E * a.H * (a.router_dtype == ARTLITE_F32 ? 4 : 2);
    const int64_t xbytes = (int64_t)a.T * a.H * (a.x_dtype == ARTLITE_BF16 ? 2 : 4);
    const void* xsrc = a.x_in ? a.x_in : a.x;
    const int64_t rc = ((rbytes + gridDim.x - 1) / gridDim.x + 15) & ~(int64_t)15;
    const int64_t r0 = rc * blockIdx.x;
    if (r0 < rbytes)
      asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(static_cast<const uint8_t*>(a.router) + r0),
                   "r"((uint32_t)min64(rc, rbytes - r0)) : "memory");
    const int64_t xc = ((xbytes + gridDim.x - 1) / gridDim.x + 15) & ~(int64_t)15;
    const int64_t x0 = xc * blockIdx.x;
    if (x0 < xbytes)
      asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(static_cast<const uint8_t*>(xsrc) + x0),
                   "r"((uint32_t)min64(xc, xbytes - x0)) : "memory");
  }
  griddep_wait();
  constexpr bool kMs = QG == ARTLITE_Q4_K;  // (then QD == QG)
  ms::Pipe pp{};
  if constexpr (kMs) {
    uint64_t* bars = reinterpret_cast<uint64_t*>(reinterpret_cast<uint8_t*>(sm) + a.stage_bytes - 64);
    pp.full = bars;
    pp.done = reinterpret_cast<int*>(bars + ms::kStages);
    pp.issued = pp.done + ms::kStages;
    pp.failed = pp.issued + 1;
    if (threadIdx.x == 0) {
      for (int i = 0; i < ms::kStages; i++) {
        ms::mbar_init(&pp.full[i], ms::kFullArrivals);
        pp.done[i] = 0;
      }
      *pp.issued = 0;
      *pp.failed = 0;
    }
  }
  // ---- 0. the layer's input norm: the rows normed into x, every CTA waits for all T (one count a row)
  if (a.x_in) {
    unsigned mine = 0;
    for (int t = blockIdx.x; t < a.T; t += gridDim.x, mine++)
      nrm::norm_rows<1>(a.x_in, a.x_dtype, a.norm_w, a.norm_dtype, a.norm_eps, a.H, t, 1, const_cast<void*>(a.x));
    nrm::norm_publish(&a.bar->norm_cnt, mine);
    if (!nrm::norm_wait(&a.bar->norm_cnt, (unsigned)a.T, a.status, 8)) return;
  }
  // ---- 1. router logits (and the tokens' x in fragment order)
  const bool tiles = a.H % 512 == 0 && E % 4 == 0;
  if (tiles) {
    router_tiles<J>(a, sm, warp, lane);  // (the staging area is free until phase 3; its end holds the mbarriers)
  } else {
    for (int u = blockIdx.x * rq::kWarps + warp; u < a.T * E; u += gridDim.x * rq::kWarps)
      router_unit(a, u / E, u % E, lane);
  }
  if constexpr (kMs) {
    const int G = a.H >> 5;
    for (int u = blockIdx.x * kThreads + threadIdx.x; u < a.T * G * 4; u += gridDim.x * kThreads) {  // (4 | kThreads)
      const int t = u & 3, grp = (u >> 2) % G, tok = (u >> 2) / G;
      const uint4 q = __ldcg(reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(a.x) + (int64_t)tok * a.H + grp * 32 + 8 * t));
      const uint32_t w[4] = {q.x, q.y, q.z, q.w};
      float v[8];
#pragma unroll
      for (int j = 0; j < 4; j++) v[2 * j] = __uint_as_float(w[j] << 16), v[2 * j + 1] = __uint_as_float(w[j] & 0xFFFF0000u);
      a.xq[u] = ms::arrange(v);
      float part = ((v[0] + v[1]) + (v[2] + v[3])) + ((v[4] + v[5]) + (v[6] + v[7]));
      part += __shfl_xor_sync(0xFFFFFFFFu, part, 1);
      part += __shfl_xor_sync(0xFFFFFFFFu, part, 2);
      if (t == 0) a.xs[u >> 2] = part;
    }
  }
  if (a.shared) {  // the shared expert's gates: a warp per token, as launch_shared_gate (combine.cu)
    for (int t = blockIdx.x * rq::kWarps + warp; t < a.T; t += gridDim.x * rq::kWarps) {
      float acc = 0.0f;
      if (a.sgate) {
        for (int c = lane * 8; c < a.H; c += 256) {
          float xv[4], xw[4];
#pragma unroll
          for (int hh = 0; hh < 2; hh++) {
            load4(a.x, a.x_dtype, (int64_t)t * a.H + c + 4 * hh, xv);
            load4(a.sgate, ARTLITE_F32, c + 4 * hh, xw);
#pragma unroll
            for (int j = 0; j < 4; j++) acc = fmaf(xv[j], xw[j], acc);
          }
        }
#pragma unroll
        for (int o = 16; o; o >>= 1) acc += __shfl_xor_sync(0xFFFFFFFFu, acc, o);
      }
      if (lane == 0) a.sh_s[t] = a.sgate ? __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-acc))) : 1.0f;
    }
  }
  if (!grid_sync(a.bar, a.status, 1)) return;
  if (a.x_in && blockIdx.x == 0 && threadIdx.x == 0) atomicExch(&a.bar->norm_cnt, 0u);  // (every CTA is past its wait)
  // ---- 2. routing and the dispatch
  const bool local = a.T <= rq::kWarps;  // every CTA routes all tokens itself
  {
    RouteArgs r{a.logits, a.T, E, E, 0, E, a.K, a.gating, a.vector_shape, local ? ids_s : a.ids, local ? w_s : a.w};
    if (local) {
      if (warp < a.T) route_row<J>(r, warp, lane);
    } else {
      if (!tiles) {  // (the router tiles route each token block as it completes: done before barrier 1)
        const int t = blockIdx.x * rq::kWarps + warp;
        if (t < a.T) route_row<J>(r, t, lane);
        if (!grid_sync(a.bar, a.status, 2)) return;
      }
      for (int p = threadIdx.x; p < P; p += kThreads) ids_s[p] = __ldcg(a.ids + p), w_s[p] = __ldcg(a.w + p);
    }
  }
  for (int i = threadIdx.x; i < (2 + rq::kWarps) * kMaxExperts; i += kThreads) cnt[i] = 0;  // cnt, run, wc
  __syncthreads();
  for (int p = threadIdx.x; p < P; p += kThreads) {
    const int32_t x = ids_s[p];
    if (x < 0 || x >= E) report(a.status, ARTLITE_EDEVICE, x, E, 1);
    else atomicAdd(&cnt[x], 1);
  }
  __syncthreads();
  {
    const int e = threadIdx.x;  // (kThreads >= E)
    const int32_t c = e < E ? cnt[e] : 0;
    int64_t tot64;
    const int64_t o = block_exclusive_scan<int64_t>(c, s64, &tot64);
    if (e < E) offs[e] = o;
    if (e == 0) offs[E] = tot64;
    int32_t tot;
    const int32_t ug = block_exclusive_scan<int32_t>(e < E ? (c + kGemvTokens - 1) / kGemvTokens * a.mult_gu : 0, s32, &tot);
    if (e < E) uo_gu[e] = ug;
    if (e == 0) uo_gu[E] = tot;
    const int32_t ud = block_exclusive_scan<int32_t>(e < E ? (c + kGemvTokens - 1) / kGemvTokens * a.mult_dn : 0, s32, &tot);
    if (e < E) uo_dn[e] = ud;
    if (e == 0) uo_dn[E] = tot;
    if (blockIdx.x == 0 && e < E) a.counts[e] = c;
  }
  __syncthreads();
  {
    const unsigned lt = (1u << lane) - 1u;
    for (int r0 = 0; r0 < P; r0 += kThreads) {
      const int p = r0 + threadIdx.x;
      int32_t x = p < P ? ids_s[p] : -1;
      const bool valid = x >= 0 && x < E;
      if (!valid) x = -1 - lane;
      const unsigned peers = __match_any_sync(0xFFFFFFFFu, x);
      const int rank = __popc(peers & lt);
      const bool leader = rank == 0;
      if (valid && leader) wc[warp * E + x] = __popc(peers);
      __syncthreads();
      if (valid) {
        int32_t pre = run[x];
        for (int w = 0; w < warp; w++) pre += wc[w * E + x];
        const int dest = (int)offs[x] + pre + rank;
        perm_s[dest] = p;
        slot_s[p] = dest;
      }
      __syncthreads();
      if (valid && leader) {
        atomicAdd(&run[x], __popc(peers));
        wc[warp * E + x] = 0;
      }
      __syncthreads();
    }
  }
  if (blockIdx.x == 0) {  // the dispatch (and, when routed locally, the routing) for the caller
    for (int p = threadIdx.x; p < P; p += kThreads) {
      a.perm[p] = perm_s[p];
      a.slot[p] = slot_s[p];
      if (local) a.ids[p] = ids_s[p], a.w[p] = w_s[p];
    }
    for (int e = threadIdx.x; e <= E; e += kThreads) a.offsets[e] = offs[e];
    if (a.gu_only)
      for (int e = threadIdx.x; e <= E; e += kThreads) a.unit_dn[e] = uo_dn[e];
  }
  // ---- 3. gate / up
  {
    ExpertGemvArgs g{};
    g.qtype = QG;
    g.w0 = a.gate;
    g.w1 = a.up;
    g.row_bytes = a.rb_gu;
    g.K = a.H;
    g.N = a.F;
    g.E = E;
    g.x = a.x;
    g.x_dtype = a.x_dtype;
    g.k = a.K;
    g.out = a.h;
    const int routed = uo_gu[E];
    const int sh_items = a.shared ? (a.T + kGemvTokens - 1) / kGemvTokens * (a.Fs / 64) : 0;
    const int total = routed + sh_items;
    const int i0 = (int)((int64_t)blockIdx.x * total / gridDim.x), i1 = (int)((int64_t)(blockIdx.x + 1) * total / gridDim.x);
    if constexpr (kMs) {
      ms::Gemv m{&a.mg, &a.mu, a.H, a.F, E, a.K, a.xq, a.xs, a.hq, a.hs, nullptr, a.natural};
      ms::run<true>(m, uo_gu, offs, perm_s, reinterpret_cast<uint8_t*>(xs), pp, i0, min(i1, routed), a.status);
      if (i1 > routed) {  // (the shared expert: one expert, every token a pair of its own, in token order)
        sh_uo[0] = 0, sh_uo[1] = sh_items, sh_off[0] = 0, sh_off[1] = a.T;
        __syncthreads();
        ms::Gemv ms_{&a.smg, &a.smu, a.H, a.Fs, 1, 1, a.xq, a.xs, a.shq, a.shs, nullptr};
        ms::run<true>(ms_, sh_uo, sh_off, a.iota, reinterpret_cast<uint8_t*>(xs), pp, max(i0, routed) - routed,
                      i1 - routed, a.status);
      }
    } else {
      rq::run_items<QG, true>(g, a.R_gu, uo_gu, offs, perm_s, xs, i0, i1);
    }
  }
  if (a.gu_only) return;  // (the down kernel and the combine follow as separate launches)
  if (!grid_sync(a.bar, a.status, 3)) return;
  // ---- 4. down
  {
    ExpertGemvArgs d{};
    d.qtype = QD;
    d.w0 = a.down;
    d.row_bytes = a.rb_dn;
    d.K = a.F;
    d.N = a.H;
    d.E = E;
    d.x = a.h;
    d.x_dtype = ARTLITE_F32;
    d.k = a.K;
    d.out = a.y;
    const int routed = uo_dn[E];
    const int sh_items = a.shared ? (a.T + kGemvTokens - 1) / kGemvTokens * (a.H / 128) : 0;
    const int total = routed + sh_items;
    const int i0 = (int)((int64_t)blockIdx.x * total / gridDim.x), i1 = (int)((int64_t)(blockIdx.x + 1) * total / gridDim.x);
    if constexpr (kMs) {
      ms::Gemv m{&a.md, nullptr, a.F, a.H, E, a.K, a.hq, a.hs, nullptr, nullptr, a.y};
      ms::run<false>(m, uo_dn, offs, perm_s, reinterpret_cast<uint8_t*>(xs), pp, i0, min(i1, routed), a.status);
      if (i1 > routed) {
        sh_uo[0] = 0, sh_uo[1] = sh_items, sh_off[0] = 0, sh_off[1] = a.T;
        __syncthreads();
        ms::Gemv ms_{&a.smd, nullptr, a.Fs, a.H, 1, 1, a.shq, a.shs, nullptr, nullptr, a.shy};
        ms::run<false>(ms_, sh_uo, sh_off, a.iota, reinterpret_cast<uint8_t*>(xs), pp, max(i0, routed) - routed,
                       i1 - routed, a.status);
      }
    } else {
      rq::run_items<QD, false>(d, a.R_dn, uo_dn, offs, perm_s, xs, i0, i1);
    }
  }
  if (!grid_sync(a.bar, a.status, 4)) return;
  griddep_launch();
  // ---- 5. combine
  {
    const int per_tok = a.H >> 3;
    for (int u = blockIdx.x * kThreads + threadIdx.x; u < a.T * per_tok; u += gridDim.x * kThreads) {
      const int t = u / per_tok, c = (u - t * per_tok) * 8;
      float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
      for (int i = 0; i < a.K; i++) {
        const float wi = w_s[t * a.K + i];
        const float4* yr = reinterpret_cast<const float4*>(a.y + (int64_t)slot_s[t * a.K + i] * a.H + c);
        const float4 y0 = __ldcg(yr), y1 = __ldcg(yr + 1);
        acc[0] = fmaf(wi, y0.x, acc[0]), acc[1] = fmaf(wi, y0.y, acc[1]);
        acc[2] = fmaf(wi, y0.z, acc[2]), acc[3] = fmaf(wi, y0.w, acc[3]);
        acc[4] = fmaf(wi, y1.x, acc[4]), acc[5] = fmaf(wi, y1.y, acc[5]);
        acc[6] = fmaf(wi, y1.z, acc[6]), acc[7] = fmaf(wi, y1.w, acc[7]);
      }
      const int64_t o = (int64_t)t * a.H + c;
      if (a.shared) {  // (the shared expert's gated rows, after the routed sum)
        const float si = a.sh_s[t];
        const float4* sr = reinterpret_cast<const float4*>(a.shy + o);
        const float4 s0 = __ldcg(sr), s1 = __ldcg(sr + 1);
        acc[0] = fmaf(si, s0.x, acc[0]), acc[1] = fmaf(si, s0.y, acc[1]);
        acc[2] = fmaf(si, s0.z, acc[2]), acc[3] = fmaf(si, s0.w, acc[3]);
        acc[4] = fmaf(si, s1.x, acc[4]), acc[5] = fmaf(si, s1.y, acc[5]);
        acc[6] = fmaf(si, s1.z, acc[6]), acc[7] = fmaf(si, s1.w, acc[7]);
      }
      if (a.res) {  // (the residual, last in the fp32 sum)
        float r[8];
        if (a.x_dtype == ARTLITE_BF16) {
          const uint4 u = __ldg(reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(a.res) + o));
          const uint32_t q[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
          for (int j = 0; j < 4; j++) r[2 * j] = __uint_as_float(q[j] << 16), r[2 * j + 1] = __uint_as_float(q[j] & 0xFFFF0000u);
        } else {
          const float4* f = reinterpret_cast<const float4*>(static_cast<const float*>(a.res) + o);
          const float4 f0 = __ldg(f), f1 = __ldg(f + 1);
          r[0] = f0.x, r[1] = f0.y, r[2] = f0.z, r[3] = f0.w, r[4] = f1.x, r[5] = f1.y, r[6] = f1.z, r[7] = f1.w;
        }
#pragma unroll
        for (int j = 0; j < 8; j++) acc[j] = __fadd_rn(acc[j], r[j]);
      }
      if (a.x_dtype == ARTLITE_BF16) {
        uint32_t q[4];
#pragma unroll
        for (int j = 0; j < 4; j++) {
          const __nv_bfloat162 b = __floats2bfloat162_rn(acc[2 * j], acc[2 * j + 1]);
          q[j] = *reinterpret_cast<const uint32_t*>(&b);
        }
        *reinterpret_cast<uint4*>(static_cast<uint16_t*>(a.out) + o) = make_uint4(q[0], q[1], q[2], q[3]);
      } else {
        float4* f = reinterpret_cast<float4*>(static_cast<float*>(a.out) + o);
        f[0] = make_float4(acc[0], acc[1], acc[2], acc[3]);
        f[1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
      }
    }
  }
}

// the GEMV staging area: the tensor-core GEMV's for Q4_K, else the register-decoding GEMV's
size_t stage_bytes(int qt, int H, int F) {
  const size_t b = qt == ARTLITE_Q4_K ? ms::smem_bytes()  // (its last 64 bytes: the stages' mbarriers)
                                      : sizeof(float) * std::max(rq::stage_floats(H), rq::stage_floats(F));
  return (b + 15) & ~(size_t)15;
}

size_t decode_smem(int qt, int H, int F) {
  return stage_bytes(qt, H, F) + sizeof(int32_t) * 4 * kMaxPairs + sizeof(int32_t) * (2 + rq::kWarps) * kMaxExperts +
         sizeof(int64_t) * (kMaxExperts + 1) + sizeof(int32_t) * 2 * (kMaxExperts + 1);
}

bool rq_type(int qt) { return qt == ARTLITE_Q4_0 || qt == ARTLITE_Q8_0 || qt == ARTLITE_Q4_K; }

}  // namespace

bool decode_fused_ok(const artlite_moe& h, const artlite_moe::Layer& L, int64_t T) {
  static const bool off = [] {
    const char* v = getenv("ARTLITE_DECODE_FUSED");
    return v && v[0] == '0';
  }();
  static const int64_t t_set = [] {  // (ARTLITE_DECODE_FUSED_MIN: the smallest batch that takes the fused kernel)
    const char* v = getenv("ARTLITE_DECODE_FUSED_MIN");
    const int64_t m = v ? atoll(v) : 0;
    return m >= 1 ? m : (int64_t)0;
  }();
  const artlite_moe_desc& d = h.d;
  // below the threshold the separate kernels, whose GEMVs spread finer items over the whole grid, are faster: below 8
  // tokens with the register-decoding GEMVs, below 16 with the small-batch tensor-core ones (measured at B = 8: 110 us
  // against the fused kernel's 117; at B = 16: 170 against 161)
  // (layers whose down runs as the separate small-batch kernel after the kernel's gate / up: from 10 tokens, between
  // the measured B = 8, chain 105 against 110 us, and B = 12, 142 against 130 us)
  // (a layer with a shared expert the kernel carries: from 3 tokens, between the measured qwen35moe B = 2, chain 55.7
  // against 61.5 us, and B = 4, 73.6 against 70.3 us; the chain runs the shared expert as a separate row group)
  const bool splits = !L.has_shared && L.qtype == ARTLITE_Q4_K && (L.down_qtype == ARTLITE_Q6_K || L.has_dm);
  const bool mss = mss_use(h, routed_weights(L), 1, d.act_dtype, d.expert_ffn);
  const int64_t t_min = t_set ? t_set : L.has_shared && mss ? 3 : mss ? (splits ? 10 : 16) : 8;
  if (L.qtype == ARTLITE_Q4_K && L.down_qtype == ARTLITE_Q6_K)  // (Q4_K_M: the kernel through gate / up, then the
                                                                 // small-batch Q6_K down kernel and the combine)
    return !off && !L.has_shared && T >= t_min && T * d.top_k <= kMaxPairs && d.n_experts <= kMaxExperts &&
           h.E_local == d.n_experts && L.has_dm_gu && d.act_dtype == ARTLITE_BF16 && d.hidden % 512 == 0 &&
           d.expert_ffn % 256 == 0 && mss_use(h, routed_weights(L), 1, d.act_dtype, d.expert_ffn) &&
           decode_smem(L.qtype, d.hidden, d.expert_ffn) <= 113 * 1024;
  const bool shared_ok = !L.has_shared || (L.sh_has_dm && L.qtype == ARTLITE_Q4_K && L.has_dm && L.sh_F % 256 == 0);
  return !off && shared_ok && T >= t_min && T * d.top_k <= kMaxPairs && d.n_experts <= kMaxExperts && h.E_local == d.n_experts &&
         rq_type(L.qtype) && L.down_qtype == L.qtype && d.hidden % 256 == 0 && d.expert_ffn % 256 == 0 &&
         gemv_rq_rows_per_warp(L.qtype, d.hidden, true) > 0 && gemv_rq_rows_per_warp(L.down_qtype, d.expert_ffn, false) > 0 &&
         (L.qtype != ARTLITE_Q4_K || (d.act_dtype == ARTLITE_BF16 && L.has_dm)) &&
         decode_smem(L.qtype, d.hidden, d.expert_ffn) <= 113 * 1024;
}

int launch_decode(artlite_moe* h, const artlite_moe::Layer& L, const void* x, void* y, int64_t T, cudaStream_t st,
                  const void* res, const NormIn* norm) {
  const artlite_moe_desc& d = h->d;
  if (!h->bar.ptr) {
    AL_TRY(h->bar.reserve(sizeof(GridBar)));
    AL_CUDA(cudaMemset(h->bar.ptr, 0, sizeof(GridBar)));
  }
  DecodeArgs a{};
  a.x = x;
  a.x_dtype = d.act_dtype;
  a.T = (int)T;
  a.H = d.hidden;
  a.E = d.n_experts;
  a.K = d.top_k;
  a.F = d.expert_ffn;
  a.router = L.router.ptr;
  a.router_dtype = L.router_qtype;
  a.bias = L.has_bias ? L.bias.as<float>() : nullptr;
  a.gating = d.gating;
  a.vector_shape = d.top_k <= 16 && d.n_experts % 16 == 0 && d.n_experts <= 512;
  a.gate = L.gate.as<uint8_t>();
  a.up = L.up.as<uint8_t>();
  a.down = L.down.as<uint8_t>();
  a.rb_gu = L.rb_gu;
  a.rb_dn = L.rb_dn;
  a.R_gu = gemv_rq_rows_per_warp(L.qtype, d.hidden, true);
  a.R_dn = gemv_rq_rows_per_warp(L.down_qtype, d.expert_ffn, false);
  a.mult_gu = a.R_gu > 0 ? (int)cdiv(d.expert_ffn, a.R_gu * rq::kWarps) : 0;
  a.mult_dn = a.R_dn > 0 ? (int)cdiv(d.hidden, a.R_dn * rq::kWarps) : 0;  // (a Q6_K down: no register GEMV)
  if (L.qtype == ARTLITE_Q4_K) {
    a.mult_gu = d.expert_ffn / 64;
    a.mult_dn = d.hidden / 128;
    a.xq = h->xp.as<uint4>();
    a.xs = reinterpret_cast<float*>(h->xp.as<uint8_t>() + sizeof(uint16_t) * T * d.hidden);
    a.hq = h->h.as<uint4>();
    a.hs = reinterpret_cast<float*>(h->h.as<uint8_t>() + sizeof(uint16_t) * T * d.top_k * d.expert_ffn);
    a.mg = L.dm_gate;
    a.mu = L.dm_up;
    a.md = L.dm_down;
  }
  a.stage_bytes = stage_bytes(L.qtype, d.hidden, d.expert_ffn);
  a.logits = h->logits.as<float>();
  a.ids = h->ids.as<int32_t>();
  a.w = h->w.as<float>();
  a.offsets = h->offsets.as<int64_t>();
  a.counts = h->counts.as<int32_t>();
  a.perm = h->perm.as<int32_t>();
  a.slot = h->slot.as<int32_t>();
  a.h = h->h.as<float>();
  a.y = h->y.as<float>();
  a.out = y;
  a.res = res;
  if (norm) {
    a.x_in = norm->x;
    a.norm_w = norm->w;
    a.norm_dtype = norm->w_dtype;
    a.norm_eps = norm->eps;
  }
  a.bar = h->bar.as<GridBar>();
  a.status = h->status.as<DevStatus>();
  a.shared = L.has_shared;
  if (L.has_shared) {
    a.smg = L.sh_dm_gate;
    a.smu = L.sh_dm_up;
    a.smd = L.sh_dm_down;
    a.Fs = L.sh_F;
    a.sgate = L.sh_has_gate ? L.sh_ginp.as<float>() : nullptr;
    a.shq = h->sh_hq.as<uint4>();
    a.shs = reinterpret_cast<float*>(h->sh_hq.as<uint8_t>() + sizeof(uint16_t) * T * L.sh_F);
    a.shy = h->sh_y.as<float>();
    a.sh_s = h->sh_s.as<float>();
    a.iota = h->sh_iota.as<int32_t>();
  }
  const bool mixed = L.qtype == ARTLITE_Q4_K && L.down_qtype == ARTLITE_Q6_K;
  // the down projection and the combine as separate launches after the fused kernel's gate / up (the small-batch
  // down kernel's whole items per CTA, each item's rows requested as the warps finish the previous one, measured
  // faster than the fused kernel's down phase: Q4_K B = 16 161 -> 154 us, B = 64 224 -> 216 us; Q6_K downs always:
  // the fused kernel has no Q6_K phase); ARTLITE_DECODE_SPLIT=0 keeps Q4_K downs (and a shared expert's) in the kernel
  static const bool split_off = [] {
    const char* v = getenv("ARTLITE_DECODE_SPLIT");
    return v && v[0] == '0';
  }();
  const bool split = mixed || (L.qtype == ARTLITE_Q4_K && L.down_qtype == ARTLITE_Q4_K && !L.has_shared && L.has_dm &&
                               !split_off);
  a.gu_only = split ? 1 : 0;
  a.natural = mixed ? 1 : 0;
  a.unit_dn = h->unit_dn.as<int32_t>();
  const size_t smem = decode_smem(L.qtype, d.hidden, d.expert_ffn);
  auto go = [&](auto kern) -> int {
    AL_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    int per_sm = 0, sms = 0;
    AL_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kThreads, smem));
    AL_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, h->dev));
    AL_CHECK(per_sm >= 1, ARTLITE_EUNSUPPORTED, "decode kernel: no CTA fits an SM (%zu B of shared memory)", smem);
    const int grid = per_sm * sms;
    AL_CHECK((T + rq::kWarps - 1) / rq::kWarps <= grid, ARTLITE_EUNSUPPORTED, "decode kernel: T %lld", (long long)T);
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeCooperative;
    at[0].val.cooperative = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    AL_CUDA(cudaLaunchKernelEx(&cfg, kern, a));
    count_launch();
    return ARTLITE_OK;
  };
  if (split) {  // gate / up in the fused kernel, then the small-batch down kernel and the combine
    AL_TRY(go(decode_kernel<ARTLITE_Q4_K, ARTLITE_Q4_K, kMaxExperts / 32>));
    MssLaunch s{};
    s.down_map = mixed ? nullptr : &L.dm_down;
    s.H = d.hidden;
    s.F = d.expert_ffn;
    s.E = d.n_experts;
    s.k = d.top_k;
    s.hq = a.hq;
    s.hs = a.hs;
    s.y = a.y;
    s.unit_dn = a.unit_dn;
    s.offsets = a.offsets;
    s.perm = a.perm;
    s.slots = (int)std::min<int64_t>(kGemvTokens, T);  // (a token's k pairs go to distinct experts)
    s.status = a.status;
    s.down_qtype = L.down_qtype;
    s.down_raw = a.down;
    s.rb_dn = L.rb_dn;
    AL_TRY(launch_mss(s, false, st));
    return launch_combine(a.y, ARTLITE_F32, a.slot, a.w, T, d.top_k, d.hidden, y, d.act_dtype, st, CombineOwn{},
                          CombineShared{}, res);
  }
#define AL_DEC(QG, QD) \
  if (L.qtype == QG && L.down_qtype == QD) return go(decode_kernel<QG, QD, kMaxExperts / 32>);
  AL_DEC(ARTLITE_Q4_0, ARTLITE_Q4_0)
  AL_DEC(ARTLITE_Q8_0, ARTLITE_Q8_0)
  AL_DEC(ARTLITE_Q4_K, ARTLITE_Q4_K)
#undef AL_DEC
  set_error("decode kernel: types %d / %d", L.qtype, L.down_qtype);
  return ARTLITE_EUNSUPPORTED;
}

}  // namespace artlite
