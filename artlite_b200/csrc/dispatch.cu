// Dispatch: the (token, slot) pairs grouped by expert, stable in pair order, as moe_plan's histogram / prefix scan /
// permute (csrc/artlite/moe_host.cpp:203-215), in three kernels over blocks of blk_pairs pairs (4096; the forward's
// 1024, for more CTAs and fewer rounds a CTA):
//   count   per block, a shared-memory histogram of its pairs' experts (ids checked: an id outside [0, E) is reported
//           through the status word as moe_plan's "expert id {x} of {E}" error, :247);
//   scan    per expert the exclusive scan over blocks (segments of blocks summed in parallel, the segments' prefix,
//           then each segment's blocks in order), then over experts (offsets), the units of work per expert and their
//           scan, the compacted list of experts with pairs;
//   rank    per block, in rounds of 256 pairs in order: within a warp the rank among lanes of the same expert
//           (__match_any_sync), across the round's warps a prefix of per-warp counts, across rounds a running count:
//           a pair's place = offsets[e] + block base[e] + running[e] + warp prefix + lane rank (stable).
// Then the reference plan's chunk deal (moe_host.cpp:216-234) for the drop-in artlite_moe_plan.
#include <algorithm>

#include "common.cuh"
#include "kernels.cuh"
#include "route.cuh"

namespace artlite {


size_t dispatch_scratch_bytes(int64_t P, int E, int blk_pairs) {
  const int64_t nblk = P ? cdiv(P, blk_pairs) : 1;
  return sizeof(int32_t) * (size_t)nblk * E;
}

__device__ __forceinline__ int64_t blk_pairs(const DispatchArgs& a) {
  return a.blk_pairs ? a.blk_pairs : kDispatchBlockPairs;
}

// (the dispatch kernels are programmatic dependents, each of the kernel before it: every one waits for that kernel's
// end before it reads or writes anything)
__global__ void __launch_bounds__(512) dispatch_count(DispatchArgs a) {
  extern __shared__ int32_t hist[];
  griddep_wait();
  griddep_launch();
  for (int e = threadIdx.x; e < a.E; e += blockDim.x) hist[e] = 0;
  __syncthreads();
  const int64_t p0 = (int64_t)blockIdx.x * blk_pairs(a);
  const int64_t p1 = min(p0 + blk_pairs(a), a.P);
  for (int64_t p = p0 + threadIdx.x; p < p1; p += blockDim.x) {
    const int32_t x = a.ids[p];
    if (x < 0 || x >= a.E)
      report(a.status, ARTLITE_EDEVICE, x, a.E, 1);
    else
      atomicAdd(&hist[x], 1);
  }
  __syncthreads();
  for (int e = threadIdx.x; e < a.E; e += blockDim.x) a.blk_counts[(int64_t)blockIdx.x * a.E + e] = hist[e];
}

// threads (segment sg, expert e): blockDim.x = Ep nseg (Ep = E rounded up to 32); segment sg takes blocks
// [sg per, (sg + 1) per): its total, the segments' prefix per expert, then its blocks' exclusive counts in place
__global__ void __launch_bounds__(1024) dispatch_scan(DispatchArgs a, int nblk) {
  __shared__ int64_t s64[32];
  __shared__ int32_t s32[32];
  __shared__ int64_t seg[1024];
  griddep_wait();
  griddep_launch();
  const int Ep = (a.E + 31) & ~31, nseg = blockDim.x / Ep;
  const int e = threadIdx.x % Ep, sg = threadIdx.x / Ep;
  const int per = (nblk + nseg - 1) / nseg, b0 = min(nblk, sg * per), b1 = min(nblk, b0 + per);
  int32_t* col = a.blk_counts + e;
  int64_t t = 0;
  if (e < a.E) {
#pragma unroll 4
    for (int b = b0; b < b1; b++) t += col[(int64_t)b * a.E];
  }
  seg[threadIdx.x] = t;
  __syncthreads();
  int64_t run = 0, pre = 0;  // (run: all segments, pre: those before sg)
  for (int s2 = 0; s2 < nseg; s2++) {
    const int64_t v = seg[s2 * Ep + e];
    run += v;
    if (s2 < sg) pre += v;
  }
  if (e < a.E)
    for (int b = b0; b < b1; b++) {
      const int32_t v = col[(int64_t)b * a.E];
      col[(int64_t)b * a.E] = (int32_t)pre;
      pre += v;
    }
  if (sg > 0) run = 0;  // (the expert-level scans below: one value an expert, from segment 0's threads)
  int64_t tot64;
  const int64_t off = block_exclusive_scan<int64_t>(e < a.E ? run : 0, s64, &tot64);
  const bool own = sg == 0 && e < a.E;
  if (own) {
    a.offsets[e] = off;
    if (a.counts) a.counts[e] = (int32_t)run;
  }
  if (threadIdx.x == 0) a.offsets[a.E] = tot64;
  if (a.unit_off) {
    const int32_t u = (own && a.unit_rows > 0) ? (int32_t)((run + a.unit_rows - 1) / a.unit_rows) * a.unit_mult : 0;
    int32_t tot;
    const int32_t uo = block_exclusive_scan<int32_t>(u, s32, &tot);
    if (own) a.unit_off[e] = uo;
    if (threadIdx.x == 0) a.unit_off[a.E] = tot;
  }
  if (a.active) {
    int32_t tot;
    const int32_t has = (own && run > 0) ? 1 : 0;
    const int32_t at = block_exclusive_scan<int32_t>(has, s32, &tot);
    if (has) a.active[at] = e;
    if (threadIdx.x == 0) *a.n_active = tot;
  }
}

__global__ void __launch_bounds__(256) dispatch_rank(DispatchArgs a) {
  extern __shared__ int32_t sm[];
  griddep_wait();
  griddep_launch();
  int32_t* wc = sm;              // [8][E] per-warp counts of the current round
  int32_t* run = sm + 8 * a.E;   // [E] pairs of this block placed so far
  for (int i = threadIdx.x; i < 9 * a.E; i += blockDim.x) sm[i] = 0;
  __syncthreads();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t p0 = (int64_t)blockIdx.x * blk_pairs(a);
  const int64_t p1 = min(p0 + blk_pairs(a), a.P);
  const int32_t* base = a.blk_counts + (int64_t)blockIdx.x * a.E;
  const unsigned lt = (1u << lane) - 1u;
  for (int64_t r0 = p0; r0 < p1; r0 += 256) {
    const int64_t p = r0 + threadIdx.x;
    int32_t x = p < p1 ? a.ids[p] : -1;
    const bool valid = x >= 0 && x < a.E;
    if (!valid) x = -1 - lane;  // (a key of its own: never grouped)
    const unsigned peers = __match_any_sync(0xFFFFFFFFu, x);
    const int rank = __popc(peers & lt);
    const bool leader = rank == 0;
    if (valid && leader) wc[warp * a.E + x] = __popc(peers);
    __syncthreads();
    if (valid) {
      int32_t pre = run[x];
      for (int w = 0; w < warp; w++) pre += wc[w * a.E + x];
      const int64_t dest = a.offsets[x] + base[x] + pre + rank;
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

int launch_dispatch(const DispatchArgs& a, cudaStream_t st) {
  AL_CHECK(a.E >= 1 && a.E <= 1024, ARTLITE_EUNSUPPORTED, "dispatch: E %d (this build: E <= 1024)", a.E);
  const int nblk = a.P ? (int)cdiv(a.P, a.blk_pairs ? a.blk_pairs : kDispatchBlockPairs) : 0;
  if (nblk) AL_TRY(launch_pdl(dispatch_count, dim3(nblk), dim3(512), a.E * sizeof(int32_t), st, a));
  const int Ep = (int)cdiv(a.E, 32) * 32;
  const int nseg = std::max(1, std::min(1024 / Ep, nblk));
  AL_TRY(launch_pdl(dispatch_scan, dim3(1), dim3(Ep * nseg), 0, st, a, nblk));
  if (nblk) AL_TRY(launch_pdl(dispatch_rank, dim3(nblk), dim3(256), 9 * (size_t)a.E * sizeof(int32_t), st, a));
  return ARTLITE_OK;
}


// ---------------------------------------------------------------- decode-sized batches: routing and dispatch in one CTA
//
// For n k <= kSmallPairs pairs (and E <= kSmallExperts): one CTA of NT threads (1024, or 256 for at most 512 pairs
// and 256 experts) routes every token (a warp per row, route.cuh) into shared memory, copies the ids and weights out
// for the caller, then histograms, scans and ranks the pairs exactly as the three dispatch kernels do for a single
// block (the same stable order), and writes both expert GEMVs' unit scans. One launch instead of six.
template <int J, int NT>
__global__ void __launch_bounds__(NT) route_dispatch_small(RouteArgs r, DispatchArgs a, int mult2, int32_t* unit_off2) {
  extern __shared__ int32_t sm[];
  griddep_wait();
  griddep_launch();
  route_dispatch_cta<J, NT>(r, a, mult2, unit_off2, sm);
}

bool small_dispatch_ok(int64_t P, int E) { return P <= kSmallPairs && E <= kSmallExperts; }

int launch_route_dispatch_small(const RouteArgs& r, const DispatchArgs& a, int mult2, int32_t* unit_off2,
                                cudaStream_t st) {
  AL_CHECK(small_dispatch_ok(a.P, a.E) && a.P == r.n * r.k, ARTLITE_EINVAL, "route_dispatch_small: P %lld E %d",
           (long long)a.P, a.E);
  AL_CHECK(a.ids == r.ids, ARTLITE_EINVAL, "route_dispatch_small: the dispatch reads the routed ids");
  const int J = (r.E + 31) / 32;
  const bool narrow = a.P <= 512 && a.E <= 256;  // (256 threads: e = threadIdx.x still covers every expert)
  const int NT = narrow ? 256 : 1024;
  const size_t smem = sizeof(int32_t) * ((NT / 32 + 2) * (size_t)a.E + 1) + sizeof(int64_t) * a.E +
                      (sizeof(int32_t) + sizeof(float)) * (size_t)a.P;
  auto go = [&](auto kern) -> int {
    AL_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    return launch_pdl(kern, dim3(1), dim3(NT), smem, st, r, a, mult2, unit_off2);
  };
  if (narrow) {
    if (J <= 1) return go(route_dispatch_small<1, 256>);
    if (J <= 2) return go(route_dispatch_small<2, 256>);
    if (J <= 4) return go(route_dispatch_small<4, 256>);
    return go(route_dispatch_small<8, 256>);
  }
  if (J <= 1) return go(route_dispatch_small<1, 1024>);
  if (J <= 2) return go(route_dispatch_small<2, 1024>);
  if (J <= 4) return go(route_dispatch_small<4, 1024>);
  if (J <= 8) return go(route_dispatch_small<8, 1024>);
  return go(route_dispatch_small<16, 1024>);
}

// ---------------------------------------------------------------- the reference plan's chunk deal

// per pair: pos and its row entry
__global__ void chunk_plan_pairs(ChunkPlanArgs a) {
  const int64_t p = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (p >= a.P) return;
  const int x = a.ids[p];
  if (x < 0 || x >= a.E) return;  // (reported by the dispatch)
  const int64_t i = a.slot[p] - a.offsets[x];
  const int64_t j = a.chunk_off[x] + i / a.chunk;  // the chunk's index in the deal
  const int c = (int)(j % a.cols);
  const int64_t kk = j / a.cols;
  if (kk >= a.cap) {
    report(a.status, ARTLITE_ECAPACITY, a.cap, 0, 0);
    return;
  }
  const int64_t at = ((int64_t)c * a.cap + kk) * a.chunk + i % a.chunk;
  a.pos[p] = at;
  a.rows[at] = (int32_t)(p / a.k);
}

// per chunk: its expert, size, padding rows; per column its count
__global__ void chunk_plan_chunks(ChunkPlanArgs a) {
  const int J = a.chunk_off[a.E];
  const int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (j < a.cols) a.counts[j] = (int32_t)min64(a.cap, j < J ? (J - j + a.cols - 1) / a.cols : 0);
  if (j >= J) return;
  int lo = 0, hi = a.E;  // the expert x with chunk_off[x] <= j < chunk_off[x + 1]
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (a.chunk_off[mid] <= j) lo = mid; else hi = mid;
  }
  const int x = lo;
  const int c = (int)(j % a.cols);
  const int64_t kk = j / a.cols;
  if (kk >= a.cap) return;
  const int64_t first = (j - a.chunk_off[x]) * a.chunk;
  const int64_t n = a.offsets[x + 1] - a.offsets[x] - first;
  const int size = (int)min64(n, a.chunk);
  a.experts[c * a.cap + kk] = x;
  a.sizes[c * a.cap + kk] = size;
  int32_t* r = a.rows + ((int64_t)c * a.cap + kk) * a.chunk;
  const int32_t t0 = a.perm[a.offsets[x] + first] / a.k;
  for (int i = size; i < a.chunk; i++) r[i] = t0;
}

int launch_chunk_plan(const ChunkPlanArgs& a, cudaStream_t st) {
  if (a.P) {
    chunk_plan_pairs<<<(unsigned)cdiv(a.P, 256), 256, 0, st>>>(a);
    AL_LAUNCHED();
  }
  // (chunks: at most P + E, and at least cols threads for the counts)
  const int64_t nj = a.P + a.E + a.cols;
  chunk_plan_chunks<<<(unsigned)cdiv(nj, 256), 256, 0, st>>>(a);
  AL_LAUNCHED();
  return ARTLITE_OK;
}

}  // namespace artlite

namespace artlite {

__global__ void __launch_bounds__(1024) unit_scan_kernel(const int32_t* counts, int E, int unit_rows, int mult,
                                                         int32_t* out) {
  __shared__ int32_t s32[32];
  griddep_wait();
  griddep_launch();
  const int e = threadIdx.x;
  const int32_t u = e < E ? (counts[e] + unit_rows - 1) / unit_rows * mult : 0;
  int32_t tot;
  const int32_t o = block_exclusive_scan<int32_t>(u, s32, &tot);
  if (e < E) out[e] = o;
  if (e == 0) out[E] = tot;
}

int launch_unit_scan(const int32_t* counts, int E, int unit_rows, int mult, int32_t* out, cudaStream_t st) {
  AL_CHECK(E >= 1 && E <= 1024 && unit_rows > 0, ARTLITE_EUNSUPPORTED, "unit scan: E %d", E);
  return launch_pdl(unit_scan_kernel, dim3(1), dim3((unsigned)cdiv(E, 32) * 32), 0, st, counts, E, unit_rows, mult,
                    out);
}

}  // namespace artlite
