// Kernel argument blocks and launchers of libartlite_moe_cuda.so (one definition per .cu file).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"

namespace artlite {

// ---------------------------------------------------------------- route.cu
struct RouteArgs {
  const float* logits;
  int64_t n, row;
  int per_col;
  int64_t pitch;
  int E, k, sigmoid, vector_shape;
  int32_t* ids;
  float* w;
};
int check_route_args(int64_t n, int per_col, int E, int k);
int launch_route(const RouteArgs& a, cudaStream_t st);

// ---------------------------------------------------------------- dispatch.cu
// Pairs p = t k + i (P = n k) grouped by expert, stable in p. Work buffers sized by dispatch_scratch_bytes.
struct DispatchArgs {
  const int32_t* ids;
  int64_t P;
  int E;
  // scratch (device)
  int32_t* blk_counts;  // [nblk][E]
  // outputs (device)
  int64_t* offsets;     // [E + 1]
  int32_t* perm;        // [P]
  int32_t* slot;        // [P]
  int32_t* counts;      // [E] pairs per expert
  // work units per expert: ceil(count / unit_rows) * unit_mult, their exclusive scan (int32 [E + 1]); unit_rows 0: none
  int unit_rows, unit_mult;
  int32_t* unit_off;
  // the compacted list of experts with pairs (int32 [E]) and their number (int32 [1]); may be null
  int32_t* active;
  int32_t* n_active;
  DevStatus* status;
  int blk_pairs;  // pairs a block of the count and rank kernels (0: kDispatchBlockPairs)
};
constexpr int kDispatchBlockPairs = 4096;
constexpr int kDispatchBlockPairsFwd = 1024;  // the forward's: more blocks, fewer rounds a block
size_t dispatch_scratch_bytes(int64_t P, int E, int blk_pairs = kDispatchBlockPairs);
int launch_dispatch(const DispatchArgs& a, cudaStream_t st);
// decode-sized batches: the routing (r) and the dispatch (a, its unit scan and a second one: mult2 / unit_off2) in one
// CTA; r.ids is a.ids
constexpr int kSmallPairs = 4096, kSmallExperts = 512;
bool small_dispatch_ok(int64_t P, int E);
int launch_route_dispatch_small(const RouteArgs& r, const DispatchArgs& a, int mult2, int32_t* unit_off2,
                                cudaStream_t st);

// The reference plan's chunk deal (moe_host.cpp:216-234) from a dispatch: experts / counts / sizes / rows / pos.
struct ChunkPlanArgs {
  const int32_t* ids;
  const int32_t* slot;
  const int32_t* perm;
  const int64_t* offsets;
  const int32_t* chunk_off;  // [E + 1] exclusive scan of ceil(count / chunk) (a dispatch with unit_rows = chunk)
  int64_t P;
  int k, E, cols, cap, chunk;
  int32_t *experts, *counts, *sizes, *rows;
  int64_t* pos;
  DevStatus* status;
};
int launch_chunk_plan(const ChunkPlanArgs& a, cudaStream_t st);

// ---------------------------------------------------------------- dequant.cu
int qtype_from_name(const char* name);
const char* qtype_name(int qtype);
int qtype_block(int qtype, int* per, int* bytes);  // values and bytes per block; ARTLITE_EUNSUPPORTED if unknown
int launch_dequant_rows(int qtype, const uint8_t* raw, int64_t n, int64_t row_bytes, int64_t cols, float* out,
                        cudaStream_t st);

// ---------------------------------------------------------------- router.cu
// logits (T x E fp32) = x (T x H, f32 or bf16) . W_r^T (E x H, f32 or bf16) (+ bias (E), if not null)
int launch_router(const void* x, int x_dtype, const void* w, int w_dtype, const float* bias, int64_t T, int H, int E,
                  float* logits, cudaStream_t st);
// the same for decode-sized batches (T <= kRouterSmallTokens, H % 4 == 0): a warp per (token, expert) over the grid
constexpr int kRouterSmallTokens = 256;
bool router_small_ok(int64_t T, int H);
// a layer's input norm done by the kernel that first reads its rows (norm.cuh): x_in the raw rows, w (H values of
// w_dtype) and eps the norm; the normed rows go to the kernel's x buffer
struct NormFuse {
  const void* x_in;
  const void* w;
  int w_dtype;
  double eps;
};
// whether launch_router_small can norm its rows itself (the CTA-per-expert form, H % 256 == 0 and T <= 16, with the
// batch's rows in a CTA's shared memory: at most 128 KiB)
bool router_small_norms(int64_t T, int H, int x_dtype);
int launch_router_small(const void* x, int x_dtype, const void* w, int w_dtype, const float* bias, int64_t T, int H,
                        int E, float* logits, cudaStream_t st, const NormFuse* norm = nullptr);

// ---------------------------------------------------------------- gemv.cu (CUDA-core dequant path)
struct ExpertGemvArgs {
  int qtype;          // weights' GGUF type
  const uint8_t* w0;  // gate rows (E F x rb_h) or down rows (E H x rb_f)
  const uint8_t* w1;  // up rows (gu only)
  int64_t row_bytes;  // bytes per weight row
  int K;              // reduction length (H for gu, F for down)
  int N;              // output rows per expert (F for gu, H for down)
  int E;
  const void* x;      // gu: the token rows (T x H, act dtype); down: h rows (P x F fp32, in dispatch order)
  int x_dtype;
  const int32_t* perm;     // dispatch order -> pair (gu: token = pair / k)
  const int64_t* offsets;  // [E + 1]
  const int32_t* unit_off; // [E + 1] items per expert, ceil(n_e / 8) * ceil(N / rt), scanned (launch_unit_scan)
  int rt;                  // weight rows per item (gemv_row_tile(N))
  const int32_t* wexp;     // (may be null) the weight expert of each of the E row groups (expert parallelism: a row
                           // group is one source rank's rows of one local expert); null: group e uses expert e
  int k;
  float* out;        // gu: h (P x F fp32, dispatch order); down: y (P x H fp32, dispatch order)
};
constexpr int kGemvTokens = 8;  // pairs per item
// weight rows per item (the register-decoding kernel's, else 16 or 8 dividing N; 0: none); items per expert and token
// group: ceil(N / rows)
int gemv_row_tile(int qtype, int K, int N, bool gu);
int launch_gemv_gu(const ExpertGemvArgs& a, cudaStream_t st);
int launch_gemv_down(const ExpertGemvArgs& a, cudaStream_t st);

// out[E + 1] = exclusive scan over experts of ceil(counts[e] / unit_rows) * mult (one CTA)
int launch_unit_scan(const int32_t* counts, int E, int unit_rows, int mult, int32_t* out, cudaStream_t st);

// ---------------------------------------------------------------- combine.cu
// out[t] = sum_i w[t, i] y[slot[t k + i]] in slot order, fp32; out f32 or bf16. y rows are f32 (y_dtype F32) or bf16.
// Rows slot in [own_lo, own_hi) come from own + (s - own_lo) rows instead of y + s rows (expert parallelism: the rank's
// own block stays where its experts wrote it); own = null: every row from y.
struct CombineOwn {
  const void* own = nullptr;
  int64_t own_lo = 0, own_hi = 0;
};
// the shared expert's term: out_t += s[t] y[t] in the same fp32 sum (y = null: none)
struct CombineShared {
  const void* y = nullptr;
  int y_dtype = 0;
  const float* s = nullptr;
};
int launch_combine(const void* y, int y_dtype, const int32_t* slot, const float* w, int64_t T, int k, int H, void* out,
                   int out_dtype, cudaStream_t st, CombineOwn own = CombineOwn{}, CombineShared sh = CombineShared{},
                   const void* res = nullptr);  // res: rows of out_dtype added last (the residual), or null
// out = rms_norm(x, w, eps) row by row (T rows of H, x and out of x_dtype; w: H values of w_dtype F32 / BF16)
int launch_norm(const void* x, int x_dtype, const void* w, int w_dtype, double eps, int64_t T, int H, void* out,
                cudaStream_t st);
// the shared expert's gates: s[t] = sigmoid(x_t . g) in fp32 (g: H values of g_dtype F32 / BF16; g = null: 1); also
// its one row group: off = {0, T}, then the count T (int32) after them
int launch_shared_gate(const void* x, int x_dtype, const void* g, int g_dtype, int64_t T, int H, float* s,
                       int64_t* off, cudaStream_t st);

// gather x rows into dispatch order: xp[i] = x[perm[i] / k] (bf16 out; x f32 or bf16); rows i in [own_lo, own_hi)
// go to own_dst + (i - own_lo) rows instead (own_dst null: all to xp)
int launch_gather(const void* x, int x_dtype, const int32_t* perm, int64_t P, int k, int H, uint16_t* xp,
                  cudaStream_t st, uint16_t* own_dst = nullptr, int64_t own_lo = 0, int64_t own_hi = 0);

// ---------------------------------------------------------------- mss.cu
// The small-batch tensor-core GEMVs (Q4_K, bf16 x): gate / up items of 32 output rows into h (fragment order + group
// sums: hq, hs), down items of 128 output rows into fp32 y, both over the dispatch's pair groups of <= 8.
struct MssLaunch {
  const CUtensorMap *gate_map, *up_map, *down_map;  // raw rows: gate / up boxes of 32 rows, down boxes of 128 rows (Q4_K)
  int H, F, E, k;
  const void* x;  // bf16 token rows; pair d's row is perm[d] / k
  uint4* hq;      // h of the pairs in fragment order (F / 32 groups a row), then
  float* hs;      // their group sums
  float* y;       // fp32 output rows (pairs x H)
  const int32_t *unit_gu, *unit_dn;  // items per expert (exclusive scans: mss_mult_* x ceil(pairs / 8))
  const int64_t* offsets;
  const int32_t* perm;
  int slots;  // token slots to stage: min(8, the most pairs an expert can get)
  DevStatus* status;
  int down_qtype;          // ARTLITE_Q4_K (down_map) or ARTLITE_Q6_K (down_raw: E H rows of rb_dn bytes)
  const uint8_t* down_raw;
  int64_t rb_dn;
};
bool mss_ok(int qtype, int down_qtype, int x_dtype, int H, int F, bool has_maps);
int mss_mult_gu(int F);
int mss_mult_dn(int H);
int launch_mss(const MssLaunch& s, bool gu, cudaStream_t st);

}  // namespace artlite
