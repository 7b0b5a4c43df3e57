// The MoE block handle (artlite_moe_create / set_weights / forward / sync / debug / destroy): raw GGUF expert blocks
// resident in HBM, per-handle workspaces sized for max_tokens, and the forward's kernel sequence on one stream:
//   router (x W_r^T, fp32) -> route (ids, w) -> dispatch (offsets, perm, slot) -> experts -> combine (y).
// The experts run on one of two paths:
//   gemv  (path 1; decode batches): CUDA-core dequant-GEMVs, fp32 dequant and accumulation (gemv.cu);
//   tc    (path 2; prefill): the token rows gathered into dispatch order (bf16), then tcgen05 grouped GEMMs over the
//         raw quantised blocks dequantised in shared memory (tc_gemm.cu), h and y in bf16.
// The order of the stages is MoEPrefill.items (src/artlite/moe/prefill.py:102-125) minus the NPU's host round trip:
// routing and dispatch run on the GPU between the router and the experts.
#include <cuda_runtime.h>
#include <stdlib.h>
#include <string.h>

#include <algorithm>
#include <chrono>
#include <memory>
#include <thread>
#include <string>
#include <vector>

#include "common.cuh"
#include "kernels.cuh"
#include "tc_gemm.cuh"
#include "block.cuh"



namespace artlite {
namespace {

int status_error(const DevStatus& s, int E) {
  if (s.code == ARTLITE_ETIMEOUT) {
    set_error("moe: a bounded device wait ran out (site %d, block %d)", s.a, s.b);
    return ARTLITE_ETIMEOUT;
  }
  if (s.code == ARTLITE_EDEVICE) {
    set_error("moe: expert id %d of %d from the routing", s.a, E);
    return ARTLITE_EDEVICE;
  }
  if (s.code) {
    set_error("moe: device status %d (%d %d %d)", s.code, s.a, s.b, s.c);
    return s.code;
  }
  return ARTLITE_OK;
}

// a bounded wait for an event recorded earlier
int wait_event(cudaEvent_t e, int timeout_ms) {
  if (timeout_ms <= 0) timeout_ms = 60000;
  const auto t0 = std::chrono::steady_clock::now();
  for (;;) {
    const cudaError_t q = cudaEventQuery(e);
    if (q == cudaSuccess) return ARTLITE_OK;
    if (q != cudaErrorNotReady) {
      set_error("moe: %s", cudaGetErrorString(q));
      return ARTLITE_ECUDA;
    }
    if (std::chrono::steady_clock::now() - t0 > std::chrono::milliseconds(timeout_ms)) {
      set_error("moe: no completion within %d ms", timeout_ms);
      return ARTLITE_ETIMEOUT;
    }
    std::this_thread::yield();
  }
}

int wait(cudaStream_t st, int timeout_ms) {
  if (timeout_ms <= 0) timeout_ms = 60000;
  cudaEvent_t e;
  AL_CUDA(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
  AL_CUDA(cudaEventRecord(e, st));
  const auto t0 = std::chrono::steady_clock::now();
  for (;;) {
    const cudaError_t q = cudaEventQuery(e);
    if (q == cudaSuccess) break;
    if (q != cudaErrorNotReady) {
      cudaEventDestroy(e);
      set_error("moe: %s", cudaGetErrorString(q));
      return ARTLITE_ECUDA;
    }
    if (std::chrono::steady_clock::now() - t0 > std::chrono::milliseconds(timeout_ms)) {
      cudaEventDestroy(e);
      set_error("moe: no completion within %d ms", timeout_ms);
      return ARTLITE_ETIMEOUT;
    }
    std::this_thread::yield();
  }
  cudaEventDestroy(e);
  return ARTLITE_OK;
}

}  // namespace
}  // namespace artlite


namespace artlite {

int wait_deadline(cudaStream_t st, int timeout_ms) { return wait(st, timeout_ms); }

bool mss_use(const artlite_moe& h, const ExpertWeights& W, int path, int x_dtype, int F);

int expert_path(const artlite_moe& h, int64_t P, const artlite_moe::Layer& L) {
  const artlite_moe_desc& d = h.d;
  const bool tc = tc_supported(L.qtype, d.hidden, d.expert_ffn) && tc_supported(L.down_qtype, d.expert_ffn, d.hidden);
  if (d.path == 1 || !tc) return 1;
  if (d.path == 2) return 2;
  // the fused decode kernel where it applies (up to 512 pairs), else tcgen05 for prefill-sized batches (on average 4
  // pairs an expert or more) and the GEMVs for decode batches
  if (decode_fused_ok(h, L, P / d.top_k)) return 1;
  // decode-sized batches of layers the fused kernel does not take (Q4_K gate / up with a Q6_K down) stay on the
  // small-batch tensor-core GEMVs up to 64 tokens
  if (P <= 64 * (int64_t)d.top_k && mss_use(h, routed_weights(L), 1, d.act_dtype, d.expert_ffn)) return 1;
  return P >= 4 * (int64_t)h.E_local ? 2 : 1;
}

// the norm done inside the kernel that first reads the rows (ARTLITE_NORM_FUSE=0: the norm kernel first, always;
// read at each forward, so that a benchmark can time both in one process)
static bool norm_fusion_on() {
  const char* v = getenv("ARTLITE_NORM_FUSE");
  return !(v && v[0] == '0');
}

int run_norm(artlite_moe* h, const NormIn& n, void* xn, int64_t T, cudaStream_t st) {
  return launch_norm(n.x, h->d.act_dtype, n.w, n.w_dtype, n.eps, T, h->d.hidden, xn, st);
}

int route_and_dispatch(artlite_moe* h, const artlite_moe::Layer& L, const void* xd, int64_t T, cudaStream_t st,
                       Marker& mk, int mult_gu, int mult_dn, const NormIn* norm) {
  const artlite_moe_desc& d = h->d;
  const int H = d.hidden, E = d.n_experts, K = d.top_k;
  if (T > 0) {
    // the norm in the CTA-per-expert router where it applies, else the norm kernel first
    const bool fuse = norm && router_small_ok(T, H) && router_small_norms(T, H, d.act_dtype) && norm_fusion_on();
    if (norm && !fuse) AL_TRY(run_norm(h, *norm, const_cast<void*>(xd), T, st));
    NormFuse nf{};
    if (fuse) nf = {norm->x, norm->w, norm->w_dtype, norm->eps};
    if (router_small_ok(T, H))
      AL_TRY(launch_router_small(xd, d.act_dtype, L.router.ptr, L.router_qtype, L.has_bias ? L.bias.as<float>() : nullptr,
                                 T, H, E, h->logits.as<float>(), st, fuse ? &nf : nullptr));
    else if (L.n_planes)
      AL_TRY(launch_router_tc(static_cast<const uint16_t*>(xd), L.planes.as<uint16_t>(), L.n_planes,
                              L.has_bias ? L.bias.as<float>() : nullptr, T, H, E, T, h->logits.as<float>(),
                              h->status.as<DevStatus>(), st));
    else
      AL_TRY(launch_router(xd, d.act_dtype, L.router.ptr, L.router_qtype, L.has_bias ? L.bias.as<float>() : nullptr,
                           T, H, E, h->logits.as<float>(), st));
  }
  AL_TRY(mk.mark());
  RouteArgs ra{h->logits.as<float>(), T, E, E, 0, E, K, d.gating, K <= 16 && E % 16 == 0 && E <= 512,
               h->ids.as<int32_t>(), h->w.as<float>()};
  DispatchArgs da{};
  da.ids = h->ids.as<int32_t>();
  da.P = T * K;
  da.E = E;
  da.blk_counts = h->blk.as<int32_t>();
  da.offsets = h->offsets.as<int64_t>();
  da.perm = h->perm.as<int32_t>();
  da.slot = h->slot.as<int32_t>();
  da.counts = h->counts.as<int32_t>();
  da.status = h->status.as<DevStatus>();
  da.blk_pairs = kDispatchBlockPairsFwd;
  if (mult_gu > 0 && T > 0) {  // decode-sized: one kernel, with the GEMVs' unit scans
    da.unit_rows = kGemvTokens;
    da.unit_mult = mult_gu;
    da.unit_off = h->unit_gu.as<int32_t>();
    AL_TRY(launch_route_dispatch_small(ra, da, mult_dn, h->unit_dn.as<int32_t>(), st));
  } else {
    AL_TRY(launch_route(ra, st));
    AL_TRY(launch_dispatch(da, st));
  }
  return mk.mark();
}

// The decode-sized plan of a forward: both GEMVs' items per expert and token group (0, 0 when the fused routing /
// dispatch kernel does not apply).
bool mss_use(const artlite_moe& h, const ExpertWeights& W, int path, int x_dtype, int F) {
  static const bool off = [] {
    const char* v = getenv("ARTLITE_DECODE_MSS");
    return v && v[0] == '0';
  }();
  return !off && path == 1 && W.ss_gate && (W.ss_down || W.down_qtype == ARTLITE_Q6_K) &&
         mss_ok(W.qtype, W.down_qtype, x_dtype, h.d.hidden, F, true);
}

void small_plan(const artlite_moe& h, const artlite_moe::Layer& L, int path, int64_t T, int* mult_gu, int* mult_dn) {
  const artlite_moe_desc& d = h.d;
  *mult_gu = *mult_dn = 0;
  if (path != 1 || T <= 0 || !small_dispatch_ok(T * d.top_k, d.n_experts) || !router_small_ok(T, d.hidden)) return;
  if (mss_use(h, routed_weights(L), path, d.act_dtype, d.expert_ffn)) {
    *mult_gu = mss_mult_gu(d.expert_ffn);
    *mult_dn = mss_mult_dn(d.hidden);
    return;
  }
  const int rt_gu = gemv_row_tile(L.qtype, d.hidden, d.expert_ffn, true);
  const int rt_dn = gemv_row_tile(L.down_qtype, d.expert_ffn, d.hidden, false);
  if (rt_gu <= 0 || rt_dn <= 0) return;
  *mult_gu = (int)cdiv(d.expert_ffn, rt_gu);
  *mult_dn = (int)cdiv(d.hidden, rt_dn);
}

int run_experts(artlite_moe* h, const ExpertWeights& L, int path, const void* x, int x_dtype, bool gathered,
                const int32_t* perm, int k, int64_t P, int E_run, const int64_t* offsets, const int32_t* counts,
                int64_t x_rows, void** y_rows, int* y_dtype, cudaStream_t st, Marker& mk, bool units_ready,
                const int32_t* wexp, int E_w, int F_run, void* y_out) {
  const artlite_moe_desc& d = h->d;
  const int H = d.hidden, F = F_run > 0 ? F_run : d.expert_ffn;
  *y_rows = y_out ? y_out : h->y.ptr;
  if (path == 1 && !wexp && mss_use(*h, L, path, x_dtype, F)) {  // the small-batch tensor-core GEMVs (no row-group map)
    *y_dtype = ARTLITE_F32;
    if (P == 0) return ARTLITE_OK;
    if (!units_ready) {
      AL_TRY(launch_unit_scan(counts, E_run, kGemvTokens, mss_mult_gu(F), h->unit_gu.as<int32_t>(), st));
      AL_TRY(launch_unit_scan(counts, E_run, kGemvTokens, mss_mult_dn(H), h->unit_dn.as<int32_t>(), st));
    }
    MssLaunch s{};
    s.gate_map = L.ss_gate;
    s.up_map = L.ss_up;
    s.down_map = L.ss_down;
    s.down_qtype = L.down_qtype;
    s.down_raw = L.down;
    s.rb_dn = L.rb_dn;
    s.H = H;
    s.F = F;
    s.E = E_run;
    s.k = k;
    s.x = x;
    s.hq = h->h.as<uint4>();
    s.hs = reinterpret_cast<float*>(h->h.as<uint8_t>() + sizeof(uint16_t) * P * F);
    s.y = static_cast<float*>(*y_rows);
    s.unit_gu = h->unit_gu.as<int32_t>();
    s.unit_dn = h->unit_dn.as<int32_t>();
    s.offsets = offsets;
    s.perm = perm;
    s.slots = (int)std::min<int64_t>(kGemvTokens, k > 1 ? P / k : P);  // (a token's k pairs go to distinct experts)
    s.status = h->status.as<DevStatus>();
    AL_TRY(launch_mss(s, true, st));
    AL_TRY(mk.mark());
    AL_TRY(launch_mss(s, false, st));
    return mk.mark();
  }
  if (path == 1) {
    *y_dtype = ARTLITE_F32;
    if (P == 0) return ARTLITE_OK;
    const int rt_gu = gemv_row_tile(L.qtype, H, F, true), rt_dn = gemv_row_tile(L.down_qtype, F, H, false);
    AL_CHECK(rt_gu > 0 && rt_dn > 0, ARTLITE_EUNSUPPORTED, "expert gemv: no row tile for F %d / H %d", F, H);
    if (!units_ready) {
      AL_TRY(launch_unit_scan(counts, E_run, kGemvTokens, (int)cdiv(F, rt_gu), h->unit_gu.as<int32_t>(), st));
      AL_TRY(launch_unit_scan(counts, E_run, kGemvTokens, (int)cdiv(H, rt_dn), h->unit_dn.as<int32_t>(), st));
    }
    ExpertGemvArgs g{};
    g.qtype = L.qtype;
    g.w0 = L.gate;
    g.w1 = L.up;
    g.row_bytes = L.rb_gu;
    g.K = H;
    g.N = F;
    g.E = E_run;
    g.x = x;
    g.x_dtype = x_dtype;
    g.perm = perm;
    g.offsets = offsets;
    g.unit_off = h->unit_gu.as<int32_t>();
    g.rt = rt_gu;
    g.wexp = wexp;
    g.k = k;
    g.out = h->h.as<float>();
    AL_TRY(launch_gemv_gu(g, st));
    AL_TRY(mk.mark());
    ExpertGemvArgs dn = g;
    dn.qtype = L.down_qtype;
    dn.w0 = L.down;
    dn.w1 = nullptr;
    dn.row_bytes = L.rb_dn;
    dn.K = F;
    dn.N = H;
    dn.x = h->h.ptr;
    dn.x_dtype = ARTLITE_F32;
    dn.unit_off = h->unit_dn.as<int32_t>();
    dn.rt = rt_dn;
    dn.out = static_cast<float*>(*y_rows);
    AL_TRY(launch_gemv_down(dn, st));
    return mk.mark();
  }
  *y_dtype = ARTLITE_BF16;
  if (P == 0) return ARTLITE_OK;
  const uint16_t* xg = static_cast<const uint16_t*>(x);
  if (!gathered) {
    AL_TRY(launch_gather(x, x_dtype, perm, P, k, H, h->xp.as<uint16_t>(), st));
    xg = h->xp.as<uint16_t>();
    x_rows = (int64_t)(h->xp.bytes / (sizeof(uint16_t) * H));
  }
  TcGemmArgs g{};
  g.qtype = L.qtype;
  g.w0 = L.gate;
  g.w1 = L.up;
  g.row_bytes = L.rb_gu;
  g.K = H;
  g.N = F;
  g.E = E_run;
  g.x = xg;
  g.x_rows = x_rows;
  g.status = h->status.as<DevStatus>();
  g.P = P;
  g.offsets = offsets;
  g.counts = counts;
  g.wexp = wexp;
  g.wE = E_w;
  g.sched = h->tiles.ptr;
  g.out = h->h.as<uint16_t>();
  AL_TRY(launch_tc_gemm(g, /*gu=*/true, st));
  AL_TRY(mk.mark());
  TcGemmArgs dn = g;
  dn.qtype = L.down_qtype;
  dn.w0 = L.down;
  dn.w1 = nullptr;
  dn.row_bytes = L.rb_dn;
  dn.K = F;
  dn.N = H;
  dn.x = h->h.as<uint16_t>();
  dn.x_rows = (int64_t)(h->h.bytes / (sizeof(uint16_t) * F));
  dn.out = static_cast<uint16_t*>(*y_rows);
  AL_TRY(launch_tc_gemm(dn, /*gu=*/false, st));
  return mk.mark();
}

// the layer's shared expert on all T tokens (one row group, token order) and its gates, for the combine
// the captured forwards name the weights' and workspaces' addresses: new weights (which may move them) drop them
void drop_graphs(artlite_moe* h) {
  for (const artlite_moe::Graph& g : h->graphs) cudaGraphExecDestroy(g.exec);
  h->graphs.clear();
}

int run_shared(artlite_moe* h, const artlite_moe::Layer& L, const void* xd, int64_t T, cudaStream_t st,
               CombineShared* sh) {
  const artlite_moe_desc& d = h->d;
  const int H = d.hidden, F = L.sh_F;
  AL_TRY(launch_shared_gate(xd, d.act_dtype, L.sh_has_gate ? L.sh_ginp.ptr : nullptr, L.sh_gate_dtype, T, H,
                            h->sh_s.as<float>(), h->sh_off.as<int64_t>(), st));
  const ExpertWeights W = shared_weights(L);
  const bool tc = T >= 64 && tc_supported(W.qtype, H, F) && tc_supported(W.down_qtype, F, H);
  int64_t* off = h->sh_off.as<int64_t>();  // (written by the gate kernel: {0, T} and the count T)
  int32_t* cnt = reinterpret_cast<int32_t*>(off + 2);
  Marker quiet{h, 0, st};
  quiet.ns = kStages;
  void* yrows;
  int ydt;
  AL_TRY(run_experts(h, W, tc ? 2 : 1, xd, d.act_dtype, false, h->sh_iota.as<int32_t>(), 1, T, 1, off, cnt, 0, &yrows,
                     &ydt, st, quiet, false, nullptr, 0, F, h->sh_y.ptr));
  sh->y = yrows;
  sh->y_dtype = ydt;
  sh->s = h->sh_s.as<float>();
  return ARTLITE_OK;
}

}  // namespace artlite

using namespace artlite;

extern "C" {
#pragma GCC visibility push(default)

int artlite_moe_create(const artlite_moe_desc* desc, artlite_moe** out) {
  AL_CHECK(desc && out, ARTLITE_EINVAL, "moe_create: null argument");
  const artlite_moe_desc& d = *desc;
  AL_CHECK(d.hidden > 0 && d.n_experts > 0 && d.top_k >= 1 && d.top_k <= d.n_experts && d.expert_ffn > 0 &&
               d.n_layers >= 1 && d.max_tokens >= 0 && (d.gating == 0 || d.gating == 1),
           ARTLITE_EINVAL, "moe_create: H %d E %d K %d F %d layers %d max_tokens %d gating %d", d.hidden,
           d.n_experts, d.top_k, d.expert_ffn, d.n_layers, d.max_tokens, d.gating);
  AL_CHECK(d.act_dtype == ARTLITE_F32 || d.act_dtype == ARTLITE_BF16, ARTLITE_EINVAL,
           "moe_create: act_dtype %d (F32 or BF16)", d.act_dtype);
  AL_CHECK(d.n_experts <= 1024 && d.top_k <= 32 && d.hidden % 256 == 0 && d.expert_ffn % 256 == 0,
           ARTLITE_EUNSUPPORTED, "moe_create: E %d K %d H %d F %d (this build: E <= 1024, K <= 32, H and F "
           "multiples of 256)", d.n_experts, d.top_k, d.hidden, d.expert_ffn);
  const int world = d.ep_world > 0 ? d.ep_world : 1;
  AL_CHECK(d.ep_rank >= 0 && d.ep_rank < world && d.n_experts % world == 0, ARTLITE_EINVAL,
           "moe_create: rank %d of %d with %d experts", d.ep_rank, world, d.n_experts);
  std::unique_ptr<artlite_moe> h(new artlite_moe);
  h->d = d;
  if (d.device >= 0) AL_CUDA(cudaSetDevice(d.device));
  AL_CUDA(cudaGetDevice(&h->dev));
  AL_CUDA(cudaStreamCreateWithFlags(&h->st, cudaStreamNonBlocking));
  AL_CUDA(cudaEventCreateWithFlags(&h->done, cudaEventDisableTiming));
  h->E_local = d.n_experts / world;
  h->e0 = d.ep_rank * h->E_local;
  h->layers.resize(d.n_layers);
  const char* tm = getenv("ARTLITE_MOE_TIMING");
  h->timing = tm && tm[0] == '1';
  h->n_stages.assign(d.n_layers, 0);
  h->paths.assign(d.n_layers, 0);
  if (h->timing) {
    h->ev.assign((size_t)d.n_layers * kStages, nullptr);
    for (cudaEvent_t& e : h->ev) AL_CUDA(cudaEventCreate(&e));
  }
  const int64_t T = d.max_tokens > 0 ? d.max_tokens : 1, P = T * d.top_k;
  const int H = d.hidden, E = d.n_experts, F = d.expert_ffn;
  AL_TRY(h->logits.reserve(sizeof(float) * T * E));
  AL_TRY(h->ids.reserve(sizeof(int32_t) * P));
  AL_TRY(h->w.reserve(sizeof(float) * P));
  AL_TRY(h->offsets.reserve(sizeof(int64_t) * (E + 1)));
  AL_TRY(h->perm.reserve(sizeof(int32_t) * P));
  AL_TRY(h->slot.reserve(sizeof(int32_t) * P));
  AL_TRY(h->counts.reserve(sizeof(int32_t) * E));
  AL_TRY(h->blk.reserve(dispatch_scratch_bytes(P, E, kDispatchBlockPairsFwd)));
  AL_TRY(h->unit_gu.reserve(sizeof(int32_t) * (E + 1)));
  AL_TRY(h->unit_dn.reserve(sizeof(int32_t) * (E + 1)));
  AL_TRY(h->status.reserve(sizeof(DevStatus)));
  AL_TRY(h->tiles.reserve(tc_sched_bytes(E)));
  // h and y hold fp32 rows (gemv) or bf16 rows (tc: at least P + 256 of them, whole 256-row token boxes)
  AL_TRY(h->h.reserve(std::max(sizeof(float) * P * F, sizeof(uint16_t) * (P + 256) * F)));
  AL_TRY(h->y.reserve(sizeof(float) * P * H));
  AL_TRY(h->xp.reserve(sizeof(uint16_t) * (P + 256) * H));
  const size_t act = d.act_dtype == ARTLITE_BF16 ? 2 : 4;
  AL_TRY(h->xin.reserve(act * T * H));
  AL_TRY(h->yout.reserve(act * T * H));
  AL_CUDA(cudaMemsetAsync(h->status.ptr, 0, sizeof(DevStatus), h->st));
  // the fused decode kernel's grid barrier, zeroed now: a forward captured into a graph must not allocate
  AL_TRY(h->bar.reserve(1024));
  AL_CUDA(cudaMemsetAsync(h->bar.ptr, 0, 1024, h->st));
  if (world > 1) AL_TRY(ep_create(h.get()));
  AL_CUDA(cudaStreamSynchronize(h->st));
  *out = h.release();
  return ARTLITE_OK;
}

int artlite_moe_set_weights(artlite_moe* h, int layer, int qtype, const void* gate, const void* up, int down_qtype,
                            const void* down, const void* router, int router_qtype) {
  AL_CHECK(h, ARTLITE_EINVAL, "moe_set_weights: null handle");
  drop_graphs(h);
  AL_CHECK(layer >= 0 && layer < (int)h->layers.size(), ARTLITE_EINVAL, "moe_set_weights: layer %d of %d", layer,
           (int)h->layers.size());
  AL_CHECK(gate && up && down && router, ARTLITE_EINVAL, "moe_set_weights: null tensor");
  AL_CHECK(router_qtype == ARTLITE_F32 || router_qtype == ARTLITE_BF16, ARTLITE_EINVAL,
           "moe_set_weights: router type %d (F32 or BF16)", router_qtype);
  int per, bytes, per_d, bytes_d;
  AL_TRY(qtype_block(qtype, &per, &bytes));
  AL_TRY(qtype_block(down_qtype, &per_d, &bytes_d));
  const artlite_moe_desc& d = h->d;
  AL_CHECK(d.hidden % per == 0 && d.expert_ffn % per_d == 0, ARTLITE_EINVAL, "moe_set_weights: H %d / F %d and blocks "
           "of %d / %d", d.hidden, d.expert_ffn, per, per_d);
  AL_CUDA(cudaSetDevice(h->dev));
  artlite_moe::Layer& L = h->layers[layer];
  L.qtype = qtype;
  L.down_qtype = down_qtype;
  L.router_qtype = router_qtype;
  L.rb_gu = (int64_t)d.hidden / per * bytes;
  L.rb_dn = (int64_t)d.expert_ffn / per_d * bytes_d;
  const int64_t F = d.expert_ffn, H = d.hidden;
  const size_t gu_bytes = (size_t)(h->E_local * F * L.rb_gu), dn_bytes = (size_t)(h->E_local * H * L.rb_dn);
  const size_t r_bytes = (size_t)d.n_experts * H * (router_qtype == ARTLITE_F32 ? 4 : 2);
  // (64 bytes of slack past each tensor: the loaders read whole 16-byte words)
  AL_TRY(L.gate.reserve(gu_bytes + 64));
  AL_TRY(L.up.reserve(gu_bytes + 64));
  AL_TRY(L.down.reserve(dn_bytes + 64));
  AL_TRY(L.router.reserve(r_bytes));
  const uint8_t* g8 = static_cast<const uint8_t*>(gate) + (size_t)(h->e0 * F * L.rb_gu);
  const uint8_t* u8 = static_cast<const uint8_t*>(up) + (size_t)(h->e0 * F * L.rb_gu);
  const uint8_t* d8 = static_cast<const uint8_t*>(down) + (size_t)(h->e0 * H * L.rb_dn);
  AL_CUDA(cudaMemcpyAsync(L.gate.ptr, g8, gu_bytes, cudaMemcpyDefault, h->st));
  AL_CUDA(cudaMemcpyAsync(L.up.ptr, u8, gu_bytes, cudaMemcpyDefault, h->st));
  AL_CUDA(cudaMemcpyAsync(L.down.ptr, d8, dn_bytes, cudaMemcpyDefault, h->st));
  AL_CUDA(cudaMemcpyAsync(L.router.ptr, router, r_bytes, cudaMemcpyDefault, h->st));
  AL_CUDA(cudaMemsetAsync(static_cast<uint8_t*>(L.gate.ptr) + gu_bytes, 0, 64, h->st));
  AL_CUDA(cudaMemsetAsync(static_cast<uint8_t*>(L.up.ptr) + gu_bytes, 0, 64, h->st));
  AL_CUDA(cudaMemsetAsync(static_cast<uint8_t*>(L.down.ptr) + dn_bytes, 0, 64, h->st));
  L.has_dm = L.has_dm_gu = false;
  if (qtype == ARTLITE_Q4_K && F % 64 == 0 && H % 128 == 0) {
    AL_TRY(make_raw_map(&L.dm_gate, L.gate.ptr, L.rb_gu, h->E_local * F, 144, 64));
    AL_TRY(make_raw_map(&L.dm_up, L.up.ptr, L.rb_gu, h->E_local * F, 144, 64));
    L.has_dm_gu = true;
    if (down_qtype == ARTLITE_Q4_K) {
      AL_TRY(make_raw_map(&L.dm_down, L.down.ptr, L.rb_dn, h->E_local * H, 144, 128));
      L.has_dm = true;
    }
  }
  L.has_ss = false;  // (the small-batch GEMVs' gate / up maps: Q4_K gate / up, whatever the down type)
  if (qtype == ARTLITE_Q4_K && F % 32 == 0 && H % 128 == 0) {
    AL_TRY(make_raw_map(&L.ss_gate, L.gate.ptr, L.rb_gu, h->E_local * F, 144, 32));
    AL_TRY(make_raw_map(&L.ss_up, L.up.ptr, L.rb_gu, h->E_local * F, 144, 32));
    L.has_ss = true;
  }
  L.n_planes = 0;
  if (router_tc_supported(d.n_experts, d.hidden, d.act_dtype)) {
    L.n_planes = router_qtype == ARTLITE_F32 ? 3 : 1;
    AL_TRY(L.planes.reserve(sizeof(uint16_t) * 3 * d.n_experts * H));
    AL_TRY(router_split(L.router.ptr, router_qtype, d.n_experts, (int)H, L.planes.as<uint16_t>(), h->st));
  }
  return wait(h->st, 0);
}

int artlite_moe_forward(artlite_moe* h, int layer, const void* x, void* y, int64_t T, void* stream) {
  AL_CHECK(h, ARTLITE_EINVAL, "moe_forward: null handle");
  AL_CHECK(layer >= 0 && layer < (int)h->layers.size() && h->layers[layer].qtype >= 0, ARTLITE_EINVAL,
           "moe_forward: layer %d has no weights", layer);
  AL_CHECK(T >= 0 && T <= (h->d.max_tokens > 0 ? h->d.max_tokens : 1), ARTLITE_EINVAL,
           "moe_forward: T %lld (max_tokens %d)", (long long)T, h->d.max_tokens);
  AL_CHECK(T == 0 || (x && y), ARTLITE_EINVAL, "moe_forward: null x / y");
  const artlite_moe_desc& d = h->d;
  const artlite_moe::Layer& L = h->layers[layer];
  const int H = d.hidden, E = d.n_experts, K = d.top_k;
  const int64_t P = T * K;
  const size_t act = d.act_dtype == ARTLITE_BF16 ? 2 : 4;
  AL_CUDA(cudaSetDevice(h->dev));
  cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : h->st;
  h->last_T = T;
  if (T == 0 && h->E_local == E) return ARTLITE_OK;  // (with expert parallelism a rank without tokens still serves)
  const bool x_dev = T > 0 && is_device_ptr(x) && ((uintptr_t)x % 16) == 0;
  const bool y_dev = T > 0 && is_device_ptr(y) && ((uintptr_t)y % 16) == 0;
  const void* xd = x;
  if (T > 0 && !x_dev) {
    AL_CUDA(cudaMemcpyAsync(h->xin.ptr, x, act * T * H, cudaMemcpyDefault, st));
    xd = h->xin.ptr;
  }
  void* yd = y_dev ? y : h->yout.ptr;
  Marker mk{h, layer, st};
  AL_TRY(mk.mark());
  // a layer with a norm: its input is added back to the output (res); the normed rows go to xn, normed by the first
  // kernel that reads them where it can (the fused decode kernel, the CTA-per-expert router), else by the norm kernel
  const void* res = nullptr;
  NormIn norm;
  if (L.has_norm && T > 0) {
    norm = NormIn{xd, L.norm_w.ptr, L.norm_dtype, L.norm_eps};
    res = xd;
    xd = h->xn.ptr;
  }
  const NormIn* nin = norm.x ? &norm : nullptr;
  if (h->E_local < E) {
    if (nin) AL_TRY(run_norm(h, norm, h->xn.ptr, T, st));
    AL_TRY(ep_forward(h, layer, xd, yd, T, st, mk, res));
  } else {
    const int path = expert_path(*h, P, L);
    h->last_path = path;
    h->paths[layer] = path;
    if (path == 1 && decode_fused_ok(*h, L, T)) {
      if (nin && !norm_fusion_on()) {
        AL_TRY(run_norm(h, norm, h->xn.ptr, T, st));
        nin = nullptr;
      }
      AL_TRY(launch_decode(h, L, xd, yd, T, st, res, nin));
    } else {
      int mult_gu, mult_dn;
      small_plan(*h, L, path, T, &mult_gu, &mult_dn);
      AL_TRY(route_and_dispatch(h, L, xd, T, st, mk, mult_gu, mult_dn, nin));
      void* yrows;
      int ydt;
      AL_TRY(run_experts(h, routed_weights(L), path, xd, d.act_dtype, false, h->perm.as<int32_t>(), K, P, E,
                         h->offsets.as<int64_t>(), h->counts.as<int32_t>(), 0, &yrows, &ydt, st, mk, mult_gu > 0));
      CombineShared sh;
      if (L.has_shared) AL_TRY(run_shared(h, L, xd, T, st, &sh));
      AL_TRY(launch_combine(yrows, ydt, h->slot.as<int32_t>(), h->w.as<float>(), T, K, H, yd, d.act_dtype, st,
                            CombineOwn{}, sh, res));
    }
  }
  AL_TRY(mk.mark());
  h->n_stages[layer] = mk.ns;
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  AL_CUDA(cudaStreamIsCapturing(st, &cs));
  if (cs == cudaStreamCaptureStatusNone) AL_CUDA(cudaEventRecord(h->done, st));
  if (T > 0 && !y_dev) {
    AL_CUDA(cudaMemcpyAsync(y, yd, act * T * H, cudaMemcpyDefault, st));
    AL_TRY(wait_deadline(st, 0));
    DevStatus s;
    AL_CUDA(cudaMemcpy(&s, h->status.ptr, sizeof s, cudaMemcpyDeviceToHost));
    if (s.code) {
      AL_CUDA(cudaMemset(h->status.ptr, 0, sizeof s));
      if (h->bar.ptr) AL_CUDA(cudaMemset(h->bar.ptr, 0, h->bar.bytes));  // (a wait that ran out may leave it mid-way)
      return status_error(s, E);
    }
  }
  return ARTLITE_OK;
}

int artlite_moe_set_router_bias(artlite_moe* h, int layer, const float* bias) {
  AL_CHECK(h, ARTLITE_EINVAL, "moe_set_router_bias: null handle");
  drop_graphs(h);
  AL_CHECK(layer >= 0 && layer < (int)h->layers.size(), ARTLITE_EINVAL, "moe_set_router_bias: layer %d of %d", layer,
           (int)h->layers.size());
  AL_CUDA(cudaSetDevice(h->dev));
  artlite_moe::Layer& L = h->layers[layer];
  if (!bias) {
    L.has_bias = false;
    return ARTLITE_OK;
  }
  AL_TRY(L.bias.reserve(sizeof(float) * h->d.n_experts));
  AL_CUDA(cudaMemcpyAsync(L.bias.ptr, bias, sizeof(float) * h->d.n_experts, cudaMemcpyDefault, h->st));
  L.has_bias = true;
  return wait(h->st, 0);
}

int artlite_moe_set_norm(artlite_moe* h, int layer, const void* w, int w_dtype, double eps) {
  AL_CHECK(h, ARTLITE_EINVAL, "moe_set_norm: null handle");
  drop_graphs(h);
  AL_CHECK(layer >= 0 && layer < (int)h->layers.size(), ARTLITE_EINVAL, "moe_set_norm: layer %d of %d", layer,
           (int)h->layers.size());
  AL_CUDA(cudaSetDevice(h->dev));
  artlite_moe::Layer& L = h->layers[layer];
  if (!w) {
    L.has_norm = false;
    return ARTLITE_OK;
  }
  AL_CHECK(w_dtype == ARTLITE_F32 || w_dtype == ARTLITE_BF16, ARTLITE_EINVAL, "moe_set_norm: weight type %d", w_dtype);
  AL_CHECK(eps >= 0.0, ARTLITE_EINVAL, "moe_set_norm: eps %g", eps);
  AL_CHECK(h->d.hidden % 8 == 0, ARTLITE_EUNSUPPORTED, "moe_set_norm: H %d (a multiple of 8)", h->d.hidden);
  const size_t wb = (w_dtype == ARTLITE_F32 ? 4 : 2) * (size_t)h->d.hidden;
  const size_t act = h->d.act_dtype == ARTLITE_BF16 ? 2 : 4;
  const int64_t T = h->d.max_tokens > 0 ? h->d.max_tokens : 1;
  AL_TRY(L.norm_w.reserve(wb));
  AL_TRY(h->xn.reserve(act * T * h->d.hidden));
  AL_CUDA(cudaMemcpyAsync(L.norm_w.ptr, w, wb, cudaMemcpyDefault, h->st));
  L.norm_dtype = w_dtype;
  L.norm_eps = eps;
  L.has_norm = true;
  return wait(h->st, 0);
}

int artlite_moe_set_shared(artlite_moe* h, int layer, int ffn, int qtype, const void* gate, const void* up,
                           int down_qtype, const void* down, const void* gate_inp, int gate_dtype) {
  AL_CHECK(h, ARTLITE_EINVAL, "moe_set_shared: null handle");
  drop_graphs(h);
  AL_CHECK(layer >= 0 && layer < (int)h->layers.size(), ARTLITE_EINVAL, "moe_set_shared: layer %d of %d", layer,
           (int)h->layers.size());
  AL_CUDA(cudaSetDevice(h->dev));
  artlite_moe::Layer& L = h->layers[layer];
  if (!gate) {
    L.has_shared = false;
    return ARTLITE_OK;
  }
  AL_CHECK(up && down && ffn > 0, ARTLITE_EINVAL, "moe_set_shared: null up / down or ffn %d", ffn);
  AL_CHECK(!gate_inp || gate_dtype == ARTLITE_F32 || gate_dtype == ARTLITE_BF16, ARTLITE_EINVAL,
           "moe_set_shared: gate type %d (F32 or BF16)", gate_dtype);
  int per, bytes, per_d, bytes_d;
  AL_TRY(qtype_block(qtype, &per, &bytes));
  AL_TRY(qtype_block(down_qtype, &per_d, &bytes_d));
  const artlite_moe_desc& d = h->d;
  const int64_t H = d.hidden, F = ffn, T = d.max_tokens > 0 ? d.max_tokens : 1;
  AL_CHECK(H % per == 0 && F % per_d == 0, ARTLITE_EINVAL, "moe_set_shared: H %lld / ffn %lld and blocks of %d / %d",
           (long long)H, (long long)F, per, per_d);
  L.sh_F = ffn;
  L.sh_qtype = qtype;
  L.sh_down_qtype = down_qtype;
  L.sh_rb_gu = H / per * bytes;
  L.sh_rb_dn = F / per_d * bytes_d;
  const size_t gu_bytes = (size_t)(F * L.sh_rb_gu), dn_bytes = (size_t)(H * L.sh_rb_dn);
  AL_TRY(L.sh_gate.reserve(gu_bytes + 64));
  AL_TRY(L.sh_up.reserve(gu_bytes + 64));
  AL_TRY(L.sh_down.reserve(dn_bytes + 64));
  AL_CUDA(cudaMemcpyAsync(L.sh_gate.ptr, gate, gu_bytes, cudaMemcpyDefault, h->st));
  AL_CUDA(cudaMemcpyAsync(L.sh_up.ptr, up, gu_bytes, cudaMemcpyDefault, h->st));
  AL_CUDA(cudaMemcpyAsync(L.sh_down.ptr, down, dn_bytes, cudaMemcpyDefault, h->st));
  AL_CUDA(cudaMemsetAsync(static_cast<uint8_t*>(L.sh_gate.ptr) + gu_bytes, 0, 64, h->st));
  AL_CUDA(cudaMemsetAsync(static_cast<uint8_t*>(L.sh_up.ptr) + gu_bytes, 0, 64, h->st));
  AL_CUDA(cudaMemsetAsync(static_cast<uint8_t*>(L.sh_down.ptr) + dn_bytes, 0, 64, h->st));
  L.sh_has_gate = gate_inp != nullptr;
  if (gate_inp) {
    const size_t gb = (size_t)H * (gate_dtype == ARTLITE_F32 ? 4 : 2);
    AL_TRY(L.sh_ginp.reserve(gb));
    AL_CUDA(cudaMemcpyAsync(L.sh_ginp.ptr, gate_inp, gb, cudaMemcpyDefault, h->st));
    L.sh_gate_dtype = gate_dtype;
  }
  // the shared run's workspaces: all T tokens as one row group (rows 0 .. T - 1 in token order)
  AL_TRY(h->sh_y.reserve(sizeof(float) * T * H));
  AL_TRY(h->sh_s.reserve(sizeof(float) * T));
  AL_TRY(h->sh_off.reserve(sizeof(int64_t) * 2 + sizeof(int32_t)));
  AL_TRY(h->h.reserve(std::max(h->h.bytes, std::max(sizeof(float) * T * F, sizeof(uint16_t) * (T + 256) * F))));
  if (h->sh_iota.bytes < sizeof(int32_t) * T) {
    AL_TRY(h->sh_iota.reserve(sizeof(int32_t) * T));
    std::vector<int32_t> io(T);
    for (int64_t i = 0; i < T; i++) io[i] = (int32_t)i;
    AL_CUDA(cudaMemcpyAsync(h->sh_iota.ptr, io.data(), sizeof(int32_t) * T, cudaMemcpyHostToDevice, h->st));
    AL_TRY(wait(h->st, 0));
  }
  L.sh_has_dm = false;
  if (qtype == ARTLITE_Q4_K && down_qtype == ARTLITE_Q4_K && F % 64 == 0 && H % 128 == 0 &&
      (!gate_inp || gate_dtype == ARTLITE_F32)) {  // (the fused decode kernel can run this shared expert)
    AL_TRY(make_raw_map(&L.sh_dm_gate, L.sh_gate.ptr, L.sh_rb_gu, F, 144, 64));
    AL_TRY(make_raw_map(&L.sh_dm_up, L.sh_up.ptr, L.sh_rb_gu, F, 144, 64));
    AL_TRY(make_raw_map(&L.sh_dm_down, L.sh_down.ptr, L.sh_rb_dn, H, 144, 128));
    AL_TRY(h->sh_hq.reserve(std::max(h->sh_hq.bytes, (size_t)(sizeof(uint16_t) * T * F + sizeof(float) * T * (F / 32)))));
    L.sh_has_dm = true;
  }
  L.sh_has_ss = false;  // (decode batches below the fused kernel: the shared expert on the small-batch GEMVs)
  if (qtype == ARTLITE_Q4_K && F % 32 == 0 && H % 128 == 0) {
    AL_TRY(make_raw_map(&L.sh_ss_gate, L.sh_gate.ptr, L.sh_rb_gu, F, 144, 32));
    AL_TRY(make_raw_map(&L.sh_ss_up, L.sh_up.ptr, L.sh_rb_gu, F, 144, 32));
    L.sh_has_ss = true;
  }
  L.has_shared = true;
  return wait(h->st, 0);
}

int artlite_moe_forward_graph(artlite_moe* h, int layer, const void* x, void* y, int64_t T, void* stream) {
  AL_CHECK(h, ARTLITE_EINVAL, "moe_forward_graph: null handle");
  AL_CHECK(h->E_local == h->d.n_experts, ARTLITE_EUNSUPPORTED,
           "moe_forward_graph: not with expert parallelism (its exchange sizes are host values of each forward)");
  AL_CHECK(T > 0 && is_device_ptr(x) && is_device_ptr(y) && ((uintptr_t)x % 16) == 0 && ((uintptr_t)y % 16) == 0,
           ARTLITE_EINVAL, "moe_forward_graph: T > 0 and 16-byte aligned device x / y");
  AL_CUDA(cudaSetDevice(h->dev));
  cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : h->st;
  for (const artlite_moe::Graph& g : h->graphs)
    if (g.layer == layer && g.T == T && g.x == x && g.y == y) {
      AL_CUDA(cudaGraphLaunch(g.exec, st));
      AL_CUDA(cudaEventRecord(h->done, st));
      h->last_T = T;
      return ARTLITE_OK;
    }
  // capture one forward on a side stream (the tensor maps and workspaces it names stay valid: the handle owns them)
  cudaStream_t cap;
  AL_CUDA(cudaStreamCreateWithFlags(&cap, cudaStreamNonBlocking));
  const bool timing = h->timing;
  h->timing = false;  // (no per-stage events inside a graph)
  cudaGraph_t graph = nullptr;
  int rc = ARTLITE_OK;
  if (cudaStreamBeginCapture(cap, cudaStreamCaptureModeThreadLocal) != cudaSuccess) {
    rc = ARTLITE_ECUDA;
    set_error("moe_forward_graph: begin capture failed");
  } else {
    rc = artlite_moe_forward(h, layer, x, y, T, cap);
    const cudaError_t e = cudaStreamEndCapture(cap, &graph);
    if (rc == ARTLITE_OK && e != cudaSuccess) {
      rc = ARTLITE_ECUDA;
      set_error("moe_forward_graph: capture failed: %s", cudaGetErrorString(e));
    }
  }
  h->timing = timing;
  cudaStreamDestroy(cap);
  if (rc != ARTLITE_OK) {
    if (graph) cudaGraphDestroy(graph);
    cudaGetLastError();
    return rc;
  }
  cudaGraphExec_t exec;
  const cudaError_t ie = cudaGraphInstantiate(&exec, graph, 0);
  cudaGraphDestroy(graph);
  AL_CHECK(ie == cudaSuccess, ARTLITE_ECUDA, "moe_forward_graph: instantiate: %s", cudaGetErrorString(ie));
  h->graphs.push_back({layer, T, x, y, exec});
  AL_CUDA(cudaGraphLaunch(exec, st));
  AL_CUDA(cudaEventRecord(h->done, st));
  return ARTLITE_OK;
}

int artlite_moe_sync(artlite_moe* h, int timeout_ms) {
  AL_CHECK(h, ARTLITE_EINVAL, "moe_sync: null handle");
  AL_CUDA(cudaSetDevice(h->dev));
  AL_TRY(wait(h->st, timeout_ms));
  AL_TRY(wait_event(h->done, timeout_ms));  // (the last forward, on whichever stream it was enqueued)
  DevStatus s;
  AL_CUDA(cudaMemcpy(&s, h->status.ptr, sizeof s, cudaMemcpyDeviceToHost));
  if (s.code) {
    AL_CUDA(cudaMemset(h->status.ptr, 0, sizeof s));
    if (h->bar.ptr) AL_CUDA(cudaMemset(h->bar.ptr, 0, h->bar.bytes));  // (a wait that ran out may leave it mid-way)
    return status_error(s, h->d.n_experts);
  }
  return ARTLITE_OK;
}

int artlite_moe_debug(artlite_moe* h, float* logits, int32_t* ids, float* weights, int64_t* offsets, int32_t* perm) {
  AL_CHECK(h, ARTLITE_EINVAL, "moe_debug: null handle");
  AL_TRY(artlite_moe_sync(h, 0));
  const int64_t T = h->last_T, P = T * h->d.top_k;
  const int E = h->d.n_experts;
  if (logits) AL_CUDA(cudaMemcpy(logits, h->logits.ptr, sizeof(float) * T * E, cudaMemcpyDefault));
  if (ids) AL_CUDA(cudaMemcpy(ids, h->ids.ptr, sizeof(int32_t) * P, cudaMemcpyDefault));
  if (weights) AL_CUDA(cudaMemcpy(weights, h->w.ptr, sizeof(float) * P, cudaMemcpyDefault));
  if (offsets) AL_CUDA(cudaMemcpy(offsets, h->offsets.ptr, sizeof(int64_t) * (E + 1), cudaMemcpyDefault));
  if (perm) AL_CUDA(cudaMemcpy(perm, h->perm.ptr, sizeof(int32_t) * P, cudaMemcpyDefault));
  return ARTLITE_OK;
}

int artlite_moe_stage_times(artlite_moe* h, int layer, float* ms, int* n_out) {
  AL_CHECK(h && ms && n_out, ARTLITE_EINVAL, "moe_stage_times: null argument");
  AL_CHECK(layer >= 0 && layer < (int)h->layers.size(), ARTLITE_EINVAL, "moe_stage_times: layer %d", layer);
  *n_out = 0;
  const int ns = h->n_stages[layer];
  if (!h->timing || ns < 2) return ARTLITE_OK;
  AL_CUDA(cudaSetDevice(h->dev));
  const cudaEvent_t* e = &h->ev[(size_t)layer * kStages];
  AL_CUDA(cudaEventSynchronize(e[ns - 1]));
  for (int i = 0; i + 1 < ns; i++) AL_CUDA(cudaEventElapsedTime(&ms[i], e[i], e[i + 1]));
  *n_out = ns - 1;
  return ARTLITE_OK;
}

int artlite_moe_path(artlite_moe* h, int layer) {
  if (!h || layer < 0 || layer >= (int)h->layers.size()) return 0;
  return h->paths[layer];
}

int artlite_moe_weights(artlite_moe* h, int layer, int which, const void** ptr, int64_t* bytes) {
  AL_CHECK(h && ptr && bytes, ARTLITE_EINVAL, "moe_weights: null argument");
  AL_CHECK(layer >= 0 && layer < (int)h->layers.size() && h->layers[layer].qtype >= 0, ARTLITE_EINVAL,
           "moe_weights: layer %d has no weights", layer);
  AL_CHECK(which >= 0 && which <= 3, ARTLITE_EINVAL, "moe_weights: tensor %d (0 gate, 1 up, 2 down, 3 router)", which);
  const artlite_moe::Layer& L = h->layers[layer];
  const int64_t F = h->d.expert_ffn, H = h->d.hidden;
  switch (which) {
    case 0: *ptr = L.gate.ptr, *bytes = h->E_local * F * L.rb_gu; break;
    case 1: *ptr = L.up.ptr, *bytes = h->E_local * F * L.rb_gu; break;
    case 2: *ptr = L.down.ptr, *bytes = h->E_local * H * L.rb_dn; break;
    default: *ptr = L.router.ptr, *bytes = h->d.n_experts * H * (L.router_qtype == ARTLITE_F32 ? 4 : 2); break;
  }
  return ARTLITE_OK;
}

int64_t artlite_moe_launch_count(void) { return artlite::launch_count(); }

int artlite_moe_destroy(artlite_moe* h) {
  if (!h) return ARTLITE_OK;
  cudaSetDevice(h->dev);
  if (!h->ep_failed) wait(h->st, 0);  // (bounded; after a failed exchange nothing is waited for)
  for (cudaEvent_t e : h->ev)
    if (e) cudaEventDestroy(e);
  if (h->done) cudaEventDestroy(h->done);
  ep_destroy(h);
  for (artlite_moe::Graph& g : h->graphs) cudaGraphExecDestroy(g.exec);
  cudaStreamDestroy(h->st);
  delete h;
  return ARTLITE_OK;
}

}  // extern "C"
