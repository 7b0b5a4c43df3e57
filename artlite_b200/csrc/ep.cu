// Expert parallelism across the GPUs of one node: rank r of W owns experts [r E / W, (r + 1) E / W) (their raw GGUF
// rows only, set_weights) and its own tokens; per layer
//   1. router, routing and the dispatch over all E experts, on the rank's tokens (block.cu: route_and_dispatch); in
//      dispatch order a rank's pairs for peer q's experts are one contiguous block;
//   2. per-expert pair counts exchanged (NCCL send / recv of E / W int32 per peer), read back to the host (the one
//      host synchronisation of the layer: NCCL message sizes are host values); the plan on the host: the send blocks,
//      and the receive buffer's layout: the peers' blocks (q ascending), then the rank's own, each expert-major as its
//      source dispatched it;
//   3. the token rows gathered (bf16): rows for peers into the send buffer at their dispatch positions, the rank's own
//      rows straight into their place in the receive buffer;
//   4. the rows exchanged with grouped ncclSend / ncclRecv, one message per peer, on a second stream, while
//   5. the local experts run on the receive buffer's W x (E / W) (source, expert) row groups, each in place against its
//      expert's weights (run_experts with a weight-expert map), no regrouping copy: at W = 2 the own groups first,
//      while the rows travel, then the peer's; at W >= 4 (the own block a small share) one run over all groups once
//      the rows are in; with ARTLITE_EP_CHUNKS > 1 the peers' groups in expert chunks, each run as its rows land.
//      From 8 ranks on the tcgen05 path (ARTLITE_EP_REGROUP=1 / 0 forces it on / off) the received rows are first
//      gathered into expert-major order (index maps built on the host from the counts), each local expert one row
//      group, so that its weights are dequantised once per full 256-token tile rather than once per source's half
//      tile, and the outputs are gathered back into the receive order;
//   6. the outputs returned by one message per peer, each landing as the contiguous block of the source rank's dispatch
//      order it came from; the rank's own block stays where its experts wrote it;
//   7. the weighted combine of the rank's own tokens, its own rows read from the expert outputs (combine.cu).
// NCCL is loaded at run time (dlopen "libnccl.so.2": the one a process that imported torch already holds, or the
// system's), so the library itself has no link-time NCCL dependency. Waits on the host are bounded: a peer that never
// sends makes the count exchange's wait run out, the communicator is aborted and the call returns ARTLITE_ETIMEOUT.
// Nothing here uses TMA multicast or reads another GPU's memory from a kernel: every byte between GPUs moves by NCCL.
#include <cstdlib>
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>

#include <algorithm>
#include <mutex>
#include <type_traits>
#include <vector>

#include "block.cuh"
#include "common.cuh"
#include "kernels.cuh"
#include "tc_gemm.cuh"

namespace artlite {
namespace {

struct Nccl {
  void* so = nullptr;
  ncclResult_t (*getUniqueId)(ncclUniqueId*) = nullptr;
  ncclResult_t (*commInitRank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  // (non-blocking communicators: present from NCCL 2.14; without them the initialisation blocks)
  ncclResult_t (*commInitRankConfig)(ncclComm_t*, int, ncclUniqueId, int, ncclConfig_t*) = nullptr;
  ncclResult_t (*commGetAsyncError)(ncclComm_t, ncclResult_t*) = nullptr;
  ncclResult_t (*commFinalize)(ncclComm_t) = nullptr;
  ncclResult_t (*commDestroy)(ncclComm_t) = nullptr;
  ncclResult_t (*commAbort)(ncclComm_t) = nullptr;
  ncclResult_t (*send)(const void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*recv)(void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*groupStart)() = nullptr;
  ncclResult_t (*groupEnd)() = nullptr;
  const char* (*errorString)(ncclResult_t) = nullptr;
};

Nccl g_nccl;
std::mutex g_nccl_mu;

int nccl(Nccl** out) {
  std::lock_guard<std::mutex> lock(g_nccl_mu);
  if (!g_nccl.so) {
    const char* env = getenv("ARTLITE_NCCL_LIB");
    void* so = dlopen(env && env[0] ? env : "libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    AL_CHECK(so, ARTLITE_ENCCL, "nccl: cannot load %s (%s)", env && env[0] ? env : "libnccl.so.2", dlerror());
    Nccl n;
    n.so = so;
    bool ok = true;
    auto sym = [&](auto& f, const char* name) {
      f = reinterpret_cast<std::remove_reference_t<decltype(f)>>(dlsym(so, name));
      ok = ok && f;
    };
    sym(n.getUniqueId, "ncclGetUniqueId");
    sym(n.commInitRank, "ncclCommInitRank");
    sym(n.commDestroy, "ncclCommDestroy");
    sym(n.commAbort, "ncclCommAbort");
    sym(n.send, "ncclSend");
    sym(n.recv, "ncclRecv");
    sym(n.groupStart, "ncclGroupStart");
    sym(n.groupEnd, "ncclGroupEnd");
    sym(n.errorString, "ncclGetErrorString");
    AL_CHECK(ok, ARTLITE_ENCCL, "nccl: a symbol is missing from the loaded library");
    sym(n.commInitRankConfig, "ncclCommInitRankConfig");
    sym(n.commGetAsyncError, "ncclCommGetAsyncError");
    sym(n.commFinalize, "ncclCommFinalize");
    if (!n.commInitRankConfig || !n.commGetAsyncError || !n.commFinalize)
      n.commInitRankConfig = nullptr, n.commGetAsyncError = nullptr, n.commFinalize = nullptr;
    g_nccl = n;
  }
  *out = &g_nccl;
  return ARTLITE_OK;
}

// (a call on a non-blocking communicator may answer ncclInProgress: accepted here, settled by nccl_settle)
#define AL_NCCL(call)                                                                               \
  do {                                                                                              \
    const ncclResult_t r_ = (call);                                                                 \
    if (r_ != ncclSuccess && r_ != ncclInProgress) {                                                \
      ::artlite::set_error("%s:%d %s: %s", __FILE__, __LINE__, #call, N->errorString(r_));          \
      return ARTLITE_ENCCL;                                                                         \
    }                                                                                               \
  } while (0)

int now_ms() {
  timespec t;
  clock_gettime(CLOCK_MONOTONIC, &t);
  return (int)(t.tv_sec * 1000 + t.tv_nsec / 1000000);
}

// Waits, up to timeout_ms, until the communicator's pending work (its initialisation, a group's enqueue) is done:
// ARTLITE_OK, ARTLITE_ENCCL (NCCL reported an error) or ARTLITE_ETIMEOUT. A blocking communicator is always settled.
int nccl_settle(Nccl* N, ncclComm_t comm, int timeout_ms, const char* what) {
  if (!N->commGetAsyncError) return ARTLITE_OK;
  const int t0 = now_ms();
  for (;;) {
    ncclResult_t st = ncclSuccess;
    const ncclResult_t r = N->commGetAsyncError(comm, &st);
    if (r != ncclSuccess) st = r;
    if (st == ncclSuccess) return ARTLITE_OK;
    if (st != ncclInProgress) {
      set_error("%s: %s", what, N->errorString(st));
      return ARTLITE_ENCCL;
    }
    if (now_ms() - t0 > timeout_ms) {
      set_error("%s: not done within %d ms", what, timeout_ms);
      return ARTLITE_ETIMEOUT;
    }
    struct timespec ts{0, 20000};
    nanosleep(&ts, nullptr);
  }
}

// the bound on a host wait for the peers (ARTLITE_EP_TIMEOUT_MS, default 30 s) and on the communicator's forming
// (ARTLITE_EP_INIT_TIMEOUT_MS, default 120 s)
int env_ms(const char* name, int dflt) {
  const char* v = getenv(name);
  const int t = v ? atoi(v) : 0;
  return t > 0 ? t : dflt;
}
int ep_timeout_ms() { return env_ms("ARTLITE_EP_TIMEOUT_MS", 30000); }

// ---------------------------------------------------------------- the peer-store exchange
//
// A push copies up to kMaxPeers blocks of rows from this GPU's memory into other GPUs' buffers (CUDA IPC mappings,
// reached over NVLink by plain 16-byte loads and stores: no TMA, no multicast), then raises each destination's flag to
// the forward's epoch: every thread fences its own stores at system scope, then its CTA counts itself done; the last
// CTA releases the flags (st.release.sys). A wait (one warp, a lane per source) acquires the flags of every peer at system scope, up to
// a deadline (about 2 s of the GPU's global timer), after which it reports ARTLITE_ETIMEOUT in the status word and
// returns: no wait here is unbounded. The blocks of a push never overlap; a buffer is written only between two
// count exchanges that both of its owner's consecutive forwards take part in, so no push can reach a buffer that its
// owner is still reading.
constexpr int kMaxPeers = 8;
struct PushArgs {
  const uint8_t* src[kMaxPeers];
  uint8_t* dst[kMaxPeers];
  int64_t n16[kMaxPeers + 1];  // exclusive prefix of the blocks' 16-byte units
  uint32_t* flag[kMaxPeers];   // the destination's flag (null: no block to that rank)
  int nb;
  uint32_t epoch;
  int* done;
};

__global__ void __launch_bounds__(512) ep_push_kernel(const PushArgs a) {
  const int64_t total = a.n16[a.nb];
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  int b = 0;
  // four 16-byte units a thread in flight (their loads issued before the stores), in increasing unit order
  for (int64_t i0 = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i0 < total; i0 += 4 * stride) {
    uint4 v[4];
    int bb[4];
#pragma unroll
    for (int u = 0; u < 4; u++) {
      const int64_t i = i0 + u * stride;
      bb[u] = -1;
      if (i < total) {
        while (i >= a.n16[b + 1]) b++;
        bb[u] = b;
        v[u] = __ldcg(reinterpret_cast<const uint4*>(a.src[b]) + (i - a.n16[b]));
      }
    }
#pragma unroll
    for (int u = 0; u < 4; u++)
      if (bb[u] >= 0) reinterpret_cast<uint4*>(a.dst[bb[u]])[i0 + u * stride - a.n16[bb[u]]] = v[u];
  }
  __threadfence_system();  // (every thread: its own stores to the peers' memory are visible system-wide first)
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    if (atomicAdd(a.done, 1) == (int)gridDim.x - 1) {
      __threadfence_system();
      for (int k = 0; k < a.nb; k++)
        if (a.flag[k]) asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(a.flag[k]), "r"(a.epoch) : "memory");
      *a.done = 0;
    }
  }
}

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// every peer's flag at flags[q] (q != r, q < W) reaching epoch; where: the report's detail
__global__ void ep_wait_kernel(const uint32_t* flags, int W, int r, uint32_t epoch, DevStatus* status, int where) {
  const int q = threadIdx.x;
  if (q >= W || q == r) return;
  const uint64_t t0 = global_ns();
  for (;;) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(flags + q) : "memory");
    if ((int32_t)(v - epoch) >= 0) return;
    if (global_ns() - t0 > 2000000000ull) {
      report(status, ARTLITE_ETIMEOUT, where, q);
      return;
    }
    __nanosleep(256);
  }
}

__global__ void iota_kernel(int32_t* p, int64_t n) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) p[i] = (int32_t)i;
}

}  // namespace

int ep_create(artlite_moe* h) {
  const artlite_moe_desc& d = h->d;
  const int W = d.ep_world, El = h->E_local, E = d.n_experts, H = d.hidden, F = d.expert_ffn, K = d.top_k;
  const int64_t T = d.max_tokens > 0 ? d.max_tokens : 1;
  const int64_t R = T * K * W;  // the most rows a rank can receive (every rank's pairs all on its experts)
  h->ep_max_rows = R;
  AL_TRY(h->ep_loff.reserve(sizeof(int64_t) * (E + 1)));  // the W El row groups' offsets in the receive buffer
  AL_TRY(h->ep_lcounts.reserve(sizeof(int32_t) * E));     // their rows
  AL_TRY(h->ep_wexp.reserve(sizeof(int32_t) * E));        // their weight experts: group q El + e -> e
  AL_TRY(h->ep_ident.reserve(sizeof(int32_t) * R));
  AL_TRY(h->xr.reserve(sizeof(uint16_t) * (R + 256) * H));  // (the tcgen05 path reads 256-row boxes)
  AL_TRY(h->xe.reserve(sizeof(uint16_t) * (R + 256) * H));
  AL_TRY(h->ep_idx.reserve(sizeof(int32_t) * 2 * R));
  AL_TRY(h->ys.reserve(sizeof(float) * T * K * H));
  // the expert workspaces hold the received rows (h: fp32 or bf16 with 256 spare rows; y: fp32 or bf16)
  AL_TRY(h->h.reserve(std::max(sizeof(float) * R * F, sizeof(uint16_t) * (R + 256) * F)));
  AL_TRY(h->y.reserve(sizeof(float) * R * H));
  AL_TRY(h->tiles.reserve(tc_sched_bytes(E)));
  AL_TRY(h->unit_gu.reserve(sizeof(int32_t) * (E + 1)));
  AL_TRY(h->unit_dn.reserve(sizeof(int32_t) * (E + 1)));
  AL_CUDA(cudaHostAlloc(reinterpret_cast<void**>(&h->hb_counts), sizeof(int32_t) * 2 * E, cudaHostAllocDefault));
  AL_CUDA(cudaHostAlloc(reinterpret_cast<void**>(&h->hb_full), sizeof(int32_t) * W * E, cudaHostAllocDefault));
  AL_TRY(h->ep_fullc.reserve(sizeof(int32_t) * W * E));
  AL_TRY(h->ep_flags.reserve(sizeof(uint32_t) * 2 * W));
  AL_TRY(h->ep_done.reserve(256));
  AL_CUDA(cudaMemsetAsync(h->ep_flags.ptr, 0, sizeof(uint32_t) * 2 * W, h->st));
  AL_CUDA(cudaMemsetAsync(h->ep_done.ptr, 0, 256, h->st));
  AL_CUDA(cudaHostAlloc(reinterpret_cast<void**>(&h->hb_loff), sizeof(int64_t) * (E + 1), cudaHostAllocDefault));
  AL_CUDA(cudaHostAlloc(reinterpret_cast<void**>(&h->hb_lcounts), sizeof(int32_t) * E, cudaHostAllocDefault));
  AL_CUDA(cudaHostAlloc(reinterpret_cast<void**>(&h->hb_idx), sizeof(int32_t) * 2 * R, cudaHostAllocDefault));
  h->ep_xoff.assign(El + 1, 0);
  if (const char* ev = std::getenv("ARTLITE_EP_REGROUP")) h->ep_regroup = ev[0] == '0' ? 0 : 1;
  h->ep_send_base.assign(W, 0);
  h->ep_recv_base.assign(W, 0);
  h->ep_send_rows.assign(W, 0);
  h->ep_recv_rows.assign(W, 0);
  AL_CUDA(cudaStreamCreateWithFlags(&h->ep_st, cudaStreamNonBlocking));
  for (cudaEvent_t& e : h->ep_ev) AL_CUDA(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
  // Expert chunks pipeline the exchanges with the peers' GEMMs, but each chunk is another pair of GEMM launches.
  // ARTLITE_EP_CHUNKS (1, 2 or 4, a divisor of the local experts) sets the count; default 1.
  h->ep_chunks = 1;
  if (const char* ev = std::getenv("ARTLITE_EP_CHUNKS")) {
    const int c = std::atoi(ev);
    if ((c == 2 || c == 4) && c <= artlite_moe::kEpChunks && El % c == 0) h->ep_chunks = c;
  }
  h->ep_cs_pos.assign((size_t)W * h->ep_chunks, 0);
  h->ep_cs_rows.assign((size_t)W * h->ep_chunks, 0);
  h->ep_cr_pos.assign((size_t)W * h->ep_chunks, 0);
  h->ep_cr_rows.assign((size_t)W * h->ep_chunks, 0);
  iota_kernel<<<(unsigned)cdiv(R, 256), 256, 0, h->st>>>(h->ep_ident.as<int32_t>(), R);
  AL_LAUNCHED();
  // the row groups' weight experts: chunk-major for the peers (chunk c, peer place qi, expert e of the chunk), then
  // the own block's El groups
  std::vector<int32_t> wexp(E);
  const int C = h->ep_chunks, Ec = El / C;
  for (int c = 0; c < C; c++)
    for (int qi = 0; qi < W - 1; qi++)
      for (int i = 0; i < Ec; i++) wexp[(c * (W - 1) + qi) * Ec + i] = c * Ec + i;
  for (int e = 0; e < El; e++) wexp[(W - 1) * El + e] = e;
  AL_CUDA(cudaMemcpyAsync(h->ep_wexp.ptr, wexp.data(), sizeof(int32_t) * E, cudaMemcpyHostToDevice, h->st));
  AL_CUDA(cudaStreamSynchronize(h->st));
  return ARTLITE_OK;
}

void ep_destroy(artlite_moe* h) {
  if (h->comm) {
    Nccl* N;
    if (nccl(&N) == ARTLITE_OK) {
      // (after a failed exchange the peers may never complete theirs: abort, which does not wait for them)
      // (a non-blocking communicator is finalized first, with a bound: one that does not settle is aborted)
      ncclComm_t c = static_cast<ncclComm_t>(h->comm);
      bool abort = h->ep_failed;
      if (!abort && N->commFinalize) {
        const ncclResult_t r = N->commFinalize(c);
        abort = (r != ncclSuccess && r != ncclInProgress) ||
                nccl_settle(N, c, ep_timeout_ms(), "expert parallelism: finalize") != ARTLITE_OK;
      }
      if (abort) N->commAbort(c);
      else N->commDestroy(c);
    }
    h->comm = nullptr;
  }
  for (uint8_t* p : h->ep_peer_xr)
    if (p) cudaIpcCloseMemHandle(p);
  for (uint8_t* p : h->ep_peer_ys)
    if (p) cudaIpcCloseMemHandle(p);
  for (uint32_t* p : h->ep_peer_flags)
    if (p) cudaIpcCloseMemHandle(p);
  h->ep_peer_xr.clear(), h->ep_peer_ys.clear(), h->ep_peer_flags.clear();
  h->ep_p2p = false;
  if (h->hb_full) cudaFreeHost(h->hb_full), h->hb_full = nullptr;
  for (cudaEvent_t& e : h->ep_ev)
    if (e) cudaEventDestroy(e), e = nullptr;
  if (h->ep_st) cudaStreamDestroy(h->ep_st), h->ep_st = nullptr;
  if (h->hb_counts) cudaFreeHost(h->hb_counts);
  if (h->hb_loff) cudaFreeHost(h->hb_loff);
  if (h->hb_lcounts) cudaFreeHost(h->hb_lcounts);
  if (h->hb_idx) cudaFreeHost(h->hb_idx);
  h->hb_idx = nullptr;
  h->hb_counts = nullptr;
  h->hb_loff = nullptr;
  h->hb_lcounts = nullptr;
}

namespace {
// One small exchange of `bytes` per rank over the communicator: every rank's `mine` into all[rank] (its own too);
// bounded waits.
int ep_allgather_host(artlite_moe* h, Nccl* N, ncclComm_t comm, const void* mine, void* all, size_t bytes) {
  const int W = h->d.ep_world, r = h->d.ep_rank;
  DevBuf buf;
  AL_TRY(buf.reserve(bytes * (W + 1)));
  uint8_t* b = buf.as<uint8_t>();
  AL_CUDA(cudaMemcpyAsync(b + bytes * W, mine, bytes, cudaMemcpyHostToDevice, h->st));
  AL_NCCL(N->groupStart());
  for (int q = 0; q < W; q++) {
    AL_NCCL(N->send(b + bytes * W, bytes, ncclUint8, q, comm, h->st));
    AL_NCCL(N->recv(b + bytes * q, bytes, ncclUint8, q, comm, h->st));
  }
  AL_NCCL(N->groupEnd());
  AL_TRY(nccl_settle(N, comm, ep_timeout_ms(), "ep_init: handle exchange"));
  AL_CUDA(cudaMemcpyAsync(all, b, bytes * W, cudaMemcpyDeviceToHost, h->st));
  const int rc = wait_deadline(h->st, ep_timeout_ms());
  if (rc == ARTLITE_ETIMEOUT) set_error("ep_init: rank %d: the handle exchange did not complete", r);
  return rc;
}

// The peer-store exchange's set-up (every rank takes part): the CUDA IPC handles of each rank's receive buffer, return
// buffer and flags go to every rank, which maps its peers' (NVLink peer access); it is used only if every rank wants
// it (by default at two ranks; ARTLITE_EP_EXCHANGE=p2p or nccl forces either way; expert chunks keep NCCL) and every
// rank mapped every peer.
int ep_p2p_setup(artlite_moe* h, Nccl* N, ncclComm_t comm) {
  const int W = h->d.ep_world, r = h->d.ep_rank;
  const char* v = getenv("ARTLITE_EP_EXCHANGE");
  struct Slot {
    int32_t ok, pad[11];
    int64_t xr_bytes, ys_bytes;  // (a push checks its block's end against the owner's buffer)
    cudaIpcMemHandle_t hx, hy, hf;
  };
  Slot m;
  memset(&m, 0, sizeof m);
  m.xr_bytes = (int64_t)h->xr.bytes;
  m.ys_bytes = (int64_t)h->ys.bytes;
  // (the default: the peer stores at two ranks, where they measured faster; NCCL from four, where they did not)
  const bool want = v && !strcmp(v, "p2p") ? true : v && !strcmp(v, "nccl") ? false : W == 2;
  m.ok = want && h->ep_chunks == 1 && W <= kMaxPeers &&
         cudaIpcGetMemHandle(&m.hx, h->xr.ptr) == cudaSuccess && cudaIpcGetMemHandle(&m.hy, h->ys.ptr) == cudaSuccess &&
         cudaIpcGetMemHandle(&m.hf, h->ep_flags.ptr) == cudaSuccess;
  cudaGetLastError();  // (a refusal above is an answer, not an error)
  std::vector<Slot> all(W);
  AL_TRY(ep_allgather_host(h, N, comm, &m, all.data(), sizeof(Slot)));
  bool ok = true;
  for (const Slot& q : all) ok = ok && q.ok;
  h->ep_peer_xr.assign(W, nullptr);
  h->ep_peer_ys.assign(W, nullptr);
  h->ep_peer_flags.assign(W, nullptr);
  h->ep_peer_xr_bytes.assign(W, 0);
  h->ep_peer_ys_bytes.assign(W, 0);
  for (int q = 0; q < W; q++) h->ep_peer_xr_bytes[q] = all[q].xr_bytes, h->ep_peer_ys_bytes[q] = all[q].ys_bytes;
  if (ok)
    for (int q = 0; q < W && ok; q++) {
      if (q == r) continue;
      void *px = nullptr, *py = nullptr, *pf = nullptr;
      ok = cudaIpcOpenMemHandle(&px, all[q].hx, cudaIpcMemLazyEnablePeerAccess) == cudaSuccess &&
           cudaIpcOpenMemHandle(&py, all[q].hy, cudaIpcMemLazyEnablePeerAccess) == cudaSuccess &&
           cudaIpcOpenMemHandle(&pf, all[q].hf, cudaIpcMemLazyEnablePeerAccess) == cudaSuccess;
      h->ep_peer_xr[q] = static_cast<uint8_t*>(px);
      h->ep_peer_ys[q] = static_cast<uint8_t*>(py);
      h->ep_peer_flags[q] = static_cast<uint32_t*>(pf);
    }
  cudaGetLastError();
  // every rank's verdict: the exchange is used only where every rank mapped every peer
  int32_t mine = ok ? 1 : 0;
  std::vector<int32_t> verdicts(W);
  AL_TRY(ep_allgather_host(h, N, comm, &mine, verdicts.data(), sizeof(int32_t)));
  bool all_ok = true;
  for (int32_t x : verdicts) all_ok = all_ok && x == 1;
  if (!all_ok) {
    for (int q = 0; q < W; q++) {
      if (h->ep_peer_xr[q]) cudaIpcCloseMemHandle(h->ep_peer_xr[q]);
      if (h->ep_peer_ys[q]) cudaIpcCloseMemHandle(h->ep_peer_ys[q]);
      if (h->ep_peer_flags[q]) cudaIpcCloseMemHandle(h->ep_peer_flags[q]);
    }
    h->ep_peer_xr.assign(W, nullptr);
    h->ep_peer_ys.assign(W, nullptr);
    h->ep_peer_flags.assign(W, nullptr);
    cudaGetLastError();
  }
  h->ep_p2p = all_ok;
  return ARTLITE_OK;
}

int ep_forward_impl(artlite_moe* h, int layer, const void* xd, void* yd, int64_t T, cudaStream_t st, Marker& mk,
                    const void* res);

}  // namespace

// The EP forward; any failure once the exchanges have begun aborts the communicator (the peers' next bounded wait
// then fails too) and leaves the handle unusable for expert parallelism, instead of a rank blocking on a peer forever.
int ep_forward(artlite_moe* h, int layer, const void* xd, void* yd, int64_t T, cudaStream_t st, Marker& mk,
               const void* res) {
  AL_CHECK(h->comm && !h->ep_failed, ARTLITE_EINVAL,
           "moe_forward: expert parallelism needs artlite_moe_ep_init first (or a previous exchange failed)");
  const int rc = ep_forward_impl(h, layer, xd, yd, T, st, mk, res);
  if (rc != ARTLITE_OK && h->comm) {
    Nccl* N;
    if (nccl(&N) == ARTLITE_OK) N->commAbort(static_cast<ncclComm_t>(h->comm));
    h->comm = nullptr;
    h->ep_failed = true;
  }
  return rc;
}

namespace {
int ep_forward_impl(artlite_moe* h, int layer, const void* xd, void* yd, int64_t T, cudaStream_t st, Marker& mk,
                    const void* res) {
  Nccl* N;
  AL_TRY(nccl(&N));
  ncclComm_t comm = static_cast<ncclComm_t>(h->comm);
  const artlite_moe_desc& d = h->d;
  const artlite_moe::Layer& L = h->layers[layer];
  const int W = d.ep_world, r = d.ep_rank, El = h->E_local, E = d.n_experts, H = d.hidden, K = d.top_k;
  const int64_t P = T * K;
  // 1: routing and the dispatch over all experts
  AL_TRY(route_and_dispatch(h, L, xd, T, st, mk));
  // 2: counts (every rank's whole count vector to every rank: the peer-store exchange places its blocks by the other
  // ranks' plans), then the plan on the host
  AL_NCCL(N->groupStart());
  for (int q = 0; q < W; q++) {
    AL_NCCL(N->send(h->counts.as<int32_t>(), E, ncclInt32, q, comm, st));
    AL_NCCL(N->recv(h->ep_fullc.as<int32_t>() + (size_t)q * E, E, ncclInt32, q, comm, st));
  }
  AL_NCCL(N->groupEnd());
  AL_TRY(nccl_settle(N, comm, ep_timeout_ms(), "expert parallelism: count exchange"));
  AL_CUDA(cudaMemcpyAsync(h->hb_full, h->ep_fullc.ptr, sizeof(int32_t) * W * E, cudaMemcpyDeviceToHost, st));
  const int tmo = ep_timeout_ms();
  const int rc = wait_deadline(st, tmo);
  if (rc == ARTLITE_ETIMEOUT) {  // a peer that never sent its counts (the caller aborts the communicator)
    set_error("expert parallelism: rank %d: the count exchange did not complete within %d ms (communicator aborted)",
              r, tmo);
    return ARTLITE_ETIMEOUT;
  }
  AL_TRY(rc);
  const int32_t* full = h->hb_full;      // [q][e]: rank q's pairs for expert e (all E)
  for (int e = 0; e < E; e++) h->hb_counts[e] = full[(size_t)r * E + e];
  for (int q = 0; q < W; q++)
    for (int e = 0; e < El; e++) h->hb_counts[E + q * El + e] = full[(size_t)q * E + r * El + e];
  const int32_t* sc = h->hb_counts;      // this rank's pairs per expert (all E)
  const int32_t* rcv = h->hb_counts + E; // [q][e]: peer q's pairs for local expert e
  std::vector<int64_t>& send_base = h->ep_send_base;
  std::vector<int64_t>& recv_base = h->ep_recv_base;
  std::vector<int64_t>& send_rows = h->ep_send_rows;
  std::vector<int64_t>& recv_rows = h->ep_recv_rows;
  // The plan. Sent blocks: in dispatch order, peer q's experts' rows are one block (send_base / send_rows), chunk c of
  // its experts a contiguous part of it. Receive buffer: chunk-major over the peers' blocks (chunk c: peer q ascending,
  // its rows of chunk c's experts as it dispatched them), then this rank's own block; the row groups in that same order
  // (group of (chunk c, peer place qi, expert) = (c (W - 1) + qi) Ec + i), so every chunk is one contiguous range of
  // groups and of rows.
  const int C = h->ep_chunks, Ec = El / C;
  int64_t sb = 0;
  for (int q = 0; q < W; q++) {
    send_base[q] = sb;
    int64_t sn = 0;
    for (int c = 0; c < C; c++) {
      int64_t n = 0;
      for (int i = 0; i < Ec; i++) {
        const int32_t v = sc[q * El + c * Ec + i];
        AL_CHECK(v >= 0, ARTLITE_EDEVICE, "expert parallelism: count %d", v);
        n += v;
      }
      h->ep_cs_pos[(size_t)q * C + c] = sb + sn;
      h->ep_cs_rows[(size_t)q * C + c] = n;
      sn += n;
    }
    send_rows[q] = sn;
    sb += sn;
  }
  int64_t rb = 0;
  for (int q = 0; q < W; q++) recv_rows[q] = 0;
  for (int c = 0; c < C; c++)
    for (int qi = 0; qi < W - 1; qi++) {
      const int q = qi < r ? qi : qi + 1;
      const int64_t start = rb;
      for (int i = 0; i < Ec; i++) {
        const int e = c * Ec + i, j = (c * (W - 1) + qi) * Ec + i;
        const int32_t v = rcv[q * El + e];
        AL_CHECK(v >= 0, ARTLITE_EDEVICE, "expert parallelism: count %d from rank %d", v, q);
        h->hb_loff[j] = rb;
        h->hb_lcounts[j] = v;
        rb += v;
      }
      h->ep_cr_pos[(size_t)q * C + c] = start;
      h->ep_cr_rows[(size_t)q * C + c] = rb - start;
      recv_rows[q] += rb - start;
    }
  recv_base[r] = rb;
  for (int e = 0; e < El; e++) {
    const int j = (W - 1) * El + e;
    const int32_t v = rcv[r * El + e];
    AL_CHECK(v >= 0, ARTLITE_EDEVICE, "expert parallelism: count %d", v);
    h->hb_loff[j] = rb;
    h->hb_lcounts[j] = v;
    rb += v;
  }
  recv_rows[r] = rb - recv_base[r];
  h->hb_loff[E] = rb;
  const int64_t Rl = rb;
  AL_CHECK(sb == P && Rl <= h->ep_max_rows, ARTLITE_EDEVICE,
           "expert parallelism: %lld rows sent of %lld, %lld received, room for %lld", (long long)sb, (long long)P,
           (long long)Rl, (long long)h->ep_max_rows);
  AL_CHECK(send_rows[r] == recv_rows[r], ARTLITE_EDEVICE, "expert parallelism: own block %lld / %lld rows",
           (long long)send_rows[r], (long long)recv_rows[r]);
  const int path = expert_path(*h, Rl, L);
  h->last_path = path;
  h->paths[layer] = path;
  // Regroup (tcgen05 path, one chunk; by default from 8 ranks, where a (source, expert) group averages about half a
  // 256-token tile): the received rows gathered into expert-major order, so that each local expert is one row group
  // and its weights are dequantised once per full tile instead of once per source; the outputs gathered back.
  const bool regroup = C == 1 && path == 2 && (h->ep_regroup > 0 || (h->ep_regroup < 0 && W >= 8));
  if (regroup) {
    int32_t* idx = h->hb_idx;                     // expert-major row -> receive-buffer row
    int32_t* inv = h->hb_idx + h->ep_max_rows;    // receive-buffer row -> expert-major row
    int64_t i = 0;
    for (int e = 0; e < El; e++) {
      h->ep_xoff[e] = i;
      for (int qi = 0; qi < W; qi++) {  // (group qi El + e: the peers' (qi < W - 1), then the own block's)
        const int j = qi * El + e;
        for (int64_t m = 0; m < h->hb_lcounts[j]; m++, i++) {
          idx[i] = (int32_t)(h->hb_loff[j] + m);
          inv[h->hb_loff[j] + m] = (int32_t)i;
        }
      }
    }
    h->ep_xoff[El] = i;
    for (int e = 0; e < El; e++) {
      h->hb_loff[e] = h->ep_xoff[e];
      h->hb_lcounts[e] = (int32_t)(h->ep_xoff[e + 1] - h->ep_xoff[e]);
    }
    h->hb_loff[El] = i;
    if (Rl) {
      AL_CUDA(cudaMemcpyAsync(h->ep_idx.ptr, idx, sizeof(int32_t) * Rl, cudaMemcpyHostToDevice, st));
      AL_CUDA(cudaMemcpyAsync(h->ep_idx.as<int32_t>() + h->ep_max_rows, inv, sizeof(int32_t) * Rl,
                              cudaMemcpyHostToDevice, st));
    }
  }
  AL_CUDA(cudaMemcpyAsync(h->ep_loff.ptr, h->hb_loff, sizeof(int64_t) * (E + 1), cudaMemcpyHostToDevice, st));
  AL_CUDA(cudaMemcpyAsync(h->ep_lcounts.ptr, h->hb_lcounts, sizeof(int32_t) * E, cudaMemcpyHostToDevice, st));
  // 3: the rows in dispatch order: the peers' blocks into the send buffer, this rank's own block into its place in the
  // receive buffer
  uint16_t* xp = h->xp.as<uint16_t>();
  uint16_t* xr = h->xr.as<uint16_t>();
  if (P)
    AL_TRY(launch_gather(xd, d.act_dtype, h->perm.as<int32_t>(), P, K, H, xp, st, xr + recv_base[r] * H, send_base[r],
                         send_base[r] + send_rows[r]));
  cudaEvent_t ev_g = h->ep_ev[0], ev_b = h->ep_ev[1];
  cudaEvent_t* ev_r = h->ep_ev + 2;      // [C] a chunk's rows received
  cudaEvent_t* ev_y = h->ep_ev + 2 + C;  // [C] a chunk's outputs ready
  AL_CUDA(cudaEventRecord(ev_g, st));
  AL_TRY(mk.mark());
  // rows a source s sends to rank q (its pairs for q's experts), from the count matrix
  auto rows_to = [&](int s, int q) {
    int64_t n = 0;
    for (int e = 0; e < El; e++) n += full[(size_t)s * E + q * El + e];
    return n;
  };
  const bool p2p = h->ep_p2p;
  const uint32_t epoch = ++h->ep_epoch;
  DevStatus* status = h->status.as<DevStatus>();
  // 4: the peers' rows, chunk by chunk, on the exchange stream
  AL_CUDA(cudaStreamWaitEvent(h->ep_st, ev_g, 0));
  if (p2p) {  // each block straight into its place in the owner's receive buffer: after the sources before this rank
    PushArgs pa{};
    int nb = 0;
    int64_t acc = 0;
    for (int q = 0; q < W; q++) {
      if (q == r) continue;
      int64_t at = 0;  // (this rank's block in q's receive buffer: the blocks of the sources before it)
      for (int s2 = 0; s2 < r; s2++)
        if (s2 != q) at += rows_to(s2, q);
      AL_CHECK((at + send_rows[q]) * H * 2 <= h->ep_peer_xr_bytes[q], ARTLITE_EDEVICE,
               "expert parallelism: rank %d's rows for rank %d end past its receive buffer (%lld rows at %lld)", r, q,
               (long long)send_rows[q], (long long)at);
      pa.src[nb] = reinterpret_cast<const uint8_t*>(xp + send_base[q] * H);
      pa.dst[nb] = h->ep_peer_xr[q] + at * H * 2;
      pa.n16[nb] = acc;
      acc += send_rows[q] * H * 2 / 16;
      pa.flag[nb] = h->ep_peer_flags[q] + r;
      nb++;
    }
    pa.n16[nb] = acc;
    pa.nb = nb;
    pa.epoch = epoch;
    pa.done = h->ep_done.as<int>();
    const unsigned grid = (unsigned)std::max<int64_t>(1, std::min<int64_t>(cdiv(acc, 512 * 4), 128));
    ep_push_kernel<<<grid, 512, 0, h->ep_st>>>(pa);
    AL_LAUNCHED();
  }
  // the peers' rows are in (the main stream): their flags (peer-store), or the exchange stream's event (NCCL)
  auto rows_in = [&](int c) -> int {
    if (!p2p) {
      AL_CUDA(cudaStreamWaitEvent(st, ev_r[c], 0));
      return ARTLITE_OK;
    }
    ep_wait_kernel<<<1, 32, 0, st>>>(h->ep_flags.as<uint32_t>(), W, r, epoch, status, 40);
    AL_LAUNCHED();
    return ARTLITE_OK;
  };
  for (int c = 0; c < C && !p2p; c++) {
    AL_NCCL(N->groupStart());
    for (int q = 0; q < W; q++) {
      if (q == r) continue;
      const size_t k = (size_t)q * C + c;
      if (h->ep_cs_rows[k])
        AL_NCCL(N->send(xp + h->ep_cs_pos[k] * H, (size_t)h->ep_cs_rows[k] * H, ncclBfloat16, q, comm, h->ep_st));
      if (h->ep_cr_rows[k])
        AL_NCCL(N->recv(xr + h->ep_cr_pos[k] * H, (size_t)h->ep_cr_rows[k] * H, ncclBfloat16, q, comm, h->ep_st));
    }
    AL_NCCL(N->groupEnd());
    AL_TRY(nccl_settle(N, comm, ep_timeout_ms(), "expert parallelism: exchange"));
    AL_CUDA(cudaEventRecord(ev_r[c], h->ep_st));
  }
  // 5: the local experts in place: the own groups while the rows travel, then each chunk of the peers' groups once its
  // rows are in, its outputs handed to the exchange stream
  void* yrows = nullptr;
  int ydt = 0;
  const int64_t* goff = h->ep_loff.as<int64_t>();
  const int32_t* gcnt = h->ep_lcounts.as<int32_t>();
  const int32_t* gexp = h->ep_wexp.as<int32_t>();
  const int64_t xr_rows = (int64_t)(h->xr.bytes / (2 * H));
  const int32_t* ident = h->ep_ident.as<int32_t>();
  Marker quiet{h, layer, st};
  quiet.ns = kStages;  // (no stage events inside the expert calls)
  const int jo = (W - 1) * El;
  if (regroup) {  // every row in: gathered expert-major, the experts, the outputs gathered back into xr's order
    AL_TRY(rows_in(0));
    uint16_t* xe = h->xe.as<uint16_t>();
    const int32_t* idx = h->ep_idx.as<int32_t>();
    if (Rl) AL_TRY(launch_gather(xr, ARTLITE_BF16, idx, Rl, 1, H, xe, st, nullptr, 0, 0));
    AL_TRY(mk.mark());
    AL_TRY(run_experts(h, routed_weights(L), path, xe, ARTLITE_BF16, true, ident, 1, Rl, El, goff, gcnt,
                       (int64_t)(h->xe.bytes / (2 * H)), &yrows, &ydt, st, quiet, false, gexp + jo, El));
    AL_CHECK(ydt == ARTLITE_BF16, ARTLITE_EUNSUPPORTED, "expert parallelism: regrouped outputs of type %d", ydt);
    if (Rl) AL_TRY(launch_gather(yrows, ARTLITE_BF16, idx + h->ep_max_rows, Rl, 1, H, xr, st, nullptr, 0, 0));
    yrows = xr;
    AL_CUDA(cudaEventRecord(ev_y[0], st));
    AL_TRY(mk.mark());
  } else {
    if (W == 2) {  // the own groups while the rows travel, then the peer's (at N >= 4 the own block is too small a
                   // share to hide the exchange behind, and one launch over all groups costs less than two)
      AL_TRY(run_experts(h, routed_weights(L), path, xr, ARTLITE_BF16, true, ident, 1, recv_rows[r], El, goff + jo,
                         gcnt + jo, xr_rows, &yrows, &ydt, st, quiet, false, gexp + jo, El));
    }
    AL_TRY(mk.mark());
    const int Gc = (W - 1) * Ec;  // groups a chunk
    for (int c = 0; c < C; c++) {
      AL_TRY(rows_in(c));
      int64_t rows = 0;
      for (int q = 0; q < W; q++)
        if (q != r) rows += h->ep_cr_rows[(size_t)q * C + c];
      const int ng = Gc + (W == 2 || c < C - 1 ? 0 : El);  // (N >= 4: the last chunk's run takes the own groups too)
      if (W != 2 && c == C - 1) rows += recv_rows[r];
      if (ng)
        AL_TRY(run_experts(h, routed_weights(L), path, xr, ARTLITE_BF16, true, ident, 1, rows, ng, goff + c * Gc,
                           gcnt + c * Gc, xr_rows, &yrows, &ydt, st, quiet, false, gexp + c * Gc, El));
      AL_CUDA(cudaEventRecord(ev_y[c], st));
    }
    AL_TRY(mk.mark());
  }
  // the shared expert on this rank's own tokens (every rank holds all of it), on the main stream while the outputs
  // travel back
  CombineShared sh;
  if (L.has_shared && T > 0) AL_TRY(run_shared(h, L, xd, T, st, &sh));
  // 6: the outputs back, chunk by chunk, each landing as the block of the source's dispatch order it came from
  const size_t el = ydt == ARTLITE_BF16 ? 2 : 4;
  const ncclDataType_t dt = ydt == ARTLITE_BF16 ? ncclBfloat16 : ncclFloat32;
  uint8_t* yo = static_cast<uint8_t*>(yrows);
  uint8_t* ys = h->ys.as<uint8_t>();
  if (p2p) {  // each source's outputs straight into its return buffer, where its dispatch order put the block for
              // this rank (after its blocks for the ranks before this one)
    AL_CUDA(cudaStreamWaitEvent(h->ep_st, ev_y[0], 0));
    PushArgs pa{};
    int nb = 0;
    int64_t acc = 0;
    for (int q = 0; q < W; q++) {
      if (q == r) continue;
      int64_t at = 0;
      for (int q2 = 0; q2 < r; q2++) at += rows_to(q, q2);
      AL_CHECK((at + h->ep_cr_rows[q]) * H * (int64_t)el <= h->ep_peer_ys_bytes[q], ARTLITE_EDEVICE,
               "expert parallelism: rank %d's outputs for rank %d end past its return buffer", r, q);
      pa.src[nb] = yo + h->ep_cr_pos[q] * H * el;
      pa.dst[nb] = h->ep_peer_ys[q] + at * H * el;
      pa.n16[nb] = acc;
      acc += h->ep_cr_rows[q] * H * (int64_t)el / 16;
      pa.flag[nb] = h->ep_peer_flags[q] + W + r;
      nb++;
    }
    pa.n16[nb] = acc;
    pa.nb = nb;
    pa.epoch = epoch;
    pa.done = h->ep_done.as<int>();
    const unsigned grid = (unsigned)std::max<int64_t>(1, std::min<int64_t>(cdiv(acc, 512 * 4), 128));
    ep_push_kernel<<<grid, 512, 0, h->ep_st>>>(pa);
    AL_LAUNCHED();
  }
  for (int c = 0; c < C && !p2p; c++) {
    AL_CUDA(cudaStreamWaitEvent(h->ep_st, ev_y[c], 0));
    AL_NCCL(N->groupStart());
    for (int q = 0; q < W; q++) {
      if (q == r) continue;
      const size_t k = (size_t)q * C + c;
      if (h->ep_cr_rows[k])
        AL_NCCL(N->send(yo + h->ep_cr_pos[k] * H * el, (size_t)h->ep_cr_rows[k] * H, dt, q, comm, h->ep_st));
      if (h->ep_cs_rows[k])
        AL_NCCL(N->recv(ys + h->ep_cs_pos[k] * H * el, (size_t)h->ep_cs_rows[k] * H, dt, q, comm, h->ep_st));
    }
    AL_NCCL(N->groupEnd());
    AL_TRY(nccl_settle(N, comm, ep_timeout_ms(), "expert parallelism: exchange"));
  }
  AL_CUDA(cudaEventRecord(ev_b, h->ep_st));
  AL_CUDA(cudaStreamWaitEvent(st, ev_b, 0));
  if (p2p) {  // every owner's outputs for this rank's rows are in
    ep_wait_kernel<<<1, 32, 0, st>>>(h->ep_flags.as<uint32_t>() + W, W, r, epoch, status, 41);
    AL_LAUNCHED();
  }
  AL_TRY(mk.mark());
  // 7: the combine of this rank's tokens (its own block read where its experts wrote it)
  CombineOwn own;
  own.own = yo + recv_base[r] * H * el;
  own.own_lo = send_base[r];
  own.own_hi = send_base[r] + send_rows[r];
  if (T) AL_TRY(launch_combine(ys, ydt, h->slot.as<int32_t>(), h->w.as<float>(), T, K, H, yd, d.act_dtype, st, own,
                               sh, res));
  return ARTLITE_OK;
}
}  // namespace

}  // namespace artlite

using namespace artlite;

extern "C" {
#pragma GCC visibility push(default)

int artlite_moe_ep_plan(const int32_t* send_counts, const int32_t* recv_counts, int world, int rank, int E,
                        int64_t* send_off, int64_t* recv_pos, int64_t* local_off, int32_t* local_counts) {
  AL_CHECK(world >= 1 && rank >= 0 && rank < world && E >= world && E % world == 0, ARTLITE_EINVAL,
           "ep_plan: rank %d of %d, E %d", rank, world, E);
  AL_CHECK(send_counts && recv_counts && send_off && recv_pos && local_off && local_counts, ARTLITE_EINVAL,
           "ep_plan: null array");
  const int El = E / world;
  int64_t o = 0;  // this rank's rows in expert order: expert e's at send_off[e]
  for (int e = 0; e < E; e++) {
    AL_CHECK(send_counts[e] >= 0, ARTLITE_EINVAL, "ep_plan: count %d of expert %d", send_counts[e], e);
    send_off[e] = o;
    o += send_counts[e];
  }
  o = 0;  // received rows grouped by local expert, then by source rank
  for (int e = 0; e < El; e++) {
    local_off[e] = o;
    int64_t n = 0;
    for (int q = 0; q < world; q++) {
      const int32_t c = recv_counts[q * El + e];
      AL_CHECK(c >= 0, ARTLITE_EINVAL, "ep_plan: count %d from rank %d", c, q);
      recv_pos[(size_t)q * El + e] = o + n;
      n += c;
    }
    AL_CHECK(n <= INT32_MAX, ARTLITE_EINVAL, "ep_plan: %lld rows for one expert", (long long)n);
    local_counts[e] = (int32_t)n;
    o += n;
  }
  local_off[El] = o;
  return ARTLITE_OK;
}

int artlite_moe_ep_unique_id(void* out, int bytes) {
  AL_CHECK(out && bytes >= (int)sizeof(ncclUniqueId), ARTLITE_EINVAL, "ep_unique_id: %d bytes (needs %d)", bytes,
           (int)sizeof(ncclUniqueId));
  Nccl* N;
  AL_TRY(nccl(&N));
  ncclUniqueId id;
  AL_NCCL(N->getUniqueId(&id));
  memcpy(out, &id, sizeof id);
  return ARTLITE_OK;
}

int artlite_moe_ep_init(artlite_moe* h, const void* unique_id, int bytes) {
  AL_CHECK(h && unique_id && bytes >= (int)sizeof(ncclUniqueId), ARTLITE_EINVAL, "ep_init: bad arguments");
  AL_CHECK(h->d.ep_world > 1, ARTLITE_EINVAL, "ep_init: the handle was created with ep_world %d", h->d.ep_world);
  Nccl* N;
  AL_TRY(nccl(&N));
  AL_CUDA(cudaSetDevice(h->dev));
  ncclUniqueId id;
  memcpy(&id, unique_id, sizeof id);
  ncclComm_t comm = nullptr;
  if (!N->commInitRankConfig) {
    AL_NCCL(N->commInitRank(&comm, h->d.ep_world, id, h->d.ep_rank));
    h->comm = comm;
    return ep_p2p_setup(h, N, comm);
  }
  // non-blocking: the host's wait for every rank to join is bounded; past it the half-formed communicator is aborted
  ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
  cfg.blocking = 0;
  AL_NCCL(N->commInitRankConfig(&comm, h->d.ep_world, id, h->d.ep_rank, &cfg));
  const int tmo = env_ms("ARTLITE_EP_INIT_TIMEOUT_MS", 120000);
  const int rc = nccl_settle(N, comm, tmo, "ep_init");
  if (rc != ARTLITE_OK) {
    N->commAbort(comm);
    if (rc == ARTLITE_ETIMEOUT)
      set_error("ep_init: rank %d of %d: the communicator did not form within %d ms (aborted)", h->d.ep_rank,
                h->d.ep_world, tmo);
    return rc;
  }
  h->comm = comm;
  const int rs = ep_p2p_setup(h, N, comm);
  if (rs != ARTLITE_OK) {  // (the peers' waits on this rank then fail too: the communicator is gone)
    N->commAbort(comm);
    h->comm = nullptr;
  }
  return rs;
}

}  // extern "C"
