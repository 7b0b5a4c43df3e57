// Expert parallelism across the GPUs of one node: rank r of W owns experts [r E / W, (r + 1) E / W) (their raw GGUF
// rows only, set_weights) and its own tokens; per layer
//   1. router, routing and the dispatch over all E experts, on the rank's tokens (block.cu: route_and_dispatch);
//   2. the token rows gathered into expert order (bf16): contiguous per destination rank;
//   3. per-expert pair counts exchanged (NCCL send / recv of E / W int32 per peer), read back to the host (the one
//      host synchronisation of the layer: NCCL message sizes are host values), the exchange plan computed on the host
//      (artlite_moe_ep_plan);
//   4. the token rows exchanged with grouped ncclSend / ncclRecv, one message per peer (a rank's rows for a peer's
//      experts are one contiguous block of its dispatch order), its own block by a device copy; the received blocks
//      (rank-major, expert-minor) copied into expert-major order by a segment-copy kernel;
//   5. the local experts on the received rows (block.cu: run_experts; the tcgen05 path or the GEMVs);
//   6. the outputs copied back into rank-major blocks (the inverse segments), one message per peer, each landing
//      as the contiguous block of the source rank's dispatch order it came from;
//   7. the weighted combine of the rank's own tokens (combine.cu).
// NCCL is loaded at run time (dlopen "libnccl.so.2": the one a process that imported torch already holds, or the
// system's), so the library itself has no link-time NCCL dependency. Waits on the host are bounded: a peer that never
// sends makes the count exchange's wait run out, the communicator is aborted and the call returns ARTLITE_ETIMEOUT.
// Nothing here uses TMA multicast or reads another GPU's memory from a kernel: every byte between GPUs moves by NCCL.
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>
#include <stdlib.h>
#include <string.h>

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
    g_nccl = n;
  }
  *out = &g_nccl;
  return ARTLITE_OK;
}

#define AL_NCCL(call)                                                                               \
  do {                                                                                              \
    const ncclResult_t r_ = (call);                                                                 \
    if (r_ != ncclSuccess) {                                                                        \
      ::artlite::set_error("%s:%d %s: %s", __FILE__, __LINE__, #call, N->errorString(r_));          \
      return ARTLITE_ENCCL;                                                                         \
    }                                                                                               \
  } while (0)

// rows of `row_bytes` (a multiple of 16) in segments: segment g's n[g] rows from src row s[g] to dst row d[g]
__global__ void __launch_bounds__(256) segment_copy_kernel(const uint8_t* src, uint8_t* dst, const int64_t* s,
                                                            const int64_t* d, const int64_t* n, int64_t row_bytes) {
  const int g = blockIdx.y;
  const int64_t rows = n[g];
  const int64_t v16 = row_bytes / 16;
  for (int64_t i = blockIdx.x; i < rows; i += gridDim.x) {
    const uint4* a = reinterpret_cast<const uint4*>(src + (s[g] + i) * row_bytes);
    uint4* b = reinterpret_cast<uint4*>(dst + (d[g] + i) * row_bytes);
    for (int64_t j = threadIdx.x; j < v16; j += blockDim.x) b[j] = a[j];
  }
}

__global__ void iota_kernel(int32_t* p, int64_t n) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) p[i] = (int32_t)i;
}

}  // namespace

int launch_segment_copy(const void* src, void* dst, const int64_t* s, const int64_t* d, const int64_t* n, int nseg,
                        int64_t row_bytes, int64_t total_rows, cudaStream_t st) {
  if (nseg == 0 || total_rows == 0) return ARTLITE_OK;
  AL_CHECK(row_bytes % 16 == 0, ARTLITE_EINVAL, "segment copy: rows of %lld bytes", (long long)row_bytes);
  const unsigned per = (unsigned)std::min<int64_t>(64, std::max<int64_t>(1, total_rows / nseg));
  segment_copy_kernel<<<dim3(per, (unsigned)nseg), 256, 0, st>>>(static_cast<const uint8_t*>(src),
                                                                  static_cast<uint8_t*>(dst), s, d, n, row_bytes);
  AL_LAUNCHED();
  return ARTLITE_OK;
}

int ep_create(artlite_moe* h) {
  const artlite_moe_desc& d = h->d;
  const int W = d.ep_world, El = h->E_local, E = d.n_experts, H = d.hidden, F = d.expert_ffn, K = d.top_k;
  const int64_t T = d.max_tokens > 0 ? d.max_tokens : 1;
  const int64_t R = T * K * W;  // the most rows a rank can receive (every rank's pairs all on its experts)
  h->ep_max_rows = R;
  AL_TRY(h->ep_rcounts.reserve(sizeof(int32_t) * E));
  AL_TRY(h->ep_loff.reserve(sizeof(int64_t) * (El + 1)));
  AL_TRY(h->ep_lcounts.reserve(sizeof(int32_t) * El));
  AL_TRY(h->ep_ident.reserve(sizeof(int32_t) * R));
  AL_TRY(h->xl.reserve(sizeof(uint16_t) * (R + 256) * H));
  AL_TRY(h->xr.reserve(sizeof(uint16_t) * R * H));
  AL_TRY(h->yr.reserve(sizeof(float) * R * H));
  AL_TRY(h->ep_seg.reserve(sizeof(int64_t) * 3 * E));
  AL_TRY(h->ys.reserve(sizeof(float) * T * K * H));
  // the expert workspaces hold the received rows (h: fp32 or bf16 with 256 spare rows; y: fp32 or bf16)
  AL_TRY(h->h.reserve(std::max(sizeof(float) * R * F, sizeof(uint16_t) * (R + 256) * F)));
  AL_TRY(h->y.reserve(sizeof(float) * R * H));
  AL_TRY(h->tiles.reserve(tc_sched_bytes(El)));
  AL_CUDA(cudaHostAlloc(reinterpret_cast<void**>(&h->hb_counts), sizeof(int32_t) * 2 * E, cudaHostAllocDefault));
  AL_CUDA(cudaHostAlloc(reinterpret_cast<void**>(&h->hb_loff), sizeof(int64_t) * (El + 1), cudaHostAllocDefault));
  AL_CUDA(cudaHostAlloc(reinterpret_cast<void**>(&h->hb_lcounts), sizeof(int32_t) * El, cudaHostAllocDefault));
  AL_CUDA(cudaHostAlloc(reinterpret_cast<void**>(&h->hb_seg), sizeof(int64_t) * 3 * E, cudaHostAllocDefault));
  h->ep_send_base.assign(W, 0);
  h->ep_recv_base.assign(W, 0);
  h->ep_send_rows.assign(W, 0);
  h->ep_recv_rows.assign(W, 0);
  iota_kernel<<<(unsigned)cdiv(R, 256), 256, 0, h->st>>>(h->ep_ident.as<int32_t>(), R);
  AL_LAUNCHED();
  h->ep_send_off.assign(E, 0);
  h->ep_recv_pos.assign((size_t)W * El, 0);
  return ARTLITE_OK;
}

void ep_destroy(artlite_moe* h) {
  if (h->comm) {
    Nccl* N;
    if (nccl(&N) == ARTLITE_OK) {
      // (after a failed exchange the peers may never complete theirs: abort, which does not wait for them)
      if (h->ep_failed) N->commAbort(static_cast<ncclComm_t>(h->comm));
      else N->commDestroy(static_cast<ncclComm_t>(h->comm));
    }
    h->comm = nullptr;
  }
  if (h->hb_counts) cudaFreeHost(h->hb_counts);
  if (h->hb_loff) cudaFreeHost(h->hb_loff);
  if (h->hb_lcounts) cudaFreeHost(h->hb_lcounts);
  if (h->hb_seg) cudaFreeHost(h->hb_seg);
  h->hb_seg = nullptr;
  h->hb_counts = nullptr;
  h->hb_loff = nullptr;
  h->hb_lcounts = nullptr;
}

namespace {
int ep_forward_impl(artlite_moe* h, int layer, const void* xd, void* yd, int64_t T, cudaStream_t st, Marker& mk);

int ep_timeout_ms() {
  const char* v = getenv("ARTLITE_EP_TIMEOUT_MS");
  const int t = v ? atoi(v) : 0;
  return t > 0 ? t : 30000;
}
}  // namespace

// The EP forward; any failure once the exchanges have begun aborts the communicator (the peers' next bounded wait
// then fails too) and leaves the handle unusable for expert parallelism, instead of a rank blocking on a peer forever.
int ep_forward(artlite_moe* h, int layer, const void* xd, void* yd, int64_t T, cudaStream_t st, Marker& mk) {
  AL_CHECK(h->comm && !h->ep_failed, ARTLITE_EINVAL,
           "moe_forward: expert parallelism needs artlite_moe_ep_init first (or a previous exchange failed)");
  const int rc = ep_forward_impl(h, layer, xd, yd, T, st, mk);
  if (rc != ARTLITE_OK && h->comm) {
    Nccl* N;
    if (nccl(&N) == ARTLITE_OK) N->commAbort(static_cast<ncclComm_t>(h->comm));
    h->comm = nullptr;
    h->ep_failed = true;
  }
  return rc;
}

namespace {
int ep_forward_impl(artlite_moe* h, int layer, const void* xd, void* yd, int64_t T, cudaStream_t st, Marker& mk) {
  Nccl* N;
  AL_TRY(nccl(&N));
  ncclComm_t comm = static_cast<ncclComm_t>(h->comm);
  const artlite_moe_desc& d = h->d;
  const artlite_moe::Layer& L = h->layers[layer];
  const int W = d.ep_world, r = d.ep_rank, El = h->E_local, E = d.n_experts, H = d.hidden, K = d.top_k;
  const int64_t P = T * K;
  // 1-2: routing and the dispatch over all experts; the rows in expert order (contiguous per destination rank)
  AL_TRY(route_and_dispatch(h, L, xd, T, st, mk));
  if (P) AL_TRY(launch_gather(xd, d.act_dtype, h->perm.as<int32_t>(), P, K, H, h->xp.as<uint16_t>(), st));
  // 3: counts, then the plan on the host
  AL_NCCL(N->groupStart());
  for (int q = 0; q < W; q++) {
    AL_NCCL(N->send(h->counts.as<int32_t>() + q * El, El, ncclInt32, q, comm, st));
    AL_NCCL(N->recv(h->ep_rcounts.as<int32_t>() + q * El, El, ncclInt32, q, comm, st));
  }
  AL_NCCL(N->groupEnd());
  AL_CUDA(cudaMemcpyAsync(h->hb_counts, h->counts.ptr, sizeof(int32_t) * E, cudaMemcpyDeviceToHost, st));
  AL_CUDA(cudaMemcpyAsync(h->hb_counts + E, h->ep_rcounts.ptr, sizeof(int32_t) * E, cudaMemcpyDeviceToHost, st));
  const int tmo = ep_timeout_ms();
  const int rc = wait_deadline(st, tmo);
  if (rc == ARTLITE_ETIMEOUT) {  // a peer that never sent its counts (the caller aborts the communicator)
    set_error("expert parallelism: rank %d: the count exchange did not complete within %d ms (communicator aborted)",
              r, tmo);
    return ARTLITE_ETIMEOUT;
  }
  AL_TRY(rc);
  AL_TRY(artlite_moe_ep_plan(h->hb_counts, h->hb_counts + E, W, r, E, h->ep_send_off.data(), h->ep_recv_pos.data(),
                             h->hb_loff, h->hb_lcounts));
  const int64_t Rl = h->hb_loff[El];
  AL_CHECK(Rl <= h->ep_max_rows, ARTLITE_EDEVICE, "expert parallelism: %lld rows received, room for %lld",
           (long long)Rl, (long long)h->ep_max_rows);
  // per rank q: the block this rank sends (its rows for q's experts, contiguous in dispatch order) and the block it
  // receives (q's rows for this rank's experts: expert-major inside); the segments (q, e) of the received blocks and
  // their places in expert-grouped order
  const int32_t* sc = h->hb_counts;
  const int32_t* rcv = h->hb_counts + E;
  int64_t* seg = h->hb_seg;  // [3][W El]: source row, destination row, rows
  std::vector<int64_t>& send_base = h->ep_send_base;
  std::vector<int64_t>& recv_base = h->ep_recv_base;
  std::vector<int64_t>& send_rows = h->ep_send_rows;
  std::vector<int64_t>& recv_rows = h->ep_recv_rows;
  int64_t rb = 0;
  for (int q = 0; q < W; q++) {
    send_base[q] = h->ep_send_off[(size_t)q * El];
    int64_t sn = 0, rn = 0;
    for (int e = 0; e < El; e++) {
      const int g = q * El + e;
      sn += sc[g];
      seg[g] = rb + rn;                                  // where (q, e)'s rows sit in the received block
      seg[W * El + g] = h->ep_recv_pos[(size_t)q * El + e];  // where they go (expert-grouped)
      seg[2 * W * El + g] = rcv[g];
      rn += rcv[g];
    }
    send_rows[q] = sn;
    recv_base[q] = rb;
    recv_rows[q] = rn;
    rb += rn;
  }
  AL_CUDA(cudaMemcpyAsync(h->ep_loff.ptr, h->hb_loff, sizeof(int64_t) * (El + 1), cudaMemcpyHostToDevice, st));
  AL_CUDA(cudaMemcpyAsync(h->ep_lcounts.ptr, h->hb_lcounts, sizeof(int32_t) * El, cudaMemcpyHostToDevice, st));
  AL_CUDA(cudaMemcpyAsync(h->ep_seg.ptr, seg, sizeof(int64_t) * 3 * W * El, cudaMemcpyHostToDevice, st));
  const int64_t* dseg = h->ep_seg.as<int64_t>();
  // 4: the token rows, one message per peer; this rank's own block by a device copy; then into expert order
  const uint16_t* xp = h->xp.as<uint16_t>();
  uint16_t* xr = h->xr.as<uint16_t>();
  uint16_t* xl = h->xl.as<uint16_t>();
  AL_NCCL(N->groupStart());
  for (int q = 0; q < W; q++) {
    if (q == r) continue;
    if (send_rows[q]) AL_NCCL(N->send(xp + send_base[q] * H, (size_t)send_rows[q] * H, ncclBfloat16, q, comm, st));
    if (recv_rows[q]) AL_NCCL(N->recv(xr + recv_base[q] * H, (size_t)recv_rows[q] * H, ncclBfloat16, q, comm, st));
  }
  AL_NCCL(N->groupEnd());
  if (send_rows[r])
    AL_CUDA(cudaMemcpyAsync(xr + recv_base[r] * H, xp + send_base[r] * H, sizeof(uint16_t) * send_rows[r] * H,
                            cudaMemcpyDeviceToDevice, st));
  AL_TRY(launch_segment_copy(xr, xl, dseg, dseg + W * El, dseg + 2 * W * El, W * El, (int64_t)H * 2, Rl, st));
  AL_TRY(mk.mark());
  // 5: the local experts
  const int path = expert_path(*h, Rl, L);
  h->last_path = path;
  h->paths[layer] = path;
  void* yrows;
  int ydt;
  AL_TRY(run_experts(h, L, path, xl, ARTLITE_BF16, true, h->ep_ident.as<int32_t>(), 1, Rl, El,
                     h->ep_loff.as<int64_t>(), h->ep_lcounts.as<int32_t>(), (int64_t)(h->xl.bytes / (2 * H)), &yrows,
                     &ydt, st, mk));
  // 6: the outputs back: into per-rank blocks (the inverse segments), one message per peer, into dispatch order
  const size_t el = ydt == ARTLITE_BF16 ? 2 : 4;
  const ncclDataType_t dt = ydt == ARTLITE_BF16 ? ncclBfloat16 : ncclFloat32;
  uint8_t* yr = h->yr.as<uint8_t>();
  uint8_t* ys = h->ys.as<uint8_t>();
  AL_TRY(launch_segment_copy(yrows, yr, dseg + W * El, dseg, dseg + 2 * W * El, W * El, (int64_t)H * el, Rl, st));
  AL_NCCL(N->groupStart());
  for (int q = 0; q < W; q++) {
    if (q == r) continue;
    if (recv_rows[q]) AL_NCCL(N->send(yr + recv_base[q] * H * el, (size_t)recv_rows[q] * H, dt, q, comm, st));
    if (send_rows[q]) AL_NCCL(N->recv(ys + send_base[q] * H * el, (size_t)send_rows[q] * H, dt, q, comm, st));
  }
  AL_NCCL(N->groupEnd());
  if (send_rows[r])
    AL_CUDA(cudaMemcpyAsync(ys + send_base[r] * H * el, yr + recv_base[r] * H * el, el * send_rows[r] * H,
                            cudaMemcpyDeviceToDevice, st));
  AL_TRY(mk.mark());
  // 7: the combine of this rank's tokens
  if (T) AL_TRY(launch_combine(ys, ydt, h->slot.as<int32_t>(), h->w.as<float>(), T, K, H, yd, d.act_dtype, st));
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
  ncclComm_t comm;
  AL_NCCL(N->commInitRank(&comm, h->d.ep_world, id, h->d.ep_rank));
  h->comm = comm;
  return ARTLITE_OK;
}

}  // extern "C"
