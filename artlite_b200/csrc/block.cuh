// The MoE block handle's state, shared by block.cu (single GPU) and ep.cu (expert parallelism over NCCL).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <vector>

#include "common.cuh"

struct artlite_moe {
  artlite_moe_desc d{};
  int dev = 0;
  cudaStream_t st = nullptr;
  int E_local = 0, e0 = 0;  // this rank's experts [e0, e0 + E_local)
  struct Layer {
    artlite::DevBuf gate, up, down, router, bias, planes;
    bool has_bias = false;
    int n_planes = 0;  // the router's bf16 planes (router_split): 3 for an F32 router, 1 for BF16
    int qtype = -1, down_qtype = -1, router_qtype = -1;
    int64_t rb_gu = 0, rb_dn = 0;
    // Q4_K: tensor maps of the raw rows for the fused decode kernel (gate / up: boxes of 64 rows, down: 128 rows,
    // one 144-byte super-block wide)
    bool has_dm = false;     // the fused decode kernel's maps of gate, up and down (Q4_K everywhere)
    bool has_dm_gu = false;  // those of gate and up (Q4_K gate / up, any down type)
    CUtensorMap dm_gate, dm_up, dm_down;
    // and for the small-batch GEMVs (mss.cu): gate / up boxes of 32 rows (down: dm_down)
    bool has_ss = false;
    CUtensorMap ss_gate, ss_up;
    // RMSNorm of the input before the router and the experts, and the input added back to the output as the residual
    // (artlite_moe_set_norm): the norm weight (H values of norm_dtype) and eps
    bool has_norm = false;
    int norm_dtype = -1;
    double norm_eps = 0;
    artlite::DevBuf norm_w;
    // the shared expert (artlite_moe_set_shared): raw rows of one SwiGLU expert of width sh_F, and its gate vector
    bool has_shared = false, sh_has_gate = false;
    int sh_F = 0, sh_qtype = -1, sh_down_qtype = -1, sh_gate_dtype = -1;
    int64_t sh_rb_gu = 0, sh_rb_dn = 0;
    artlite::DevBuf sh_gate, sh_up, sh_down, sh_ginp;
    // Q4_K shared experts: tensor maps of its raw rows for the fused decode kernel (as dm_* for the routed experts)
    bool sh_has_dm = false;
    CUtensorMap sh_dm_gate, sh_dm_up, sh_dm_down;
    bool sh_has_ss = false;           // the small-batch GEMVs' gate / up maps of the shared expert (Q4_K gate / up)
    CUtensorMap sh_ss_gate, sh_ss_up;
  };
  std::vector<Layer> layers;
  // workspaces
  artlite::DevBuf xin, yout, logits, ids, w, offsets, perm, slot, counts, blk, unit_gu, unit_dn, status;
  artlite::DevBuf h, y, xp, tiles;
  artlite::DevBuf xn;  // the normed input rows (layers with artlite_moe_set_norm)
  artlite::DevBuf bar;  // the fused decode kernel's grid barrier (zeroed once; left zeroed by every complete run)
  artlite::DevBuf sh_y, sh_s, sh_iota, sh_off;  // the shared expert's outputs (T rows), gates (T), 0..T-1, {0, T} / {T}
  artlite::DevBuf sh_hq;  // the fused decode kernel's shared-expert h rows (fragment order, then their group sums)
  int64_t last_T = 0;
  int last_path = 0;
  // recorded on the forward's stream at the end of every forward (and graph replay): artlite_moe_sync waits for it,
  // so that a forward enqueued on a caller's stream is waited for before the status word is read
  cudaEvent_t done = nullptr;
  bool timing = false;
  std::vector<cudaEvent_t> ev;  // [n_layers][kStages]: the last forward of each layer, read without a sync
  std::vector<int> n_stages;    // per layer
  std::vector<int> paths;       // per layer: the expert path of its last forward
  // CUDA graphs of whole forwards (artlite_moe_forward_graph), keyed by (layer, T, x, y, stream)
  struct Graph {
    int layer;
    int64_t T;
    const void* x;
    void* y;
    cudaGraphExec_t exec;
  };
  std::vector<Graph> graphs;
  // expert parallelism (ep.cu): the NCCL communicator, exchange buffers, pinned host copies of the counts
  void* comm = nullptr;                // ncclComm_t
  cudaStream_t ep_st = nullptr;        // the exchanges' stream (overlapping the experts)
  static constexpr int kEpChunks = 4;  // the peers' row groups in up to this many expert chunks (pipelined)
  int ep_chunks = 1;
  cudaEvent_t ep_ev[2 + 2 * kEpChunks] = {};  // rows gathered, returns in, per chunk: rows in, outputs ready
  artlite::DevBuf ep_loff, ep_lcounts, ep_wexp, ep_ident, xr, ys;
  artlite::DevBuf ep_idx, xe;          // the regroup's row maps (2 x ep_max_rows) and expert-major rows
  int32_t* hb_idx = nullptr;           // pinned: the same maps, built on the host
  int ep_regroup = -1;                 // rows regrouped expert-major before the experts: -1 from 8 ranks, 0 no, 1 yes
  std::vector<int64_t> ep_xoff;        // [E_local + 1] the expert-major groups' offsets
  int32_t* hb_counts = nullptr;        // pinned: [E] this rank's pairs per expert, then [world x E_local] received
  int64_t* hb_loff = nullptr;          // pinned: [world E_local + 1] the received row groups' offsets
  int32_t* hb_lcounts = nullptr;       // pinned: [world E_local] their rows
  std::vector<int64_t> ep_send_base, ep_recv_base, ep_send_rows, ep_recv_rows;  // per peer: blocks sent / received
  std::vector<int64_t> ep_cs_pos, ep_cs_rows, ep_cr_pos, ep_cr_rows;  // per (peer, chunk): sent / received blocks
  int64_t ep_max_rows = 0;             // rows a rank can receive: max_tokens K world
  bool ep_failed = false;              // an exchange failed: the communicator is aborted, never waited for
  // the peer-store exchange (ep.cu): the rows and outputs written straight into the peers' receive buffers by this
  // library's kernels over NVLink (CUDA IPC mappings), each block followed by a flag in the peer's flag array
  artlite::DevBuf ep_flags;            // [2 world] u32: rows in from source q at q, outputs in from owner q at world + q
  artlite::DevBuf ep_done;             // the push kernels' count of finished CTAs (zero, left zero)
  artlite::DevBuf ep_fullc;            // [world][E] every rank's pairs per expert (the count exchange)
  int32_t* hb_full = nullptr;          // pinned: the same
  std::vector<uint8_t*> ep_peer_xr, ep_peer_ys;  // per rank: its receive / return buffer (null for this rank)
  std::vector<uint32_t*> ep_peer_flags;
  std::vector<int64_t> ep_peer_xr_bytes, ep_peer_ys_bytes;  // their sizes
  bool ep_p2p = false;                 // rows and outputs by the peer-store kernels (else NCCL send / recv)
  uint32_t ep_epoch = 0;               // forwards so far (the flags' value for the current one)
};


namespace artlite {

constexpr int kStages = 8;

// per-stage CUDA events of a forward (ARTLITE_MOE_TIMING=1)
struct Marker {
  artlite_moe* h;
  int layer;
  cudaStream_t st;
  int ns = 0;
  int mark() {
    if (h->timing && ns < kStages) {
      const cudaError_t e = cudaEventRecord(h->ev[(size_t)layer * kStages + ns++], st);
      if (e != cudaSuccess) {
        set_error("event record: %s", cudaGetErrorString(e));
        return ARTLITE_ECUDA;
      }
    }
    return ARTLITE_OK;
  }
};

// the raw rows one run of the expert GEMMs reads: the routed experts of a layer, or its shared expert
struct ExpertWeights {
  int qtype, down_qtype;
  const uint8_t *gate, *up, *down;
  int64_t rb_gu, rb_dn;
  const CUtensorMap *ss_gate, *ss_up, *ss_down;  // the small-batch GEMVs' maps (null: none)
};
inline ExpertWeights routed_weights(const artlite_moe::Layer& L) {
  return {L.qtype, L.down_qtype, L.gate.as<uint8_t>(), L.up.as<uint8_t>(), L.down.as<uint8_t>(), L.rb_gu, L.rb_dn,
          L.has_ss ? &L.ss_gate : nullptr, L.has_ss ? &L.ss_up : nullptr, L.has_dm ? &L.dm_down : nullptr};
}
inline ExpertWeights shared_weights(const artlite_moe::Layer& L) {
  return {L.sh_qtype, L.sh_down_qtype, L.sh_gate.as<uint8_t>(), L.sh_up.as<uint8_t>(), L.sh_down.as<uint8_t>(),
          L.sh_rb_gu, L.sh_rb_dn, L.sh_has_ss ? &L.sh_ss_gate : nullptr, L.sh_has_ss ? &L.sh_ss_up : nullptr,
          L.sh_has_dm ? &L.sh_dm_down : nullptr};
}
// the small-batch tensor-core GEMVs apply (GEMV path, Q4_K with maps, bf16 x; ARTLITE_DECODE_MSS=0 turns them off)
bool mss_use(const artlite_moe& h, const ExpertWeights& W, int path, int x_dtype, int F);

// router logits, routing and the dispatch over all E experts of T tokens x (device, act dtype) into the handle's
// logits / ids / w / offsets / perm / slot / counts
// mult_gu > 0: the decode-sized path (the small router when it applies, routing and dispatch in one kernel, which also
// writes the GEMVs' unit scans: mult_gu / mult_dn items per expert and token group)
// A layer's input norm, when the forward has one: the raw rows x, the weight w (H values of w_dtype) and eps; the
// normed rows go to the handle's xn buffer, which the forward passes on as its x. The kernel that first reads the rows
// norms them where it can (the fused decode kernel, the CTA-per-expert router); otherwise the norm kernel runs first.
struct NormIn {
  const void* x = nullptr;
  const void* w = nullptr;
  int w_dtype = 0;
  double eps = 0;
};
int run_norm(artlite_moe* h, const NormIn& n, void* xn, int64_t T, cudaStream_t st);

// norm (may be null): the layer's input norm, x its output buffer (the norm fused into the router where it can be)
int route_and_dispatch(artlite_moe* h, const artlite_moe::Layer& L, const void* x, int64_t T, cudaStream_t st,
                       Marker& mk, int mult_gu = 0, int mult_dn = 0, const NormIn* norm = nullptr);

// F_run (0: the block's expert_ffn) the experts' width; y_out (null: the handle's y buffer) where the output rows go.
// wexp (device, may be null): the weight expert of each of the E_run row groups (expert parallelism: a group is one
// source rank's rows of one local expert), E_w the experts the weights hold (0: E_run).
// The experts of a forward over P rows for E_run experts (offsets / counts on the device): rows are the tokens x
// through perm / k (gathered = false), or already gathered bf16 rows in expert order (gathered = true, perm = the
// identity, k = 1). Output rows in the same order into *y_rows (the handle's y buffer), fp32 (GEMV path) or bf16
// (tcgen05 path) in *y_dtype.
int run_experts(artlite_moe* h, const ExpertWeights& W, int path, const void* x, int x_dtype, bool gathered,
                const int32_t* perm, int k, int64_t P, int E_run, const int64_t* offsets, const int32_t* counts,
                int64_t x_rows, void** y_rows, int* y_dtype, cudaStream_t st, Marker& mk, bool units_ready = false,
                const int32_t* wexp = nullptr, int E_w = 0, int F_run = 0, void* y_out = nullptr);

// destroys the captured forwards (their addresses may be stale after new weights)
void drop_graphs(artlite_moe* h);

// which expert path a forward of P pairs takes
int expert_path(const artlite_moe& h, int64_t P, const artlite_moe::Layer& L);

// a bounded wait for the work enqueued on st so far
int wait_deadline(cudaStream_t st, int timeout_ms);

// expert parallelism (ep.cu)
int ep_create(artlite_moe* h);
int ep_forward(artlite_moe* h, int layer, const void* x, void* y, int64_t T, cudaStream_t st, Marker& mk,
               const void* res = nullptr);
// the layer's shared expert over all T tokens (its gated rows for the combine); with expert parallelism every rank
// holds the whole shared expert and runs it on its own tokens
struct CombineShared;
int run_shared(artlite_moe* h, const artlite_moe::Layer& L, const void* xd, int64_t T, cudaStream_t st,
               CombineShared* sh);
void ep_destroy(artlite_moe* h);

// the fused decode-batch forward (decode.cu): whether it applies, and the launch (x, y device, act dtype)
bool decode_fused_ok(const artlite_moe& h, const artlite_moe::Layer& L, int64_t T);
// norm (may be null): the layer's input norm, done in the kernel's phase 0 with x its output buffer
int launch_decode(artlite_moe* h, const artlite_moe::Layer& L, const void* x, void* y, int64_t T, cudaStream_t st,
                  const void* res = nullptr, const NormIn* norm = nullptr);

}  // namespace artlite
