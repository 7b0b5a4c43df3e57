/*
 * artlite_moe.h: the C ABI of libartlite_moe_cuda.so, the B200 (sm_100a) implementation of artlite's GGUF
 * mixture-of-experts block. Plain C types only (no torch, no CUDA types in the signatures); every function returns
 * an int status (0 = ok, negative = ARTLITE_E*) and leaves a message for artlite_moe_last_error().
 *
 * Pointer arguments of the drop-in entry points may point to host memory (the reference's numpy buffers: staged
 * through device memory by the library, the call returns when the results are back) or to device memory of the
 * current CUDA device (used in place; the call still returns when the work is done, so that errors are reported).
 *
 * Reference interfaces replaced (artlite-project/artlite):
 *   artlite_moe_route      <- artlite::moe_route   csrc/artlite/moe_host.h:13-14,
 *                             bound as _native.moe_route  csrc/bindings/moe.cpp:20-36
 *   artlite_moe_plan       <- artlite::moe_plan    csrc/artlite/moe_host.h:21-22,
 *                             bound as _native.moe_plan   csrc/bindings/moe.cpp:37-59
 *   artlite_dequant_rows   <- artlite::dequant_rows csrc/artlite/dequant.h:16 (bound as _native.dequant_rows)
 *   artlite_dequant_supported <- artlite::dequant_supported csrc/artlite/dequant.h:11
 *   artlite_moe_create / set_weights / forward / destroy
 *                          <- the block the reference composes from MoEPrefill.items + host_route / host_streams
 *                             (src/artlite/moe/prefill.py:102-195) and defines in its oracle ref.moe_ffn
 *                             (tests/moe/ref.py:43-52); the reference has no single-call equivalent.
 *   artlite_moe_last_error <- the message of artlite::Error (csrc/artlite/error.h:10-12), which the reference's
 *                             bindings translate to the Python exception artlite.Error (csrc/bindings/errors.cpp).
 */
#ifndef ARTLITE_MOE_H
#define ARTLITE_MOE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* status codes */
#define ARTLITE_OK 0
#define ARTLITE_EINVAL -1     /* bad argument: the reference's artlite::Error cases (e.g. "moe_route: k 9 of E 8") */
#define ARTLITE_ECAPACITY -2  /* moe_plan: a column needs more than cap chunks (moe_host.cpp:223) */
#define ARTLITE_ECUDA -3      /* a CUDA runtime / driver call failed */
#define ARTLITE_ENCCL -4      /* an NCCL call failed (expert-parallel exchange) */
#define ARTLITE_ETIMEOUT -5   /* a bounded wait ran out (host event wait, device flag wait) */
#define ARTLITE_EDEVICE -6    /* a kernel reported a bad input through its status word (e.g. an expert id >= E) */
#define ARTLITE_EUNSUPPORTED -7 /* a shape or type this build does not implement */

/* ggml tensor type ids (gguf_model.py:385-390) accepted by the block */
#define ARTLITE_F32 0
#define ARTLITE_F16 1
#define ARTLITE_Q4_0 2
#define ARTLITE_Q4_1 3
#define ARTLITE_Q8_0 8
#define ARTLITE_Q3_K 11
#define ARTLITE_Q4_K 12
#define ARTLITE_Q5_K 13
#define ARTLITE_Q6_K 14
#define ARTLITE_IQ4_NL 20
#define ARTLITE_IQ4_XS 23
#define ARTLITE_BF16 30

/* The message of the last failed call on this thread ("" if none). */
const char* artlite_moe_last_error(void);

/* Library version string. */
const char* artlite_moe_version(void);

/*
 * Routing (drop-in for artlite::moe_route, moe_host.h:9-14): per token t of n, the k largest of E fp32 logits (expert
 * e at logits[t row + (e / per_col) pitch + e % per_col]), largest first, ties to the lower id, -0 equal to +0;
 * weights e^(l - l_max) over the k in double, normalised in numpy's pairwise order, rounded to fp32 (sigmoid != 0:
 * sigmoid(l) over their sum, at least 2^-14). ids (n x k) int32, weights (n x k) fp32. E <= 1024, k <= 32.
 */
int artlite_moe_route(const float* logits, int64_t n, int64_t row, int per_col, int64_t pitch, int E, int k,
                      int sigmoid, int32_t* ids, float* weights);

/*
 * The plan (drop-in for artlite::moe_plan, moe_host.h:16-22): an expert's (token, slot) pairs in token order, in
 * chunks of at most `chunk`, dealt to the cols columns in turn, expert by expert: experts (cols x cap), counts (cols),
 * sizes (cols x cap), rows (cols x cap x chunk; padding repeats the chunk's first token), pos (n x k) =
 * (c cap + kk) chunk + j. ARTLITE_EINVAL on an id outside [0, E); ARTLITE_ECAPACITY when a column needs more than cap
 * chunks (the reference's two artlite::Error cases, moe_host.cpp:207,223).
 */
int artlite_moe_plan(const int32_t* ids, int64_t n, int k, int E, int cols, int cap, int chunk, int32_t* experts,
                     int32_t* counts, int32_t* sizes, int32_t* rows, int64_t* pos);

/*
 * The expert-contiguous dispatch the block runs on the GPU (the histogram / scan / stable permute at the head of
 * moe_plan, moe_host.cpp:203-215): offsets (E + 1, int64) the exclusive scan of the per-expert pair counts, perm
 * (n k, int32) the pairs t k + i in expert-then-pair order, slot (n k, int32) the position of each pair in perm.
 */
int artlite_moe_dispatch(const int32_t* ids, int64_t n, int k, int E, int64_t* offsets, int32_t* perm,
                         int32_t* slot);

/*
 * The same dispatch for callers that must not allocate device memory while they run (a serving loop that reserves its
 * memory budget at start-up, code whose device memory a framework's caching allocator owns): it allocates nothing.
 * No counterpart in the reference. ids, offsets, perm and slot must be device memory of the current device (host,
 * pinned, managed and other GPUs' buffers are rejected with ARTLITE_EINVAL before anything is launched); the
 * scratch is a 1 MiB static device array of this library (held on every GPU that loads it until exit), so a call
 * takes at most ceil(n k / 4096) E <= 262144 block counts (n k <= 8,388,608 pairs at E = 128) and rejects more with
 * ARTLITE_EINVAL. The first call on a device looks the array's address up (cudaGetSymbolAddress) for that device; make
 * it before any stream capture. Enqueued on `stream` (NULL: the default stream), then waited for (at most 60 s:
 * ARTLITE_ETIMEOUT); an expert id outside [0, E) returns ARTLITE_EINVAL. Every call shares the array, so calls that
 * overlap on the GPU race.
 */
int artlite_moe_dispatch_noalloc(const int32_t* ids, int64_t n, int k, int E, int64_t* offsets, int32_t* perm,
                                 int32_t* slot, void* stream);

/* Whether artlite_dequant_rows reads a GGUF type name ("Q4_0", "Q8_0", "Q4_K", ...; dequant.h:9-11). */
int artlite_dequant_supported(const char* qtype);

/*
 * n GGUF rows of qtype (row_bytes apart from raw) dequantised into out (n x cols fp32), with the fp32 operations of
 * the reference's dequant_rows in their order (dequant.h:13-16): bit-identical values.
 */
int artlite_dequant_rows(const char* qtype, const uint8_t* raw, int64_t n, int64_t row_bytes, int64_t cols,
                         float* out);

/* ---------------------------------------------------------------- the block */

typedef struct artlite_moe artlite_moe;

typedef struct {
  int32_t hidden;        /* H */
  int32_t n_experts;     /* E (<= 1024) */
  int32_t top_k;         /* K (<= 32) */
  int32_t expert_ffn;    /* F */
  int32_t n_layers;      /* weight slots (a stack of blocks, each with its own weights) */
  int32_t gating;        /* 0 softmax, 1 sigmoid (moe/plan.py:25-36) */
  int32_t act_dtype;     /* x and y: ARTLITE_F32 or ARTLITE_BF16 */
  int32_t max_tokens;    /* the largest T a forward takes (sizes the workspaces) */
  int32_t device;        /* CUDA device ordinal (-1: the current one) */
  int32_t path;          /* 0 auto, 1 the CUDA-core dequant-GEMV path, 2 the tcgen05 grouped-GEMM path */
  int32_t ep_rank;       /* expert parallelism: this rank and the world (1: all experts local) */
  int32_t ep_world;
} artlite_moe_desc;

int artlite_moe_create(const artlite_moe_desc* desc, artlite_moe** out);

/*
 * Layer `layer`'s weights, the GGUF tensors' raw bytes exactly as the file holds them (GGUFFile.tensor(name).raw,
 * gguf_model.py:494-506), copied verbatim to HBM, no conversion: gate / up = blk.L.ffn_{gate,up}_exps.weight (E F rows
 * of H values), down = blk.L.ffn_down_exps.weight (E H rows of F values), router = blk.L.ffn_gate_inp.weight (E x H,
 * router_qtype ARTLITE_F32 or ARTLITE_BF16). Host or device pointers. With ep_world > 1 only this rank's experts'
 * rows are read (experts [rank E / world, (rank + 1) E / world)).
 */
int artlite_moe_set_weights(artlite_moe* h, int layer, int qtype, const void* gate, const void* up,
                            int down_qtype, const void* down, const void* router, int router_qtype);

/*
 * An optional per-expert bias (E fp32, host or device; NULL removes it) added to layer `layer`'s router logits before
 * the routing (a load-skew fixture: the benchmark's Zipf-skewed prefill). The reference's router has none
 * (tests/moe/ref.py:11-14: "no selection bias"); without this call the block has none either.
 */
int artlite_moe_set_router_bias(artlite_moe* h, int layer, const float* bias);

/*
 * Layer `layer`'s input norm and residual (the MoE layer's place in the reference's decoder: the post-attention
 * RMSNorm feeds the router and the experts, GatherNormOperator, src/artlite/moe/gather.py:142-289, and the combined
 * delta is added back to the residual stream, moe/gather.py:11-17): with a norm weight w (H values of w_dtype
 * ARTLITE_F32 or ARTLITE_BF16, host or device; NULL removes it) every forward computes
 *   x_n = rms_norm(x, w, eps) = float32(x / sqrt(mean(x^2) + eps)) * w   (tests/np_ops.py:27-32: the mean in float64)
 * in the activation dtype, routes and runs the experts on x_n, and returns y = x + the routed (and shared) sum, one
 * fp32 sum rounded once. Without this call the block has neither (the benchmark's configs have none).
 */
int artlite_moe_set_norm(artlite_moe* h, int layer, const void* w, int w_dtype, double eps);

/*
 * Layer `layer`'s shared expert (the reference's ref.shared_expert, tests/moe/ref.py:55-60; llama.cpp's
 * ffn_shexp_gated): raw GGUF rows gate / up = blk.L.ffn_{gate,up}_shexp.weight (ffn rows of H values, qtype), down =
 * blk.L.ffn_down_shexp.weight (H rows of ffn values, down_qtype), and gate_inp = blk.L.ffn_gate_inp_shexp.weight (H
 * values of gate_dtype ARTLITE_F32 / ARTLITE_BF16; NULL: no gate). The layer's output becomes the routed sum +
 * sigmoid(gate_inp . x) swiglu(x), both in one fp32 sum rounded once. Host or device pointers; gate = NULL removes the
 * shared expert. With expert parallelism (ep_world > 1) every rank holds the whole shared expert and runs it on its
 * own tokens while the routed rows travel.
 */
int artlite_moe_set_shared(artlite_moe* h, int layer, int ffn, int qtype, const void* gate, const void* up,
                           int down_qtype, const void* down, const void* gate_inp, int gate_dtype);

/*
 * y (T x H) = the block of layer `layer` on x (T x H), act_dtype both: router logits x W_r^T (fp32), routing,
 * dispatch, SwiGLU experts, weighted combine. Host or device x / y; `stream` a cudaStream_t (NULL: the handle's own).
 * With host pointers the call returns when y is back; with device pointers it returns after enqueueing (errors of
 * the enqueued work surface at the next call or at artlite_moe_sync).
 */
int artlite_moe_forward(artlite_moe* h, int layer, const void* x, void* y, int64_t T, void* stream);

/*
 * The same forward as a CUDA graph (device x / y only, no expert parallelism): the first call with a given
 * (layer, T, x, y) captures one forward and instantiates it, every later call launches the graph on `stream` (NULL:
 * the handle's). For decode batches, whose kernels are short enough that launch gaps dominate.
 */
int artlite_moe_forward_graph(artlite_moe* h, int layer, const void* x, void* y, int64_t T, void* stream);

/* Wait (bounded by timeout_ms; <= 0: 60 s) for the handle's work, its last forward included on whichever stream it
 * was enqueued, and report any device-side status (a bounded device wait that ran out: ARTLITE_ETIMEOUT; an expert
 * id out of range: ARTLITE_EDEVICE); the status word is cleared after it is reported. */
int artlite_moe_sync(artlite_moe* h, int timeout_ms);

/*
 * The last forward's routing and dispatch, for the bit-exact checks (any pointer may be NULL): logits (T x E fp32),
 * ids / weights (T x K), offsets (E + 1, int64), perm (T K, int32).
 */
int artlite_moe_debug(artlite_moe* h, float* logits, int32_t* ids, float* weights, int64_t* offsets, int32_t* perm);

/*
 * Per-stage device times (ms) of layer `layer`'s last forward, from CUDA events recorded between its kernels on the
 * forward's stream when the handle was created with ARTLITE_MOE_TIMING=1 (n_out = 0 otherwise): router; route +
 * dispatch; then gate/up, down, combine (GEMV path) or gather + gate/up, down, combine (tcgen05 path). n_out <= 7.
 */
int artlite_moe_stage_times(artlite_moe* h, int layer, float* ms, int* n_out);

/* The expert path layer `layer`'s last forward took: 1 the GEMV path (the fused decode kernel, the small-batch
 * tensor-core GEMVs or the register-decoding GEMVs), 2 the tcgen05 grouped GEMM (0: none yet). */
int artlite_moe_path(artlite_moe* h, int layer);

/*
 * Where layer `layer`'s tensor `which` lives in device memory, as set_weights copied it (the GGUF bytes verbatim, no
 * conversion; GGUFFile.tensor's raw view, gguf_model.py:494-506): 0 ffn_gate_exps, 1 ffn_up_exps, 2 ffn_down_exps
 * (this rank's experts' rows), 3 ffn_gate_inp (the router). *bytes excludes the zeroed slack past the tensor.
 */
int artlite_moe_weights(artlite_moe* h, int layer, int which, const void** ptr, int64_t* bytes);

/* Kernels this library has launched in this process so far (all handles and entry points). */
int64_t artlite_moe_launch_count(void);

int artlite_moe_destroy(artlite_moe* h);

/* ---------------------------------------------------------------- expert parallelism (ep_world > 1)
 * The reference runs on one NPU and has no counterpart (its closest analogue is the 8-column deal of moe_plan,
 * moe_host.cpp:216-234, an intra-device split). One process per GPU; rank r of W owns experts [r E / W, (r + 1) E / W)
 * and its own tokens; artlite_moe_forward exchanges token rows and expert outputs with NCCL (loaded at run time:
 * libnccl.so.2, or ARTLITE_NCCL_LIB). */

/* A new NCCL unique id (NCCL_UNIQUE_ID_BYTES = 128 bytes into out): made on one rank, shared with the others. */
int artlite_moe_ep_unique_id(void* out, int bytes);

/* Joins the handle (created with ep_world = W, ep_rank = r) to the communicator of unique_id; collective over the W
 * ranks. */
int artlite_moe_ep_init(artlite_moe* h, const void* unique_id, int bytes);

/*
 * The exchange plan of one rank (host only, no GPU): send_counts (E) this rank's pairs per expert; recv_counts
 * (world x E / world) the pairs each rank sends for this rank's experts. Out: send_off (E) each expert's first row in
 * this rank's expert-ordered rows; recv_pos (world x E / world) where the rows from rank q for local expert e land in
 * the received rows (grouped by local expert, then by rank); local_off (E / world + 1) / local_counts (E / world) the
 * received rows per local expert. (The block's own forward keeps the received blocks source-major and runs each
 * (source rank, local expert) row group in place, or from 8 ranks gathers them into this expert-grouped layout first;
 * the plan gives the layout to callers that exchange rows themselves.)
 */
int artlite_moe_ep_plan(const int32_t* send_counts, const int32_t* recv_counts, int world, int rank, int E,
                        int64_t* send_off, int64_t* recv_pos, int64_t* local_off, int32_t* local_counts);

#ifdef __cplusplus
}
#endif

#endif /* ARTLITE_MOE_H */
