// The tcgen05 grouped expert GEMM (tc_gemm.cu): declarations.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"

namespace artlite {

struct TcGemmArgs {
  int qtype;              // the weights' GGUF type (Q4_0, Q8_0, Q4_K)
  const uint8_t* w0;      // gu: gate rows (E F x row_bytes); down: down rows (E H x row_bytes)
  const uint8_t* w1;      // gu: up rows
  int64_t row_bytes;
  int K;                  // reduction (gu: H, down: F)
  int N;                  // weight rows per expert (gu: F, down: H)
  int E;
  const uint16_t* x;      // bf16 rows in dispatch order (gu: gathered tokens, P x H; down: h, P x F)
  int64_t x_rows;         // rows the x buffer holds (>= P + 256: the token tiles read whole 256-row boxes)
  int64_t P;
  const int64_t* offsets; // [E + 1] the E row groups' first rows in x
  const int32_t* counts;  // [E]
  const int32_t* wexp;    // (may be null) each row group's weight expert (expert parallelism); null: group e, expert e
  int wE;                 // experts in the weight tensors (0: E)
  void* sched;            // tc_sched_bytes(E) of device scratch (the tile scan)
  uint16_t* out;          // bf16 rows in dispatch order (gu: h, P x F; down: y, P x H)
  DevStatus* status;
};

// a 2D tensor map over raw rows (rows x row_bytes, 16-byte multiples), box box_rows x box_bytes, no swizzle
int make_raw_map(CUtensorMap* m, const void* base, int64_t row_bytes, int64_t rows, int box_bytes, int box_rows);

// whether the tcgen05 path reads this type at these shapes (K, N multiples of 256 / 128)
bool tc_supported(int qtype, int K, int N);
size_t tc_sched_bytes(int E);
int launch_tc_gemm(const TcGemmArgs& a, bool gu, cudaStream_t st);

// The router on the tensor cores: logits (T x E fp32) = x (T x H bf16, x_rows >= T + 128 rows readable) . W^T from
// the bf16 planes of W (router_split: 3 for an fp32 W, 1 for a bf16 W), + bias (E, may be null).
bool router_tc_supported(int E, int H, int x_dtype);
int router_split(const void* w, int w_dtype, int E, int H, uint16_t* planes, cudaStream_t st);
int launch_router_tc(const uint16_t* x, const uint16_t* planes, int n_planes, const float* bias, int64_t T, int H,
                     int E, int64_t x_rows, float* logits, DevStatus* status, cudaStream_t st);

}  // namespace artlite
