// The CUDA-core expert path (decode batches and small T): per expert, a dequant-GEMV over its tokens, fp32 exact
// dequant (quant.cuh) and fp32 accumulation, read straight from the raw GGUF blocks.
//
// Semantics: ref.moe_ffn / swiglu (tests/moe/ref.py:21-24,43-52): h = silu(x W_g^T) * (x W_u^T), y = h W_d^T, per
// (token, slot) pair, the weighted sum in the combine (combine.cu).
//
// Work: an item is (expert e, row tile of RT weight rows, group of up to NT of e's pairs); the dispatch's scan gives
// every expert ceil(n_e / NT) * (N / RT) items (unit_off). A persistent grid takes contiguous item ranges, so that
// consecutive items of a CTA share their tokens (x staged once) and walk the expert's rows. The next item's raw rows
// (one contiguous byte range per tensor, widened to 16-byte bounds) stream into shared memory by cp.async while the
// current item computes; a warp takes RT / 8 rows, its lanes the row's 32-groups, x from shared memory in a padded
// layout (33 floats per group: conflict-free across lanes).
#include <cuda_bf16.h>

#include "common.cuh"
#include "kernels.cuh"
#include "quant.cuh"
#include "rq.cuh"

namespace artlite {


namespace {

constexpr int kWarps = 8;

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  const unsigned s = (unsigned)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(s), "l"(gmem));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N)); }

__device__ __forceinline__ float load_act(const void* x, int dtype, int64_t i) {
  if (dtype == ARTLITE_BF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(x)[i]);
  return reinterpret_cast<const float*>(x)[i];
}

__device__ __forceinline__ float silu(float g) { return __fdiv_rn(g, __fadd_rn(1.0f, expf(-g))); }

struct Item {
  int e, tg, rt;
};

__device__ __forceinline__ Item item_of(const int32_t* unit_off, int E, int ntile, int i) {
  int lo = 0, hi = E;  // the largest e with unit_off[e] <= i
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (unit_off[mid] <= i) lo = mid; else hi = mid;
  }
  const int li = i - unit_off[lo];
  return {lo, li / ntile, li % ntile};
}

// stage the raw bytes of rows [r0, r0 + rows) of a row-major tensor (row_bytes apart, 16-byte aligned base) into
// dst; returns the offset of row r0 in dst
__device__ __forceinline__ int stage_rows(uint8_t* dst, const uint8_t* base, int64_t r0, int rows, int64_t rb) {
  const int64_t b0 = r0 * rb, b1 = (r0 + rows) * rb;
  const int64_t a0 = b0 & ~(int64_t)15, a1 = (b1 + 15) & ~(int64_t)15;
  const int n16 = (int)((a1 - a0) >> 4);
  for (int i = threadIdx.x; i < n16; i += blockDim.x) cp_async16(dst + 16 * i, base + a0 + 16 * (int64_t)i);
  return (int)(b0 - a0);
}

}  // namespace

template <int QT, bool GU, int NT>
__global__ void __launch_bounds__(kWarps * 32) expert_gemv(ExpertGemvArgs a, const int32_t* unit_off, int RT,
                                                           int raw_bytes) {
  extern __shared__ __align__(16) uint8_t smem[];
  const int G = a.K / 32;
  float* xs = reinterpret_cast<float*>(smem);                            // [NT][G][33]
  uint8_t* raw = smem + sizeof(float) * NT * G * 33;                    // [2 stages][GU ? 2 : 1][raw_bytes]
  const int ntile = a.N / RT;
  const int total = unit_off[a.E];
  const int per = (total + gridDim.x - 1) / gridDim.x;
  const int i0 = blockIdx.x * per, i1 = min(total, i0 + per);
  if (i0 >= i1) return;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nt_tensors = GU ? 2 : 1;
  const int stage_bytes = nt_tensors * raw_bytes;

  int offs[2][2];  // per stage, per tensor: the first row's offset in the staged bytes
  auto stage = [&](int i, int buf) {
    const Item it = item_of(unit_off, a.E, ntile, i);
    const int64_t r0 = (int64_t)(a.wexp ? a.wexp[it.e] : it.e) * a.N + (int64_t)it.rt * RT;
    offs[buf][0] = stage_rows(raw + buf * stage_bytes, a.w0, r0, RT, a.row_bytes);
    if (GU) offs[buf][1] = stage_rows(raw + buf * stage_bytes + raw_bytes, a.w1, r0, RT, a.row_bytes);
    cp_async_commit();
  };

  stage(i0, 0);
  int cur_e = -1, cur_tg = -1, nt = 0;
  int64_t d0 = 0;  // dispatch index of the group's first pair
  for (int i = i0; i < i1; i++) {
    const int buf = (i - i0) & 1;
    if (i + 1 < i1) {
      stage(i + 1, buf ^ 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    const Item it = item_of(unit_off, a.E, ntile, i);
    if (it.e != cur_e || it.tg != cur_tg) {  // stage this group's activations (fp32, padded)
      cur_e = it.e;
      cur_tg = it.tg;
      const int64_t o = a.offsets[it.e];
      const int64_t n_e = a.offsets[it.e + 1] - o;
      d0 = o + (int64_t)it.tg * NT;
      nt = (int)min64(NT, n_e - (int64_t)it.tg * NT);
      for (int idx = threadIdx.x; idx < nt * a.K; idx += blockDim.x) {
        const int n = idx / a.K, c = idx % a.K;
        const int64_t src_row = GU ? (int64_t)(a.perm[d0 + n] / a.k) : d0 + n;
        xs[(n * G + c / 32) * 33 + c % 32] = load_act(a.x, a.x_dtype, src_row * a.K + c);
      }
    }
    __syncthreads();
    const uint8_t* st0 = raw + buf * stage_bytes + offs[buf][0];
    const uint8_t* st1 = raw + buf * stage_bytes + raw_bytes + (GU ? offs[buf][1] : 0);
    for (int rr = warp; rr < RT; rr += kWarps) {
      float acc0[NT], acc1[NT];
#pragma unroll
      for (int n = 0; n < NT; n++) acc0[n] = acc1[n] = 0.0f;
      const uint8_t* row0 = st0 + (int64_t)rr * a.row_bytes;
      const uint8_t* row1 = st1 + (int64_t)rr * a.row_bytes;
      for (int g = lane; g < G; g += 32) {
        float w0[32];
        dq_group<QT>(row0, g, w0);
        if (GU) {
          float w1[32];
          dq_group<QT>(row1, g, w1);
#pragma unroll
          for (int n = 0; n < NT; n++) {
            if (n < nt) {
              const float* xv = xs + (n * G + g) * 33;
              float s0 = 0.0f, s1 = 0.0f;
#pragma unroll
              for (int j = 0; j < 32; j++) {
                s0 = fmaf(w0[j], xv[j], s0);
                s1 = fmaf(w1[j], xv[j], s1);
              }
              acc0[n] += s0;
              acc1[n] += s1;
            }
          }
        } else {
#pragma unroll
          for (int n = 0; n < NT; n++) {
            if (n < nt) {
              const float* xv = xs + (n * G + g) * 33;
              float s0 = 0.0f;
#pragma unroll
              for (int j = 0; j < 32; j++) s0 = fmaf(w0[j], xv[j], s0);
              acc0[n] += s0;
            }
          }
        }
      }
#pragma unroll
      for (int n = 0; n < NT; n++) {
#pragma unroll
        for (int o = 16; o; o >>= 1) {
          acc0[n] += __shfl_xor_sync(0xFFFFFFFFu, acc0[n], o);
          if (GU) acc1[n] += __shfl_xor_sync(0xFFFFFFFFu, acc1[n], o);
        }
      }
      if (lane < nt) {
        float v0 = acc0[0], v1 = acc1[0];
#pragma unroll
        for (int n = 1; n < NT; n++)
          if (lane == n) v0 = acc0[n], v1 = acc1[n];
        const int r = it.rt * RT + rr;
        a.out[(d0 + lane) * a.N + r] = GU ? __fmul_rn(silu(v0), v1) : v0;
      }
    }
    __syncthreads();  // (the next prefetch overwrites this stage)
  }
}


template <int QT, bool GU>
__global__ void __launch_bounds__(rq::kWarps * 32, 2) expert_gemv_rq(ExpertGemvArgs a, int R) {
  extern __shared__ __align__(16) float sm[];
  float* xs = sm;
  int32_t* uo = reinterpret_cast<int32_t*>(sm + rq::stage_floats(a.K));  // [E + 1]
  griddep_wait();
  griddep_launch();
  for (int i = threadIdx.x; i <= a.E; i += blockDim.x) uo[i] = a.unit_off[i];
  __syncthreads();
  const int total = uo[a.E];
  const int i0 = (int)((int64_t)blockIdx.x * total / gridDim.x), i1 = (int)((int64_t)(blockIdx.x + 1) * total / gridDim.x);
  rq::run_items<QT, GU>(a, R, uo, a.offsets, a.perm, xs, i0, i1);
}

// rows per warp of the register-decoding kernel (0: the type or shape goes to the staged kernel)
int gemv_rq_rows_per_warp(int qtype, int K, bool gu) {
  if (!(qtype == ARTLITE_Q4_0 || qtype == ARTLITE_Q8_0 || qtype == ARTLITE_Q4_K) || K % 256 || K <= 0) return 0;
  return 32 / (K / 256) / (gu ? 2 : 1);
}

namespace {

template <bool GU>
int launch_gemv(const ExpertGemvArgs& a, const int32_t* unit_off, int rt, cudaStream_t st) {
  constexpr int NT = kGemvTokens;
  const int R = gemv_rq_rows_per_warp(a.qtype, a.K, GU);
  if (R > 0 && rt == R * rq::kWarps) {
    const size_t smem = sizeof(float) * rq::stage_floats(a.K) + sizeof(int32_t) * (a.E + 1);
    int dev, sms;
    AL_CUDA(cudaGetDevice(&dev));
    AL_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    auto go = [&](auto kern) -> int {
      AL_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
      int per_sm = 0;
      AL_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, rq::kWarps * 32, smem));
      return launch_pdl(kern, dim3(std::max(1, per_sm) * sms), dim3(rq::kWarps * 32), smem, st, a, R);
    };
    if (a.qtype == ARTLITE_Q4_0) return go(expert_gemv_rq<ARTLITE_Q4_0, GU>);
    if (a.qtype == ARTLITE_Q8_0) return go(expert_gemv_rq<ARTLITE_Q8_0, GU>);
    return go(expert_gemv_rq<ARTLITE_Q4_K, GU>);
  }
  int per, bytes;
  AL_TRY(qtype_block(a.qtype, &per, &bytes));
  AL_CHECK(a.K % 32 == 0 && a.K % per == 0 && a.N % rt == 0, ARTLITE_EUNSUPPORTED, "expert gemv: K %d N %d RT %d",
           a.K, a.N, rt);
  const int raw_bytes = (int)(((int64_t)rt * a.row_bytes + 32 + 15) & ~15);
  const size_t smem = sizeof(float) * NT * (a.K / 32) * 33 + 2 * (GU ? 2 : 1) * (size_t)raw_bytes;
  AL_CHECK(smem <= 227 * 1024, ARTLITE_EUNSUPPORTED, "expert gemv: %zu B of shared memory (K %d, RT %d)", smem, a.K, rt);
  int dev, sms;
  AL_CUDA(cudaGetDevice(&dev));
  AL_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  const int grid = sms;
  auto go = [&](auto kern) -> int {
    AL_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    kern<<<grid, kWarps * 32, smem, st>>>(a, unit_off, rt, raw_bytes);
    AL_LAUNCHED();
    return ARTLITE_OK;
  };
  switch (a.qtype) {
    case ARTLITE_Q4_0: return go(expert_gemv<ARTLITE_Q4_0, GU, NT>);
    case ARTLITE_Q4_1: return go(expert_gemv<ARTLITE_Q4_1, GU, NT>);
    case ARTLITE_Q8_0: return go(expert_gemv<ARTLITE_Q8_0, GU, NT>);
    case ARTLITE_Q4_K: return go(expert_gemv<ARTLITE_Q4_K, GU, NT>);
    case ARTLITE_Q5_K: return go(expert_gemv<ARTLITE_Q5_K, GU, NT>);
    case ARTLITE_Q6_K: return go(expert_gemv<ARTLITE_Q6_K, GU, NT>);
    case ARTLITE_Q3_K: return go(expert_gemv<ARTLITE_Q3_K, GU, NT>);
    case ARTLITE_IQ4_NL: return go(expert_gemv<ARTLITE_IQ4_NL, GU, NT>);
    case ARTLITE_IQ4_XS: return go(expert_gemv<ARTLITE_IQ4_XS, GU, NT>);
    case ARTLITE_F32: return go(expert_gemv<ARTLITE_F32, GU, NT>);
    case ARTLITE_F16: return go(expert_gemv<ARTLITE_F16, GU, NT>);
    case ARTLITE_BF16: return go(expert_gemv<ARTLITE_BF16, GU, NT>);
    default: break;
  }
  set_error("expert gemv: GGUF type %d", a.qtype);
  return ARTLITE_EUNSUPPORTED;
}

}  // namespace

int gemv_row_tile(int qtype, int K, int N, bool gu) {
  const int R = gemv_rq_rows_per_warp(qtype, K, gu);
  if (R > 0) return R * rq::kWarps;
  for (int rt : {16, 8})
    if (N % rt == 0) return rt;
  return 0;
}

int launch_gemv_gu(const ExpertGemvArgs& a, cudaStream_t st) {
  return launch_gemv<true>(a, a.unit_off, a.rt, st);
}
int launch_gemv_down(const ExpertGemvArgs& a, cudaStream_t st) {
  return launch_gemv<false>(a, a.unit_off, a.rt, st);
}

}  // namespace artlite
