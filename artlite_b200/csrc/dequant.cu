// Row dequant on the GPU (the drop-in artlite_dequant_rows, csrc/artlite/dequant.h:13-16): one thread per 32 values,
// the exact fp32 decode of quant.cuh.
#include <string.h>

#include "common.cuh"
#include "kernels.cuh"
#include "quant.cuh"

namespace artlite {

namespace {
struct Named {
  const char* name;
  int qtype;
};
constexpr Named kNames[] = {{"F32", ARTLITE_F32},   {"F16", ARTLITE_F16},   {"BF16", ARTLITE_BF16},
                            {"Q4_0", ARTLITE_Q4_0}, {"Q4_1", ARTLITE_Q4_1}, {"Q8_0", ARTLITE_Q8_0},
                            {"Q4_K", ARTLITE_Q4_K}, {"Q5_K", ARTLITE_Q5_K}, {"Q6_K", ARTLITE_Q6_K},
                            {"Q3_K", ARTLITE_Q3_K}, {"IQ4_NL", ARTLITE_IQ4_NL}, {"IQ4_XS", ARTLITE_IQ4_XS}};
}  // namespace

int qtype_from_name(const char* name) {
  if (!name) return -1;
  for (const Named& n : kNames)
    if (!strcmp(n.name, name)) return n.qtype;
  return -1;
}

const char* qtype_name(int qtype) {
  for (const Named& n : kNames)
    if (n.qtype == qtype) return n.name;
  return "?";
}

int qtype_block(int qtype, int* per, int* bytes) {
  *per = q_per(qtype);
  *bytes = q_bytes(qtype);
  AL_CHECK(*per > 0, ARTLITE_EUNSUPPORTED, "GGUF type %d is not read by this build", qtype);
  return ARTLITE_OK;
}

template <int QT>
__global__ void dequant_rows_kernel(const uint8_t* raw, int64_t n, int64_t row_bytes, int64_t cols, float* out) {
  const int64_t groups = cols / 32;
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n * groups) return;
  const int64_t r = i / groups, g = i % groups;
  float v[32];
  dq_group<QT>(raw + r * row_bytes, (int)g, v);
  float4* o = reinterpret_cast<float4*>(out + r * cols + 32 * g);
#pragma unroll
  for (int j = 0; j < 8; j++) o[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
}

// plain types with cols not a multiple of 32: one thread per value
template <int QT>
__global__ void dequant_plain_kernel(const uint8_t* raw, int64_t n, int64_t row_bytes, int64_t cols, float* out) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n * cols) return;
  const int64_t r = i / cols, c = i % cols;
  const uint8_t* p = raw + r * row_bytes + c * q_bytes(QT);
  float v;
  if constexpr (QT == ARTLITE_F32) v = __uint_as_float((uint32_t)(p[0] | (p[1] << 8) | (p[2] << 16) | ((uint32_t)p[3] << 24)));
  else if constexpr (QT == ARTLITE_F16) v = f16_at(p);
  else v = __uint_as_float((uint32_t)(p[0] | (p[1] << 8)) << 16);
  out[i] = v;
}

int launch_dequant_rows(int qtype, const uint8_t* raw, int64_t n, int64_t row_bytes, int64_t cols, float* out,
                        cudaStream_t st) {
  int per, bytes;
  AL_TRY(qtype_block(qtype, &per, &bytes));
  AL_CHECK(cols % per == 0 && cols / per * bytes <= row_bytes, ARTLITE_EINVAL,
           "dequant_rows: %lld columns of rows of %lld B", (long long)cols, (long long)row_bytes);
  if (n == 0 || cols == 0) return ARTLITE_OK;
  const bool plain = per == 1;
  // (raw and out are the library's own aligned staging buffers or 16-byte aligned device pointers: the C ABI layer
  // stages anything else)
  const bool plain_aligned = plain && (cols % 32 == 0) && (row_bytes % 4 == 0) && qtype == ARTLITE_F32;
  if (plain && !plain_aligned) {
    const unsigned grid = (unsigned)cdiv(n * cols, 256);
    if (qtype == ARTLITE_F32) dequant_plain_kernel<ARTLITE_F32><<<grid, 256, 0, st>>>(raw, n, row_bytes, cols, out);
    else if (qtype == ARTLITE_F16) dequant_plain_kernel<ARTLITE_F16><<<grid, 256, 0, st>>>(raw, n, row_bytes, cols, out);
    else dequant_plain_kernel<ARTLITE_BF16><<<grid, 256, 0, st>>>(raw, n, row_bytes, cols, out);
    AL_LAUNCHED();
    return ARTLITE_OK;
  }
  const unsigned grid = (unsigned)cdiv(n * (cols / 32), 128);
  switch (qtype) {
    case ARTLITE_Q4_0: dequant_rows_kernel<ARTLITE_Q4_0><<<grid, 128, 0, st>>>(raw, n, row_bytes, cols, out); break;
    case ARTLITE_Q4_1: dequant_rows_kernel<ARTLITE_Q4_1><<<grid, 128, 0, st>>>(raw, n, row_bytes, cols, out); break;
    case ARTLITE_Q8_0: dequant_rows_kernel<ARTLITE_Q8_0><<<grid, 128, 0, st>>>(raw, n, row_bytes, cols, out); break;
    case ARTLITE_Q4_K: dequant_rows_kernel<ARTLITE_Q4_K><<<grid, 128, 0, st>>>(raw, n, row_bytes, cols, out); break;
    case ARTLITE_Q5_K: dequant_rows_kernel<ARTLITE_Q5_K><<<grid, 128, 0, st>>>(raw, n, row_bytes, cols, out); break;
    case ARTLITE_Q6_K: dequant_rows_kernel<ARTLITE_Q6_K><<<grid, 128, 0, st>>>(raw, n, row_bytes, cols, out); break;
    case ARTLITE_Q3_K: dequant_rows_kernel<ARTLITE_Q3_K><<<grid, 128, 0, st>>>(raw, n, row_bytes, cols, out); break;
    case ARTLITE_IQ4_NL: dequant_rows_kernel<ARTLITE_IQ4_NL><<<grid, 128, 0, st>>>(raw, n, row_bytes, cols, out); break;
    case ARTLITE_IQ4_XS: dequant_rows_kernel<ARTLITE_IQ4_XS><<<grid, 128, 0, st>>>(raw, n, row_bytes, cols, out); break;
    default: dequant_rows_kernel<ARTLITE_F32><<<grid, 128, 0, st>>>(raw, n, row_bytes, cols, out); break;
  }
  AL_LAUNCHED();
  return ARTLITE_OK;
}

}  // namespace artlite
