// The C ABI (include/artlite_moe.h): argument checks with the reference's error cases and messages, host / device
// pointer staging, the block handle and its forward.
#include <cuda_runtime.h>
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <atomic>
#include <chrono>
#include <mutex>
#include <thread>
#include <string>
#include <vector>

#include <cstdlib>

#include "common.cuh"
#include "kernels.cuh"

namespace artlite {

static thread_local std::string g_error;

void set_error(const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  g_error = buf;
}

std::string& last_error() { return g_error; }

static std::atomic<int64_t> g_launches{0};
int64_t launch_count() { return g_launches.load(); }
void count_launch(int n) { g_launches += n; }

bool pdl_enabled() {
  static const bool on = [] {
    const char* v = getenv("ARTLITE_PDL");
    return !(v && v[0] == '0');
  }();
  return on;
}

bool is_device_ptr(const void* p) {
  if (!p) return false;
  cudaPointerAttributes at;
  if (cudaPointerGetAttributes(&at, p) != cudaSuccess) {
    cudaGetLastError();  // (clear: an unknown host pointer on older runtimes)
    return false;
  }
  return at.type == cudaMemoryTypeDevice || at.type == cudaMemoryTypeManaged;
}

int DevBuf::reserve(size_t n) {
  if (n <= bytes && ptr) return ARTLITE_OK;
  release();
  const size_t want = n ? ((n + 255) & ~(size_t)255) : 256;
  AL_CUDA(cudaMalloc(&ptr, want));
  bytes = want;
  return ARTLITE_OK;
}

void DevBuf::release() {
  if (ptr) cudaFree(ptr);
  ptr = nullptr;
  bytes = 0;
}

namespace {

// An argument buffer: used in place when it is device memory aligned to `align`, else staged in a device buffer.
struct Arg {
  explicit Arg(DevBuf& b) : buf(b) {}
  void* dev = nullptr;
  const void* user = nullptr;
  size_t bytes = 0;
  bool staged = false;
  DevBuf& buf;
  int in(const void* p, size_t n, cudaStream_t st, size_t align = 16, bool force_stage = false) {
    user = p;
    bytes = n;
    if (!force_stage && p && is_device_ptr(p) && ((uintptr_t)p % align) == 0) {
      dev = const_cast<void*>(p);
      return ARTLITE_OK;
    }
    staged = true;
    AL_TRY(buf.reserve(n + 16));
    dev = buf.ptr;
    if (n && p) AL_CUDA(cudaMemcpyAsync(dev, p, n, cudaMemcpyDefault, st));
    return ARTLITE_OK;
  }
  int out(void* p, size_t n, size_t align = 16) {
    user = p;
    bytes = n;
    if (p && is_device_ptr(p) && ((uintptr_t)p % align) == 0) {
      dev = p;
      return ARTLITE_OK;
    }
    staged = true;
    AL_TRY(buf.reserve(n + 16));
    dev = buf.ptr;
    return ARTLITE_OK;
  }
  int back(cudaStream_t st) {
    if (staged && bytes && user) AL_CUDA(cudaMemcpyAsync(const_cast<void*>(user), dev, bytes, cudaMemcpyDefault, st));
    return ARTLITE_OK;
  }
  template <class T>
  T* as() const { return static_cast<T*>(dev); }
};

// a bounded wait for a stream (cudaStreamQuery polling with a deadline)
int wait_stream(cudaStream_t st, int timeout_ms) {
  if (timeout_ms <= 0) timeout_ms = 60000;
  const auto t0 = std::chrono::steady_clock::now();
  for (;;) {
    const cudaError_t e = cudaStreamQuery(st);
    if (e == cudaSuccess) return ARTLITE_OK;
    if (e != cudaErrorNotReady) {
      set_error("stream: %s", cudaGetErrorString(e));
      return ARTLITE_ECUDA;
    }
    if (std::chrono::steady_clock::now() - t0 > std::chrono::milliseconds(timeout_ms)) {
      set_error("stream wait: no completion within %d ms", timeout_ms);
      return ARTLITE_ETIMEOUT;
    }
    std::this_thread::yield();
  }
}

// the per-thread stream and status word of the drop-in entry points
struct Scratch {
  int dev = -1;
  cudaStream_t st = nullptr;
  DevBuf status, blk, offsets, perm, slot, counts, chunk_off, ids;
  DevBuf stage[6];  // argument staging (Arg)
  int init() {
    int d;
    AL_CUDA(cudaGetDevice(&d));
    if (st && d == dev) return ARTLITE_OK;
    if (st) {
      cudaStreamDestroy(st);
      status.release(); blk.release(); offsets.release(); perm.release(); slot.release(); counts.release();
      chunk_off.release(); ids.release();
      for (DevBuf& b : stage) b.release();
    }
    dev = d;
    AL_CUDA(cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking));
    AL_TRY(status.reserve(sizeof(DevStatus)));
    return ARTLITE_OK;
  }
  int read_status(DevStatus* s) {
    AL_CUDA(cudaMemcpyAsync(s, status.ptr, sizeof(DevStatus), cudaMemcpyDeviceToHost, st));
    AL_TRY(wait_stream(st, 0));
    return ARTLITE_OK;
  }
};

thread_local Scratch g_scratch;

int plan_status(const DevStatus& s, int E, int cap) {
  if (s.code == ARTLITE_EDEVICE) {
    set_error("moe_plan: expert id %d of %d", s.a, E);
    return ARTLITE_EINVAL;
  }
  if (s.code == ARTLITE_ECAPACITY) {
    set_error("moe_plan: more than %d chunks in a column", cap);
    return ARTLITE_ECAPACITY;
  }
  if (s.code) {
    set_error("device status %d (%d %d %d)", s.code, s.a, s.b, s.c);
    return s.code;
  }
  return ARTLITE_OK;
}

// the dispatch of P pairs' ids (device) into the scratch's offsets / perm / slot / counts (+ chunk scan)
int run_dispatch(Scratch& S, const int32_t* ids, int64_t P, int E, int chunk) {
  AL_TRY(S.blk.reserve(dispatch_scratch_bytes(P, E)));
  AL_TRY(S.offsets.reserve(sizeof(int64_t) * (E + 1)));
  AL_TRY(S.perm.reserve(sizeof(int32_t) * (P + 1)));
  AL_TRY(S.slot.reserve(sizeof(int32_t) * (P + 1)));
  AL_TRY(S.counts.reserve(sizeof(int32_t) * E));
  AL_TRY(S.chunk_off.reserve(sizeof(int32_t) * (E + 1)));
  AL_CUDA(cudaMemsetAsync(S.status.ptr, 0, sizeof(DevStatus), S.st));
  DispatchArgs d{};
  d.ids = ids;
  d.P = P;
  d.E = E;
  d.blk_counts = S.blk.as<int32_t>();
  d.offsets = S.offsets.as<int64_t>();
  d.perm = S.perm.as<int32_t>();
  d.slot = S.slot.as<int32_t>();
  d.counts = S.counts.as<int32_t>();
  d.unit_rows = chunk;
  d.unit_mult = 1;
  d.unit_off = chunk > 0 ? S.chunk_off.as<int32_t>() : nullptr;
  d.status = S.status.as<DevStatus>();
  return launch_dispatch(d, S.st);
}

}  // namespace
}  // namespace artlite

using namespace artlite;

extern "C" {
#pragma GCC visibility push(default)

const char* artlite_moe_last_error(void) { return g_error.c_str(); }

const char* artlite_moe_version(void) { return "artlite-b200-moe 0.1 (sm_100a)"; }

int artlite_moe_route(const float* logits, int64_t n, int64_t row, int per_col, int64_t pitch, int E, int k,
                      int sigmoid, int32_t* ids, float* weights) {
  AL_TRY(check_route_args(n, per_col, E, k));
  if (n == 0) return ARTLITE_OK;
  AL_CHECK(logits && ids && weights, ARTLITE_EINVAL, "moe_route: null array");
  Scratch& S = g_scratch;
  AL_TRY(S.init());
  const int64_t nl = (n - 1) * row + (int64_t)(E / per_col - 1) * pitch + per_col;
  Arg lg(S.stage[0]), oi(S.stage[1]), ow(S.stage[2]);
  AL_TRY(lg.in(logits, sizeof(float) * nl, S.st, 4));
  AL_TRY(oi.out(ids, sizeof(int32_t) * n * k, 4));
  AL_TRY(ow.out(weights, sizeof(float) * n * k, 4));
  RouteArgs a{lg.as<float>(), n, row, per_col, pitch, E, k, sigmoid != 0,
              k <= 16 && per_col % 16 == 0 && E % per_col == 0 && E <= 512, oi.as<int32_t>(), ow.as<float>()};
  AL_TRY(launch_route(a, S.st));
  AL_TRY(oi.back(S.st));
  AL_TRY(ow.back(S.st));
  return wait_stream(S.st, 0);
}

int artlite_moe_dispatch(const int32_t* ids, int64_t n, int k, int E, int64_t* offsets, int32_t* perm,
                         int32_t* slot) {
  AL_CHECK(n >= 0 && k >= 1 && E >= 1, ARTLITE_EINVAL, "moe_dispatch: n %lld k %d E %d", (long long)n, k, E);
  AL_CHECK(E <= 1024, ARTLITE_EUNSUPPORTED, "moe_dispatch: E %d (this build: E <= 1024)", E);
  AL_CHECK(offsets && (n == 0 || (ids && perm && slot)), ARTLITE_EINVAL, "moe_dispatch: null array");
  Scratch& S = g_scratch;
  AL_TRY(S.init());
  const int64_t P = n * k;
  Arg ai(S.stage[0]);
  AL_TRY(ai.in(ids, sizeof(int32_t) * P, S.st, 4));
  AL_TRY(run_dispatch(S, ai.as<int32_t>(), P, E, 0));
  AL_CUDA(cudaMemcpyAsync(offsets, S.offsets.ptr, sizeof(int64_t) * (E + 1), cudaMemcpyDefault, S.st));
  if (P) {
    AL_CUDA(cudaMemcpyAsync(perm, S.perm.ptr, sizeof(int32_t) * P, cudaMemcpyDefault, S.st));
    AL_CUDA(cudaMemcpyAsync(slot, S.slot.ptr, sizeof(int32_t) * P, cudaMemcpyDefault, S.st));
  }
  DevStatus s;
  AL_TRY(S.read_status(&s));
  return plan_status(s, E, 0);
}

int artlite_moe_plan(const int32_t* ids, int64_t n, int k, int E, int cols, int cap, int chunk, int32_t* experts,
                     int32_t* counts, int32_t* sizes, int32_t* rows, int64_t* pos) {
  AL_CHECK(n >= 0 && k >= 1 && E >= 1 && cols >= 1 && cap >= 0 && chunk >= 1, ARTLITE_EINVAL,
           "moe_plan: n %lld k %d E %d cols %d cap %d chunk %d", (long long)n, k, E, cols, cap, chunk);
  AL_CHECK(E <= 1024, ARTLITE_EUNSUPPORTED, "moe_plan: E %d (this build: E <= 1024)", E);
  AL_CHECK(counts && (n == 0 || (ids && experts && sizes && rows && pos)), ARTLITE_EINVAL, "moe_plan: null array");
  Scratch& S = g_scratch;
  AL_TRY(S.init());
  const int64_t P = n * k;
  Arg ai(S.stage[0]), ae(S.stage[1]), ac(S.stage[2]), as(S.stage[3]), ar(S.stage[4]), ap(S.stage[5]);
  AL_TRY(ai.in(ids, sizeof(int32_t) * P, S.st, 4));
  AL_TRY(ae.out(experts, sizeof(int32_t) * cols * cap, 4));
  AL_TRY(ac.out(counts, sizeof(int32_t) * cols, 4));
  AL_TRY(as.out(sizes, sizeof(int32_t) * cols * cap, 4));
  AL_TRY(ar.out(rows, sizeof(int32_t) * (int64_t)cols * cap * chunk, 4));
  AL_TRY(ap.out(pos, sizeof(int64_t) * P, 8));
  AL_TRY(run_dispatch(S, ai.as<int32_t>(), P, E, chunk));
  ChunkPlanArgs c{ai.as<int32_t>(), S.slot.as<int32_t>(), S.perm.as<int32_t>(), S.offsets.as<int64_t>(),
                  S.chunk_off.as<int32_t>(), P, k, E, cols, cap, chunk, ae.as<int32_t>(), ac.as<int32_t>(),
                  as.as<int32_t>(), ar.as<int32_t>(), ap.as<int64_t>(), S.status.as<DevStatus>()};
  AL_TRY(launch_chunk_plan(c, S.st));
  for (Arg* a : {&ae, &ac, &as, &ar, &ap}) AL_TRY(a->back(S.st));
  DevStatus s;
  AL_TRY(S.read_status(&s));
  return plan_status(s, E, cap);
}

int artlite_dequant_supported(const char* qtype) { return qtype_from_name(qtype) >= 0 ? 1 : 0; }

int artlite_dequant_rows(const char* qtype, const uint8_t* raw, int64_t n, int64_t row_bytes, int64_t cols,
                         float* out) {
  const int qt = qtype_from_name(qtype);
  AL_CHECK(qt >= 0, ARTLITE_EINVAL, "dequant_rows: no native %s", qtype ? qtype : "(null)");
  int per, bytes;
  AL_TRY(qtype_block(qt, &per, &bytes));
  AL_CHECK(n >= 0 && cols >= 0 && cols % per == 0 && cols / per * bytes <= row_bytes, ARTLITE_EINVAL,
           "dequant_rows: %lld columns of rows of %lld B", (long long)cols, (long long)row_bytes);
  if (n == 0 || cols == 0) return ARTLITE_OK;
  Scratch& S = g_scratch;
  AL_TRY(S.init());
  Arg ar(S.stage[0]), ao(S.stage[1]);
  // (the block decoders read fp32 planes 4-aligned and write float4: stage anything less aligned)
  AL_TRY(ar.in(raw, (size_t)(n * row_bytes), S.st, 16, row_bytes % 16 != 0));
  AL_TRY(ao.out(out, sizeof(float) * n * cols, 16));
  AL_TRY(launch_dequant_rows(qt, ar.as<uint8_t>(), n, row_bytes, cols, ao.as<float>(), S.st));
  AL_TRY(ao.back(S.st));
  return wait_stream(S.st, 0);
}

}  // extern "C"
