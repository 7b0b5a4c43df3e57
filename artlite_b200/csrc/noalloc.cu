// artlite_moe_dispatch_noalloc: the expert dispatch (histogram / scan / stable permute, dispatch.cu) with its scratch
// in this file's static device array instead of memory the library allocates.
//
// Who needs it: callers that must not allocate device memory once they run. A serving loop that reserves its whole
// memory budget at start-up and forbids allocation per request; code whose device memory belongs to a framework's
// caching allocator (PyTorch's and the like), where a raw cudaMalloc bypasses the framework's accounting and limits
// and a cudaFree stalls the whole device until it drains. artlite_moe_dispatch cannot serve them: it grows device
// buffers on demand and stages host arrays through them.
//
// The scratch: kNoAllocScratchBytes (1 MiB + the status word) in g_noalloc_scratch, which every GPU that loads this
// library holds until the process exits. It takes a block count per 4096 pairs per expert, so a call needs
// ceil(n k / 4096) x E <= kNoAllocMaxCounts; larger calls are rejected with ARTLITE_EINVAL and a message. Every call
// shares the array and it keeps the last call's contents: the status word is cleared at the start of each call and
// the counts are overwritten in full, but two calls that overlap on the GPU (other streams, other host threads, other
// handles) race on it.
#include <cuda_runtime.h>

#include <chrono>
#include <mutex>
#include <thread>

#include "common.cuh"
#include "kernels.cuh"

namespace artlite {
namespace {

constexpr int64_t kNoAllocMaxCounts = 262144;  // int32 block counts: 1 MiB
constexpr size_t kNoAllocScratchBytes = sizeof(int32_t) * kNoAllocMaxCounts + 256;

// [0, 256): the status word (DevStatus); [256, ...): the per-block counts
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
void* g_addr[kMaxDevices] = {};  // the array's device address, per device (set up once, the device current)

int scratch_address(int dev, uint8_t** out) {
  AL_CHECK(dev >= 0 && dev < kMaxDevices, ARTLITE_EUNSUPPORTED, "dispatch_noalloc: device %d (at most %d)", dev,
           kMaxDevices);
  std::lock_guard<std::mutex> lock(g_mu);
  if (!g_addr[dev]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    AL_CHECK(e == cudaSuccess && p, ARTLITE_ECUDA, "dispatch_noalloc: cudaGetSymbolAddress on device %d: %s", dev,
             cudaGetErrorString(e));
    g_addr[dev] = p;
  }
  *out = static_cast<uint8_t*>(g_addr[dev]);
  return ARTLITE_OK;
}

// device memory of device `dev` (not host, pinned, managed or another GPU's memory: the kernels would fault on a
// buffer of another device without peer access, and host memory is not reachable at these addresses)
bool on_device(const void* p, int dev) {
  cudaPointerAttributes at;
  if (cudaPointerGetAttributes(&at, p) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  return at.type == cudaMemoryTypeDevice && at.device == dev;
}

}  // namespace
}  // namespace artlite

using namespace artlite;

extern "C" {
#pragma GCC visibility push(default)

int artlite_moe_dispatch_noalloc(const int32_t* ids, int64_t n, int k, int E, int64_t* offsets, int32_t* perm,
                                 int32_t* slot, void* stream) {
  AL_CHECK(n >= 0 && k >= 1 && E >= 1, ARTLITE_EINVAL, "dispatch_noalloc: n %lld k %d E %d", (long long)n, k, E);
  AL_CHECK(E <= 1024, ARTLITE_EUNSUPPORTED, "dispatch_noalloc: E %d (this build: E <= 1024)", E);
  // (the pair count is bounded before it is formed: n k must not wrap)
  AL_CHECK(n <= kNoAllocMaxCounts * (int64_t)kDispatchBlockPairs / k, ARTLITE_EINVAL,
           "dispatch_noalloc: %lld tokens x %d slots exceed the static scratch (at most %lld pairs)", (long long)n, k,
           (long long)(kNoAllocMaxCounts / E * kDispatchBlockPairs));
  const int64_t P = n * k;
  const int64_t nblk = P ? cdiv(P, kDispatchBlockPairs) : 0;
  AL_CHECK(nblk * E <= kNoAllocMaxCounts, ARTLITE_EINVAL,
           "dispatch_noalloc: %lld pairs of %d experts need %lld block counts; the static scratch holds %lld (at most "
           "%lld pairs at this E)", (long long)P, E, (long long)(nblk * E), (long long)kNoAllocMaxCounts,
           (long long)(kNoAllocMaxCounts / E * kDispatchBlockPairs));
  int dev;
  AL_CUDA(cudaGetDevice(&dev));
  AL_CHECK(offsets && on_device(offsets, dev) && (P == 0 || (ids && perm && slot && on_device(ids, dev) &&
                                                              on_device(perm, dev) && on_device(slot, dev))),
           ARTLITE_EINVAL, "dispatch_noalloc: ids / offsets / perm / slot must be device memory of the current device");
  uint8_t* scratch;
  AL_TRY(scratch_address(dev, &scratch));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  DevStatus* status = reinterpret_cast<DevStatus*>(scratch);
  AL_CUDA(cudaMemsetAsync(status, 0, sizeof(DevStatus), st));
  DispatchArgs d{};
  d.ids = ids;
  d.P = P;
  d.E = E;
  d.blk_counts = reinterpret_cast<int32_t*>(scratch + 256);
  d.offsets = offsets;
  d.perm = perm;
  d.slot = slot;
  d.status = status;
  AL_TRY(launch_dispatch(d, st));
  // the call returns when its kernels are done: the stream is polled against a deadline, and the status word is read
  // only once the stream is idle (a copy that has nothing to wait for)
  const auto t0 = std::chrono::steady_clock::now();
  for (;;) {
    const cudaError_t q = cudaStreamQuery(st);
    if (q == cudaSuccess) break;
    AL_CHECK(q == cudaErrorNotReady, ARTLITE_ECUDA, "dispatch_noalloc: %s", cudaGetErrorString(q));
    AL_CHECK(std::chrono::steady_clock::now() - t0 < std::chrono::seconds(60), ARTLITE_ETIMEOUT,
             "dispatch_noalloc: no completion within 60 s");
    std::this_thread::yield();
  }
  DevStatus s{};
  AL_CUDA(cudaMemcpy(&s, status, sizeof s, cudaMemcpyDeviceToHost));
  AL_CHECK(s.code != ARTLITE_EDEVICE, ARTLITE_EINVAL, "dispatch_noalloc: expert id %d of %d", s.a, E);
  AL_CHECK(s.code == 0, s.code, "dispatch_noalloc: device status %d", s.code);
  return ARTLITE_OK;
}

}  // extern "C"
