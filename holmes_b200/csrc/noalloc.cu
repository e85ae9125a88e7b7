// holmes_rescale_noalloc: rescale with library-owned scratch, for callers that cannot allocate.
//
// holmes_rescale needs comps * N words of device scratch for the inverse NTT of the dropped limb, and
// expects the caller to pass them in.  Some callers cannot produce such a buffer on demand: a host runtime
// that owns the whole device memory pool and forbids allocations outside it (a serving engine that
// reserves HBM up front), or a latency-critical loop where cudaMalloc / cudaFree would synchronise the
// device and stall every other stream.  This entry point takes the scratch from a fixed array compiled
// into the library instead, so a call allocates nothing.
//
// The array is a file-scope __device__ variable of kNoallocScratchWords words (2 MiB).  Every GPU that
// loads the library holds those 2 MiB until the process exits.  A kernel cannot be handed the host-side
// name of the array (that is only a host stand-in for the symbol), so the first call on each device, with
// that device current, looks up its device address with cudaGetSymbolAddress and caches it; that first
// call should therefore happen before any stream capture.  The cached address assumes one primary-context
// lifetime per device and process: after cudaDeviceReset the array lives at an address this cache does not
// know, so the library must not be called again in that process.  All calls share the one array: two calls that
// overlap on the GPU (different streams, no ordering between them) race on it.  The inverse NTT writes
// every scratch word it later reads, so stale contents from an earlier call are never used and nothing
// needs clearing.
#include <mutex>

#include "../../include/holmes_cuda.h"
#include "ops.h"

constexpr size_t kNoallocScratchWords = (size_t)4 << 16;  // four 2^16-word polynomials
static __device__ __align__(256) holmes::u64 g_noalloc_scratch[kNoallocScratchWords];

namespace {

constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mutex;
holmes::u64* g_noalloc_ptr[kMaxDevices] = {};

// Device address of the scratch array on the current device (looked up once per device).
int noalloc_scratch(holmes::u64** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return (int)e;
  if (dev < 0 || dev >= kMaxDevices) return -8;
  std::lock_guard<std::mutex> lock(g_noalloc_mutex);
  if (!g_noalloc_ptr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return (int)e;
    g_noalloc_ptr[dev] = (holmes::u64*)p;
  }
  *out = g_noalloc_ptr[dev];
  return 0;
}

}  // namespace

extern "C" int holmes_rescale_noalloc(void* ctx, const uint64_t* in, long long in_stride, uint64_t* out,
                                      long long out_stride, int cur, int comps, void* stream) {
  if (!ctx || !in || !out || comps < 1) return -1;
  const holmes::HolmesCtx& c = *(const holmes::HolmesCtx*)ctx;
  if ((size_t)comps * (size_t)c.n > kNoallocScratchWords) return -6;  // more than the fixed scratch holds
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return (int)e;
  if (dev != c.device) return -7;  // the context's tables live on another device
  holmes::u64* scratch = nullptr;
  const int rc = noalloc_scratch(&scratch);
  if (rc) return rc;
  return holmes::rescale(c, in, in_stride, out, out_stride, cur, comps, scratch, (cudaStream_t)stream);
}
