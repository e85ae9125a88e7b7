// Modular reduce-scatter over peer memory (one process per GPU, CUDA IPC mappings, plain loads and stores).
//
// Each rank holds its partial sums of every item in one buffer that the other ranks have mapped with
// cudaIpcOpenMemHandle (opened by the READING process with its own device current, so the mapping belongs to the
// device whose kernels read it).  The owner of an item range sums every rank's partials of that range modulo q:
// the NCCL sum is not a modular sum, and this replaces an all-to-all of raw limbs plus a second pass over HBM.
//
// Ordering is carried by 64-bit epoch flags in each rank's flag block (flag 0: "my partials of this epoch are
// written"; flag 2 + s: "rank s has finished reading my partials of this epoch"), written with release stores at
// system scope after a system fence and read with acquire loads.  Every wait is bounded by a clock64 budget: a wait
// that runs out writes the index of the flag it gave up on (plus one) into a device status word and returns, and the
// summing kernel does nothing when the status is set, so a missing peer turns into an error the host reads rather
// than a hung GPU.  Only plain loads and stores touch peer memory here.
#include <cuda_runtime.h>

#include <cstring>

#include "../../include/holmes_cuda.h"
#include "ops.h"

namespace holmes {

namespace {

__device__ __forceinline__ u64 ld_acquire_sys(const u64* p) {
  u64 v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys(u64* p, u64 v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

constexpr int kMaxPeers = 16;

inline unsigned peer_grid(size_t work, int threads) {
  const size_t blocks = (work + threads - 1) / threads;
  return (unsigned)(blocks < 148 * 8 ? (blocks ? blocks : 1) : 148 * 8);
}
struct FlagPtrs {
  u64* p[kMaxPeers];
};
struct PeerSrcs {
  const u64* p[kMaxPeers];
};

// one thread per flag: store the epoch after every earlier write of this stream is visible system-wide
__global__ void k_peer_signal(FlagPtrs f, int count, u64 epoch) {
  const int i = threadIdx.x;
  if (i < count) {
    __threadfence_system();
    st_release_sys(f.p[i], epoch);
  }
}

// one thread per flag: spin until flag >= epoch or the cycle budget runs out (then status = index + 1)
__global__ void k_peer_wait(FlagPtrs f, int count, u64 epoch, long long budget, int* status) {
  const int i = threadIdx.x;
  if (i >= count) return;
  const long long start = clock64();
  while (ld_acquire_sys(f.p[i]) < epoch) {
    if (clock64() - start > budget) {
      atomicCAS(status, 0, i + 1);
      return;
    }
    __nanosleep(256);
  }
}

// out = sum_r src_r mod q over [items][limbs][N] (item stride item_stride in every source and in out), skipped when
// a wait before it gave up
__global__ void k_peer_modsum(PeerSrcs s, int nsrc, u64* __restrict__ out, int items, int limbs, long long item_stride,
                              int log_n, const Mod* __restrict__ mods, const int* __restrict__ status) {
  if (*(volatile const int*)status) return;
  const size_t per_item = (size_t)limbs << log_n;
  const size_t total = (size_t)items * per_item / 2;
  for (size_t t = blockIdx.x * (size_t)blockDim.x + threadIdx.x; t < total; t += (size_t)gridDim.x * blockDim.x) {
    const size_t w = 2 * t;
    const unsigned wl = (unsigned)(w >> log_n);
    const int item = (int)(wl / (unsigned)limbs), limb = (int)(wl - (unsigned)item * limbs);
    const size_t off = item * item_stride + ((size_t)limb << log_n) + (w & (((size_t)1 << log_n) - 1));
    const u64 q = mods[limb].q;
    u64 a = 0, b = 0;
    for (int k = 0; k < nsrc; ++k) {
      const ulonglong2 x = *reinterpret_cast<const ulonglong2*>(s.p[k] + off);
      a = add_mod(a, x.x, q);
      b = add_mod(b, x.y, q);
    }
    *reinterpret_cast<ulonglong2*>(out + off) = make_ulonglong2(a, b);
  }
}

}  // namespace
}  // namespace holmes

using namespace holmes;

extern "C" {

int holmes_peer_alloc(unsigned long long bytes, void** ptr_out) {
  if (!ptr_out || bytes == 0) return -1;
  cudaError_t e = cudaMalloc(ptr_out, (size_t)bytes);
  if (e == cudaSuccess) e = cudaMemset(*ptr_out, 0, (size_t)bytes);
  return (int)e;
}

int holmes_peer_free(void* ptr) {
  if (!ptr) return -1;
  return (int)cudaFree(ptr);
}

int holmes_ipc_export(const void* dev_ptr, void* handle_out) {
  if (!dev_ptr || !handle_out) return -1;
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, const_cast<void*>(dev_ptr));
  if (e != cudaSuccess) return (int)e;
  memcpy(handle_out, &h, sizeof(h));
  return 0;
}

int holmes_ipc_import(const void* handle, void** ptr_out) {
  if (!handle || !ptr_out) return -1;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  return (int)cudaIpcOpenMemHandle(ptr_out, h, cudaIpcMemLazyEnablePeerAccess);
}

int holmes_ipc_close(void* ptr) {
  if (!ptr) return -1;
  return (int)cudaIpcCloseMemHandle(ptr);
}

int holmes_peer_signal(uint64_t* const* flags, int count, uint64_t epoch, void* stream) {
  if (!flags || count < 1 || count > kMaxPeers) return -1;
  FlagPtrs f{};
  for (int i = 0; i < count; ++i) {
    if (!flags[i]) return -1;
    f.p[i] = flags[i];
  }
  count_launch();
  k_peer_signal<<<1, 32, 0, (cudaStream_t)stream>>>(f, count, epoch);
  return (int)cudaGetLastError();
}

int holmes_peer_wait(const uint64_t* const* flags, int count, uint64_t epoch, long long budget_cycles, int* status,
                     void* stream) {
  if (!flags || !status || count < 1 || count > kMaxPeers || budget_cycles < 1) return -1;
  FlagPtrs f{};
  for (int i = 0; i < count; ++i) {
    if (!flags[i]) return -1;
    f.p[i] = const_cast<u64*>(flags[i]);
  }
  count_launch();
  k_peer_wait<<<1, 32, 0, (cudaStream_t)stream>>>(f, count, epoch, budget_cycles, status);
  return (int)cudaGetLastError();
}

int holmes_modreduce_scatter(void* ctx, const uint64_t* const* srcs, int nsrc, uint64_t* out, int items, int limbs,
                             long long item_stride, const int* status, void* stream) {
  if (!ctx || !srcs || !out || !status || nsrc < 1 || nsrc > kMaxPeers) return -1;
  const HolmesCtx& c = *(const HolmesCtx*)ctx;
  if (items < 1 || limbs < 1 || limbs > c.L || item_stride < (long long)limbs * c.n) return -2;
  PeerSrcs s{};
  for (int k = 0; k < nsrc; ++k) {
    if (!srcs[k]) return -1;
    s.p[k] = srcs[k];
  }
  const size_t work = ((size_t)items * limbs * c.n) / 2;
  count_launch();
  k_peer_modsum<<<peer_grid(work, 256), 256, 0, (cudaStream_t)stream>>>(s, nsrc, out, items, limbs, item_stride,
                                                                        c.log_n, c.d_mod, status);
  return (int)cudaGetLastError();
}

}  // extern "C"
