// Batched negacyclic NTT / inverse NTT for 64-bit RNS limbs, one thread-block cluster per polynomial.
//
// Convention (the reference's, bench/cmp/kernels/holmes_encode.cu:65-71): forward round l pairs
// words n and n + 2^(logN-1-l) with root tw[2^l + (n >> (logN-l))], tw[k] = psi^bitrev(k); the
// inverse runs the Gentleman-Sande rounds in reverse with psi^-bitrev(k) and a final N^-1.
//
// B200 layout.  A polynomial of N = 2^16 words is 512 KB, more than one CTA's shared memory, so a
// cluster of CL = N / 8192 CTAs holds it: CTA r keeps the contiguous segment [r S, (r+1) S),
// S = 8192 words = 64 KB (three CTAs per SM).  The first log2(CL) forward rounds pair words of
// different segments; they run as one register-resident radix-CL pass over "columns" (the CL words
// j, S + j, 2S + j, ...) straight from global memory, and the results are scattered into the owners'
// shared memory through distributed shared memory.  The remaining log2(S) rounds are local
// radix-16 / radix-8 passes through shared memory.  The inverse mirrors this: local passes, then the
// cross-segment column pass gathers through DSMEM, applies N^-1 and writes global memory.  HBM sees
// one read and one write of every word.  For N <= 8192 a single CTA holds the polynomial.
//
// Fusion points.  A Load functor produces word n of polynomial p (`ld.load(ld.prep(p), n)`, called once
// per word, in coalesced order) and a Store functor consumes the final canonical word
// (`st.store(st.prep(p), n, v)`); `prep` hoists the per-polynomial constants into registers.  So
// base conversions, inner products, automorphisms and rescale arithmetic run inside the NTT kernel
// instead of in separate passes over HBM.
#pragma once
#include <cooperative_groups.h>

#include "common.cuh"

// Two 512-thread CTAs per SM (64 registers each, a few spilled words) measured 20-37% faster than one
// CTA per SM with no spills across the NTT kernel family at N = 2^16.
#ifndef HOLMES_NTT_MINB
#define HOLMES_NTT_MINB 2
#endif

namespace holmes {
namespace cg = cooperative_groups;

template <int LOGN>
struct NttGeom {
  static constexpr int N = 1 << LOGN;
  static constexpr int LOGCL = LOGN > 13 ? LOGN - 13 : 0;
  static constexpr int CL = 1 << LOGCL;
  static constexpr int LOGS = LOGN - LOGCL;
  static constexpr int S = 1 << LOGS;
  static constexpr int THREADS = (S / 16) < 32 ? 32 : (S / 16);
  static constexpr int SMEM = S * 8;
  // resident 512-thread CTAs per SM asked of the register allocator (2: 64 registers per thread)
  static constexpr int MINB = HOLMES_NTT_MINB;
};

#define HOLMES_NTT_BOUNDS(LOGN) __launch_bounds__(NttGeom<LOGN>::THREADS, NttGeom<LOGN>::MINB)

// XOR swizzle of the low 4 bits by bits 4..7: every radix-16 / radix-8 access pattern of a warp
// touches 16 distinct 8-byte bank pairs per half-warp.
__device__ __forceinline__ int swz(int x) { return x ^ ((x >> 4) & 15); }

// Per-launch constants shared by every NTT kernel.
struct NttTables {
  const Tw* tw;   // [T][N] forward (psi^bitrev) or inverse (psi^-bitrev) twiddles
  const Mod* mod; // [T]
};

// ---------------------------------------------------------------------------------------------------------
// butterflies
// Butterflies on lazy values below 8q (forward) / 4q (inverse) with the three-product Shoup estimate
// (shoup_lazy4, common.cuh): its quotient is at most 2 short, so the product lies in [0, 4q), and one
// conditional subtraction of 4q per butterfly keeps the bounds (8q < 2^63 for q < 2^60).
__device__ __forceinline__ void bf_fwd(u64& x, u64& y, Tw t, u64 q, u64 q4) {
  if (x >= q4) x -= q4;
  const u64 v = shoup_lazy4(y, t, q);
  y = x + q4 - v;
  x = x + v;
}
__device__ __forceinline__ void bf_inv(u64& x, u64& y, Tw t, u64 q, u64 q4) {
  u64 u = x + y;
  if (u >= q4) u -= q4;
  const u64 d = x + q4 - y;
  y = shoup_lazy4(d, t, q);
  x = u;
}
__device__ __forceinline__ u64 canon8(u64 x, u64 q) {
  if (x >= (q << 2)) x -= (q << 2);
  if (x >= (q << 1)) x -= (q << 1);
  if (x >= q) x -= q;
  return x;
}
__device__ __forceinline__ u64 canon2(u64 x, u64 q) { return x >= q ? x - q : x; }

// ---------------------------------------------------------------------------------------------------------
// One local pass of R rounds starting at global round L0 over this CTA's segment (global word offset
// seg0).  Group gid covers the 2^R words base + (k << s), s = LOGN - L0 - R.  For round L0 + r the root
// index 2^(L0+r) + (n >> (LOGN-L0-r)) of word k is (B0 << r) + (k >> (R - r)) with
// B0 = 2^L0 + ((seg0 + base) >> (s + R)): the 2^r roots of a round are contiguous.
template <int LOGN, int R, bool INV, int L0>
__device__ __forceinline__ void local_pass(u64* sh, int seg0, const Tw* __restrict__ tw, u64 q) {
  using G = NttGeom<LOGN>;
  constexpr int M = 1 << R;
  constexpr int GROUPS = G::S >> R;
  constexpr int s = LOGN - L0 - R;
  const u64 q4 = q << 2;
  for (int gid = threadIdx.x; gid < GROUPS; gid += G::THREADS) {
    const int lo = gid & ((1 << s) - 1);
    const int base = lo | ((gid >> s) << (s + R));
    const int b0 = (1 << L0) + (seg0 >> (s + R)) + (gid >> s);
    u64 x[M];
#pragma unroll
    for (int k = 0; k < M; ++k) x[k] = sh[swz(base + (k << s))];
    if constexpr (!INV) {
#pragma unroll
      for (int r = 0; r < R; ++r) {
        const int h = M >> (r + 1);
        const Tw* tr = tw + (b0 << r);
#pragma unroll
        for (int k = 0; k < M; ++k) {
          if (k & h) continue;
          bf_fwd(x[k], x[k + h], tr[k >> (R - r)], q, q4);
        }
      }
    } else {
#pragma unroll
      for (int r = R - 1; r >= 0; --r) {
        const int h = M >> (r + 1);
        const Tw* tr = tw + (b0 << r);
#pragma unroll
        for (int k = 0; k < M; ++k) {
          if (k & h) continue;
          bf_inv(x[k], x[k + h], tr[k >> (R - r)], q, q4);
        }
      }
    }
#pragma unroll
    for (int k = 0; k < M; ++k) sh[swz(base + (k << s))] = x[k];
  }
  __syncthreads();
}

// Pass schedule for the local rounds: radix-16 passes, the remainder as radix-8 passes.
struct PassSched {
  int n;
  int r[8];
  int off[8];
};
__host__ __device__ constexpr PassSched make_sched(int rt, int first) {
  PassSched p{0, {0, 0, 0, 0, 0, 0, 0, 0}, {0, 0, 0, 0, 0, 0, 0, 0}};
  const int n4 = rt / 4, rem = rt % 4;
  int sizes[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  int c = 0;
  if (rem == 0) { for (int i = 0; i < n4; ++i) sizes[c++] = 4; }
  else if (rem == 3) { for (int i = 0; i < n4; ++i) sizes[c++] = 4; sizes[c++] = 3; }
  else if (rem == 2) { for (int i = 0; i < n4 - 1; ++i) sizes[c++] = 4; sizes[c++] = 3; sizes[c++] = 3; }
  else { for (int i = 0; i < n4 - 2; ++i) sizes[c++] = 4; sizes[c++] = 3; sizes[c++] = 3; sizes[c++] = 3; }
  int l0 = first;
  for (int i = 0; i < c; ++i) { p.r[i] = sizes[i]; p.off[i] = l0; l0 += sizes[i]; }
  p.n = c;
  return p;
}

template <int LOGN, bool INV, int I>
__device__ __forceinline__ void run_passes(u64* sh, int seg0, const Tw* __restrict__ tw, u64 q) {
  using G = NttGeom<LOGN>;
  constexpr PassSched sc = make_sched(G::LOGS, G::LOGCL);
  if constexpr (!INV) {
    if constexpr (I < sc.n) {
      local_pass<LOGN, sc.r[I], false, sc.off[I]>(sh, seg0, tw, q);
      run_passes<LOGN, false, I + 1>(sh, seg0, tw, q);
    }
  } else {
    if constexpr (I >= 0) {
      local_pass<LOGN, sc.r[I], true, sc.off[I]>(sh, seg0, tw, q);
      run_passes<LOGN, true, I - 1>(sh, seg0, tw, q);
    }
  }
}

template <int LOGN, bool INV>
__device__ __forceinline__ void local_rounds(u64* sh, int seg0, const Tw* __restrict__ tw, u64 q) {
  using G = NttGeom<LOGN>;
  constexpr PassSched sc = make_sched(G::LOGS, G::LOGCL);
  if constexpr (!INV) run_passes<LOGN, false, 0>(sh, seg0, tw, q);
  else run_passes<LOGN, true, sc.n - 1>(sh, seg0, tw, q);
}

// ---------------------------------------------------------------------------------------------------------
// Forward NTT of polynomial `poly` with modulus index `mi`.  Block layout: blockIdx.x = poly * CL + rank.
template <int LOGN, class LD, class ST>
__device__ __forceinline__ void ntt_forward_body(int poly, int mi, const NttTables& T, const LD& ld, const ST& st) {
  using G = NttGeom<LOGN>;
  extern __shared__ u64 sh[];
  const Mod m = T.mod[mi];
  const u64 q = m.q;
  const Tw* __restrict__ tw = T.tw + (size_t)mi * G::N;
  const auto ls = ld.prep(poly);
  int rank = 0;
  if constexpr (G::CL > 1) {
    cg::cluster_group cluster = cg::this_cluster();
    rank = (int)cluster.block_rank();
    // every CTA of the cluster must be running before its shared memory is written remotely
    cluster.sync();
    // cross-segment rounds 0 .. LOGCL-1 on columns j in [rank S/CL, (rank+1) S/CL)
    constexpr int COLS = G::S / G::CL;
    const u64 q4 = q << 2;
    // the cross rounds use only the CL - 1 twiddles tw[1 .. CL-1]
    Tw ct[G::CL];
#pragma unroll
    for (int i = 1; i < G::CL; ++i) ct[i] = tw[i];
    for (int c = threadIdx.x; c < COLS; c += G::THREADS) {
      const int j = rank * COLS + c;
      u64 x[G::CL];
#pragma unroll
      for (int r = 0; r < G::CL; ++r) x[r] = ld.load(ls, r * G::S + j);
#pragma unroll
      for (int l = 0; l < G::LOGCL; ++l) {
        const int h = G::CL >> (l + 1);
#pragma unroll
        for (int r = 0; r < G::CL; ++r) {
          if (r & h) continue;
          bf_fwd(x[r], x[r + h], ct[(1 << l) + (r >> (G::LOGCL - l))], q, q4);
        }
      }
      // scatter: word r S + j belongs to CTA r, local index j
#pragma unroll
      for (int r = 0; r < G::CL; ++r) {
        u64* dst = cluster.map_shared_rank(sh, r);
        dst[swz(j)] = x[r];
      }
    }
    cluster.sync();
  } else {
    for (int i = threadIdx.x; i < G::S; i += G::THREADS) sh[swz(i)] = ld.load(ls, i);
    __syncthreads();
  }
  const int seg0 = rank * G::S;
  local_rounds<LOGN, false>(sh, seg0, tw, q);
  const auto ss = st.prep(poly);
  for (int i = threadIdx.x; i < G::S; i += G::THREADS) st.store(ss, seg0 + i, canon8(sh[swz(i)], q));
}

// Inverse NTT; `scale` is the final per-polynomial multiplier (N^-1, or N^-1 times a constant).
template <int LOGN, class LD, class ST>
__device__ __forceinline__ void ntt_inverse_body(int poly, int mi, Tw scale, const NttTables& T, const LD& ld,
                                                 const ST& st) {
  using G = NttGeom<LOGN>;
  extern __shared__ u64 sh[];
  const Mod m = T.mod[mi];
  const u64 q = m.q;
  const Tw* __restrict__ tw = T.tw + (size_t)mi * G::N;
  int rank = 0;
  if constexpr (G::CL > 1) rank = (int)cg::this_cluster().block_rank();
  const int seg0 = rank * G::S;
  {
    const auto ls = ld.prep(poly);
    for (int i = threadIdx.x; i < G::S; i += G::THREADS) sh[swz(i)] = ld.load(ls, seg0 + i);
  }
  __syncthreads();
  local_rounds<LOGN, true>(sh, seg0, tw, q);
  const auto ss = st.prep(poly);
  if constexpr (G::CL > 1) {
    cg::cluster_group cluster = cg::this_cluster();
    cluster.sync();
    constexpr int COLS = G::S / G::CL;
    const u64 q4 = q << 2;
    Tw ct[G::CL];
#pragma unroll
    for (int i = 1; i < G::CL; ++i) ct[i] = tw[i];
    for (int c = threadIdx.x; c < COLS; c += G::THREADS) {
      const int j = rank * COLS + c;
      u64 x[G::CL];
#pragma unroll
      for (int r = 0; r < G::CL; ++r) x[r] = cluster.map_shared_rank(sh, r)[swz(j)];
#pragma unroll
      for (int l = G::LOGCL - 1; l >= 0; --l) {
        const int h = G::CL >> (l + 1);
#pragma unroll
        for (int r = 0; r < G::CL; ++r) {
          if (r & h) continue;
          bf_inv(x[r], x[r + h], ct[(1 << l) + (r >> (G::LOGCL - l))], q, q4);
        }
      }
#pragma unroll
      for (int r = 0; r < G::CL; ++r) st.store(ss, r * G::S + j, canon2(shoup_lazy(x[r], scale, q), q));
    }
    // keep every CTA's shared memory alive until all remote reads of it are done
    cluster.sync();
  } else {
    for (int i = threadIdx.x; i < G::S; i += G::THREADS) st.store(ss, i, canon2(shoup_lazy(sh[swz(i)], scale, q), q));
  }
}

// ---------------------------------------------------------------------------------------------------------
// Launch helper: grid = polys * CL CTAs, cluster (CL, 1, 1), S * 8 bytes of dynamic shared memory.
template <class K, class... Args>
inline cudaError_t launch_ntt(K kernel, int logn_cl, int threads, int smem, int polys, cudaStream_t st,
                              Args... args) {
  if (polys <= 0) return cudaSuccess;
  cudaError_t e = set_smem_once((const void*)kernel, smem);
  if (e != cudaSuccess) return e;
  const int cl = 1 << logn_cl;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(polys * cl), 1, 1);
  cfg.blockDim = dim3((unsigned)threads, 1, 1);
  cfg.dynamicSmemBytes = (size_t)smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = (unsigned)cl;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  count_launch();
  return cudaLaunchKernelEx(&cfg, kernel, args...);
}

}  // namespace holmes
