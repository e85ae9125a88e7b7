// Cluster-free NTT for N = 2^16 as two passes over a 256 x 256 view (the "four-step" order of the same
// butterflies): word n = 256 i + j is row i, column j.
//
//   forward  pass A (columns): rounds 0..7 pair rows i, i + 2^(7-l) of one column with the root
//            tw[2^l + (i >> (8 - l))]: the same 255 roots for every column;
//            pass B (rows):    rounds 8..15 pair words j, j + 2^(15-l) of one row with tw[2^l + (256 i + j) >> (16 - l)].
//   inverse  pass B' (rows, rounds 15..8), then pass A' (columns, rounds 7..0) with the final scale.
//
// These are exactly the rounds, pairs and roots of ntt_forward_body / ntt_inverse_body (ntt.cuh), so the results
// are word for word the same; only the schedule differs.  Each pass is its own launch of 16 CTAs per polynomial
// (256 threads, 16 columns or 16 rows of 256 words, 32 KB of shared memory, three CTAs per SM), with no
// cluster: an 8-CTA cluster of the one-launch NTT cannot tile a GPC's SMs and leaves about a tenth of the B200's
// CTA slots idle, and it needs two cluster-wide barriers plus four shared-memory passes where this needs two or
// three block barriers per pass.  The price is one extra round trip of the polynomial between the passes, written
// to an "intermediate" buffer (the pass-A output, in place where the kernel allows) that the second launch reads;
// the kernels are bound by the integer multiply pipe with HBM at 10-20%, so that traffic is cheap.
//
// A thread holds 16 words of one column (or row) in registers for four rounds (radix 16), exchanges them through
// shared memory once, and does the other four rounds; loads and stores are 16 consecutive words per half-warp.
// Load functors see every word once (ld.load(ls, n)) and store functors every final word (st.store(ss, n, v)),
// in coalesced order, as in ntt.cuh.
#pragma once
#include "ntt.cuh"

namespace holmes {

struct Ntt16 {
  static constexpr int THREADS = 256;
  static constexpr int CTAS = 16;          // per polynomial and pass
  static constexpr int SMEM = 4096 * 8;    // 16 x 256 words
#ifndef HOLMES_NTT16_MINB
#define HOLMES_NTT16_MINB 3
#endif
  static constexpr int MINB = HOLMES_NTT16_MINB;  // resident CTAs per SM asked of the register allocator (3: 80 registers)
};

// tile index of (row-in-tile r, word w < 256) for the row passes: the low 4 bits of w are XORed with its bits 4..7
__device__ __forceinline__ int rsw(int r, int w) { return (r << 8) | (w ^ ((w >> 4) & 15)); }

// ---- forward pass A: columns 16 cb .. +15 of polynomial p; ld -> inter (lazy values below 8q)
template <class LD>
__device__ __forceinline__ void fwd16_cols(int p, int cb, int mi, const NttTables& T, const LD& ld, u64* inter) {
  __shared__ __align__(16) u64 sh[4096];  // [256 rows][16 columns]
  const Mod md = T.mod[mi];
  const u64 q = md.q, q4 = q << 2;
  const Tw* __restrict__ tw = T.tw + ((size_t)mi << 16);
  const int t = threadIdx.x, c = t & 15, col = (cb << 4) | c;
  u64 x[16];
  {
    const auto ls = ld.prep(p);
    const int i0 = t >> 4;
#pragma unroll
    for (int k = 0; k < 16; ++k) x[k] = ld.load(ls, ((i0 + 16 * k) << 8) | col);
    // rounds 0..3: rows i0 + 16 k, pairs k, k + (8 >> l), root tw[2^l + (k >> (4 - l))]
#pragma unroll
    for (int l = 0; l < 4; ++l) {
      const int h = 8 >> l;
#pragma unroll
      for (int k = 0; k < 16; ++k) {
        if (k & h) continue;
        bf_fwd(x[k], x[k + h], tw[(1 << l) + (k >> (4 - l))], q, q4);
      }
    }
#pragma unroll
    for (int k = 0; k < 16; ++k) sh[((i0 + 16 * k) << 4) | c] = x[k];
  }
  __syncthreads();
  const int i1 = t >> 4;
#pragma unroll
  for (int k = 0; k < 16; ++k) x[k] = sh[((16 * i1 + k) << 4) | c];
  // rounds 4..7: rows 16 i1 + k, pairs k, k + (1 << (7 - l)), root tw[2^l + (i1 << (l - 4)) + (k >> (8 - l))]
#pragma unroll
  for (int l = 4; l < 8; ++l) {
    const int h = 1 << (7 - l);
    const Tw* tr = tw + (1 << l) + (i1 << (l - 4));
#pragma unroll
    for (int k = 0; k < 16; ++k) {
      if (k & h) continue;
      bf_fwd(x[k], x[k + h], tr[k >> (8 - l)], q, q4);
    }
  }
#pragma unroll
  for (int k = 0; k < 16; ++k) inter[((16 * i1 + k) << 8) | col] = x[k];
}

// ---- forward pass B: rows 16 rb .. +15 of polynomial p; inter -> st (canonical words)
template <class ST>
__device__ __forceinline__ void fwd16_rows(int p, int rb, int mi, const NttTables& T, const u64* inter,
                                           const ST& st) {
  __shared__ __align__(16) u64 sh[4096];  // [16 rows][256 words], swizzled
  const Mod md = T.mod[mi];
  const u64 q = md.q, q4 = q << 2;
  const Tw* __restrict__ tw = T.tw + ((size_t)mi << 16);
  const int t = threadIdx.x, r = t >> 4, s = t & 15, row = (rb << 4) | r;
  const u64* src = inter + ((size_t)row << 8);
  u64 x[16];
#pragma unroll
  for (int k = 0; k < 16; ++k) x[k] = src[s + 16 * k];
  // rounds 8..11: words s + 16 k, pairs k, k + (8 >> (l - 8)), root tw[2^l + (row << (l - 8)) + (k >> (12 - l))]
#pragma unroll
  for (int l = 8; l < 12; ++l) {
    const int h = 8 >> (l - 8);
    const Tw* tr = tw + (1 << l) + (row << (l - 8));
#pragma unroll
    for (int k = 0; k < 16; ++k) {
      if (k & h) continue;
      bf_fwd(x[k], x[k + h], tr[k >> (12 - l)], q, q4);
    }
  }
#pragma unroll
  for (int k = 0; k < 16; ++k) sh[rsw(r, s + 16 * k)] = x[k];
  __syncthreads();
#pragma unroll
  for (int k = 0; k < 16; ++k) x[k] = sh[rsw(r, 16 * s + k)];
  // rounds 12..15: words 16 s + k, pairs k, k + (8 >> (l - 12)),
  // root tw[2^l + (row << (l - 8)) + (s << (l - 12)) + (k >> (16 - l))]
#pragma unroll
  for (int l = 12; l < 16; ++l) {
    const int h = 8 >> (l - 12);
    const Tw* tr = tw + (1 << l) + (row << (l - 8)) + (s << (l - 12));
#pragma unroll
    for (int k = 0; k < 16; ++k) {
      if (k & h) continue;
      bf_fwd(x[k], x[k + h], tr[k >> (16 - l)], q, q4);
    }
  }
  // back through shared memory so the stores run along the row
  __syncthreads();
#pragma unroll
  for (int k = 0; k < 16; ++k) sh[rsw(r, 16 * s + k)] = x[k];
  __syncthreads();
  const auto ss = st.prep(p);
#pragma unroll
  for (int k = 0; k < 16; ++k) {
    const int w = s + 16 * k;
    st.store(ss, (row << 8) | w, canon8(sh[rsw(r, w)], q));
  }
}

// ---- inverse pass B': rows 16 rb .. +15; ld -> inter (values below 4q)
template <class LD>
__device__ __forceinline__ void inv16_rows(int p, int rb, int mi, const NttTables& T, const LD& ld, u64* inter) {
  __shared__ __align__(16) u64 sh[4096];
  const Mod md = T.mod[mi];
  const u64 q = md.q, q4 = q << 2;
  const Tw* __restrict__ tw = T.tw + ((size_t)mi << 16);
  const int t = threadIdx.x, r = t >> 4, s = t & 15, row = (rb << 4) | r;
  u64 x[16];
  {
    const auto ls = ld.prep(p);
#pragma unroll
    for (int k = 0; k < 16; ++k) {
      const int w = s + 16 * k;
      sh[rsw(r, w)] = ld.load(ls, (row << 8) | w);
    }
  }
  __syncthreads();
#pragma unroll
  for (int k = 0; k < 16; ++k) x[k] = sh[rsw(r, 16 * s + k)];
  // rounds 15..12 on words 16 s + k
#pragma unroll
  for (int l = 15; l >= 12; --l) {
    const int h = 8 >> (l - 12);
    const Tw* tr = tw + (1 << l) + (row << (l - 8)) + (s << (l - 12));
#pragma unroll
    for (int k = 0; k < 16; ++k) {
      if (k & h) continue;
      bf_inv(x[k], x[k + h], tr[k >> (16 - l)], q, q4);
    }
  }
  __syncthreads();
#pragma unroll
  for (int k = 0; k < 16; ++k) sh[rsw(r, 16 * s + k)] = x[k];
  __syncthreads();
#pragma unroll
  for (int k = 0; k < 16; ++k) x[k] = sh[rsw(r, s + 16 * k)];
  // rounds 11..8 on words s + 16 k
#pragma unroll
  for (int l = 11; l >= 8; --l) {
    const int h = 8 >> (l - 8);
    const Tw* tr = tw + (1 << l) + (row << (l - 8));
#pragma unroll
    for (int k = 0; k < 16; ++k) {
      if (k & h) continue;
      bf_inv(x[k], x[k + h], tr[k >> (12 - l)], q, q4);
    }
  }
  u64* dst = inter + ((size_t)row << 8);
#pragma unroll
  for (int k = 0; k < 16; ++k) dst[s + 16 * k] = x[k];
}

// ---- inverse pass A': columns 16 cb .. +15; inter -> scale -> st (canonical words)
template <class ST>
__device__ __forceinline__ void inv16_cols(int p, int cb, int mi, Tw scale, const NttTables& T, const u64* inter,
                                           const ST& st) {
  __shared__ __align__(16) u64 sh[4096];
  const Mod md = T.mod[mi];
  const u64 q = md.q, q4 = q << 2;
  const Tw* __restrict__ tw = T.tw + ((size_t)mi << 16);
  const int t = threadIdx.x, c = t & 15, col = (cb << 4) | c;
  const int i1 = t >> 4;
  u64 x[16];
#pragma unroll
  for (int k = 0; k < 16; ++k) x[k] = inter[((16 * i1 + k) << 8) | col];
  // rounds 7..4 on rows 16 i1 + k
#pragma unroll
  for (int l = 7; l >= 4; --l) {
    const int h = 1 << (7 - l);
    const Tw* tr = tw + (1 << l) + (i1 << (l - 4));
#pragma unroll
    for (int k = 0; k < 16; ++k) {
      if (k & h) continue;
      bf_inv(x[k], x[k + h], tr[k >> (8 - l)], q, q4);
    }
  }
#pragma unroll
  for (int k = 0; k < 16; ++k) sh[((16 * i1 + k) << 4) | c] = x[k];
  __syncthreads();
  const int i0 = t >> 4;
#pragma unroll
  for (int k = 0; k < 16; ++k) x[k] = sh[((i0 + 16 * k) << 4) | c];
  // rounds 3..0 on rows i0 + 16 k
#pragma unroll
  for (int l = 3; l >= 0; --l) {
    const int h = 8 >> l;
#pragma unroll
    for (int k = 0; k < 16; ++k) {
      if (k & h) continue;
      bf_inv(x[k], x[k + h], tw[(1 << l) + (k >> (4 - l))], q, q4);
    }
  }
  const auto ss = st.prep(p);
#pragma unroll
  for (int k = 0; k < 16; ++k) st.store(ss, ((i0 + 16 * k) << 8) | col, canon2(shoup_lazy(x[k], scale, q), q));
}

// Launch of one pass: grid = polys * 16 CTAs (block b: polynomial b / 16, column or row block b % 16), no cluster.
template <class K, class... Args>
inline cudaError_t launch_ntt16(K kernel, int polys, cudaStream_t st, Args... args) {
  if (polys <= 0) return cudaSuccess;
  count_launch();
  kernel<<<(unsigned)(polys * Ntt16::CTAS), Ntt16::THREADS, 0, st>>>(args...);
  return cudaGetLastError();
}

}  // namespace holmes
