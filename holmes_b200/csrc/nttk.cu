// NTT-family kernels: every operation whose cost is dominated by a forward or inverse NTT, with its
// elementwise pre- and post-processing fused into the NTT's global loads and stores.
//
//   plain NTT / iNTT              batched [items][limbs][N]
//   ModUp                         iNTT(c1) * N^-1 (Q_j/q_k)^-1  ->  per digit: base conversion of
//                                 every target limb (k_conv, which also writes the digit's own limbs),
//                                 then their forward NTTs in place.  A digit's Q rows carry the factor
//                                 P^-1 mod q_i of the later ModDown (own limbs: c1 * P^-1; converted
//                                 limbs: constants (Q_j/q_k) P^-1 mod q_i), so it is paid once per ModUp
//                                 rather than once per key switch of a hoisted set
//   key switch (hybrid, ModDown)  inner products of every Q and P limb, both components, digits through the
//                                 automorphism, addends folded in (k_ks_inner, elementwise); P limbs: iNTT
//                                 with N^-1 (P/p_k)^-1; base conversion P->q_i with constants p_k^-1 mod q_i
//                                 (k_conv); Q limbs: NTT with "out -= conversion" fused into its store
//   The base conversions run as their own elementwise pass: one thread keeps a coefficient's source
//   words in registers for every target limb, where the NTT's load phase (fused before) recomputed its
//   splits per target and stalled on 8 scattered loads per word with few registers to spare.
//   rescale                       iNTT of the last limb; centred reduction fused into the NTT of the
//                                 other limbs, (c - v) q_last^-1 fused into its store
//   encode                        llround(v * scale) and the signed reduction fused into the NTT load
//   decrypt, keygen, encrypt      c0 + c1 s / CBD error sampling fused into the NTT load; the key /
//                                 ciphertext assembly fused into the store
#include <map>
#include <mutex>
#include <tuple>

#include "ntt.cuh"
#include "ntt16.cuh"
#include "ops.h"
#include "sampler.cuh"

namespace holmes {

constexpr int MAXA = 24;  // largest digit width (alpha) and special-limb count K supported

#define HOLMES_LOGN_SWITCH(logn, MACRO) \
  switch (logn) {                       \
    case 10: MACRO(10);                 \
    case 11: MACRO(11);                 \
    case 12: MACRO(12);                 \
    case 13: MACRO(13);                 \
    case 14: MACRO(14);                 \
    case 15: MACRO(15);                 \
    case 16: MACRO(16);                 \
    default: return -1;                 \
  }

// --------------------------------------------------------------------------------------------- functors
struct LdPlain {
  const u64* src;
  PolyMap pm;
  struct S { const u64* p; };
  __device__ S prep(int p) const { return S{src + pm.off(p)}; }
  __device__ u64 load(const S& s, int n) const { return s.p[n]; }
};
struct StPlain {
  u64* dst;
  PolyMap pm;
  struct S { u64* p; };
  __device__ S prep(int p) const { return S{dst + pm.off(p)}; }
  __device__ void store(const S& s, int n, u64 v) const { s.p[n] = v; }
};

// --------------------------------------------------------------------------------------------- N = 2^16, two passes
// The kernels below run the NTTs of N = 2^16 as two launches (ntt16.cuh); MOD maps a polynomial to its modulus
// index, SC to its final inverse scale, IM to the intermediate the first pass writes and the second reads.
struct IMRows {
  u64* base;
  __device__ u64* at(int p) const { return base + ((size_t)p << 16); }
};
struct IMPlain {
  u64* base;
  PolyMap pm;
  __device__ u64* at(int p) const { return base + pm.off(p); }
};
struct ModPlain {
  PolyMap pm;
  __device__ int operator()(int p) const { return pm.mod(p); }
};
struct ScLimb {  // scale[limb of p] or scale[modulus of p]
  const Tw* scale;
  int by_limb;
  PolyMap pm;
  __device__ Tw operator()(int p) const { return scale[by_limb ? p % pm.limbs : pm.mod(p)]; }
};
template <int MINB, class MOD, class LD, class IM>
__global__ void __launch_bounds__(Ntt16::THREADS, MINB) k16_fwd_a(NttTables T, MOD mo, LD ld, IM im) {
  const int p = blockIdx.x >> 4;
  fwd16_cols(p, blockIdx.x & 15, mo(p), T, ld, im.at(p));
}
template <int MINB, class MOD, class IM, class ST>
__global__ void __launch_bounds__(Ntt16::THREADS, MINB) k16_fwd_b(NttTables T, MOD mo, IM im, ST st) {
  const int p = blockIdx.x >> 4;
  fwd16_rows(p, blockIdx.x & 15, mo(p), T, im.at(p), st);
}
template <int MINB, class MOD, class LD, class IM>
__global__ void __launch_bounds__(Ntt16::THREADS, MINB) k16_inv_b(NttTables T, MOD mo, LD ld, IM im) {
  const int p = blockIdx.x >> 4;
  inv16_rows(p, blockIdx.x & 15, mo(p), T, ld, im.at(p));
}
template <int MINB, class MOD, class SC, class IM, class ST>
__global__ void __launch_bounds__(Ntt16::THREADS, MINB) k16_inv_a(NttTables T, MOD mo, SC sc, IM im, ST st) {
  const int p = blockIdx.x >> 4;
  inv16_cols(p, blockIdx.x & 15, mo(p), sc(p), T, im.at(p), st);
}
// forward: ld -> im (pass A), im -> st (pass B); inverse: ld -> im (pass B'), im -> scale -> st (pass A').
// MINB: resident CTAs per SM asked of the register allocator (3: 80 registers; 4: 64).
template <int MINB = Ntt16::MINB, class MOD, class LD, class IM, class ST>
static int ntt16_forward(NttTables T, MOD mo, LD ld, IM im, ST st, int polys, cudaStream_t s) {
  cudaError_t e = launch_ntt16(k16_fwd_a<MINB, MOD, LD, IM>, polys, s, T, mo, ld, im);
  if (e == cudaSuccess) e = launch_ntt16(k16_fwd_b<MINB, MOD, IM, ST>, polys, s, T, mo, im, st);
  return (int)e;
}
template <int MINB = Ntt16::MINB, class MOD, class SC, class LD, class IM, class ST>
static int ntt16_inverse(NttTables T, MOD mo, SC sc, LD ld, IM im, ST st, int polys, cudaStream_t s) {
  cudaError_t e = launch_ntt16(k16_inv_b<MINB, MOD, LD, IM>, polys, s, T, mo, ld, im);
  if (e == cudaSuccess) e = launch_ntt16(k16_inv_a<MINB, MOD, SC, IM, ST>, polys, s, T, mo, sc, im, st);
  return (int)e;
}
// resident CTAs per SM of the key switch's two-pass NTTs
#ifndef HOLMES_KS16_MINB
#define HOLMES_KS16_MINB 3
#endif

// --------------------------------------------------------------------------------------------- base conversion
// out_t[n] = sum_{a < w} y_a[n] H[a][mi(t)] mod q_mi(t) for every target t < ntgt of every item, coefficient form.
// Target t is limb r = t (t < skip_lo) or t + w (above), of modulus index mi = r (r < cur) or L + r - cur.  One
// thread reads the w source words of one coefficient once, splits them into 30-bit halves, and produces every
// target from constants pre-split in shared memory (four fused wide multiply-adds per product, w <= 16 products
// per 64-bit sum; wider digits fold once after the 16th product), then one Barrett fold per output, left lazy in
// [0, 8 q) for the forward NTT that follows.
// Used by the key switch (P -> Q) and ModUp (digit -> complement), whose NTTs then load plainly.  With `own`
// set (ModUp) the same thread also writes the skipped rows skip_lo + a: own_a * own_scale[a] mod q_(skip_lo + a).
struct ConvArgs {
  const u64* y;     // source limb a of item i at y + i * y_item + a * N
  long long y_item;
  u64* out;         // target limb r of item i at out + i * out_item + r * N
  long long out_item;
  const u64* H;     // H[a * h_row + mi]
  int h_row;
  int w, ntgt, skip_lo, cur, L, items;
  const u64* own;   // optional: row a of item i at own + i * own_item + a * N
  long long own_item;
  const Tw* own_scale;
};
// Grid (blocks, groups): block row y takes targets [y tpg, (y + 1) tpg), so a conversion of few items (one
// ciphertext: 256 blocks of coefficients) still spreads over every SM; each group re-reads its coefficients' W source
// words (from L2) and computes the same sums, so the split changes nothing in the results.
template <int W>
__global__ void __launch_bounds__(256) k_conv(ConvArgs a, int log_n, const Mod* __restrict__ mods) {
  extern __shared__ uint2 hs[];  // [targets of this group][W]: the split constant of source a for target t
  const int N = 1 << log_n;
  const int tpg = (a.ntgt + gridDim.y - 1) / gridDim.y;
  const int t0 = blockIdx.y * tpg, t1 = min(a.ntgt, t0 + tpg);
  for (int e = threadIdx.x; e < (t1 - t0) * W; e += blockDim.x) {
    const int t = t0 + e / W, k = e % W;
    const int r = t < a.skip_lo ? t : t + W;
    const int mi = r < a.cur ? r : a.L + r - a.cur;
    const u64 h = a.H[(size_t)k * a.h_row + mi];
    hs[e] = make_uint2((uint32_t)(h & ((1ull << 30) - 1)), (uint32_t)(h >> 30));
  }
  __syncthreads();
  const size_t total = (size_t)a.items << log_n;
  for (size_t g = blockIdx.x * (size_t)blockDim.x + threadIdx.x; g < total; g += (size_t)gridDim.x * blockDim.x) {
    const int item = (int)(g >> log_n);
    const int n = (int)(g & (N - 1));
    const u64* yp = a.y + item * a.y_item + n;
    uint2 ys[W];
#pragma unroll
    for (int k = 0; k < W; ++k) {
      const u64 v = yp[(size_t)k << log_n];
      ys[k] = make_uint2((uint32_t)(v & ((1ull << 30) - 1)), (uint32_t)(v >> 30));
    }
    u64* op = a.out + item * a.out_item + n;
    if (a.own && blockIdx.y == 0) {
      const u64* src = a.own + item * a.own_item + n;
#pragma unroll
      for (int k = 0; k < W; ++k) {
        const Mod& m = mods[a.skip_lo + k];
        op[(size_t)(a.skip_lo + k) << log_n] = shoup(src[(size_t)k << log_n], a.own_scale[k], m.q);
      }
    }
    for (int t = t0; t < t1; ++t) {
      const uint2* h = hs + (t - t0) * W;
      const int r = t < a.skip_lo ? t : t + W;
      const int mi = r < a.cur ? r : a.L + r - a.cur;
      Split4 s{0, 0, 0, 0};
#pragma unroll
      for (int k = 0; k < W; ++k) {
        if (k == 16) {  // 16 products of 30-bit halves fill the 64-bit sums: fold lazily and restart from the split
          const u64 v = fold_split_lazy(s, mods[mi]);
          s = Split4{v & ((1ull << 30) - 1), v >> 30, 0, 0};
        }
        const uint2 c = h[k];
        s.s00 += (u64)ys[k].x * c.x;
        s.sa += (u64)ys[k].x * c.y;
        s.sb += (u64)ys[k].y * c.x;
        s.s11 += (u64)ys[k].y * c.y;
      }
      op[(size_t)r << log_n] = fold_split_lazy(s, mods[mi]);
    }
  }
}
template <int W>
static int conv_launch_w(const HolmesCtx& c, const ConvArgs& a, cudaStream_t st) {
  const size_t work = (size_t)a.items << c.log_n;
  size_t blocks = (work + 255) / 256;
  if (blocks > 148 * 8) blocks = 148 * 8;
  // target groups: enough blocks for every SM to hold several, at least 4 targets per group
  int groups = (int)((148 * 8 + blocks - 1) / blocks);
  groups = std::max(1, std::min(groups, a.ntgt / 4));
  const int tpg = (a.ntgt + groups - 1) / groups;
  groups = (a.ntgt + tpg - 1) / tpg;
  const size_t smem = (size_t)tpg * W * sizeof(uint2);
  count_launch();
  k_conv<W><<<dim3((unsigned)blocks, (unsigned)groups), 256, smem, st>>>(a, c.log_n, c.d_mod);
  return (int)cudaGetLastError();
}
static int conv_launch(const HolmesCtx& c, const ConvArgs& a, cudaStream_t st) {
  if (a.ntgt < 1) return -3;
  switch (a.w) {
    case 1: return conv_launch_w<1>(c, a, st);
    case 2: return conv_launch_w<2>(c, a, st);
    case 3: return conv_launch_w<3>(c, a, st);
    case 4: return conv_launch_w<4>(c, a, st);
    case 5: return conv_launch_w<5>(c, a, st);
    case 6: return conv_launch_w<6>(c, a, st);
    case 7: return conv_launch_w<7>(c, a, st);
    case 8: return conv_launch_w<8>(c, a, st);
    case 9: return conv_launch_w<9>(c, a, st);
    case 10: return conv_launch_w<10>(c, a, st);
    case 11: return conv_launch_w<11>(c, a, st);
    case 12: return conv_launch_w<12>(c, a, st);
    case 13: return conv_launch_w<13>(c, a, st);
    case 14: return conv_launch_w<14>(c, a, st);
    case 15: return conv_launch_w<15>(c, a, st);
    case 16: return conv_launch_w<16>(c, a, st);
    case 17: return conv_launch_w<17>(c, a, st);
    case 18: return conv_launch_w<18>(c, a, st);
    case 19: return conv_launch_w<19>(c, a, st);
    case 20: return conv_launch_w<20>(c, a, st);
    case 21: return conv_launch_w<21>(c, a, st);
    case 22: return conv_launch_w<22>(c, a, st);
    case 23: return conv_launch_w<23>(c, a, st);
    case 24: return conv_launch_w<24>(c, a, st);
    default: return -3;
  }
}
// Plain load / in-place store of the target limbs of one ModUp digit (poly p = item * ntgt + t).
struct DigitRows {
  u64* base;
  long long item;
  int lo, w, ntgt, log_n;
  struct S { u64* p; };
  __device__ int row(int p) const {
    const int t = p % ntgt;
    return t < lo ? t : t + w;
  }
  __device__ S prep(int p) const { return S{base + (p / ntgt) * item + ((size_t)row(p) << log_n)}; }
  __device__ u64 load(const S& s, int n) const { return s.p[n]; }
  __device__ void store(const S& s, int n, u64 v) const { s.p[n] = v; }
};
struct ModDigit {
  DigitRows d;
  int cur, L;
  __device__ int operator()(int p) const {
    const int r = d.row(p);
    return r < cur ? r : L + r - cur;
  }
};
struct IMDigit {
  DigitRows d;
  __device__ u64* at(int p) const { return d.prep(p).p; }
};
template <int LOGN>
__global__ void HOLMES_NTT_BOUNDS(LOGN) k_digit_ntt(NttTables T, DigitRows d, int cur, int L) {
  const int p = blockIdx.x / NttGeom<LOGN>::CL;
  const int r = d.row(p);
  ntt_forward_body<LOGN>(p, r < cur ? r : L + r - cur, T, d, d);
}
// Plain load of the converted Q limbs of the key switch (poly p = (item * 2 + c) * cur + i).
struct LdRows {
  const u64* base;
  int log_n;
  struct S { const u64* p; };
  __device__ S prep(int p) const { return S{base + ((size_t)p << log_n)}; }
  __device__ u64 load(const S& s, int n) const { return s.p[n]; }
};

template <int LOGN>
__global__ void HOLMES_NTT_BOUNDS(LOGN) k_fwd_plain(NttTables T, PolyMap pm, LdPlain ld, StPlain st) {
  const int p = blockIdx.x / NttGeom<LOGN>::CL;
  ntt_forward_body<LOGN>(p, pm.mod(p), T, ld, st);
}
template <int LOGN>
__global__ void HOLMES_NTT_BOUNDS(LOGN) k_inv_plain(NttTables T, PolyMap pm, const Tw* scale,
                                                                       int scale_by_limb, LdPlain ld, StPlain st) {
  const int p = blockIdx.x / NttGeom<LOGN>::CL;
  const int mi = pm.mod(p);
  ntt_inverse_body<LOGN>(p, mi, scale[scale_by_limb ? p % pm.limbs : mi], T, ld, st);
}

int ntt_plain(const HolmesCtx& c, const u64* src, u64* dst, PolyMap pm, int polys, bool inverse, cudaStream_t st) {
  NttTables T{inverse ? c.d_itw : c.d_tw, c.d_mod};
  LdPlain ld{src, pm};
  StPlain sp{dst, pm};
  if (c.log_n == 16) {
    return inverse ? ntt16_inverse(T, ModPlain{pm}, ScLimb{c.d_ninv, 0, pm}, ld, IMPlain{dst, pm}, sp, polys, st)
                   : ntt16_forward(T, ModPlain{pm}, ld, IMPlain{dst, pm}, sp, polys, st);
  }
#define L_(LG)                                                                                                   \
  {                                                                                                              \
    using G = NttGeom<LG>;                                                                                       \
    return inverse ? (int)launch_ntt(k_inv_plain<LG>, G::LOGCL, G::THREADS, G::SMEM, polys, st, T, pm, c.d_ninv, \
                                     0, ld, sp)                                                                  \
                   : (int)launch_ntt(k_fwd_plain<LG>, G::LOGCL, G::THREADS, G::SMEM, polys, st, T, pm, ld, sp);  \
  }
  HOLMES_LOGN_SWITCH(c.log_n, L_)
#undef L_
}

// --------------------------------------------------------------------------------------------- ModUp
// Base conversion of one digit's scaled coefficients y_a (a < w) to modulus m: sum_a y_a hat_a mod m.
// Polynomial p of a digit launch: item p / ntgt, target limb t (the digit's own limbs skipped).
int modup(const HolmesCtx& c, const u64* c1, long long c1_item, int cur, int items, u64* digits, long long dig_item,
          u64* scratch, cudaStream_t st) {
  if (cur < 1 || cur > c.L || items < 1) return -2;
  if (c.alpha > MAXA || c.K > MAXA) return -3;
  const int N = c.n, A = c.alpha, K = c.K;
  const long long y_item = (long long)cur * N;
  // y_k = iNTT(c1_k) * N^-1 (Q_j / q_k)^-1 -> scratch [items][cur][N]
  {
    NttTables T{c.d_itw, c.d_mod};
    PolyMap pm = poly_map(cur, c1_item, N, 0);
    PolyMap ps = poly_map(cur, y_item, N, 0);
    LdPlain ld{c1, pm};
    StPlain sp{scratch, ps};
    if (c.log_n == 16) {
      const int e = ntt16_inverse(T, ModPlain{pm}, ScLimb{c.mu_scale(cur), 1, pm}, ld, IMPlain{scratch, ps}, sp,
                                  items * cur, st);
      if (e) return e;
    } else {
#define L_(LG)                                                                                                     \
  {                                                                                                                \
    using G = NttGeom<LG>;                                                                                         \
    cudaError_t e = launch_ntt(k_inv_plain<LG>, G::LOGCL, G::THREADS, G::SMEM, items * cur, st, T, pm,           \
                               c.mu_scale(cur), 1, ld, sp);                                                        \
    if (e != cudaSuccess) return (int)e;                                                                           \
    break;                                                                                                         \
  }
      HOLMES_LOGN_SWITCH(c.log_n, L_)
#undef L_
    }
  }
  const int beta = c.beta(cur);
  const size_t dstride = (size_t)(cur + K) * N;
  // The digits' chains (conversion, then NTT of its targets) are independent once the iNTT above is done: with few
  // items one chain fills a fraction of the GPU, so digit j > 0 runs on side stream (j - 1) % 3 after an event on
  // `st`, and `st` waits for every side chain before returning.
  const bool fan = beta > 1 && items <= 2 && c.log_n == 16;
  if (fan) {
    const int e = ensure_side(c);
    if (e) return e;
    HOLMES_CUDA_TRY(cudaEventRecord(c.ev[0], st));
    for (int k = 0; k < HolmesCtx::kSide && k + 1 < beta; ++k) HOLMES_CUDA_TRY(cudaStreamWaitEvent(c.side[k], c.ev[0], 0));
  }
  const cudaStream_t main_st = st;
  for (int j = 0; j < beta; ++j) {
    const int lo = j * A, w = std::min(A, cur - lo);
    u64* dj = digits + (size_t)j * dstride;
    NttTables T{c.d_tw, c.d_mod};
    const int ntgt = cur + K - w;
    st = fan && j > 0 ? c.side[(j - 1) % HolmesCtx::kSide] : main_st;
    // the digit's own limbs are the input limbs times P^-1, written by the conversion kernel
    ConvArgs ca{scratch + (size_t)lo * N, y_item, dj, dig_item, c.mu_hat(cur) + (size_t)j * A * c.T, c.T,
                w, ntgt, lo, cur, c.L, items, c1 + (size_t)lo * N, c1_item, c.d_md_pinv + lo};
    {
      const int e = conv_launch(c, ca, st);
      if (e) return e;
    }
    DigitRows dr{dj, dig_item, lo, w, ntgt, c.log_n};
    const int polys = items * ntgt;
    if (c.log_n == 16) {
      const int e = ntt16_forward(T, ModDigit{dr, cur, c.L}, dr, IMDigit{dr}, dr, polys, st);
      if (e) return e;
      continue;
    }
#define L_(LG)                                                                                                   \
  {                                                                                                              \
    using G = NttGeom<LG>;                                                                                       \
    cudaError_t e = launch_ntt(k_digit_ntt<LG>, G::LOGCL, G::THREADS, G::SMEM, polys, st, T, dr, cur, c.L);     \
    if (e != cudaSuccess) return (int)e;                                                                         \
    break;                                                                                                       \
  }
    HOLMES_LOGN_SWITCH(c.log_n, L_)
#undef L_
  }
  if (fan) {
    const int used = std::min(HolmesCtx::kSide, beta - 1);
    for (int k = 0; k < used; ++k) {
      HOLMES_CUDA_TRY(cudaEventRecord(c.ev[1 + k], c.side[k]));
      HOLMES_CUDA_TRY(cudaStreamWaitEvent(main_st, c.ev[1 + k], 0));
    }
  }
  return 0;
}

// --------------------------------------------------------------------------------------------- key switch
// Inner products, one thread per (item, limb r of Q u P, word n) and both components at once (each digit word is
// read once): acc_c = sum_j D_j[r][perm(n)] key_c[j][r'][n], r' = r (Q limb) or cap + k (special limb k = r - cur).
//   Q limbs:  out_c[r][n] = acc_c + perm(add_c)[r][n] + post_c[r][n] (mod q_r); the digits' Q rows carry P^-1,
//             so after the ModDown NTT below subtracts its conversion this is the key-switched ciphertext.
//   P limbs:  scratch[item][c][k][n] = acc_c mod p_k, the input of the ModDown inverse NTT.
// The memory-latency-bound loads run here, at full occupancy, instead of inside the NTTs' loads and stores.
struct KsInnerArgs {
  const u64* digits;
  long long dig_item;
  const u64* key;
  const u64* add0;
  const u64* add1;
  long long add_item;
  const u64* post0;
  const u64* post1;
  long long post_item;
  u64* out0;
  u64* out1;
  long long out_item;
  u64* p0;        // P limb k of component c of item i at p_c + i * p_item + k * N
  u64* p1;
  long long p_item;
  const Tw* qscale;  // optional: Q outputs times qscale[r] (P mod q_r for the extended basis)
  u64 galois;
  int cur, cap, K, L, beta, key_beta, items;
};
// grid (N / 256, rows): a thread takes word n of limb r for every item, so each key word is read (and split)
// once when beta <= MAXB (MAXB = 0: keys re-read per item, any beta); digits, addends and outputs stream per item
template <int MAXB>
__global__ void __launch_bounds__(256) k_ks_inner(KsInnerArgs a, int log_n, const Mod* __restrict__ mods) {
  constexpr int KB = MAXB > 0 ? MAXB : 1;
  const int rows = a.cur + a.K;
  const size_t dstep = (size_t)rows << log_n, kstep = (size_t)(a.cap + a.K) << log_n;
  const size_t kcomp = (size_t)a.key_beta * kstep;
  const int n = blockIdx.x * blockDim.x + threadIdx.x;
  const int r = blockIdx.y;
  const u32 src = a.galois > 1 ? automorph_src((u32)n, a.galois, log_n) : (u32)n;
  const bool qlimb = r < a.cur;
  const int kr = qlimb ? r : a.cap + (r - a.cur);
  const Mod m = mods[qlimb ? r : a.L + (r - a.cur)];
  const u64* kp = a.key + ((size_t)kr << log_n) + n;
  uint2 kb[KB], ka[KB];  // the beta key words of (r, n) per component, split into 30-bit halves
  if constexpr (MAXB > 0) {
#pragma unroll
    for (int j = 0; j < MAXB; ++j) {
      if (j < a.beta) {
        const u64 x = kp[j * kstep], y = kp[kcomp + j * kstep];
        kb[j] = make_uint2((uint32_t)x & ((1u << 30) - 1), (uint32_t)(x >> 30));
        ka[j] = make_uint2((uint32_t)y & ((1u << 30) - 1), (uint32_t)(y >> 30));
      }
    }
  }
  const size_t roff = (size_t)r << log_n;
  // Software pipeline over the items (MAXB = 2, the linear path's beta): the next item's digit words and addends are
  // loaded before this item's products and stores, so two items' loads are in flight (the stores would otherwise
  // keep the compiler from moving the loads up, the outputs not being declared distinct from the inputs).  At
  // MAXB = 5 the prefetched words would take the kernel from 70 to 110 registers, so it keeps the plain loop.
  constexpr bool PIPE = MAXB == 2;
  u64 dnext[KB];
  u64 anext0 = 0, anext1 = 0;
  auto fetch = [&](int item) {
    const u64* d = a.digits + item * a.dig_item + roff + src;
#pragma unroll
    for (int j = 0; j < KB; ++j)
      if (j < a.beta) dnext[j] = d[j * dstep];
    if (qlimb) {
      const size_t ao = item * a.add_item + roff + src;
      anext0 = a.add0 ? a.add0[ao] : 0;
      anext1 = a.add1 ? a.add1[ao] : 0;
    }
  };
  if constexpr (PIPE) fetch(0);
  for (int item = 0; item < a.items; ++item) {
    const u64* d = a.digits + item * a.dig_item + roff + src;
    Split4 s0{0, 0, 0, 0}, s1{0, 0, 0, 0};
    u64 acur0 = 0, acur1 = 0;
    if constexpr (MAXB > 0) {
      u64 dcur[KB];
      if constexpr (PIPE) {
#pragma unroll
        for (int j = 0; j < KB; ++j) dcur[j] = dnext[j];
        acur0 = anext0;
        acur1 = anext1;
        if (item + 1 < a.items) fetch(item + 1);
      }
#pragma unroll
      for (int j = 0; j < MAXB; ++j) {
        if (j < a.beta) {
          const u64 dv = PIPE ? dcur[j] : d[j * dstep];
          const uint32_t d0 = (uint32_t)dv & ((1u << 30) - 1), d1 = (uint32_t)(dv >> 30);
          s0.s00 += (u64)d0 * kb[j].x;
          s0.sa += (u64)d0 * kb[j].y;
          s0.sb += (u64)d1 * kb[j].x;
          s0.s11 += (u64)d1 * kb[j].y;
          s1.s00 += (u64)d0 * ka[j].x;
          s1.sa += (u64)d0 * ka[j].y;
          s1.sb += (u64)d1 * ka[j].x;
          s1.s11 += (u64)d1 * ka[j].y;
        }
      }
    } else {
      for (int j = 0; j < a.beta; ++j) {
        const u64 dv = d[j * dstep];
        split_mac(s0, dv, kp[j * kstep]);
        split_mac(s1, dv, kp[kcomp + j * kstep]);
      }
    }
    if (qlimb) {
      u64 u0 = fold_split(s0, m), u1 = fold_split(s1, m);
      if constexpr (PIPE) {
        if (a.add0) u0 = add_mod(u0, acur0, m.q);
        if (a.add1) u1 = add_mod(u1, acur1, m.q);
      } else {
        const size_t ao = item * a.add_item + roff;
        if (a.add0) u0 = add_mod(u0, a.add0[ao + src], m.q);
        if (a.add1) u1 = add_mod(u1, a.add1[ao + src], m.q);
      }
      const size_t po = item * a.post_item + roff + n;
      if (a.post0) u0 = add_mod(u0, a.post0[po], m.q);
      if (a.post1) u1 = add_mod(u1, a.post1[po], m.q);
      if (a.qscale) {
        u0 = shoup(u0, a.qscale[r], m.q);
        u1 = shoup(u1, a.qscale[r], m.q);
      }
      const size_t oo = item * a.out_item + roff + n;
      a.out0[oo] = u0;
      a.out1[oo] = u1;
    } else {
      const size_t po = item * a.p_item + ((size_t)(r - a.cur) << log_n) + n;
      a.p0[po] = fold_split(s0, m);
      a.p1[po] = fold_split(s1, m);
    }
  }
}
struct StScratch {
  u64* dst;
  int log_n;
  struct S { u64* p; };
  __device__ S prep(int p) const { return S{dst + ((size_t)p << log_n)}; }
  __device__ void store(const S& s, int n, u64 v) const { s.p[n] = v; }
};
// ModDown, P limbs: scratch [items][2][K][N] in place, iNTT * N^-1 (P/p_k)^-1
template <int LOGN>
__global__ void HOLMES_NTT_BOUNDS(LOGN) k_ks_p(NttTables T, const Tw* md_scale, int L, int K, LdRows ld,
                                              StScratch st) {
  const int p = blockIdx.x / NttGeom<LOGN>::CL;
  const int k = (p % (2 * K)) % K;
  ntt_inverse_body<LOGN>(p, L + k, md_scale[k], T, ld, st);
}

// ModDown, Q limbs: conv_c[i] = NTT(sum_k y_c[k] p_k^-1 mod q_i) (k_conv, then a plain-load NTT); the store
// subtracts it from what k_ks_inner left in out_c: out = inner + perm(add) + post - conv.  With the inner product
// over the digits' P^-1-scaled Q rows, that is (inner - sum_k y_k (P/p_k)) P^-1 + perm(add) + post, the ModDown.
struct StKsSub {
  u64* out0;
  u64* out1;
  long long out_item;
  const Mod* mods;
  int cur, log_n;
  struct S {
    u64* o;
    u64 q;
  };
  __device__ S prep(int p) const {
    const int item = p / (2 * cur), r = p % (2 * cur), c = r / cur, i = r % cur;
    return S{(c ? out1 : out0) + item * out_item + ((size_t)i << log_n), mods[i].q};
  }
  __device__ void store(const S& s, int n, u64 v) const { s.o[n] = sub_mod(s.o[n], v, s.q); }
};
// resident CTAs per SM for the key-switch NTTs (their stores read as well as write)
#ifndef HOLMES_KS_MINB
#define HOLMES_KS_MINB HOLMES_NTT_MINB
#endif
template <int LOGN>
__global__ void __launch_bounds__(NttGeom<LOGN>::THREADS, HOLMES_KS_MINB) k_ks_q(NttTables T, LdRows ld,
                                                                                   StKsSub st) {
  const int p = blockIdx.x / NttGeom<LOGN>::CL;
  ntt_forward_body<LOGN>(p, (p % (2 * st.cur)) % st.cur, T, ld, st);
}

struct ModKsP {
  int L, K;
  __device__ int operator()(int p) const { return L + (p % (2 * K)) % K; }
};
struct ScKsP {
  const Tw* md_scale;
  int K;
  __device__ Tw operator()(int p) const { return md_scale[(p % (2 * K)) % K]; }
};
struct ModKsQ {
  int cur;
  __device__ int operator()(int p) const { return (p % (2 * cur)) % cur; }
};

// One ciphertext (the reference's rotations are per ciphertext): nothing is reused across items, so every load of
// a word -- the beta digit words, both components' key words, the addends -- is issued before the first product
// (three times beta independent loads in flight per thread), and the kernel is held to 64 registers for four CTAs per
// SM; the multi-item kernel keeps the key words in registers across items instead (70 registers, three CTAs per SM,
// gathered digit loads one item at a time).  Same sums, same residues.
template <int MAXB>
__global__ void __launch_bounds__(256, 4) k_ks_inner1(KsInnerArgs a, int log_n, const Mod* __restrict__ mods) {
  const size_t dstep = (size_t)(a.cur + a.K) << log_n, kstep = (size_t)(a.cap + a.K) << log_n;
  const size_t kcomp = (size_t)a.key_beta * kstep;
  const int n = blockIdx.x * blockDim.x + threadIdx.x;
  const int r = blockIdx.y;
  const u32 src = a.galois > 1 ? automorph_src((u32)n, a.galois, log_n) : (u32)n;
  const bool qlimb = r < a.cur;
  const int kr = qlimb ? r : a.cap + (r - a.cur);
  const Mod m = mods[qlimb ? r : a.L + (r - a.cur)];
  const u64* kp = a.key + ((size_t)kr << log_n) + n;
  const size_t roff = (size_t)r << log_n;
  const u64* d = a.digits + roff + src;
  u64 dv[MAXB], k0[MAXB], k1[MAXB];
#pragma unroll
  for (int j = 0; j < MAXB; ++j) {
    if (j < a.beta) {
      dv[j] = d[j * dstep];
      k0[j] = kp[j * kstep];
      k1[j] = kp[kcomp + j * kstep];
    }
  }
  u64 ad0 = 0, ad1 = 0;
  if (qlimb) {
    if (a.add0) ad0 = a.add0[roff + src];
    if (a.add1) ad1 = a.add1[roff + src];
  }
  Split4 s0{0, 0, 0, 0}, s1{0, 0, 0, 0};
#pragma unroll
  for (int j = 0; j < MAXB; ++j) {
    if (j < a.beta) {
      split_mac(s0, dv[j], k0[j]);
      split_mac(s1, dv[j], k1[j]);
    }
  }
  if (qlimb) {
    u64 u0 = fold_split(s0, m), u1 = fold_split(s1, m);
    if (a.add0) u0 = add_mod(u0, ad0, m.q);
    if (a.add1) u1 = add_mod(u1, ad1, m.q);
    if (a.post0) u0 = add_mod(u0, a.post0[roff + n], m.q);
    if (a.post1) u1 = add_mod(u1, a.post1[roff + n], m.q);
    if (a.qscale) {
      u0 = shoup(u0, a.qscale[r], m.q);
      u1 = shoup(u1, a.qscale[r], m.q);
    }
    a.out0[roff + n] = u0;
    a.out1[roff + n] = u1;
  } else {
    const size_t po = ((size_t)(r - a.cur) << log_n) + n;
    a.p0[po] = fold_split(s0, m);
    a.p1[po] = fold_split(s1, m);
  }
}

static int ks_inner_launch(const HolmesCtx& c, const KsInnerArgs& ia, cudaStream_t st) {
  if (c.n < 256) return -5;
  if (ia.beta > 16) return -3;   // the split sums hold 16 products
  count_launch();
  const dim3 grid((unsigned)(c.n / 256), (unsigned)(ia.cur + ia.K));
  // (the generic loop, k_ks_inner<0>, fits 5 CTAs per SM at 50 registers but measured 2% slower than these on the
  // config-3 layer's single-ciphertext key switches: its loads wait one digit at a time)
  static const bool single = [] {   // A/B timing: HOLMES_KS_INNER1=0 keeps single items on the multi-item kernel
    const char* v = getenv("HOLMES_KS_INNER1");
    return !(v && v[0] == '0');
  }();
  if (ia.items == 1 && ia.beta <= 5 && single) {
    if (ia.beta <= 2) k_ks_inner1<2><<<grid, 256, 0, st>>>(ia, c.log_n, c.d_mod);
    else k_ks_inner1<5><<<grid, 256, 0, st>>>(ia, c.log_n, c.d_mod);
    return (int)cudaGetLastError();
  }
  if (ia.beta <= 2) k_ks_inner<2><<<grid, 256, 0, st>>>(ia, c.log_n, c.d_mod);
  else if (ia.beta <= 5) k_ks_inner<5><<<grid, 256, 0, st>>>(ia, c.log_n, c.d_mod);
  else k_ks_inner<0><<<grid, 256, 0, st>>>(ia, c.log_n, c.d_mod);
  return (int)cudaGetLastError();
}

// ModDown tail: P-limb inner products in scratch [items][2][K][N] (coefficients' NTT form, canonical), Q outputs
// out_c already holding what the conversion is subtracted from.  P iNTT in place, P -> Q conversion into
// scratch + items 2 K N, Q NTT with "out -= conversion".
static int moddown_tail(const HolmesCtx& c, u64* scratch, u64* out0, u64* out1, long long out_item, int cur, int items,
                        cudaStream_t st) {
  const int K = c.K;
  {
    NttTables T{c.d_itw, c.d_mod};
    LdRows ld{scratch, c.log_n};
    StScratch ss{scratch, c.log_n};
    const int polys = items * 2 * K;
    if (c.log_n == 16) {
      const int e = ntt16_inverse<HOLMES_KS16_MINB>(T, ModKsP{c.L, K}, ScKsP{c.d_md_scale, K}, ld, IMRows{scratch},
                                                    ss, polys, st);
      if (e) return e;
    } else {
#define L_(LG)                                                                                                   \
  {                                                                                                              \
    using G = NttGeom<LG>;                                                                                       \
    cudaError_t e = launch_ntt(k_ks_p<LG>, G::LOGCL, G::THREADS, G::SMEM, polys, st, T, c.d_md_scale, c.L, K, ld, \
                               ss);                                                                              \
    if (e != cudaSuccess) return (int)e;                                                                         \
    break;                                                                                                       \
  }
      HOLMES_LOGN_SWITCH(c.log_n, L_)
#undef L_
    }
  }
  u64* conv = scratch + (size_t)items * 2 * K * c.n;  // [items][2][cur][N], coefficient form
  {
    ConvArgs ca{scratch, (long long)K * c.n, conv, (long long)cur * c.n, c.d_md_hat, c.L,
                K, cur, cur, cur, c.L, items * 2, nullptr, 0, nullptr};
    const int e = conv_launch(c, ca, st);
    if (e) return e;
  }
  {
    NttTables T{c.d_tw, c.d_mod};
    LdRows ld{conv, c.log_n};
    StKsSub sq{out0, out1, out_item, c.d_mod, cur, c.log_n};
    const int polys = items * 2 * cur;
    if (c.log_n == 16) return ntt16_forward<HOLMES_KS16_MINB>(T, ModKsQ{cur}, ld, IMRows{conv}, sq, polys, st);
#define L_(LG)                                                                                        \
  {                                                                                                   \
    using G = NttGeom<LG>;                                                                            \
    cudaError_t e = launch_ntt(k_ks_q<LG>, G::LOGCL, G::THREADS, G::SMEM, polys, st, T, ld, sq);       \
    if (e != cudaSuccess) return (int)e;                                                              \
    break;                                                                                            \
  }
    HOLMES_LOGN_SWITCH(c.log_n, L_)
#undef L_
  }
  return 0;
}

int ks_apply(const HolmesCtx& c, const KsArgs& a, cudaStream_t st) {
  if (a.cur < 1 || a.cur > a.key_cap || a.key_cap > c.L) return -2;
  if (c.alpha > MAXA || c.K > MAXA) return -3;
  if (a.items < 1) return -4;
  const int beta = c.beta(a.cur), key_beta = c.beta(a.key_cap), K = c.K;
  const u64 g = a.galois <= 1 ? 1 : a.galois;
  KsInnerArgs ia{a.digits, a.dig_item, a.key, a.add0, a.add1, a.add_item, a.post0, a.post1, a.post_item, a.out0,
                 a.out1, a.out_item, a.scratch, a.scratch + (size_t)K * c.n, (long long)2 * K * c.n, nullptr, g,
                 a.cur, a.key_cap, K, c.L, beta, key_beta, a.items};
  const int e = ks_inner_launch(c, ia, st);
  if (e) return e;
  return moddown_tail(c, a.scratch, a.out0, a.out1, a.out_item, a.cur, a.items, st);
}

// Key switch without the ModDown: out_c [items][cur + K][N] over Q u P (Q limbs first) =
//   Q limbs: P perm(add_c) + inner_c (the digits' Q rows carry P^-1, so this is P (u) with u the Q output above),
//   P limbs: inner_c.
int ks_apply_ext(const HolmesCtx& c, const KsArgs& a, cudaStream_t st) {
  if (a.cur < 1 || a.cur > a.key_cap || a.key_cap > c.L) return -2;
  if (c.alpha > MAXA || c.K > MAXA) return -3;
  if (a.items < 1) return -4;
  const int beta = c.beta(a.cur), key_beta = c.beta(a.key_cap);
  const u64 g = a.galois <= 1 ? 1 : a.galois;
  KsInnerArgs ia{a.digits, a.dig_item, a.key, a.add0, a.add1, a.add_item, a.post0, a.post1, a.post_item, a.out0,
                 a.out1, a.out_item, a.out0 + (size_t)a.cur * c.n, a.out1 + (size_t)a.cur * c.n, a.out_item,
                 c.d_pmodq_tw, g, a.cur, a.key_cap, c.K, c.L, beta, key_beta, a.items};
  return ks_inner_launch(c, ia, st);
}

// ModDown of extended-basis ciphertexts in_c [items][cur + K][N] (Q limbs first) to out_c [items][cur][N]:
// (in_Q - conv(iNTT(in_P))) P^-1.  The Q part is scaled by P^-1 into out first (the conversion's constants
// p_k^-1 mod q_i already carry P^-1), the P part copied into scratch.
__global__ void k_ext_split(const u64* __restrict__ in0, const u64* __restrict__ in1, long long in_item,
                            u64* __restrict__ out0, u64* __restrict__ out1, long long out_item, u64* __restrict__ scr,
                            int cur, int K, int log_n, const Tw* __restrict__ pinv, const Mod* __restrict__ mods) {
  const int n = blockIdx.x * blockDim.x + threadIdx.x;
  const int r = blockIdx.y, item = blockIdx.z;
  const size_t src = item * in_item + ((size_t)r << log_n) + n;
  if (r < cur) {
    const u64 q = mods[r].q;
    const size_t dst = item * out_item + ((size_t)r << log_n) + n;
    out0[dst] = shoup(in0[src], pinv[r], q);
    out1[dst] = shoup(in1[src], pinv[r], q);
  } else {
    const size_t dst = (((size_t)item * 2 * K + (r - cur)) << log_n) + n;
    scr[dst] = in0[src];
    scr[dst + ((size_t)K << log_n)] = in1[src];
  }
}
int moddown_ext(const HolmesCtx& c, const u64* in0, const u64* in1, long long in_item, int cur, u64* out0, u64* out1,
                long long out_item, int items, u64* scratch, cudaStream_t st) {
  if (cur < 1 || cur > c.L) return -2;
  if (items < 1 || items > 65535 || c.n < 256) return -4;
  count_launch();
  k_ext_split<<<dim3((unsigned)(c.n / 256), (unsigned)(cur + c.K), (unsigned)items), 256, 0, st>>>(
      in0, in1, in_item, out0, out1, out_item, scratch, cur, c.K, c.log_n, c.d_md_pinv, c.d_mod);
  HOLMES_CUDA_TRY(cudaGetLastError());
  return moddown_tail(c, scratch, out0, out1, out_item, cur, items, st);
}

// --------------------------------------------------------------------------------------------- rescale
struct LdRescale {
  const u64* x;  // scratch [comps][N]: coefficients of the last limb
  const Mod* mods;
  u64 ql;
  int cur, log_n;
  struct S {
    const u64* x;
    Mod m;
    u64 qlm;
  };
  __device__ S prep(int p) const {
    const int e = p / (cur - 1), i = p % (cur - 1);
    S s;
    s.x = x + ((size_t)e << log_n);
    s.m = mods[i];
    s.qlm = reduce128(0, ql, s.m);
    return s;
  }
  __device__ u64 load(const S& s, int n) const {
    const u64 v = s.x[n];
    const u64 r = reduce128(0, v, s.m);
    return v > (ql >> 1) ? sub_mod(r, s.qlm, s.m.q) : r;
  }
};
// Store of the rescale, with the post-operations of EasyFHE's homo_mul_relin_rescale_postop fused in
// (operators/nonlinear/polynomial.py:139-193): r = (a - v) q_L^-1, then r = 2r (dbl), r -= sub (item e, limb i at
// sub + e sub_stride + i N: a modulus drop of a deeper ciphertext is only its stride), r += cst[i].
struct StRescale {
  const u64* in;
  long long in_stride;
  u64* out;
  long long out_stride;
  const Mod* mods;
  const Tw* qinv;
  int cur, log_n;
  const u64* sub = nullptr;
  long long sub_stride = 0;
  const u64* cst = nullptr;
  int dbl = 0;
  struct S {
    const u64* a;
    const u64* b;
    u64* o;
    u64 q, k;
    Tw t;
  };
  __device__ S prep(int p) const {
    const int e = p / (cur - 1), i = p % (cur - 1);
    S s;
    s.a = in + e * in_stride + ((size_t)i << log_n);
    s.b = sub ? sub + e * sub_stride + ((size_t)i << log_n) : nullptr;
    s.o = out + e * out_stride + ((size_t)i << log_n);
    s.q = mods[i].q;
    s.k = cst ? cst[i] : 0;
    s.t = qinv[i];
    return s;
  }
  __device__ void store(const S& s, int n, u64 v) const {
    u64 r = shoup(sub_mod(s.a[n], v, s.q), s.t, s.q);
    if (dbl) r = add_mod(r, r, s.q);
    if (s.b) r = sub_mod(r, s.b[n], s.q);
    s.o[n] = add_mod(r, s.k, s.q);
  }
};
template <int LOGN>
__global__ void HOLMES_NTT_BOUNDS(LOGN) k_rescale(NttTables T, LdRescale ld, StRescale st) {
  const int p = blockIdx.x / NttGeom<LOGN>::CL;
  ntt_forward_body<LOGN>(p, p % (ld.cur - 1), T, ld, st);
}

int rescale(const HolmesCtx& c, const u64* in, long long in_stride, u64* out, long long out_stride, int cur, int comps,
            u64* scratch, cudaStream_t st, int dbl, const u64* sub, long long sub_stride, const u64* cst) {
  if (cur < 2 || cur > c.L) return -2;
  const int N = c.n;
  if (c.log_n == 16) {
    // the two-pass NTTs: 16 CTAs per polynomial and pass instead of one 8-CTA cluster, so a rescale of one or two
    // ciphertexts still spreads over the GPU; the forward NTT's intermediate lives in `out` (each second-pass CTA
    // reads its rows before its store overwrites them)
    const PolyMap pin = poly_map(1, in_stride, N, cur - 1);
    const PolyMap pscr = poly_map(1, N, N, cur - 1);
    {
      NttTables T{c.d_itw, c.d_mod};
      const int e = ntt16_inverse(T, ModPlain{pin}, ScLimb{c.d_ninv, 0, pin}, LdPlain{in + (size_t)(cur - 1) * N, pin},
                                  IMPlain{scratch, pscr}, StPlain{scratch, pscr}, comps, st);
      if (e) return e;
    }
    NttTables T{c.d_tw, c.d_mod};
    const PolyMap pim = poly_map(cur - 1, out_stride, N, 0);
    LdRescale ld{scratch, c.d_mod, c.q[cur - 1], cur, c.log_n};
    StRescale sr{in, in_stride, out, out_stride, c.d_mod, c.rs_qinv(cur), cur, c.log_n, sub, sub_stride, cst, dbl};
    return ntt16_forward(T, ModPlain{pim}, ld, IMPlain{out, pim}, sr, comps * (cur - 1), st);
  }
  {
    NttTables T{c.d_itw, c.d_mod};
    PolyMap pin = poly_map(1, in_stride, N, cur - 1);
    PolyMap pout = poly_map(1, N, N, cur - 1);
    LdPlain ld{in + (size_t)(cur - 1) * N, pin};
    StPlain sp{scratch, pout};
#define L_(LG)                                                                                                   \
  {                                                                                                              \
    using G = NttGeom<LG>;                                                                                       \
    cudaError_t e = launch_ntt(k_inv_plain<LG>, G::LOGCL, G::THREADS, G::SMEM, comps, st, T, pin, c.d_ninv, 0,   \
                               ld, sp);                                                                          \
    if (e != cudaSuccess) return (int)e;                                                                         \
    break;                                                                                                       \
  }
    HOLMES_LOGN_SWITCH(c.log_n, L_)
#undef L_
  }
  {
    NttTables T{c.d_tw, c.d_mod};
    LdRescale ld{scratch, c.d_mod, c.q[cur - 1], cur, c.log_n};
    StRescale sr{in, in_stride, out, out_stride, c.d_mod, c.rs_qinv(cur), cur, c.log_n, sub, sub_stride, cst, dbl};
    const int polys = comps * (cur - 1);
#define L_(LG)                                                                                      \
  {                                                                                                 \
    using G = NttGeom<LG>;                                                                          \
    return (int)launch_ntt(k_rescale<LG>, G::LOGCL, G::THREADS, G::SMEM, polys, st, T, ld, sr);     \
  }
    HOLMES_LOGN_SWITCH(c.log_n, L_)
#undef L_
  }
}

// --------------------------------------------------------------------------------------------- mod raise
// Bootstrapping's first step: a ciphertext modulo q0 alone is read as integer coefficients in
// (-q0/2, q0/2] and re-expressed modulo q_0 .. q_{raise-1}: iNTT of limb 0, centred lift fused into the NTT
// load of every raised limb.
struct LdLift {
  const u64* x;  // scratch [comps][N]: coefficients mod q0
  const Mod* mods;
  u64 q0;
  int raise, log_n;
  struct S {
    const u64* x;
    Mod m;
    u64 q0m;
  };
  __device__ S prep(int p) const {
    S s;
    s.x = x + ((size_t)(p / raise) << log_n);
    s.m = mods[p % raise];
    s.q0m = reduce128(0, q0, s.m);
    return s;
  }
  __device__ u64 load(const S& s, int n) const {
    const u64 v = s.x[n];
    const u64 r = reduce128(0, v, s.m);
    return v > (q0 >> 1) ? sub_mod(r, s.q0m, s.m.q) : r;
  }
};
template <int LOGN>
__global__ void HOLMES_NTT_BOUNDS(LOGN) k_modraise(NttTables T, LdLift ld, StPlain st) {
  const int p = blockIdx.x / NttGeom<LOGN>::CL;
  ntt_forward_body<LOGN>(p, p % ld.raise, T, ld, st);
}

int modraise(const HolmesCtx& c, const u64* in, long long in_stride, u64* out, long long out_stride, int raise,
             int comps, u64* scratch, cudaStream_t st) {
  if (raise < 2 || raise > c.L || comps < 1) return -2;
  const int N = c.n;
  {
    NttTables T{c.d_itw, c.d_mod};
    PolyMap pin = poly_map(1, in_stride, N, 0);
    PolyMap pout = poly_map(1, N, N, 0);
    LdPlain ld{in, pin};
    StPlain sp{scratch, pout};
#define L_(LG)                                                                                                 \
  {                                                                                                            \
    using G = NttGeom<LG>;                                                                                     \
    cudaError_t e = launch_ntt(k_inv_plain<LG>, G::LOGCL, G::THREADS, G::SMEM, comps, st, T, pin, c.d_ninv, 0, \
                               ld, sp);                                                                        \
    if (e != cudaSuccess) return (int)e;                                                                       \
    break;                                                                                                     \
  }
    HOLMES_LOGN_SWITCH(c.log_n, L_)
#undef L_
  }
  NttTables T{c.d_tw, c.d_mod};
  LdLift ld{scratch, c.d_mod, c.q[0], raise, c.log_n};
  StPlain sp{out, poly_map(raise, out_stride, N, 0)};
#define L_(LG)                                                                                         \
  {                                                                                                    \
    using G = NttGeom<LG>;                                                                             \
    return (int)launch_ntt(k_modraise<LG>, G::LOGCL, G::THREADS, G::SMEM, comps * raise, st, T, ld, sp); \
  }
  HOLMES_LOGN_SWITCH(c.log_n, L_)
#undef L_
}

// --------------------------------------------------------------------------------------------- encode
// Coefficient n of a row: Re(u[n / gap]) for n < N/2, Im(u[(n - N/2) / gap]) above, 0 off the gap grid;
// rounded with llround(v * scale) (bench/cmp/kernels/holmes_encode.cu:136-159) and reduced mod q_i.
// Two steps: k_round_rows rounds every coefficient once per row (the 2^61 range check included) into the
// storage of the row's last output limb; the forward NTTs of the other limbs then load those integers, and the
// last limb's NTT runs afterwards in place (a cluster loads all its words before any CTA of it stores).  The
// rounding is thus paid once per coefficient rather than once per limb.
__global__ void k_round_rows(const double* __restrict__ u, long long row_stride, int rows, int gap_log, int log_n,
                             double scale, u64* out, long long out_row_stride, int* flag) {
  const int half = 1 << (log_n - 1);
  const size_t total = (size_t)rows << log_n;
  for (size_t g = blockIdx.x * (size_t)blockDim.x + threadIdx.x; g < total; g += (size_t)gridDim.x * blockDim.x) {
    const int r = (int)(g >> log_n), n = (int)(g & ((1u << log_n) - 1));
    const int im = n >= half;
    const int k = n - im * half;
    i64 m = 0;
    if (!(k & ((1 << gap_log) - 1))) {
      const double v = __dmul_rn(u[r * row_stride + 2 * (k >> gap_log) + im], scale);
      if (fabs(v) < 2305843009213693952.0) {
        m = (i64)llround(v);
      } else {
        *flag = 1;
      }
    }
    out[r * out_row_stride + n] = (u64)m;
  }
}
// Load of a rounded coefficient m (|m| < 2^61) as a representative below 8 q (the forward NTT's input range):
// m itself or m + 8 q when every modulus of the launch has 8 q > 2^61 (WIDE), a signed Barrett reduction
// otherwise.
template <bool WIDE>
struct LdRounded {
  const u64* base;       // row r's integers at base + r * row_stride
  long long row_stride;
  const Mod* mods;
  int cur, first;        // poly p = (r, first + p % (cur - first))
  struct S {
    const i64* r;
    Mod m;
  };
  __device__ S prep(int p) const {
    const int w = cur - first;
    S s;
    s.r = reinterpret_cast<const i64*>(base + (p / w) * row_stride);
    s.m = mods[first + p % w];
    return s;
  }
  __device__ u64 load(const S& s, int n) const {
    const i64 m = s.r[n];
    if constexpr (WIDE) {
      return m >= 0 ? (u64)m : (u64)m + (s.m.q << 3);
    } else {
      const u64 a = reduce_wide(0, m >= 0 ? (u64)m : (u64)(-m), s.m);
      return m >= 0 ? a : (a ? s.m.q - a : 0);
    }
  }
};
struct ModEnc {
  int first, w;
  __device__ int operator()(int p) const { return first + p % w; }
};
template <int LOGN, bool WIDE>
__global__ void HOLMES_NTT_BOUNDS(LOGN) k_encode(NttTables T, LdRounded<WIDE> ld, StPlain st) {
  const int p = blockIdx.x / NttGeom<LOGN>::CL;
  ntt_forward_body<LOGN>(p, ld.first + p % (ld.cur - ld.first), T, ld, st);
}

// The encode on explicit tables: output limb l has twiddles tw + l N and modulus mods[l]; qs (host, may be null)
// lets a limb take the direct signed load when 8 q > 2^61.
static int encode_rows_tables(const Tw* tw, const Mod* mods, const u64* qs, int log_n, const double* u,
                              long long row_stride, int rows, int slots, double scale, int cur, u64* out,
                              long long out_row_stride, int* flag, cudaStream_t st) {
  const int n = 1 << log_n;
  if (slots < 1 || slots > n / 2 || (slots & (slots - 1))) return -3;
  if (out_row_stride < (long long)cur * n) return -4;
  int gap_log = 0;
  while ((slots << (gap_log + 1)) < n) ++gap_log;
  u64* ints = out + (size_t)(cur - 1) * n;  // row r's integers at ints + r * out_row_stride
  {
    const size_t work = (size_t)rows << log_n;
    size_t blocks = (work + 255) / 256;
    if (blocks > 148 * 16) blocks = 148 * 16;
    count_launch();
    k_round_rows<<<(unsigned)blocks, 256, 0, st>>>(u, row_stride, rows, gap_log, log_n, scale, ints, out_row_stride,
                                                    flag);
    HOLMES_CUDA_TRY(cudaGetLastError());
  }
  NttTables T{tw, mods};
  // limbs 0 .. cur-2 from the integers, then limb cur-1 in place
  for (int pass = 0; pass < 2; ++pass) {
    const int first = pass ? cur - 1 : 0, last = pass ? cur : cur - 1;
    if (last <= first) continue;
    bool wide = qs != nullptr;
    for (int l = first; l < last && wide; ++l) wide = (qs[l] << 3) > (1ull << 61);
    LdRounded<true> lw{ints, out_row_stride, mods, last, first};
    LdRounded<false> ln{ints, out_row_stride, mods, last, first};
    PolyMap pm = poly_map(last - first, out_row_stride, n, 0);
    StPlain sp{out + (size_t)first * n, pm};
    const int polys = rows * (last - first);
    if (log_n == 16) {
      const int e = wide ? ntt16_forward(T, ModEnc{first, last - first}, lw, IMPlain{out + (size_t)first * n, pm}, sp,
                                         polys, st)
                         : ntt16_forward(T, ModEnc{first, last - first}, ln, IMPlain{out + (size_t)first * n, pm}, sp,
                                         polys, st);
      if (e) return e;
      continue;
    }
#define L_(LG)                                                                                                   \
  {                                                                                                              \
    using G = NttGeom<LG>;                                                                                       \
    cudaError_t e = wide ? launch_ntt(k_encode<LG, true>, G::LOGCL, G::THREADS, G::SMEM, polys, st, T, lw, sp)  \
                         : launch_ntt(k_encode<LG, false>, G::LOGCL, G::THREADS, G::SMEM, polys, st, T, ln, sp); \
    if (e != cudaSuccess) return (int)e;                                                                         \
    break;                                                                                                       \
  }
    HOLMES_LOGN_SWITCH(log_n, L_)
#undef L_
  }
  return 0;
}

int encode_rows(const HolmesCtx& c, const double* u, long long row_stride, int rows, int slots, double scale, int cur,
                u64* out, long long out_row_stride, int* flag, cudaStream_t st, int mod_first) {
  if (cur < 1 || mod_first < 0 || mod_first + cur > c.T) return -2;
  // output limb l has modulus mod_first + l: the tables are taken from there on
  return encode_rows_tables(c.d_tw + (size_t)mod_first * c.n, c.d_mod + mod_first, c.q.data() + mod_first, c.log_n,
                            u, row_stride, rows, slots, scale, cur, out, out_row_stride, flag, st);
}

// The reference's in-tree encode ABI (bench/cmp/kernels/holmes_encode.cu:240-285), context-free: the caller's
// per-limb primes / Barrett ratios and exponents and its root tables (psi^bitrev(k) and their Shoup companions,
// [limbs][N]) are gathered once per table address into this engine's interleaved form (cached per device).
__global__ void k_gather_tables(const u64* __restrict__ roots, const u64* __restrict__ roots_shoup,
                                const u64* __restrict__ primes, const u64* __restrict__ ratios,
                                const u64* __restrict__ ks, int limbs, int log_n, Tw* __restrict__ tw,
                                Mod* __restrict__ mods) {
  const size_t total = (size_t)limbs << log_n;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x)
    tw[i] = Tw{roots[i], roots_shoup[i]};
  const size_t t = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (t < (size_t)limbs) mods[t] = Mod{primes[t], ratios[t], (u32)(ks[t] - 64), 0};
}
__device__ int g_stage2_range;  // the 2^61 range flag of encode_stage2 calls (the reference checks on the host)
int encode_stage2(u64* out, const double* in, long long in_stride, int rows, double sf, int limbs, const u64* primes,
                  const u64* ratios, const u64* ks, const u64* roots, const u64* roots_shoup, int* flag,
                  cudaStream_t st) {
  constexpr int kLogN = 16;
  if (limbs < 1 || rows < 0) return -2;
  if (rows == 0) return 0;
  if (!flag) HOLMES_CUDA_TRY(cudaGetSymbolAddress((void**)&flag, g_stage2_range));
  struct Entry {
    Tw* tw;
    Mod* mods;
  };
  static std::mutex mu;
  static std::map<std::tuple<int, const void*, const void*, int>, Entry> cache;
  int dev = 0;
  HOLMES_CUDA_TRY(cudaGetDevice(&dev));
  Entry e{};
  {
    std::lock_guard<std::mutex> lock(mu);
    const auto key = std::make_tuple(dev, (const void*)roots, (const void*)primes, limbs);
    auto it = cache.find(key);
    if (it == cache.end()) {
      HOLMES_CUDA_TRY(cudaMalloc(&e.tw, ((size_t)limbs << kLogN) * sizeof(Tw)));
      HOLMES_CUDA_TRY(cudaMalloc(&e.mods, (size_t)limbs * sizeof(Mod)));
      count_launch();
      k_gather_tables<<<148 * 4, 256, 0, st>>>(roots, roots_shoup, primes, ratios, ks, limbs, kLogN, e.tw, e.mods);
      HOLMES_CUDA_TRY(cudaGetLastError());
      cache.emplace(key, e);
    } else {
      e = it->second;
    }
  }
  // full slots (N / 2 complex values per row, interleaved), the generic signed reduction (no host moduli)
  return encode_rows_tables(e.tw, e.mods, nullptr, kLogN, in, in_stride, rows, 1 << (kLogN - 1), sf, limbs, out,
                            (long long)limbs << kLogN, flag, st);
}

// --------------------------------------------------------------------------------------------- decrypt
struct LdDecrypt {
  const u64* c0;
  const u64* c1;
  const u64* s;
  const Mod* mods;
  int log_n;
  struct S {
    const u64* a;
    const u64* b;
    const u64* sk;
    Mod m;
  };
  __device__ S prep(int p) const {
    const size_t o = (size_t)p << log_n;
    return S{c0 + o, c1 + o, s + o, mods[p]};
  }
  __device__ u64 load(const S& s, int n) const { return add_mod(s.a[n], mul_mod(s.b[n], s.sk[n], s.m), s.m.q); }
};
template <int LOGN>
__global__ void HOLMES_NTT_BOUNDS(LOGN) k_decrypt(NttTables T, const Tw* ninv, LdDecrypt ld,
                                                                     StScratch st) {
  const int p = blockIdx.x / NttGeom<LOGN>::CL;
  ntt_inverse_body<LOGN>(p, p, ninv[p], T, ld, st);
}
int decrypt_coef(const HolmesCtx& c, const u64* c0, const u64* c1, int cur, u64* out, cudaStream_t st) {
  if (cur < 1 || cur > c.L) return -2;
  NttTables T{c.d_itw, c.d_mod};
  LdDecrypt ld{c0, c1, c.d_secret, c.d_mod, c.log_n};
  StScratch ss{out, c.log_n};
#define L_(LG)                                                                                          \
  {                                                                                                     \
    using G = NttGeom<LG>;                                                                              \
    return (int)launch_ntt(k_decrypt<LG>, G::LOGCL, G::THREADS, G::SMEM, cur, st, T, c.d_ninv, ld, ss); \
  }
  HOLMES_LOGN_SWITCH(c.log_n, L_)
#undef L_
}

// --------------------------------------------------------------------------------------------- secret / keys
struct LdSigned {
  const i64* v;
  const Mod* mods;
  struct S { Mod m; };
  __device__ S prep(int p) const { return S{mods[p]}; }
  __device__ u64 load(const S& s, int n) const { return signed_residue(v[n], s.m); }
};
template <int LOGN>
__global__ void HOLMES_NTT_BOUNDS(LOGN) k_secret(NttTables T, LdSigned ld, StScratch st) {
  const int p = blockIdx.x / NttGeom<LOGN>::CL;
  ntt_forward_body<LOGN>(p, p, T, ld, st);
}

void host_secret_coeffs(const HolmesCtx& c, std::vector<i64>& s);

int secret_ntt(HolmesCtx& c, cudaStream_t st) {
  std::vector<i64> s;
  host_secret_coeffs(c, s);
  i64* d = nullptr;
  HOLMES_CUDA_TRY(cudaMalloc(&d, sizeof(i64) * c.n));
  HOLMES_CUDA_TRY(cudaMemcpy(d, s.data(), sizeof(i64) * c.n, cudaMemcpyHostToDevice));
  NttTables T{c.d_tw, c.d_mod};
  LdSigned ld{d, c.d_mod};
  StScratch ss{c.d_secret, c.log_n};
  int rc = 0;
#define L_(LG)                                                                                           \
  {                                                                                                      \
    using G = NttGeom<LG>;                                                                               \
    rc = (int)launch_ntt(k_secret<LG>, G::LOGCL, G::THREADS, G::SMEM, c.T, st, T, ld, ss);              \
    break;                                                                                               \
  }
  HOLMES_LOGN_SWITCH(c.log_n, L_)
#undef L_
  cudaError_t e = cudaStreamSynchronize(st);
  cudaFree(d);
  return rc ? rc : (int)e;
}

// uniform part of a key / ciphertext: out[row][n] for `rows` rows, modulus index of row r given by the map
__global__ void k_sample_uniform(u64* out, int rows, int log_n, u64 seed, u32 domain, u32 tag, u32 digit_word,
                                 PolyMap pm, const Mod* mods) {
  const size_t total = (size_t)rows << log_n;
  for (size_t idx = blockIdx.x * (size_t)blockDim.x + threadIdx.x; idx < total; idx += (size_t)gridDim.x * blockDim.x) {
    const int r = (int)(idx >> log_n), n = (int)(idx & ((1u << log_n) - 1));
    const int mi = pm.mod(r);
    out[idx] = sample_uniform(seed, domain, tag, digit_word | (u32)mi, (u32)n, mods[mi]);
  }
}

struct LdError {
  u64 seed;
  u32 domain, tag, word;
  const Mod* mods;
  PolyMap pm;
  struct S { Mod m; };
  __device__ S prep(int p) const { return S{mods[pm.mod(p)]}; }
  __device__ u64 load(const S& s, int n) const { return signed_residue(sample_cbd(seed, domain, tag, word, (u32)n), s.m); }
};
// key digit: b = e - a s + [modulus in digit] (P mod q) t,  t = sigma_g(s) (g > 1) or s^2 (g == 0)
struct StKey {
  u64* b;
  const u64* a;
  const u64* s;
  const u64* p_mod_q;
  const Mod* mods;
  PolyMap pm;
  u64 g;
  int lo, hi, L, log_n;
  struct S {
    u64* b;
    const u64* a;
    const u64* s;
    Mod m;
    int in_digit;
    u64 pq;
  };
  __device__ S prep(int p) const {
    const int mi = pm.mod(p);
    S st;
    st.b = b + ((size_t)p << log_n);
    st.a = a + ((size_t)p << log_n);
    st.s = s + ((size_t)mi << log_n);
    st.m = mods[mi];
    st.in_digit = mi < L && mi >= lo && mi < hi;
    st.pq = st.in_digit ? p_mod_q[mi] : 0;
    return st;
  }
  __device__ void store(const S& st, int n, u64 e) const {
    u64 v = sub_mod(e, mul_mod(st.a[n], st.s[n], st.m), st.m.q);
    if (st.in_digit) {
      const u64 t = g > 1 ? st.s[automorph_src((u32)n, g, log_n)] : mul_mod(st.s[n], st.s[n], st.m);
      v = add_mod(v, mul_mod(st.pq, t, st.m), st.m.q);
    }
    st.b[n] = v;
  }
};
template <int LOGN>
__global__ void HOLMES_NTT_BOUNDS(LOGN) k_keygen(NttTables T, LdError ld, StKey st) {
  const int p = blockIdx.x / NttGeom<LOGN>::CL;
  ntt_forward_body<LOGN>(p, st.pm.mod(p), T, ld, st);
}

int keygen(const HolmesCtx& c, u64 galois, int cap, u64* key, cudaStream_t st) {
  if (cap < 1 || cap > c.L) return -2;
  const int N = c.n, K = c.K, rows = cap + K, kb = c.beta(cap);
  const size_t digit_words = (size_t)rows * N;
  const u32 tag = (u32)galois;
  for (int j = 0; j < kb; ++j) {
    u64* bj = key + (size_t)j * digit_words;
    u64* aj = key + ((size_t)kb + j) * digit_words;
    PolyMap pm = poly_map(rows, 0, N, 0, cap, c.L);
    count_launch();
    k_sample_uniform<<<592, 256, 0, st>>>(aj, rows, c.log_n, c.seed, 2, tag, (u32)j << 16, pm, c.d_mod);
    HOLMES_CUDA_TRY(cudaGetLastError());
    NttTables T{c.d_tw, c.d_mod};
    LdError ld{c.seed, 3, tag, ((u32)j << 16) | 0xFFFFu, c.d_mod, pm};
    const int lo = j * c.alpha, hi = std::min(lo + c.alpha, c.L);
    StKey sk{bj, aj, c.d_secret, c.d_p_mod_q, c.d_mod, pm, galois, lo, hi, c.L, c.log_n};
#define L_(LG)                                                                                          \
  {                                                                                                     \
    using G = NttGeom<LG>;                                                                              \
    cudaError_t e = launch_ntt(k_keygen<LG>, G::LOGCL, G::THREADS, G::SMEM, rows, st, T, ld, sk);       \
    if (e != cudaSuccess) return (int)e;                                                                \
    break;                                                                                              \
  }
    HOLMES_LOGN_SWITCH(c.log_n, L_)
#undef L_
  }
  return 0;
}

// encryption: c1 = a (uniform), c0 = e - a s + m
struct StEnc {
  u64* c0;
  const u64* a;
  const u64* s;
  const u64* m;
  const Mod* mods;
  int log_n;
  struct S {
    u64* c0;
    const u64* a;
    const u64* s;
    const u64* m;
    Mod md;
  };
  __device__ S prep(int p) const {
    const size_t o = (size_t)p << log_n;
    return S{c0 + o, a + o, s + o, m + o, mods[p]};
  }
  __device__ void store(const S& s, int n, u64 e) const {
    s.c0[n] = add_mod(sub_mod(e, mul_mod(s.a[n], s.s[n], s.md), s.md.q), s.m[n], s.md.q);
  }
};
template <int LOGN>
__global__ void HOLMES_NTT_BOUNDS(LOGN) k_encrypt(NttTables T, LdError ld, StEnc st) {
  const int p = blockIdx.x / NttGeom<LOGN>::CL;
  ntt_forward_body<LOGN>(p, p, T, ld, st);
}

int encrypt(const HolmesCtx& c, const u64* m, int cur, u64 counter, u64* c0, u64* c1, cudaStream_t st) {
  if (cur < 1 || cur > c.L) return -2;
  PolyMap pm = poly_map(cur, 0, c.n, 0);
  count_launch();
  k_sample_uniform<<<592, 256, 0, st>>>(c1, cur, c.log_n, c.seed, 4, (u32)counter, 0u, pm, c.d_mod);
  HOLMES_CUDA_TRY(cudaGetLastError());
  NttTables T{c.d_tw, c.d_mod};
  LdError ld{c.seed, 5, (u32)counter, 0xFFFFu, c.d_mod, pm};
  StEnc se{c0, c1, c.d_secret, m, c.d_mod, c.log_n};
#define L_(LG)                                                                                  \
  {                                                                                             \
    using G = NttGeom<LG>;                                                                      \
    return (int)launch_ntt(k_encrypt<LG>, G::LOGCL, G::THREADS, G::SMEM, cur, st, T, ld, se);  \
  }
  HOLMES_LOGN_SWITCH(c.log_n, L_)
#undef L_
}

}  // namespace holmes
