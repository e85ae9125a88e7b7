// Kernels that are not NTT-shaped: elementwise RNS arithmetic, the BSGS plaintext multiply-accumulate,
// the CKKS special FFT of the encoder, diagonal packing, and the mod-q sum of peer partials.
#include <cstdlib>

#include "ops.h"

namespace holmes {

static inline int grid_for(size_t work, int threads) {
  count_launch();  // every grid_for result feeds exactly one launch
  size_t b = (work + threads - 1) / threads;
  if (b > 148 * 16) b = 148 * 16;
  return (int)(b ? b : 1);
}

// --------------------------------------------------------------------------------------------- elementwise
// Two words per thread (16-byte accesses); words of limb l of item i at i * item + l * N.
__global__ void k_elementwise(int op, const u64* __restrict__ a, const u64* __restrict__ b, u64* __restrict__ o,
                              int items, int limbs, long long ai, long long bi, long long oi, int log_n,
                              const Mod* __restrict__ mods) {
  const size_t per_item = (size_t)limbs << log_n;
  const size_t total = (size_t)items * per_item / 2;
  for (size_t t = blockIdx.x * (size_t)blockDim.x + threadIdx.x; t < total; t += (size_t)gridDim.x * blockDim.x) {
    const size_t w = 2 * t;
    const unsigned wl = (unsigned)(w >> log_n);  // item * limbs + limb (32-bit division)
    const int item = (int)(wl / (unsigned)limbs), limb = (int)(wl - (unsigned)item * limbs);
    const size_t r = ((size_t)limb << log_n) | (w & (((size_t)1 << log_n) - 1));
    const Mod m = mods[limb];
    const ulonglong2 x = *reinterpret_cast<const ulonglong2*>(a + item * ai + r);
    ulonglong2 y = make_ulonglong2(0, 0);
    if (op != EW_NEG) y = *reinterpret_cast<const ulonglong2*>(b + item * bi + r);
    ulonglong2 z;
    switch (op) {
      case EW_ADD: z = make_ulonglong2(add_mod(x.x, y.x, m.q), add_mod(x.y, y.y, m.q)); break;
      case EW_SUB: z = make_ulonglong2(sub_mod(x.x, y.x, m.q), sub_mod(x.y, y.y, m.q)); break;
      case EW_MUL: z = make_ulonglong2(mul_mod(x.x, y.x, m), mul_mod(x.y, y.y, m)); break;
      default: z = make_ulonglong2(x.x ? m.q - x.x : 0, x.y ? m.q - x.y : 0); break;
    }
    *reinterpret_cast<ulonglong2*>(o + item * oi + r) = z;
  }
}

// Tensor product of two ciphertexts (before relinearisation): d0 = a0 b0, d1 = a0 b1 + a1 b0, d2 = a1 b1 (mod q_l),
// two words per thread; each operand word is read once.
__global__ void k_tensor(const u64* __restrict__ a0, const u64* __restrict__ a1, long long ai,
                         const u64* __restrict__ b0, const u64* __restrict__ b1, long long bi, u64* __restrict__ d0,
                         u64* __restrict__ d1, u64* __restrict__ d2, long long di, int items, int limbs, int log_n,
                         const Mod* __restrict__ mods) {
  const size_t per_item = (size_t)limbs << log_n;
  const size_t total = (size_t)items * per_item / 2;
  for (size_t t = blockIdx.x * (size_t)blockDim.x + threadIdx.x; t < total; t += (size_t)gridDim.x * blockDim.x) {
    const size_t w = 2 * t;
    const unsigned wl = (unsigned)(w >> log_n);
    const int item = (int)(wl / (unsigned)limbs), limb = (int)(wl - (unsigned)item * limbs);
    const size_t r = ((size_t)limb << log_n) | (w & (((size_t)1 << log_n) - 1));
    const Mod m = mods[limb];
    const ulonglong2 x0 = *reinterpret_cast<const ulonglong2*>(a0 + item * ai + r);
    const ulonglong2 x1 = *reinterpret_cast<const ulonglong2*>(a1 + item * ai + r);
    const ulonglong2 y0 = *reinterpret_cast<const ulonglong2*>(b0 + item * bi + r);
    const ulonglong2 y1 = *reinterpret_cast<const ulonglong2*>(b1 + item * bi + r);
    const size_t o = item * di + r;
    *reinterpret_cast<ulonglong2*>(d0 + o) = make_ulonglong2(mul_mod(x0.x, y0.x, m), mul_mod(x0.y, y0.y, m));
    *reinterpret_cast<ulonglong2*>(d1 + o) =
        make_ulonglong2(add_mod(mul_mod(x0.x, y1.x, m), mul_mod(x1.x, y0.x, m), m.q),
                        add_mod(mul_mod(x0.y, y1.y, m), mul_mod(x1.y, y0.y, m), m.q));
    *reinterpret_cast<ulonglong2*>(d2 + o) = make_ulonglong2(mul_mod(x1.x, y1.x, m), mul_mod(x1.y, y1.y, m));
  }
}
int tensor_product(const HolmesCtx& c, const u64* a0, const u64* a1, long long a_item, const u64* b0, const u64* b1,
                   long long b_item, u64* d0, u64* d1, u64* d2, long long d_item, int items, int limbs,
                   cudaStream_t st) {
  if (limbs < 1 || limbs > c.T || items < 1) return -2;
  if ((a_item | b_item | d_item) & 1) return -2;
  const size_t work = ((size_t)items * limbs * c.n) / 2;
  k_tensor<<<grid_for(work, 256), 256, 0, st>>>(a0, a1, a_item, b0, b1, b_item, d0, d1, d2, d_item, items, limbs,
                                                c.log_n, c.d_mod);
  return (int)cudaGetLastError();
}

int elementwise(const HolmesCtx& c, int op, const u64* a, const u64* b, u64* out, int items, int limbs,
                long long a_item, long long b_item, long long o_item, cudaStream_t st) {
  if (limbs < 1 || limbs > c.T || items < 1) return -2;
  const size_t work = ((size_t)items * limbs * c.n) / 2;
  k_elementwise<<<grid_for(work, 256), 256, 0, st>>>(op, a, b, out, items, limbs, a_item, b_item, o_item, c.log_n,
                                                      c.d_mod);
  return (int)cudaGetLastError();
}

// multiply by X^(N/2): NTT word k holds the evaluation at psi^(2 bitrev(k)+1), and
// psi^((2 bitrev(k)+1) N/2) = psi^(N/2) for k < N/2 (bitrev(k) even), -psi^(N/2) above.
__global__ void k_mul_i(const u64* __restrict__ a, u64* __restrict__ o, int items, int limbs, long long ai,
                        long long oi, int log_n, const Mod* __restrict__ mods, const Tw* __restrict__ unit,
                        const Tw* __restrict__ unit_neg) {
  const size_t per_item = (size_t)limbs << log_n;
  const size_t total = (size_t)items * per_item;
  const size_t half = (size_t)1 << (log_n - 1);
  for (size_t w = blockIdx.x * (size_t)blockDim.x + threadIdx.x; w < total; w += (size_t)gridDim.x * blockDim.x) {
    const unsigned wl = (unsigned)(w >> log_n);  // item * limbs + limb (32-bit division)
    const int item = (int)(wl / (unsigned)limbs);
    const size_t r = ((size_t)(wl - (unsigned)item * limbs) << log_n) | (w & (((size_t)1 << log_n) - 1));
    const int limb = (int)(r >> log_n);
    const size_t n = r & (((size_t)1 << log_n) - 1);
    const u64 q = mods[limb].q;
    o[item * oi + r] = shoup(a[item * ai + r], n < half ? unit[limb] : unit_neg[limb], q);
  }
}
int mul_i(const HolmesCtx& c, const u64* a, u64* out, int items, int limbs, long long a_item, long long o_item,
          cudaStream_t st) {
  if (limbs < 1 || limbs > c.T || items < 1) return -2;
  const size_t work = (size_t)items * limbs * c.n;
  k_mul_i<<<grid_for(work, 256), 256, 0, st>>>(a, out, items, limbs, a_item, o_item, c.log_n, c.d_mod, c.d_unit,
                                                c.d_unit_neg);
  return (int)cudaGetLastError();
}

__global__ void k_automorph(const u64* __restrict__ a, u64* __restrict__ o, u64 g, int items, int limbs, long long ai,
                            long long oi, int log_n) {
  const size_t per_item = (size_t)limbs << log_n;
  const size_t total = (size_t)items * per_item;
  for (size_t w = blockIdx.x * (size_t)blockDim.x + threadIdx.x; w < total; w += (size_t)gridDim.x * blockDim.x) {
    const unsigned wl = (unsigned)(w >> log_n);  // item * limbs + limb (32-bit division)
    const int item = (int)(wl / (unsigned)limbs);
    const size_t r = ((size_t)(wl - (unsigned)item * limbs) << log_n) | (w & (((size_t)1 << log_n) - 1));
    const size_t row = r >> log_n << log_n;
    const u32 n = (u32)(r - row);
    o[item * oi + r] = a[item * ai + row + automorph_src(n, g, log_n)];
  }
}
int automorph(const HolmesCtx& c, const u64* a, u64* out, u64 galois, int items, int limbs, long long a_item,
              long long o_item, cudaStream_t st) {
  if (limbs < 1 || items < 1 || !(galois & 1)) return -2;
  const size_t work = (size_t)items * limbs * c.n;
  k_automorph<<<grid_for(work, 256), 256, 0, st>>>(a, out, galois, items, limbs, a_item, o_item, c.log_n);
  return (int)cudaGetLastError();
}

// multiply limb l by the constant consts[l] (canonical residues)
__global__ void k_mul_const(const u64* __restrict__ a, const u64* __restrict__ k, u64* __restrict__ o, int items,
                            int limbs, long long ai, long long oi, int log_n, const Mod* __restrict__ mods) {
  const size_t per_item = (size_t)limbs << log_n;
  const size_t total = (size_t)items * per_item;
  for (size_t w = blockIdx.x * (size_t)blockDim.x + threadIdx.x; w < total; w += (size_t)gridDim.x * blockDim.x) {
    const unsigned wl = (unsigned)(w >> log_n);  // item * limbs + limb (32-bit division)
    const int item = (int)(wl / (unsigned)limbs);
    const size_t r = ((size_t)(wl - (unsigned)item * limbs) << log_n) | (w & (((size_t)1 << log_n) - 1));
    const int limb = (int)(r >> log_n);
    o[item * oi + r] = mul_mod(a[item * ai + r], k[limb], mods[limb]);
  }
}
int mul_const(const HolmesCtx& c, const u64* a, const u64* consts, u64* out, int items, int limbs, long long a_item,
              long long o_item, cudaStream_t st) {
  if (limbs < 1 || limbs > c.T || items < 1) return -2;
  const size_t work = (size_t)items * limbs * c.n;
  k_mul_const<<<grid_for(work, 256), 256, 0, st>>>(a, consts, out, items, limbs, a_item, o_item, c.log_n, c.d_mod);
  return (int)cudaGetLastError();
}

// out[g][l][n] = sum_k w[g][k][l] * a[k][l][n] mod q_l (the Chebyshev / Paterson-Stockmeyer linear combination,
// grouped_scalar_weighted_acc): grid (N / 256, limbs, groups), radix-2^30 split products folded every 16 terms.
__global__ void k_weighted_acc(const u64* __restrict__ a, long long ai, int nk, const u64* __restrict__ w,
                               u64* __restrict__ o, long long oi, int limbs, int log_n, const Mod* __restrict__ mods) {
  const int n = blockIdx.x * blockDim.x + threadIdx.x;
  const int l = blockIdx.y, g = blockIdx.z;
  const Mod m = mods[l];
  const u64* ap = a + ((size_t)l << log_n) + n;
  const u64* wp = w + ((size_t)g * nk) * limbs + l;
  Split4 s{0, 0, 0, 0};
  for (int k = 0; k < nk; ++k) {
    split_mac(s, ap[k * ai], wp[(size_t)k * limbs]);
    if ((k & 15) == 15 && k + 1 < nk) {  // restart from a representative below 8 q: 16 more products fit
      const u64 r = fold_split_lazy(s, m);
      s = Split4{r & ((1ull << 30) - 1), r >> 30, 0, 0};
    }
  }
  o[g * oi + ((size_t)l << log_n) + n] = fold_split(s, m);
}
int weighted_acc(const HolmesCtx& c, const u64* a, long long a_item, int nk, const u64* w, u64* out, long long o_item,
                 int groups, int limbs, cudaStream_t st) {
  if (limbs < 1 || limbs > c.T || nk < 1 || groups < 1 || groups > 65535 || c.n < 256) return -2;
  count_launch();
  k_weighted_acc<<<dim3((unsigned)(c.n / 256), (unsigned)limbs, (unsigned)groups), 256, 0, st>>>(
      a, a_item, nk, w, out, o_item, limbs, c.log_n, c.d_mod);
  return (int)cudaGetLastError();
}

__global__ void k_add_const(const u64* __restrict__ a, const u64* __restrict__ k, u64* __restrict__ o, int items,
                            int limbs, long long ai, long long oi, int log_n, const Mod* __restrict__ mods) {
  const size_t per_item = (size_t)limbs << log_n;
  const size_t total = (size_t)items * per_item;
  for (size_t w = blockIdx.x * (size_t)blockDim.x + threadIdx.x; w < total; w += (size_t)gridDim.x * blockDim.x) {
    const unsigned wl = (unsigned)(w >> log_n);  // item * limbs + limb (32-bit division)
    const int item = (int)(wl / (unsigned)limbs);
    const size_t r = ((size_t)(wl - (unsigned)item * limbs) << log_n) | (w & (((size_t)1 << log_n) - 1));
    const int limb = (int)(r >> log_n);
    o[item * oi + r] = add_mod(a[item * ai + r], k[limb], mods[limb].q);
  }
}
int add_const(const HolmesCtx& c, const u64* a, const u64* consts, u64* out, int items, int limbs, long long a_item,
              long long o_item, cudaStream_t st) {
  if (limbs < 1 || limbs > c.T || items < 1) return -2;
  const size_t work = (size_t)items * limbs * c.n;
  k_add_const<<<grid_for(work, 256), 256, 0, st>>>(a, consts, out, items, limbs, a_item, o_item, c.log_n, c.d_mod);
  return (int)cudaGetLastError();
}

// Per-limb constants passed by value in the launch's parameter space: a scalar product or sum needs no device
// copy of its residues (an upload from pageable host memory would make the host wait for the stream).
struct ConstRow {
  u64 v[HOLMES_CONST_LIMBS];
};
// op CONST_ADD: o = a + k; CONST_MUL: o = a * k; CONST_AXPY: o = o + a * k (mod q_limb); two words per thread.
__global__ void k_const_op(int op, const u64* __restrict__ a, u64* __restrict__ o, int items, int limbs, long long ai,
                           long long oi, int log_n, const Mod* __restrict__ mods, const __grid_constant__ ConstRow k) {
  const size_t per_item = (size_t)limbs << log_n;
  const size_t total = (size_t)items * per_item / 2;
  for (size_t t = blockIdx.x * (size_t)blockDim.x + threadIdx.x; t < total; t += (size_t)gridDim.x * blockDim.x) {
    const size_t w = 2 * t;
    const unsigned wl = (unsigned)(w >> log_n);
    const int item = (int)(wl / (unsigned)limbs), limb = (int)(wl - (unsigned)item * limbs);
    const size_t r = ((size_t)limb << log_n) | (w & (((size_t)1 << log_n) - 1));
    const Mod m = mods[limb];
    const u64 c = k.v[limb];
    const ulonglong2 x = *reinterpret_cast<const ulonglong2*>(a + item * ai + r);
    ulonglong2* dst = reinterpret_cast<ulonglong2*>(o + item * oi + r);
    ulonglong2 z;
    if (op == CONST_ADD) {
      z = make_ulonglong2(add_mod(x.x, c, m.q), add_mod(x.y, c, m.q));
    } else if (op == CONST_MUL) {
      z = make_ulonglong2(mul_mod(x.x, c, m), mul_mod(x.y, c, m));
    } else {
      const ulonglong2 y = *dst;
      z = make_ulonglong2(add_mod(y.x, mul_mod(x.x, c, m), m.q), add_mod(y.y, mul_mod(x.y, c, m), m.q));
    }
    *dst = z;
  }
}
int const_op(const HolmesCtx& c, int op, const u64* a, const u64* host_consts, u64* out, int items, int limbs,
             long long a_item, long long o_item, cudaStream_t st) {
  if (op < CONST_ADD || op > CONST_AXPY || limbs < 1 || limbs > c.T || limbs > HOLMES_CONST_LIMBS || items < 1)
    return -2;
  if ((a_item | o_item) & 1) return -2;   // 16-byte accesses
  ConstRow k;
  for (int l = 0; l < limbs; ++l) k.v[l] = host_consts[l];
  const size_t work = (size_t)items * limbs * c.n / 2;
  k_const_op<<<grid_for(work, 256), 256, 0, st>>>(op, a, out, items, limbs, a_item, o_item, c.log_n, c.d_mod, k);
  return (int)cudaGetLastError();
}

// --------------------------------------------------------------------------------------------- BSGS MAC
// res[c][g][i][limb][j] = sum_b pts[g nb + b][limb][j] * baby_i[b][c][limb][j]  (mod q_limb)
// (semantics of the reference's mac_multi, bench/cmp/kernels/holmes_mac.cu:1-13, 116-190).
// Block: 32 consecutive words x 8 inputs; each thread keeps TG giants x 2 components as 128-bit lazy
// sums (reduced every 16 baby steps: 16 products of canonical residues stay below 14 2^k).  Warps of
// one block read the same plaintext words, so the plaintext row is fetched from HBM once per block
// and served from L1 to the other inputs.
template <int TG>
__global__ void __launch_bounds__(256) k_bsgs_mac(u64* __restrict__ res, InPtrs in, long long bstride, int nb,
                                                  int inputs, int G, const u64* __restrict__ pts, long long pstride,
                                                  int limbs, ModSrc ms, int log_n) {
  const int lane = threadIdx.x & 31, wi = threadIdx.x >> 5;
  const int itiles = (inputs + 7) / 8;
  const int j = (blockIdx.x / itiles) * 32 + lane;
  const int i = (blockIdx.x % itiles) * 8 + wi;
  const int limb = blockIdx.y, g0 = blockIdx.z * TG;
  if (i >= inputs) return;
  const Mod m = ms.get(limb);
  const size_t lj = ((size_t)limb << log_n) + j;
  const u64* __restrict__ b0 = in.c0[i] + lj;
  const u64* __restrict__ b1 = in.c1[i] + lj;
  const u64* pp[TG];
#pragma unroll
  for (int g = 0; g < TG; ++g) pp[g] = pts + (size_t)(g0 + g < G ? g0 + g : g0) * nb * pstride + lj;
  U128 acc[2][TG];
#pragma unroll
  for (int g = 0; g < TG; ++g) acc[0][g] = acc[1][g] = U128{0, 0};
  for (int b = 0; b < nb; ++b) {
    const u64 v0 = b0[(size_t)b * bstride], v1 = b1[(size_t)b * bstride];
#pragma unroll
    for (int g = 0; g < TG; ++g) {
      const u64 w = __ldg(pp[g] + (size_t)b * pstride);
      mac128(acc[0][g], v0, w);
      mac128(acc[1][g], v1, w);
    }
    if ((b & 15) == 15) {
#pragma unroll
      for (int g = 0; g < TG; ++g) {
        acc[0][g] = U128{reduce128(acc[0][g], m), 0};
        acc[1][g] = U128{reduce128(acc[1][g], m), 0};
      }
    }
  }
  const size_t is = (size_t)limbs << log_n, gs = (size_t)inputs * is;
#pragma unroll
  for (int g = 0; g < TG; ++g) {
    if (g0 + g >= G) break;
    res[((size_t)0 * G + g0 + g) * gs + (size_t)i * is + lj] = reduce128(acc[0][g], m);
    res[((size_t)1 * G + g0 + g) * gs + (size_t)i * is + lj] = reduce128(acc[1][g], m);
  }
}

// ---------------------------------------------------------------------------------------------------------
// k_bsgs_mac2: the same result with radix-2^30 partial products.
//
// Every residue a < 2^60 splits as a = a1 2^30 + a0 with a0, a1 < 2^30, so each of the four partial products
// a0 b0, a0 b1, a1 b0, a1 b1 is below 2^60 and is one 32 x 32 -> 64-bit multiply-add into a 64-bit sum; 16 of
// them (plus a carried value below 2^30) still fit in 64 bits.  A thread keeps, per output, the four sums
// S00, SA (a0 b1), SB (a1 b0), S11 and every 16 baby steps folds
//     V = S00 + (SA + SB) 2^30 + S11 2^60  (< 16 q^2 + q),
// reduces V mod q with the 128-bit Barrett step (common.cuh) and restarts the sums from the two 30-bit
// halves of the residue.  That is 4 multiply-adds per product plus a fold amortised over 16 steps,
// instead of a full 64 x 64 -> 128-bit product and a 128-bit add.
//
// Block: 256 threads = 8 warps over 32 consecutive words of one limb; warp w takes input i0 + w/2 and the
// giant half w % 2 (4 giants) of an 8-giant group, both ciphertext components.  The plaintext words of the
// 8 giants are staged in shared memory 16 baby steps at a time (cp.async, double-buffered) and split into
// (a0 | a1 << 32) once per block, so each is fetched from HBM once per 4 inputs and split once.
constexpr int kMacSB = 16;      // baby steps per stage
constexpr int kMacGG = 8;       // giants per block
constexpr int kMacIW = 4;       // inputs per block
constexpr int kMacStageWords = kMacGG * kMacSB * 32;

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  const unsigned s = (unsigned)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(s), "l"(gmem));
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;\n" ::); }

// acc += a * b for 32-bit a, b and a 64-bit accumulator: one wide multiply-add
__device__ __forceinline__ void mad_wide(u64& acc, u32 a, u32 b) {
  asm("mad.wide.u32 %0, %1, %2, %0;" : "+l"(acc) : "r"(a), "r"(b));
}
__device__ __forceinline__ void mad_split(Split4& acc, u32 a0, u32 a1, u64 bp) {
  const u32 b0 = (u32)bp, b1 = (u32)(bp >> 32);
  mad_wide(acc.s00, a0, b0);
  mad_wide(acc.sa, a0, b1);
  mad_wide(acc.sb, a1, b0);
  mad_wide(acc.s11, a1, b1);
}
__device__ __forceinline__ void restart_split(Split4& acc, u64 r) {
  acc.s00 = r & ((1ull << 30) - 1);
  acc.sa = r >> 30;
  acc.sb = 0;
  acc.s11 = 0;
}

__global__ void __launch_bounds__(256, 2) k_bsgs_mac2(u64* __restrict__ res, InPtrs in, long long bstride, int nb,
                                                      int inputs, int G, const u64* __restrict__ pts, long long pstride,
                                                      int limbs, ModSrc ms, int log_n) {
  extern __shared__ __align__(16) u64 mac_smem[];
  u64(*stage)[kMacStageWords] = reinterpret_cast<u64(*)[kMacStageWords]>(mac_smem);
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int itiles = (inputs + kMacIW - 1) / kMacIW;
  const int j0 = (blockIdx.x / itiles) * 32;
  const int i = (blockIdx.x % itiles) * kMacIW + (w >> 1);
  const int half = w & 1;
  const int limb = blockIdx.y, g0 = blockIdx.z * kMacGG;
  const Mod m = ms.get(limb);
  const size_t lpos = ((size_t)limb << log_n) + j0;
  const bool active = i < inputs;
  const u64* __restrict__ b0p = in.c0[active ? i : 0] + lpos + lane;
  const u64* __restrict__ b1p = in.c1[active ? i : 0] + lpos + lane;

  // staging: 8 giants x 16 steps x 32 words = 2048 16-byte chunks; thread t copies chunks t + 256 k
  auto issue_stage = [&](int s, int buf) {
#pragma unroll
    for (int k = 0; k < kMacStageWords / 2 / 256; ++k) {
      const int chunk = threadIdx.x + 256 * k;
      const int g = chunk / (kMacSB * 16), r = chunk % (kMacSB * 16);
      const int bb = r / 16, c = r % 16;
      const int b = s * kMacSB + bb;
      if (b < nb) {
        const int gg = g0 + g < G ? g0 + g : g0;
        cp_async16(&stage[buf][(g * kMacSB + bb) * 32 + 2 * c], pts + ((size_t)gg * nb + b) * pstride + lpos + 2 * c);
      }
    }
    asm volatile("cp.async.commit_group;\n" ::);
  };
  auto split_stage = [&](int buf) {
#pragma unroll
    for (int k = 0; k < kMacStageWords / 2 / 256; ++k) {
      const int chunk = threadIdx.x + 256 * k;
      u64* p = &stage[buf][chunk * 2];
      const u64 x = p[0], y = p[1];
      p[0] = (x & ((1ull << 30) - 1)) | ((x >> 30) << 32);
      p[1] = (y & ((1ull << 30) - 1)) | ((y >> 30) << 32);
    }
  };

  Split4 acc[2][4];
#pragma unroll
  for (int c = 0; c < 2; ++c)
#pragma unroll
    for (int g = 0; g < 4; ++g) acc[c][g] = Split4{0, 0, 0, 0};

  const int nstages = (nb + kMacSB - 1) / kMacSB;
  issue_stage(0, 0);
  for (int s = 0; s < nstages; ++s) {
    const int buf = s & 1;
    cp_async_wait_all();
    split_stage(buf);
    __syncthreads();
    if (s + 1 < nstages) issue_stage(s + 1, buf ^ 1);
    const int steps = nb - s * kMacSB < kMacSB ? nb - s * kMacSB : kMacSB;
    if (active) {
      const u64* sp = &stage[buf][(half * 4) * kMacSB * 32 + lane];
      u64 n0 = b0p[(size_t)(s * kMacSB) * bstride], n1 = b1p[(size_t)(s * kMacSB) * bstride];
      for (int bb = 0; bb < steps; ++bb) {
        const u64 v0 = n0, v1 = n1;
        if (bb + 1 < steps) {
          n0 = b0p[(size_t)(s * kMacSB + bb + 1) * bstride];
          n1 = b1p[(size_t)(s * kMacSB + bb + 1) * bstride];
        }
        const u32 x0 = (u32)(v0 & ((1ull << 30) - 1)), x1 = (u32)(v0 >> 30);
        const u32 y0 = (u32)(v1 & ((1ull << 30) - 1)), y1 = (u32)(v1 >> 30);
#pragma unroll
        for (int g = 0; g < 4; ++g) {
          const u64 bp = sp[(g * kMacSB + bb) * 32];
          mad_split(acc[0][g], x0, x1, bp);
          mad_split(acc[1][g], y0, y1, bp);
        }
      }
#pragma unroll
      for (int c = 0; c < 2; ++c)
#pragma unroll
        for (int g = 0; g < 4; ++g) restart_split(acc[c][g], fold_split(acc[c][g], m));
    }
    __syncthreads();  // the buffer is refilled by the next stage's copies
  }
  if (!active) return;
  const size_t is = (size_t)limbs << log_n, gs = (size_t)inputs * is;
#pragma unroll
  for (int g = 0; g < 4; ++g) {
    const int gg = g0 + half * 4 + g;
    if (gg >= G) break;
#pragma unroll
    for (int c = 0; c < 2; ++c) {
      const u64 r = (acc[c][g].sa << 30) | acc[c][g].s00;  // restart_split left the canonical residue here
      res[((size_t)c * G + gg) * gs + (size_t)i * is + lpos + lane] = r;
    }
  }
}

// ---------------------------------------------------------------------------------------------------------
// k_bsgs_mac3: k_bsgs_mac2's arithmetic with the baby words staged as well.
//
// Measured on B200: the 32 x 32 -> 64-bit wide multiply-add (and mul.hi) issues at quarter rate, about 32 per
// clock per SM, so a product (four of them) costs 16 cycles of a warp's multiply pipe and the multiply-add
// ceiling is 8 products per clock per SM.  Three things keep the kernel near it:
//   * the baby words of the block's IW inputs join the plaintext words of its 8 giants in a 3-deep cp.async
//     ring of 8-step stages, so two stages of multiply-adds are in flight while one is consumed (k_bsgs_mac2
//     read the babies straight from HBM one step ahead and every warp waited on them);
//   * each thread splits the words it copied into (low 30 bits, high 30 bits) pairs in place once they land;
//     a product of two such pairs is then four fused wide multiply-adds, whereas splitting a 64-bit word in
//     registers right before the multiply costs the compiler about eight extra instructions per product;
//   * the sums are folded lazily (a representative below 8 q, restarted from its split; one accumulator per step
//     of every other stage) except at the last fold.
// Tiles: IW inputs x 8 giants per block, GPT giants per thread (HOLMES_MAC_TILE="IWxGPT" selects one for A/B
// timing; 4x4 is the default, 10.5 ms per 512-row chunk of 16 ciphertexts at 13 limbs).
constexpr int kM3SB = 8;   // baby steps per stage
constexpr int kM3NS = 3;   // stages in the ring

// Tile of k_bsgs_mac3: IW inputs per block, GPT of the 8 giants per thread (both components), so
// 8 / GPT warps per input and IW * 8 / GPT warps per block.
template <int GPT>
struct MacAcc {
  u64 s00[2 * GPT], sa[2 * GPT], sb[2 * GPT], s11[2 * GPT];  // index c * GPT + g
};
// one baby step on words pre-split into (low 30 bits, high 30 bits) pairs: every 32 x 32 -> 64-bit
// product is one fused wide multiply-add into a 64-bit sum
template <int GPT>
__device__ __forceinline__ void m3_step(MacAcc<GPT>& A, const uint2* bb, const uint2* pt, int st) {
  const uint2 x = bb[st * 32], y = bb[(kM3SB + st) * 32];
#pragma unroll
  for (int g = 0; g < GPT; ++g) {
    const uint2 p = pt[(g * kM3SB + st) * 32];
    A.s00[g] += (u64)x.x * p.x;
    A.sa[g] += (u64)x.x * p.y;
    A.sb[g] += (u64)x.y * p.x;
    A.s11[g] += (u64)x.y * p.y;
    A.s00[GPT + g] += (u64)y.x * p.x;
    A.sa[GPT + g] += (u64)y.x * p.y;
    A.sb[GPT + g] += (u64)y.y * p.x;
    A.s11[GPT + g] += (u64)y.y * p.y;
  }
}
// lazy fold of accumulator K alone (a representative below 8 q, restarted from its split): issued between the
// products of a step, one accumulator at a time, so its temporaries never pile up
template <int K, int GPT>
__device__ __forceinline__ void m3_fold_one(MacAcc<GPT>& A, const Mod& m) {
  const Split4 s{A.s00[K], A.sa[K], A.sb[K], A.s11[K]};
  const u64 r = fold_split_lazy(s, m);
  A.s00[K] = r & ((1ull << 30) - 1);
  A.sa[K] = r >> 30;
  A.sb[K] = 0;
  A.s11[K] = 0;
}
template <bool CANON, int GPT>
__device__ __forceinline__ void m3_fold(MacAcc<GPT>& A, const Mod& m) {
#pragma unroll
  for (int k = 0; k < 2 * GPT; ++k) {
    const Split4 s{A.s00[k], A.sa[k], A.sb[k], A.s11[k]};
    // the full-width Barrett here (the last, canonical fold of all sums at once): with reduce_wide the 4x4 tile
    // spills
    u64 hi, lo;
    split_fold128(s, hi, lo);
    const u64 r = CANON ? reduce128(hi, lo, m) : reduce128_lazy(hi, lo, m);
    A.s00[k] = r & ((1ull << 30) - 1);
    A.sa[k] = r >> 30;
    A.sb[k] = 0;
    A.s11[k] = 0;
  }
}
template <int GPT, int K>
__device__ __forceinline__ void m3_fold_at(MacAcc<GPT>& A, int st, const Mod& m) {
  if constexpr (K < 2 * GPT) {
    if (st == K) m3_fold_one<K, GPT>(A, m);
    else m3_fold_at<GPT, K + 1>(A, st, m);
  }
}
// one stage of `steps` (<= 8) baby steps; FOLD: accumulator st folded after step st
template <int GPT, bool FOLD>
__device__ __forceinline__ void m3_stage(MacAcc<GPT>& A, const uint2* bb, const uint2* pt, int steps, const Mod& m) {
  static_assert(2 * GPT <= kM3SB, "one fold slot per step");
#pragma unroll
  for (int st = 0; st < kM3SB; ++st) {
    if (st < steps) {
      m3_step<GPT>(A, bb, pt, st);
      if constexpr (FOLD) m3_fold_at<GPT, 0>(A, st, m);
    }
  }
}
// the words w at p, p + 1 become the pairs (w mod 2^30, w >> 30) in place
__device__ __forceinline__ void split_words(u64* p) {
  const ulonglong2 v = *reinterpret_cast<const ulonglong2*>(p);
  ulonglong2 o;
  o.x = (v.x & ((1ull << 30) - 1)) | ((v.x >> 30) << 32);
  o.y = (v.y & ((1ull << 30) - 1)) | ((v.y >> 30) << 32);
  *reinterpret_cast<ulonglong2*>(p) = o;
}

template <int IW, int GPT, int GG = kMacGG>
struct M3Geom {
  static constexpr int THREADS = IW * (GG / GPT) * 32;
  static constexpr int PT_WORDS = GG * kM3SB * 32;
  static constexpr int BB_WORDS = IW * 2 * kM3SB * 32;
  static constexpr int STAGE_WORDS = PT_WORDS + BB_WORDS;
  static constexpr int SMEM = kM3NS * STAGE_WORDS * 8;
  static constexpr int MINB = (228 * 1024) / (SMEM + 1024) < 4 ? (228 * 1024) / (SMEM + 1024) : 4;
};

template <int IW, int GPT, int GG = kMacGG>
__global__ void __launch_bounds__(M3Geom<IW, GPT, GG>::THREADS, M3Geom<IW, GPT, GG>::MINB)
    k_bsgs_mac3(u64* __restrict__ res, InPtrs in, long long bstride, int nb, int inputs, int G,
                const u64* __restrict__ pts, long long pstride, int limbs, ModSrc ms, int log_n) {
  using Geo = M3Geom<IW, GPT, GG>;
  constexpr int WPI = GG / GPT;  // warps per input
  extern __shared__ __align__(16) u64 mac_smem[];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int itiles = (inputs + IW - 1) / IW;
  const int j0 = (blockIdx.x / itiles) * 32;
  const int i0 = (blockIdx.x % itiles) * IW;
  const int iw = w / WPI, gq = w % WPI;
  const int limb = blockIdx.y, g0 = blockIdx.z * GG;
  const Mod m = ms.get(limb);
  const size_t lpos = ((size_t)limb << log_n) + j0;
  const bool active = i0 + iw < inputs;
  const int nstages = (nb + kM3SB - 1) / kM3SB;

  // Stage s -> ring slot s % kM3NS.  16-byte chunk c of a region holds its words 2c, 2c + 1: plaintext chunk
  // c is giant c / 128, step (c / 16) % 8, words 2 (c % 16) .. +1 of the 32; baby chunk c is input c / 256,
  // component (c / 128) % 2, step (c / 16) % 8.  Thread t copies (and later splits) chunks t + THREADS k; their
  // stage-0 sources are computed once, stage s adds s * 8 rows.
  constexpr int PCH = Geo::PT_WORDS / 2 / Geo::THREADS, BCH = Geo::BB_WORDS / 2 / Geo::THREADS;
  const u64* psrc[PCH];
  int pstep[PCH];
  const u64* bsrc[BCH];
  int bstep[BCH];
#pragma unroll
  for (int k = 0; k < PCH; ++k) {
    const int c = threadIdx.x + Geo::THREADS * k;
    const int g = c / (kM3SB * 16), st = (c / 16) % kM3SB;
    const int gg = g0 + g < G ? g0 + g : g0;
    psrc[k] = pts + ((size_t)gg * nb + st) * pstride + lpos + 2 * (c % 16);
    pstep[k] = st;
  }
#pragma unroll
  for (int k = 0; k < BCH; ++k) {
    const int c = threadIdx.x + Geo::THREADS * k;
    const int ii = c / (2 * kM3SB * 16), comp = (c / (kM3SB * 16)) % 2, st = (c / 16) % kM3SB;
    const bool ok = i0 + ii < inputs;
    bsrc[k] = ok ? (comp ? in.c1[i0 + ii] : in.c0[i0 + ii]) + (size_t)st * bstride + lpos + 2 * (c % 16) : nullptr;
    bstep[k] = st;
  }
  auto issue_stage = [&](int s) {
    if (s < nstages) {
      u64* pt = mac_smem + (size_t)(s % kM3NS) * Geo::STAGE_WORDS;
      u64* bb = pt + Geo::PT_WORDS;
      const size_t po = (size_t)s * kM3SB * pstride, bo = (size_t)s * kM3SB * bstride;
      const int left = nb - s * kM3SB;
#pragma unroll
      for (int k = 0; k < PCH; ++k)
        if (pstep[k] < left) cp_async16(pt + 2 * (threadIdx.x + Geo::THREADS * k), psrc[k] + po);
#pragma unroll
      for (int k = 0; k < BCH; ++k)
        if (bsrc[k] && bstep[k] < left) cp_async16(bb + 2 * (threadIdx.x + Geo::THREADS * k), bsrc[k] + bo);
    }
    asm volatile("cp.async.commit_group;\n" ::);  // an empty group past the end keeps the wait count uniform
  };

  MacAcc<GPT> A;
#pragma unroll
  for (int k = 0; k < 2 * GPT; ++k) A.s00[k] = A.sa[k] = A.sb[k] = A.s11[k] = 0;

#pragma unroll
  for (int s = 0; s < kM3NS - 1; ++s) issue_stage(s);
  for (int s = 0; s < nstages; ++s) {
    asm volatile("cp.async.wait_group %0;\n" ::"n"(kM3NS - 2));
    {  // this thread's copies of stage s have landed: split them in place
      u64* pt = mac_smem + (size_t)(s % kM3NS) * Geo::STAGE_WORDS;
      u64* bb = pt + Geo::PT_WORDS;
      const int left = nb - s * kM3SB;
#pragma unroll
      for (int k = 0; k < PCH; ++k)
        if (pstep[k] < left) split_words(pt + 2 * (threadIdx.x + Geo::THREADS * k));
#pragma unroll
      for (int k = 0; k < BCH; ++k)
        if (bsrc[k] && bstep[k] < left) split_words(bb + 2 * (threadIdx.x + Geo::THREADS * k));
    }
    __syncthreads();  // stage s is split and visible to every thread; slot (s - 1) % kM3NS is no longer read
    issue_stage(s + kM3NS - 1);
    const int steps = nb - s * kM3SB < kM3SB ? nb - s * kM3SB : kM3SB;
    if (active) {
      const u64* base = mac_smem + (size_t)(s % kM3NS) * Geo::STAGE_WORDS;
      const uint2* pt = reinterpret_cast<const uint2*>(base) + (gq * GPT) * kM3SB * 32 + lane;
      const uint2* bb = reinterpret_cast<const uint2*>(base + Geo::PT_WORDS) + (iw * 2) * kM3SB * 32 + lane;
      // In odd stages accumulator k is folded (lazily) right after step k's products, so every sum takes at most
      // 16 products between folds: 8 - k - 1 + 8 + k + 1 across full stages, and in a short last stage of
      // `steps` babies either k < steps (folded in it) or 8 - k - 1 + 8 + steps <= 15.  The last fold of the
      // kernel is canonical.
      const bool odd = s & 1;
      if (steps == kM3SB) {
        if (odd) {
          m3_stage<GPT, true>(A, bb, pt, kM3SB, m);
        } else {
#pragma unroll
          for (int st = 0; st < kM3SB; ++st) m3_step<GPT>(A, bb, pt, st);
        }
      } else {
        if (odd) m3_stage<GPT, true>(A, bb, pt, steps, m);
        else m3_stage<GPT, false>(A, bb, pt, steps, m);
      }
      if (s == nstages - 1) m3_fold<true, GPT>(A, m);
    }
  }
  asm volatile("cp.async.wait_all;\n" ::);
  if (!active) return;
  const int i = i0 + iw;
  const size_t is = (size_t)limbs << log_n, gs = (size_t)inputs * is;
#pragma unroll
  for (int g = 0; g < GPT; ++g) {
    const int gg = g0 + gq * GPT + g;
    if (gg >= G) break;
#pragma unroll
    for (int c = 0; c < 2; ++c) {
      const u64 r = (A.sa[c * GPT + g] << 30) | A.s00[c * GPT + g];  // the last fold left the canonical residue
      res[((size_t)c * G + gg) * gs + (size_t)i * is + lpos + lane] = r;
    }
  }
}

constexpr int kMacTile1 = 12;   // default tiles (IW x GPT) for one and two inputs
constexpr int kMacTile2 = 24;

template <int IW, int GPT, int GG = kMacGG>
static int launch_mac3(u64* res, const InPtrs& in, long long bstride, int nb, int inputs, int groups, const u64* pts,
                       long long pstride, int limbs, const ModSrc& ms, int log_n, int n, cudaStream_t st) {
  using Geo = M3Geom<IW, GPT, GG>;
  cudaError_t e = set_smem_once((const void*)k_bsgs_mac3<IW, GPT, GG>, Geo::SMEM);
  if (e != cudaSuccess) return (int)e;
  dim3 grid((unsigned)((n / 32) * ((inputs + IW - 1) / IW)), (unsigned)limbs, (unsigned)((groups + GG - 1) / GG));
  count_launch();
  k_bsgs_mac3<IW, GPT, GG><<<grid, Geo::THREADS, Geo::SMEM, st>>>(res, in, bstride, nb, inputs, groups, pts, pstride,
                                                                   limbs, ms, log_n);
  return (int)cudaGetLastError();
}

int bsgs_mac(ModSrc ms, u64* res, const u64* const* c0s, const u64* const* c1s,
             long long bstride, int nb, int inputs, const u64* pts, long long pstride, int groups, int limbs, int n,
             cudaStream_t st) {
  if (inputs < 1 || inputs > kMaxInputs) return -1;
  if (nb < 1) return -2;
  if (groups < 1) return -3;
  if (n < 1024 || (n & (n - 1))) return -5;
  int log_n = 0;
  while ((1 << log_n) < n) ++log_n;
  InPtrs in;
  for (int i = 0; i < kMaxInputs; ++i) {
    in.c0[i] = c0s[i < inputs ? i : 0];
    in.c1[i] = c1s[i < inputs ? i : 0];
  }
  // HOLMES_MAC_TC=1 selects the tensor-core kernel (mac_tc.cu) for the shapes it takes.  It is bit-exact but
  // measured slower than k_bsgs_mac3 at the bench shape (20 vs 10.5 ms per 512-row chunk of 16 ciphertexts): with
  // 4 coefficients per item (TMEM holds two items' accumulators) its operand gathers are 32-byte sectors from
  // 2560 rows per item and it stays latency-bound on them (tensor pipe ~2% busy).
  const char* tc = getenv("HOLMES_MAC_TC");
  if (tc && tc[0] == '1') {
    int lg = 0;
    while ((1 << lg) < n) ++lg;
    const int r = bsgs_mac_tc(ms, res, in, bstride, nb, inputs, pts, pstride, groups, limbs, lg, st);
    if (r != -7) return r;
  }
  if (getenv("HOLMES_MAC_V1")) {  // the first-generation kernel, kept for A/B timing
    constexpr int TG = 8;
    dim3 grid((unsigned)((n / 32) * ((inputs + 7) / 8)), (unsigned)limbs, (unsigned)((groups + TG - 1) / TG));
    count_launch();
    k_bsgs_mac<TG><<<grid, 256, 0, st>>>(res, in, bstride, nb, inputs, groups, pts, pstride, limbs, ms, log_n);
    return (int)cudaGetLastError();
  }
  dim3 grid((unsigned)((n / 32) * ((inputs + kMacIW - 1) / kMacIW)), (unsigned)limbs,
            (unsigned)((groups + kMacGG - 1) / kMacGG));
  // cp.async moves 16-byte chunks: every staged row must start on a 16-byte boundary
  bool aligned = ((uintptr_t)pts % 16 == 0) && (pstride % 2 == 0) && (bstride % 2 == 0);
  for (int i = 0; i < inputs; ++i) aligned = aligned && ((uintptr_t)in.c0[i] % 16 == 0) && ((uintptr_t)in.c1[i] % 16 == 0);
  if (!aligned || getenv("HOLMES_MAC_V2")) {
    const int smem = 2 * kMacStageWords * 8;
    cudaError_t e = set_smem_once((const void*)k_bsgs_mac2, smem);
    if (e != cudaSuccess) return (int)e;
    count_launch();
    k_bsgs_mac2<<<grid, 256, smem, st>>>(res, in, bstride, nb, inputs, groups, pts, pstride, limbs, ms, log_n);
    return (int)cudaGetLastError();
  }
  // the tile's inputs match the call's: a 4-input tile given one input leaves three quarters of its warps idle (the
  // reference's operators MAC one ciphertext per call)
  const char* cfg = getenv("HOLMES_MAC_TILE");  // A/B timing of tile shapes: "IWxGPT"
  const int c = cfg && cfg[0] && cfg[1] == 'x' ? atoi(cfg) * 10 + atoi(cfg + 2)
                                                : (inputs == 1 ? kMacTile1 : inputs == 2 ? kMacTile2 : 44);
  // one giant (a bootstrap transform level: the diagonals of one level summed): a tile of one giant per block, not
  // eight copies of it
  if (!(cfg && cfg[0]) && groups == 1 && inputs == 1)
    return launch_mac3<1, 1, 1>(res, in, bstride, nb, inputs, groups, pts, pstride, limbs, ms, log_n, n, st);
  switch (c) {
    case 11: return launch_mac3<1, 1>(res, in, bstride, nb, inputs, groups, pts, pstride, limbs, ms, log_n, n, st);
    case 12: return launch_mac3<1, 2>(res, in, bstride, nb, inputs, groups, pts, pstride, limbs, ms, log_n, n, st);
    case 14: return launch_mac3<1, 4>(res, in, bstride, nb, inputs, groups, pts, pstride, limbs, ms, log_n, n, st);
    case 22: return launch_mac3<2, 2>(res, in, bstride, nb, inputs, groups, pts, pstride, limbs, ms, log_n, n, st);
    case 24: return launch_mac3<2, 4>(res, in, bstride, nb, inputs, groups, pts, pstride, limbs, ms, log_n, n, st);
    case 42: return launch_mac3<4, 2>(res, in, bstride, nb, inputs, groups, pts, pstride, limbs, ms, log_n, n, st);
    default: return launch_mac3<4, 4>(res, in, bstride, nb, inputs, groups, pts, pstride, limbs, ms, log_n, n, st);
  }
}

// --------------------------------------------------------------------------------------------- gathered MAC
// The attention sparse-BSGS MAC (the reference's holmes_mac_gather, bench/cmp/kernels/holmes_mac.cu:276-347): group k
// sums rows seg[k] <= r < seg[k + 1], row r multiplying plaintext row prow[r] by baby idx[r] of every input:
//   res[c][k][i][l][n] = sum_r pts[prow[r]][l][n] * baby_i[idx[r]][c][l][n]  (mod q_l).
// Grid (N / 256 * input tiles, limbs, K); TI inputs per thread, both components; radix-2^30 split products, sums
// restarted from a representative below 8 q every 16 rows, canonical at the end (the same residues).
template <int TI>
__global__ void __launch_bounds__(256) k_mac_gather(u64* __restrict__ res, InPtrs in, long long bstride,
                                                    const int* __restrict__ idx, const int* __restrict__ prow,
                                                    const int* __restrict__ seg, int inputs, int K,
                                                    const u64* __restrict__ pts, long long pstride, int limbs,
                                                    ModSrc ms, int log_n) {
  const int ntile = (inputs + TI - 1) / TI;
  const int n = (blockIdx.x / ntile) * 256 + threadIdx.x, i0 = (blockIdx.x % ntile) * TI;
  const int limb = blockIdx.y, k = blockIdx.z;
  const Mod m = ms.get(limb);
  const size_t ln = ((size_t)limb << log_n) + n;
  const int r0 = seg[k], r1 = seg[k + 1];
  Split4 acc[TI][2];
  const u64* cp[TI][2];
#pragma unroll
  for (int t = 0; t < TI; ++t) {
    const int i = i0 + t < inputs ? i0 + t : i0;
    cp[t][0] = in.c0[i] + ln;
    cp[t][1] = in.c1[i] + ln;
#pragma unroll
    for (int c = 0; c < 2; ++c) acc[t][c] = Split4{0, 0, 0, 0};
  }
  for (int r = r0, cnt = 1; r < r1; ++r, ++cnt) {
    const u64 w = pts[(size_t)prow[r] * pstride + ln];
    const size_t bo = (size_t)idx[r] * bstride;
#pragma unroll
    for (int t = 0; t < TI; ++t)
#pragma unroll
      for (int c = 0; c < 2; ++c) split_mac(acc[t][c], cp[t][c][bo], w);
    if ((cnt & 15) == 0 && r + 1 < r1) {
#pragma unroll
      for (int t = 0; t < TI; ++t)
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          const u64 v = fold_split_lazy(acc[t][c], m);
          acc[t][c] = Split4{v & ((1ull << 30) - 1), v >> 30, 0, 0};
        }
    }
  }
  const size_t is = (size_t)limbs << log_n, gs = (size_t)inputs * is;
#pragma unroll
  for (int t = 0; t < TI; ++t) {
    const int i = i0 + t;
    if (i >= inputs) break;
#pragma unroll
    for (int c = 0; c < 2; ++c) res[((size_t)c * K + k) * gs + (size_t)i * is + ln] = fold_split(acc[t][c], m);
  }
}
int mac_gather(ModSrc ms, u64* res, const u64* const* c0s, const u64* const* c1s, long long bstride, const int* idx,
               const int* prow, const int* seg, int inputs, int K, const u64* pts, long long pstride, int ti,
               int limbs, int log_n, cudaStream_t st) {
  if (inputs < 1 || inputs > kMaxInputs) return -1;
  if (K < 1 || K > 65535) return -3;
  if (limbs < 1 || log_n < 8) return -2;
  InPtrs in;
  for (int i = 0; i < kMaxInputs; ++i) {
    in.c0[i] = c0s[i < inputs ? i : 0];
    in.c1[i] = c1s[i < inputs ? i : 0];
  }
  const unsigned nblk = (1u << log_n) / 256;
#define L_(TI)                                                                                                  \
  {                                                                                                             \
    count_launch();                                                                                             \
    k_mac_gather<TI><<<dim3(nblk * ((inputs + TI - 1) / TI), limbs, K), 256, 0, st>>>(                          \
        res, in, bstride, idx, prow, seg, inputs, K, pts, pstride, limbs, ms, log_n);                           \
    return (int)cudaGetLastError();                                                                             \
  }
  if (ti == 1) L_(1)
  if (ti == 2) L_(2)
  if (ti == 4) L_(4)
#undef L_
  return -4;
}

// --------------------------------------------------------------------------------------------- special FFT
// Inverse CKKS embedding of `slots` complex values per row (Cheon-Kim-Kim-Song 2017 "special FFT"):
// butterfly sweeps len = slots .. 2 with twiddle ksi[(4 len - rot[j] mod 4 len) * M / (4 len)], then
// bit reversal and a 1 / slots scale.  Every double operation is written out with _rn intrinsics in
// the same order as the CPU restatement, so both produce identical bits.
// One butterfly of stage `len` on the pair (x, x + len / 2), x the lower index: j = x mod len / 2, root
// ksi[(4 len - rot[j] mod 4 len) M / (4 len)], read from the per-stage table (context.cu).
__device__ __forceinline__ void fft_bfly(double2& a, double2& b, int j, int len, const double2* __restrict__ ftw) {
  const double2 w = ftw[(len >> 1) - 1 + j];
  const double wr = w.x, wi = w.y;
  const double ur = __dadd_rn(a.x, b.x), ui = __dadd_rn(a.y, b.y);
  const double vr = __dsub_rn(a.x, b.x), vi = __dsub_rn(a.y, b.y);
  const double p1 = __dmul_rn(vr, wr), p2 = __dmul_rn(vi, wi), p3 = __dmul_rn(vr, wi), p4 = __dmul_rn(vi, wr);
  a = make_double2(ur, ui);
  b = make_double2(__dsub_rn(p1, p2), __dadd_rn(p3, p4));
}
// One CTA per row.  Stages whose pairs lie more than kFftBlock apart run first as one pass over global memory
// (each thread takes the 2^G elements x0 + m kFftBlock, G <= 3, through all G of them); then each block of
// kFftBlock consecutive elements is staged in shared memory for the remaining stages (they stay inside it), and
// the bit reversal with the 1 / slots scale ends the row.  Same butterflies in the same stage order as the
// one-sweep-per-stage form, so the same bits.
constexpr int kFftBlock = 4096;  // complex elements: 64 KB of shared memory
__global__ void __launch_bounds__(512) k_fft_special_inv(double* __restrict__ z, long long row_stride, int slots,
                                                         int log_slots, const double2* __restrict__ ftw) {
  extern __shared__ double2 fb[];
  double2* r = reinterpret_cast<double2*>(z + blockIdx.x * row_stride);
  const int bs = slots < kFftBlock ? slots : kFftBlock;
  // global stages: len = slots .. 2 bs
  if (slots > bs) {
    const int G = log_slots - 12;  // 1..3 (slots <= 2^15)
    const int groups = slots >> G;  // = bs
    for (int x0 = threadIdx.x; x0 < groups; x0 += blockDim.x) {
      double2 v[8];
      for (int m = 0; m < (1 << G); ++m) v[m] = r[x0 + m * bs];
      for (int g = G - 1; g >= 0; --g) {  // len = bs 2^(g+1), pairs m, m + 2^g
        const int len = bs << (g + 1), half = len >> 1;
        for (int m = 0; m < (1 << G); ++m) {
          if (m & (1 << g)) continue;
          const int x = x0 + m * bs;
          fft_bfly(v[m], v[m + (1 << g)], x & (half - 1), len, ftw);
        }
      }
      for (int m = 0; m < (1 << G); ++m) r[x0 + m * bs] = v[m];
    }
    __syncthreads();
  }
  // block stages: len = bs .. 2 inside each block of bs elements
  for (int base = 0; base < slots; base += bs) {
    for (int i = threadIdx.x; i < bs; i += blockDim.x) fb[i] = r[base + i];
    __syncthreads();
    for (int len = bs; len >= 2; len >>= 1) {
      const int half = len >> 1;
      for (int t = threadIdx.x; t < bs / 2; t += blockDim.x) {
        const int j = t & (half - 1);
        const int i = (t / half) * len;
        fft_bfly(fb[i + j], fb[i + j + half], j, len, ftw);
      }
      __syncthreads();
    }
    for (int i = threadIdx.x; i < bs; i += blockDim.x) r[base + i] = fb[i];
    __syncthreads();
  }
  const double inv = 1.0 / (double)slots;
  for (int i = threadIdx.x; i < slots; i += blockDim.x) {
    const int j = (int)(__brev((unsigned)i) >> (32 - log_slots));
    if (i < j) {
      const double2 a = r[i], b = r[j];
      r[i] = make_double2(__dmul_rn(b.x, inv), __dmul_rn(b.y, inv));
      r[j] = make_double2(__dmul_rn(a.x, inv), __dmul_rn(a.y, inv));
    } else if (i == j) {
      const double2 a = r[i];
      r[i] = make_double2(__dmul_rn(a.x, inv), __dmul_rn(a.y, inv));
    }
  }
}

int fft_special_inv(const HolmesCtx& c, double* z, long long row_stride, int rows, int slots, cudaStream_t st) {
  if (slots < 2 || slots > c.n / 2 || (slots & (slots - 1))) return -3;
  if (slots > 8 * kFftBlock) return -3;
  if (rows < 1) return 0;
  int log_slots = 0;
  while ((1 << log_slots) < slots) ++log_slots;
  const int bs = slots < kFftBlock ? slots : kFftBlock;
  const int threads = bs / 2 < 512 ? (bs / 2 < 32 ? 32 : bs / 2) : 512;
  const size_t smem = (size_t)bs * sizeof(double2);
  HOLMES_CUDA_TRY(set_smem_once((const void*)k_fft_special_inv, (int)smem));
  count_launch();
  k_fft_special_inv<<<rows, threads, smem, st>>>(z, row_stride, slots, log_slots,
                                                 reinterpret_cast<const double2*>(c.d_fft_tw));
  return (int)cudaGetLastError();
}

// --------------------------------------------------------------------------------------------- packing
// Diagonal rows of one chunk (llama3fhe/operators/linear/weight.py:122-154,
// gpu_packer.py:157-200): row(g, b)[s] = W[(f - g B) mod D, (f + b + lane_shift lane) mod D],
// f = s / lanes, lane = s % lanes, g = giant_base + row / B, b = row % B.  Output complex
// interleaved [rows][slots][2]; a real weight gives zero imaginary parts.
// weight kind: 0 float64 real, 1 complex128, 2 float32 real (widened exactly to double)
__global__ void k_pack(const double* __restrict__ w, int kind, int dim, int lanes, int baby, int giant_base,
                       int lane_shift, int slots, double* __restrict__ out, long long row_stride) {
  const int row = blockIdx.y;
  const int g = giant_base + row / baby, b = row % baby;
  double2* o = reinterpret_cast<double2*>(out + row * row_stride);
  for (int s = blockIdx.x * blockDim.x + threadIdx.x; s < slots; s += gridDim.x * blockDim.x) {
    const int f = s / lanes, lane = s - f * lanes;
    int of = (f - g * baby) % dim;
    if (of < 0) of += dim;
    const int inf = (int)(((long long)f + b + (long long)lane_shift * lane) % dim);
    const long long idx = (long long)of * dim + inf;
    if (kind == 1)
      o[s] = reinterpret_cast<const double2*>(w)[idx];
    else if (kind == 2)
      o[s] = make_double2((double)reinterpret_cast<const float*>(w)[idx], 0.0);
    else
      o[s] = make_double2(w[idx], 0.0);
  }
}
int pack_diagonals(const double* weight, int weight_complex, int dim, int lanes, int baby, int giant_base,
                   int giant_count, int lane_shift, int slots, double* out, long long row_stride, cudaStream_t st) {
  if (dim < 1 || lanes < 1 || baby < 1 || giant_count < 1 || giant_base < 0) return -2;
  if (weight_complex < 0 || weight_complex > 2) return -2;
  dim3 grid((unsigned)((slots + 255) / 256 < 64 ? (slots + 255) / 256 : 64), (unsigned)(giant_count * baby));
  count_launch();
  k_pack<<<grid, 256, 0, st>>>(weight, weight_complex, dim, lanes, baby, giant_base, lane_shift, slots, out,
                               row_stride);
  return (int)cudaGetLastError();
}

// Structured diagonal rows: the physical square map is never built.  Output row r = physical row `of` of the
// square matrix takes its real part from source real_source[of] at logical row real_row[of] (scaled by
// real_scale[of]) and its imaginary part likewise; physical column `inf` reads logical columns real_column[inf] /
// imag_column[inf] (negative = zero) scaled by column_scale[inf].  Sources are float32 or float64 matrices with
// element strides.
__device__ __forceinline__ double struct_load(const StructSources& S, long long src, long long row, long long col) {
  if (src < 0 || src >= S.count || col < 0) return 0.0;
  const long long off = row * S.row_stride[src] + col * S.col_stride[src];
  return S.fp32 ? (double)reinterpret_cast<const float*>(S.p[src])[off]
                : reinterpret_cast<const double*>(S.p[src])[off];
}
__global__ void k_pack_structured(StructSources S, StructMaps M, int dim, int lanes, int baby, int giant_base,
                                  int lane_shift, int slots, double* __restrict__ out, long long row_stride) {
  const int row = blockIdx.y;
  const int g = giant_base + row / baby, b = row % baby;
  double2* o = reinterpret_cast<double2*>(out + row * row_stride);
  for (int s = blockIdx.x * blockDim.x + threadIdx.x; s < slots; s += gridDim.x * blockDim.x) {
    const int f = s / lanes, lane = s - f * lanes;
    int of = (f - g * baby) % dim;
    if (of < 0) of += dim;
    const int inf = (int)(((long long)f + b + (long long)lane_shift * lane) % dim);
    const double cs = M.column_scale[inf];
    double re = struct_load(S, M.real_source[of], M.real_row[of], M.real_column[inf]);
    double im = struct_load(S, M.imag_source[of], M.imag_row[of], M.imag_column[inf]);
    re = __dmul_rn(re, __dmul_rn(M.real_scale[of], cs));
    im = __dmul_rn(im, __dmul_rn(M.imag_scale[of], cs));
    o[s] = make_double2(re, im);
  }
}
int pack_structured(const StructSources& S, const StructMaps& M, int dim, int lanes, int baby, int giant_base,
                    int giant_count, int lane_shift, int slots, double* out, long long row_stride, cudaStream_t st) {
  if (dim < 1 || lanes < 1 || baby < 1 || giant_count < 1 || giant_base < 0) return -2;
  if (S.count < 1 || S.count > 3) return -2;
  dim3 grid((unsigned)((slots + 255) / 256 < 64 ? (slots + 255) / 256 : 64), (unsigned)(giant_count * baby));
  count_launch();
  k_pack_structured<<<grid, 256, 0, st>>>(S, M, dim, lanes, baby, giant_base, lane_shift, slots, out, row_stride);
  return (int)cudaGetLastError();
}

// --------------------------------------------------------------------------------------------- mod-q sum
constexpr int kMaxSrc = 16;
struct SrcPtrs {
  const u64* p[kMaxSrc];
};
__global__ void k_modsum(SrcPtrs s, int nsrc, u64* __restrict__ out, int items, int limbs, long long item_stride,
                         int log_n, const Mod* __restrict__ mods) {
  const size_t per_item = (size_t)limbs << log_n;
  const size_t total = (size_t)items * per_item / 2;
  for (size_t t = blockIdx.x * (size_t)blockDim.x + threadIdx.x; t < total; t += (size_t)gridDim.x * blockDim.x) {
    const size_t w = 2 * t;
    const unsigned wl = (unsigned)(w >> log_n);  // item * limbs + limb (32-bit division)
    const int item = (int)(wl / (unsigned)limbs), limb = (int)(wl - (unsigned)item * limbs);
    const size_t r = ((size_t)limb << log_n) | (w & (((size_t)1 << log_n) - 1));
    const u64 q = mods[limb].q;
    const size_t off = item * item_stride + r;
    u64 a = 0, b = 0;
    for (int k = 0; k < nsrc; ++k) {
      const ulonglong2 x = *reinterpret_cast<const ulonglong2*>(s.p[k] + off);
      a = add_mod(a, x.x, q);
      b = add_mod(b, x.y, q);
    }
    *reinterpret_cast<ulonglong2*>(out + off) = make_ulonglong2(a, b);
  }
}
int modsum(const HolmesCtx& c, const u64* const* srcs, int nsrc, u64* out, int items, int limbs, long long item_stride,
           cudaStream_t st) {
  if (nsrc < 1 || nsrc > kMaxSrc) return -2;
  SrcPtrs s;
  for (int k = 0; k < kMaxSrc; ++k) s.p[k] = srcs[k < nsrc ? k : 0];
  const size_t work = ((size_t)items * limbs * c.n) / 2;
  k_modsum<<<grid_for(work, 256), 256, 0, st>>>(s, nsrc, out, items, limbs, item_stride, c.log_n, c.d_mod);
  return (int)cudaGetLastError();
}

}  // namespace holmes
