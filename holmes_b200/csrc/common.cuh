// Shared types and 64-bit modular arithmetic for libholmes_cuda (sm_100a).
//
// Residues are uint64 words of primes q < 2^60 (the reference's 59/60-bit production primes and
// the ~50-bit sweep primes).  Three reductions are used:
//   * Shoup multiplication by a constant w with w' = floor(w 2^64 / q): a w - floor(a w' / 2^64) q
//     lies in [0, 2q) for every a < 2^64;
//   * Barrett reduction of a 128-bit x with mu = floor(2^k / q), k = floor(log2 q) + 63 (the
//     reference's ctx.barret_ratio / barret_k convention, bench/cmp/kernels/holmes_mac.cu:23-40):
//     est = floor(x mu / 2^k) (computed exactly from the top 128 bits of x mu) undershoots
//     floor(x / q) by less than x / 2^k + 1, so for x < 14 2^k -- e.g. 16 products of canonical
//     residues with q < 2^60, or 12 products of a 60-bit source residue with a 50-bit target
//     constant -- the remainder x - est q stays below 16 q < 2^64 and four conditional
//     subtractions (8q, 4q, 2q, q) make it canonical;
//   * radix-2^30 split sums (Split4) reduce through a cheaper Barrett on the top 66 bits (reduce_wide);
//   * the NTT butterflies use a three-product Shoup estimate (shoup_lazy4) and keep lazy values below
//     8q (forward) / 4q (inverse), Harvey-style.
#pragma once
#include <atomic>
#include <cstdint>
#include <map>
#include <mutex>
#include <utility>
#include <cuda_runtime.h>

namespace holmes {

// Kernels launched by this library since load (read through holmes_launch_count).
inline std::atomic<unsigned long long>& launch_counter() {
  static std::atomic<unsigned long long> c{0};
  return c;
}
inline void count_launch() { launch_counter().fetch_add(1, std::memory_order_relaxed); }

// Raise a kernel's dynamic shared memory limit once per device: the attribute stays set on the function for the
// context, so later launches skip the driver call.
inline cudaError_t set_smem_once(const void* fn, int bytes) {
  static std::mutex mu;
  static std::map<std::pair<int, const void*>, int> done;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  std::lock_guard<std::mutex> g(mu);
  auto it = done.find({dev, fn});
  if (it != done.end() && it->second >= bytes) return cudaSuccess;
  e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess) done[{dev, fn}] = bytes;
  return e;
}

typedef uint64_t u64;
typedef int64_t i64;
typedef uint32_t u32;

// A constant and its Shoup companion, stored together so one 16-byte load fetches both.
struct __align__(16) Tw {
  u64 w, ws;
};

struct Mod {
  u64 q;      // prime
  u64 mu;     // floor(2^k / q)
  u32 shift;  // k - 64 = floor(log2 q) - 1
  u32 pad;
};

__device__ __forceinline__ u64 add_mod(u64 a, u64 b, u64 q) {
  u64 s = a + b;
  return s >= q ? s - q : s;
}
__device__ __forceinline__ u64 sub_mod(u64 a, u64 b, u64 q) { return a >= b ? a - b : a + q - b; }

// Modulus of limb l either from a context table or from the reference's three per-limb arrays
// (ctx.primes / ctx.barret_ratio / ctx.barret_k, bench/cmp/holmes_multi_mac.py:140-141).
struct ModSrc {
  const Mod* mods;
  int first;
  const u64* primes;
  const u64* ratios;
  const u64* ks;
  int ext_cur = 0;  // > 0: limb l >= ext_cur is special limb ext_L + l - ext_cur (extended basis Q u P)
  int ext_L = 0;
  __device__ __forceinline__ Mod get(int limb) const {
    if (mods) return mods[ext_cur > 0 && limb >= ext_cur ? ext_L + limb - ext_cur : first + limb];
    Mod m;
    m.q = primes[limb];
    m.mu = ratios[limb];
    m.shift = (u32)(ks[limb] - 64);
    m.pad = 0;
    return m;
  }
};

// a * w mod q, result in [0, 2q)
__device__ __forceinline__ u64 shoup_lazy(u64 a, Tw t, u64 q) {
  const u64 hi = __umul64hi(a, t.ws);
  return a * t.w - hi * q;
}
// a * w mod q in [0, 4q) with three of the four 32 x 32 partial products of a w': dropping
// hi(a0 w'0) and the carries of the middle column makes the quotient at most 2 short.  The 32-bit
// wide/high multiplies issue at quarter rate on sm_100, so this saves a quarter of the quotient cost.
__device__ __forceinline__ u64 shoup_lazy4(u64 a, Tw t, u64 q) {
  const uint32_t a0 = (uint32_t)a, a1 = (uint32_t)(a >> 32);
  const uint32_t s0 = (uint32_t)t.ws, s1 = (uint32_t)(t.ws >> 32);
  const u64 qt = (u64)a1 * s1 + __umulhi(a0, s1) + __umulhi(a1, s0);
  return a * t.w - qt * q;
}
__device__ __forceinline__ u64 shoup(u64 a, Tw t, u64 q) {
  const u64 r = shoup_lazy(a, t, q);
  return r >= q ? r - q : r;
}

// 128-bit accumulator helpers
struct U128 {
  u64 lo, hi;
};
__device__ __forceinline__ void mac128(U128& acc, u64 a, u64 b) {
  const u64 plo = a * b, phi = __umul64hi(a, b);
  asm("add.cc.u64 %0, %0, %2;\n\taddc.u64 %1, %1, %3;" : "+l"(acc.lo), "+l"(acc.hi) : "l"(plo), "l"(phi));
}

// x = hi:lo mod q for x < 14 2^k (see header)
__device__ __forceinline__ u64 reduce128(u64 hi, u64 lo, const Mod& m) {
  const u64 t0 = __umul64hi(lo, m.mu);
  const u64 t1lo = hi * m.mu, t1hi = __umul64hi(hi, m.mu);
  u64 mid, top;
  asm("add.cc.u64 %0, %2, %3;\n\taddc.u64 %1, %4, 0;" : "=l"(mid), "=l"(top) : "l"(t0), "l"(t1lo), "l"(t1hi));
  const u64 est = (mid >> m.shift) | (top << (64 - m.shift));
  u64 r = lo - est * m.q;
  const u64 q = m.q;
  if (r >= (q << 3)) r -= (q << 3);
  if (r >= (q << 2)) r -= (q << 2);
  if (r >= (q << 1)) r -= (q << 1);
  if (r >= q) r -= q;
  return r;
}
// the same estimate without the conditional subtractions: a representative of x mod q in [0, 16 q)
__device__ __forceinline__ u64 reduce128_lazy(u64 hi, u64 lo, const Mod& m) {
  const u64 t0 = __umul64hi(lo, m.mu);
  const u64 t1lo = hi * m.mu, t1hi = __umul64hi(hi, m.mu);
  u64 mid, top;
  asm("add.cc.u64 %0, %2, %3;\n\taddc.u64 %1, %4, 0;" : "=l"(mid), "=l"(top) : "l"(t0), "l"(t1lo), "l"(t1hi));
  const u64 est = (mid >> m.shift) | (top << (64 - m.shift));
  return lo - est * m.q;
}
__device__ __forceinline__ u64 mul_mod(u64 a, u64 b, const Mod& m) { return reduce128(__umul64hi(a, b), a * b, m); }
__device__ __forceinline__ u64 reduce128(const U128& x, const Mod& m) { return reduce128(x.hi, x.lo, m); }

// Radix-2^30 partial-product sums.  A residue below 2^60 splits as a1 2^30 + a0 (a0, a1 < 2^30); the four
// partial products of two such residues are below 2^60, so up to 16 of each accumulate in one 64-bit word
// (one fused 32 x 32 -> 64-bit wide multiply-add each).  V = S00 + (SA + SB) 2^30 + S11 2^60.
struct Split4 {
  u64 s00, sa, sb, s11;
};
__device__ __forceinline__ void split_fold128(const Split4& acc, u64& hi, u64& lo) {
  lo = acc.s00;
  hi = 0;
  const u64 a_lo = acc.sa << 30, a_hi = acc.sa >> 34;
  const u64 b_lo = acc.sb << 30, b_hi = acc.sb >> 34;
  const u64 c_lo = acc.s11 << 60, c_hi = acc.s11 >> 4;
  asm("add.cc.u64 %0, %0, %2;\n\taddc.u64 %1, %1, %3;" : "+l"(lo), "+l"(hi) : "l"(a_lo), "l"(a_hi));
  asm("add.cc.u64 %0, %0, %2;\n\taddc.u64 %1, %1, %3;" : "+l"(lo), "+l"(hi) : "l"(b_lo), "l"(b_hi));
  asm("add.cc.u64 %0, %0, %2;\n\taddc.u64 %1, %1, %3;" : "+l"(lo), "+l"(hi) : "l"(c_lo), "l"(c_hi));
}
// acc += a b in split form, for a, b < 2^60
__device__ __forceinline__ void split_mac(Split4& acc, u64 a, u64 b) {
  const uint32_t a0 = (uint32_t)a & ((1u << 30) - 1), a1 = (uint32_t)(a >> 30);
  const uint32_t b0 = (uint32_t)b & ((1u << 30) - 1), b1 = (uint32_t)(b >> 30);
  acc.s00 += (u64)a0 * b0;
  acc.sa += (u64)a0 * b1;
  acc.sb += (u64)a1 * b0;
  acc.s11 += (u64)a1 * b1;
}
// x = hi:lo mod q as a representative in [0, 8 q), for x < 2^(66 + shift) (shift = floor(log2 q) - 1): e.g. 16
// products of residues below 2^60 with residues of q, plus a representative below 8 q.  Classic Barrett on the
// top bits: t = floor(x / 2^shift) < 2^66 and est = floor(t mu / 2^64), mu = floor(2^(shift + 64) / q) <= 2^63,
// taken as t's top two bits times mu plus three of the four 32 x 32 partial products of t's low word and mu.
// Truncating x and mu costs est at most 4 + 1/2 (x / 2^(shift + 64) < 4, 2^shift / q <= 1/2), the dropped
// product and carries at most 2 more, so est >= floor(x / q) - 7 and x - est q < 8 q.  Five quarter-rate
// multiplies against twelve for reduce128.
__device__ __forceinline__ u64 reduce_wide_lazy(u64 hi, u64 lo, const Mod& m) {
  const uint32_t sh = m.shift;
  const u64 t = (lo >> sh) | (hi << (64 - sh));
  const uint32_t th = (uint32_t)(hi >> sh);  // < 4
  const uint32_t t0 = (uint32_t)t, t1 = (uint32_t)(t >> 32);
  const uint32_t m0 = (uint32_t)m.mu, m1 = (uint32_t)(m.mu >> 32);
  u64 est = (u64)t1 * m1 + __umulhi(t0, m1) + __umulhi(t1, m0);
  est += (u64)th * m.mu;
  return lo - est * m.q;
}
__device__ __forceinline__ u64 reduce_wide(u64 hi, u64 lo, const Mod& m) {
  u64 r = reduce_wide_lazy(hi, lo, m);
  const u64 q = m.q;
  if (r >= (q << 2)) r -= (q << 2);
  if (r >= (q << 1)) r -= (q << 1);
  if (r >= q) r -= q;
  return r;
}
// V mod q, canonical, for V < 2^(66 + shift) (e.g. 16 products of residues below 2^60 and q)
__device__ __forceinline__ u64 fold_split(const Split4& acc, const Mod& m) {
  u64 hi, lo;
  split_fold128(acc, hi, lo);
  return reduce_wide(hi, lo, m);
}
// V mod q as a representative in [0, 8 q): restarting the sums from its split (S00 < 2^30, SA < 2^33) leaves
// room for 16 more products below 2^60 in every sum
__device__ __forceinline__ u64 fold_split_lazy(const Split4& acc, const Mod& m) {
  u64 hi, lo;
  split_fold128(acc, hi, lo);
  return reduce_wide_lazy(hi, lo, m);
}

// bit reversal of the low `bits` bits
__device__ __forceinline__ u32 brev_bits(u32 v, int bits) { return __brev(v) >> (32 - bits); }

// Source word of the NTT-domain automorphism X -> X^g: out[k] = in[perm(k)], where word k holds the
// evaluation at psi^(2 bitrev(k) + 1) (forward NTT with bit-reversed root powers).
__device__ __forceinline__ u32 automorph_src(u32 k, u64 g, int log_n) {
  const u32 mask = (2u << log_n) - 1u;
  const u32 e = (u32)(((2ull * brev_bits(k, log_n) + 1ull) * g) & mask);
  return brev_bits((e - 1u) >> 1, log_n);
}

}  // namespace holmes

#define HOLMES_CUDA_TRY(expr)                         \
  do {                                                \
    cudaError_t _e = (expr);                          \
    if (_e != cudaSuccess) return (int)_e;            \
  } while (0)
