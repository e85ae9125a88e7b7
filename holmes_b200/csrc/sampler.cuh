// Deterministic key / encryption randomness: a ChaCha20 keystream (RFC 8439 block function) keyed by
// the context seed, nonce = (domain, tag, word), block counter = word group.  Host code and kernels
// compute identical values, so a seeded context is reproducible word for word.
//   domain 1 secret, 2 key uniform part, 3 key error, 4 encryption uniform part, 5 encryption error;
//   tag = Galois element (0 for relinearisation) or encryption counter; word = (digit << 16) | modulus
//   index for uniform words, (digit << 16) | 0xFFFF for errors (shared by every modulus).
// Uniform residue of coefficient i: (w[2(i&3)+1] : w[2(i&3)]) of block i/4, a 128-bit value mod q.
// Error of coefficient i: centred binomial with eta = 21 from word i&7 of block i/8.
#pragma once
#include "common.cuh"

namespace holmes {

__device__ __forceinline__ u32 rotl32d(u32 x, int r) { return __funnelshift_l(x, x, r); }

__device__ __forceinline__ void chacha_block(u64 seed, u32 domain, u32 tag, u32 word, u32 counter, u32 out[16]) {
  const u32 s[16] = {0x61707865u, 0x3320646eu, 0x79622d32u, 0x6b206574u, (u32)seed, (u32)(seed >> 32), 0x6d6c6f68u,
                     0x62323030u, 0u, 0u, 0u, 0u, counter, domain, tag, word};
  u32 x[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) x[i] = s[i];
#define DQR(a, b, c, d)                                          \
  x[a] += x[b]; x[d] ^= x[a]; x[d] = rotl32d(x[d], 16);           \
  x[c] += x[d]; x[b] ^= x[c]; x[b] = rotl32d(x[b], 12);           \
  x[a] += x[b]; x[d] ^= x[a]; x[d] = rotl32d(x[d], 8);            \
  x[c] += x[d]; x[b] ^= x[c]; x[b] = rotl32d(x[b], 7);
#pragma unroll 1
  for (int r = 0; r < 10; ++r) {
    DQR(0, 4, 8, 12) DQR(1, 5, 9, 13) DQR(2, 6, 10, 14) DQR(3, 7, 11, 15)
    DQR(0, 5, 10, 15) DQR(1, 6, 11, 12) DQR(2, 7, 8, 13) DQR(3, 4, 9, 14)
  }
#undef DQR
#pragma unroll
  for (int i = 0; i < 16; ++i) out[i] = x[i] + s[i];
}

__device__ __forceinline__ u64 chacha_word(const u32 b[16], int w) { return (u64)b[2 * w] | ((u64)b[2 * w + 1] << 32); }

__device__ __forceinline__ u64 sample_uniform(u64 seed, u32 domain, u32 tag, u32 word, u32 i, const Mod& m) {
  u32 b[16];
  chacha_block(seed, domain, tag, word, i >> 2, b);
  const u64 lo = chacha_word(b, 2 * (i & 3)), hi = chacha_word(b, 2 * (i & 3) + 1);
  return reduce128(reduce128(0, hi, m), lo, m);
}

__device__ __forceinline__ i64 sample_cbd(u64 seed, u32 domain, u32 tag, u32 word, u32 i) {
  u32 b[16];
  chacha_block(seed, domain, tag, word, i >> 3, b);
  const u64 r = chacha_word(b, i & 7), m21 = (1ull << 21) - 1;
  return (i64)__popcll(r & m21) - (i64)__popcll((r >> 21) & m21);
}

__device__ __forceinline__ u64 signed_residue(i64 v, const Mod& m) {
  if (v >= 0) return reduce128(0, (u64)v, m);
  const u64 r = reduce128(0, (u64)(-v), m);
  return r ? m.q - r : 0;
}

}  // namespace holmes
