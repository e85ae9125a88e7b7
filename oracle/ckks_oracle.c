/*
 * ckks_oracle.c -- CPU restatement of the RNS-CKKS arithmetic on the Holmes hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the product (holmes_b200/, libholmes_cuda) links,
 * loads or calls this file; only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline
 * leg (and `bench.py --impl reference`) use it, as the checker and as the timed CPU baseline.
 *
 * Every routine is written for clarity first: exact 128-bit arithmetic (`% q`) instead of the
 * Barrett/Shoup tricks of the CUDA kernels, so a residue computed here is the canonical value in
 * [0, q) that any correct implementation of the same mathematical definition must produce.
 * The conventions follow the reference's own kernels, which document EasyFHE's:
 *   - Barrett constants ratio = floor(2^k / p), k = floor(log2 p) + 63
 *       (bench/cmp/kernels/holmes_mac.cu:23-40, holmes_multi_mac.py:126-128 ctx.barret_ratio/k);
 *   - forward NTT round l pairs n and n + 2^(logN-1-l) with root roots[2^l + (n >> (logN-l))],
 *     roots in bit-reversed power order, outputs canonical (holmes_encode.cu:24-78, 200-226);
 *   - encode: coefficient n < slots is Re(u_n), n >= slots is Im(u_{n-slots}) (gap 1 at full
 *     slots), rounded with llround(v * scale), reduced per limb (holmes_encode.cu:108-159;
 *     bench/cmp/holmes_fast_encode.py:63-112 for the 2^61 range limit);
 *   - MAC: res = sum_b pt[g*B+b] * baby[b] mod q (holmes_mac.cu:1-13, 116-190).
 * The special FFT is the published HEAAN/CKKS embedding (Cheon-Kim-Kim-Song 2017), restated
 * here; EasyFHE's own FFT operation order is not available, so encode parity with the
 * reference binary is unpinned (see the oracle header in oracle/oracle.py).
 *
 * Compiled with -ffp-contract=off so every double operation rounds exactly as written; the
 * CUDA encode uses __dmul_rn/__dadd_rn in the same expression order.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

typedef uint64_t u64;
typedef int64_t i64;
typedef unsigned __int128 u128;

/* ------------------------------------------------------------------ modular basics */
static inline u64 add_mod(u64 a, u64 b, u64 q) { u64 s = a + b; return s >= q ? s - q : s; }
static inline u64 sub_mod(u64 a, u64 b, u64 q) { return a >= b ? a - b : a + q - b; }
static inline u64 mul_mod(u64 a, u64 b, u64 q) { return (u64)(((u128)a * b) % q); }

u64 orc_pow_mod(u64 a, u64 e, u64 q) {
  u64 r = 1 % q;
  a %= q;
  while (e) {
    if (e & 1) r = mul_mod(r, a, q);
    a = mul_mod(a, a, q);
    e >>= 1;
  }
  return r;
}

u64 orc_inv_mod(u64 a, u64 q) { return orc_pow_mod(a, q - 2, q); } /* q prime */

static int miller_rabin(u64 n, u64 a) {
  if (n % a == 0) return n == a;
  u64 d = n - 1;
  int s = 0;
  while ((d & 1) == 0) { d >>= 1; ++s; }
  u64 x = orc_pow_mod(a, d, n);
  if (x == 1 || x == n - 1) return 1;
  for (int i = 1; i < s; ++i) {
    x = mul_mod(x, x, n);
    if (x == n - 1) return 1;
  }
  return 0;
}

int orc_is_prime(u64 n) {
  static const u64 bases[] = {2, 3, 5, 7, 11, 13, 17, 19, 23, 29, 31, 37};
  if (n < 2) return 0;
  for (unsigned i = 0; i < sizeof(bases) / sizeof(bases[0]); ++i)
    if (!miller_rabin(n, bases[i])) return 0;
  return 1;
}

/* Primes q = 1 (mod 2N) below 2^bits, largest first, skipping `exclude`. */
int orc_gen_primes(int log_n, int bits, int count, const u64* exclude, int n_exclude, u64* out) {
  const u64 m = 2ULL << log_n;
  u64 c = (((1ULL << bits) - 1) / m) * m + 1;
  if (c >= (1ULL << bits)) c -= m;
  int found = 0;
  while (found < count && c > m) {
    int skip = 0;
    for (int i = 0; i < n_exclude; ++i) skip |= (exclude[i] == c);
    if (!skip && orc_is_prime(c)) out[found++] = c;
    c -= m;
  }
  return found == count ? 0 : -1;
}

/* Smallest x >= 2 whose x^((q-1)/2N) has order exactly 2N; returns that power (psi). */
u64 orc_find_psi(u64 q, int log_n) {
  const u64 two_n = 2ULL << log_n;
  for (u64 x = 2;; ++x) {
    u64 psi = orc_pow_mod(x, (q - 1) / two_n, q);
    if (orc_pow_mod(psi, two_n >> 1, q) == q - 1) return psi;
  }
}

static inline u64 bitrev(u64 v, int bits) {
  u64 r = 0;
  for (int i = 0; i < bits; ++i) { r = (r << 1) | (v & 1); v >>= 1; }
  return r;
}

/* roots[k] = psi^bitrev(k), iroots[k] = psi^-bitrev(k), k < N. */
void orc_make_roots(u64 q, u64 psi, int log_n, u64* roots, u64* iroots) {
  const u64 n = 1ULL << log_n;
  const u64 ipsi = orc_inv_mod(psi, q);
  u64* pw = (u64*)malloc(sizeof(u64) * n);
  u64* ipw = (u64*)malloc(sizeof(u64) * n);
  pw[0] = 1; ipw[0] = 1;
  for (u64 i = 1; i < n; ++i) { pw[i] = mul_mod(pw[i - 1], psi, q); ipw[i] = mul_mod(ipw[i - 1], ipsi, q); }
  for (u64 k = 0; k < n; ++k) { roots[k] = pw[bitrev(k, log_n)]; iroots[k] = ipw[bitrev(k, log_n)]; }
  free(pw); free(ipw);
}

/* ------------------------------------------------------------------ NTT */
static void ntt_one(u64* a, int log_n, u64 q, const u64* roots) {
  const u64 n = 1ULL << log_n;
  for (u64 m = 1, t = n >> 1; m < n; m <<= 1, t >>= 1) {
    for (u64 i = 0; i < m; ++i) {
      const u64 w = roots[m + i];
      for (u64 j = 2 * i * t; j < 2 * i * t + t; ++j) {
        const u64 u = a[j], v = mul_mod(a[j + t], w, q);
        a[j] = add_mod(u, v, q);
        a[j + t] = sub_mod(u, v, q);
      }
    }
  }
}

static void intt_one(u64* a, int log_n, u64 q, const u64* iroots) {
  const u64 n = 1ULL << log_n;
  for (u64 m = n >> 1, t = 1; m >= 1; m >>= 1, t <<= 1) {
    for (u64 i = 0; i < m; ++i) {
      const u64 w = iroots[m + i];
      for (u64 j = 2 * i * t; j < 2 * i * t + t; ++j) {
        const u64 u = a[j], v = a[j + t];
        a[j] = add_mod(u, v, q);
        a[j + t] = mul_mod(sub_mod(u, v, q), w, q);
      }
    }
  }
  const u64 ninv = orc_inv_mod(n % q, q);
  for (u64 j = 0; j < n; ++j) a[j] = mul_mod(a[j], ninv, q);
}

/* `count` polynomials of N words each, all modulo q. */
void orc_ntt(u64* a, int log_n, u64 q, const u64* roots, int count) {
  const u64 n = 1ULL << log_n;
#pragma omp parallel for schedule(static)
  for (int c = 0; c < count; ++c) ntt_one(a + (u64)c * n, log_n, q, roots);
}

void orc_intt(u64* a, int log_n, u64 q, const u64* iroots, int count) {
  const u64 n = 1ULL << log_n;
#pragma omp parallel for schedule(static)
  for (int c = 0; c < count; ++c) intt_one(a + (u64)c * n, log_n, q, iroots);
}

/* ------------------------------------------------------------------ elementwise */
void orc_add(const u64* a, const u64* b, u64* out, u64 n, u64 q) {
  for (u64 i = 0; i < n; ++i) out[i] = add_mod(a[i], b[i], q);
}
void orc_sub(const u64* a, const u64* b, u64* out, u64 n, u64 q) {
  for (u64 i = 0; i < n; ++i) out[i] = sub_mod(a[i], b[i], q);
}
void orc_mul(const u64* a, const u64* b, u64* out, u64 n, u64 q) {
#pragma omp parallel for schedule(static)
  for (i64 i = 0; i < (i64)n; ++i) out[i] = mul_mod(a[i], b[i], q);
}
void orc_mul_scalar(const u64* a, u64 s, u64* out, u64 n, u64 q) {
  for (u64 i = 0; i < n; ++i) out[i] = mul_mod(a[i], s, q);
}
/* out[i] = (a[i] * b[i] + c[i]) mod q */
void orc_mul_add(const u64* a, const u64* b, const u64* c, u64* out, u64 n, u64 q) {
#pragma omp parallel for schedule(static)
  for (i64 i = 0; i < (i64)n; ++i) out[i] = add_mod(mul_mod(a[i], b[i], q), c[i], q);
}
/* signed integers -> residues */
void orc_reduce_signed(const i64* v, u64* out, u64 n, u64 q) {
  for (u64 i = 0; i < n; ++i) {
    i64 r = v[i] % (i64)q;
    out[i] = (u64)(r < 0 ? r + (i64)q : r);
  }
}

/* ------------------------------------------------------------------ automorphisms
 * A forward-NTT output word k holds the evaluation at psi^(2 bitrev(k) + 1).  X -> X^g maps the
 * evaluation at psi^e to the one at psi^(e g), so out[k] = in[k'] with
 * 2 bitrev(k') + 1 = (2 bitrev(k) + 1) g mod 2N.  g odd. */
void orc_automorph_ntt(const u64* in, u64* out, int log_n, u64 g, int count) {
  const u64 n = 1ULL << log_n, mask = 2 * n - 1;
  for (u64 k = 0; k < n; ++k) {
    const u64 e = ((2 * bitrev(k, log_n) + 1) * g) & mask;
    const u64 src = bitrev((e - 1) >> 1, log_n);
    for (int c = 0; c < count; ++c) out[(u64)c * n + k] = in[(u64)c * n + src];
  }
}
/* coefficient domain: coefficient i moves to i g mod 2N, negated when that lands in [N, 2N) */
void orc_automorph_coeff(const u64* in, u64* out, int log_n, u64 g, u64 q) {
  const u64 n = 1ULL << log_n, mask = 2 * n - 1;
  for (u64 i = 0; i < n; ++i) {
    const u64 j = (i * g) & mask;
    if (j < n) out[j] = in[i];
    else out[j - n] = in[i] ? q - in[i] : 0;
  }
}

/* ------------------------------------------------------------------ fast base conversion
 * in: `na` source limbs (coefficient domain) of N words; inv_hat[k] = (Qhat_k)^-1 mod q_k;
 * hat_mod[k * nb + t] = Qhat_k mod p_t.  out[t][i] = sum_k [in_k[i] inv_hat_k]_{q_k} Qhat_k mod p_t. */
void orc_base_conv(const u64* in, int na, const u64* qa, const u64* inv_hat, int nb, const u64* pb,
                   const u64* hat_mod, u64* out, int log_n) {
  const u64 n = 1ULL << log_n;
#pragma omp parallel for schedule(static)
  for (i64 i = 0; i < (i64)n; ++i) {
    u64 y[64];
    for (int k = 0; k < na; ++k) y[k] = mul_mod(in[(u64)k * n + i], inv_hat[k], qa[k]);
    for (int t = 0; t < nb; ++t) {
      u128 acc = 0;
      for (int k = 0; k < na; ++k) acc += (u128)y[k] * (hat_mod[k * nb + t] % pb[t]);
      out[(u64)t * n + i] = (u64)(acc % pb[t]);
    }
  }
}

/* ------------------------------------------------------------------ BSGS multiply-accumulate
 * res[g][i] = sum_{b<nb} pt[g*nb + b][i] * baby[b][i] mod q over one limb's words: pt [G*nb][n],
 * baby [nb][n] (strides in words), res [G][n]. */
void orc_bsgs_mac(const u64* pt, u64 pt_stride, const u64* baby, u64 baby_stride, int nb, int G, u64* res,
                  u64 res_stride, u64 n, u64 q) {
#pragma omp parallel for schedule(static)
  for (int g = 0; g < G; ++g) {
    for (u64 i = 0; i < n; ++i) {
      u128 acc = 0;
      for (int b = 0; b < nb; ++b) {
        acc += (u128)pt[(u64)(g * nb + b) * pt_stride + i] * baby[(u64)b * baby_stride + i];
        if ((b & 15) == 15) acc %= q;
      }
      res[(u64)g * res_stride + i] = (u64)(acc % q);
    }
  }
}

/* ------------------------------------------------------------------ special FFT (CKKS embedding)
 * rot_group[j] = 5^j mod M (j < N/2), ksi_re/ksi_im[k] = cos/sin(2 pi k / M) (k < M). */
static void bit_reverse_c(double* re, double* im, int n) {
  int bits = 0;
  while ((1 << bits) < n) ++bits;
  for (int i = 0; i < n; ++i) {
    int j = (int)bitrev((u64)i, bits);
    if (i < j) {
      double t = re[i]; re[i] = re[j]; re[j] = t;
      t = im[i]; im[i] = im[j]; im[j] = t;
    }
  }
}

void orc_fft_special_inv(double* re, double* im, int n, u64 m_order, const u64* rot_group, const double* ksi_re,
                         const double* ksi_im) {
  for (int len = n; len >= 2; len >>= 1) {
    const int half = len >> 1;
    const u64 lenq = (u64)len << 2, stride = m_order / lenq;
    for (int i = 0; i < n; i += len) {
      for (int j = 0; j < half; ++j) {
        const u64 k = (lenq - (rot_group[j] % lenq)) * stride;
        const double ar = re[i + j], ai = im[i + j];
        const double br = re[i + j + half], bi = im[i + j + half];
        const double ur = ar + br, ui = ai + bi;
        const double vr = ar - br, vi = ai - bi;
        const double wr = ksi_re[k], wi = ksi_im[k];
        const double p1 = vr * wr, p2 = vi * wi, p3 = vr * wi, p4 = vi * wr;
        re[i + j] = ur; im[i + j] = ui;
        re[i + j + half] = p1 - p2; im[i + j + half] = p3 + p4;
      }
    }
  }
  bit_reverse_c(re, im, n);
  const double inv = 1.0 / (double)n;
  for (int i = 0; i < n; ++i) { re[i] = re[i] * inv; im[i] = im[i] * inv; }
}

void orc_fft_special(double* re, double* im, int n, u64 m_order, const u64* rot_group, const double* ksi_re,
                     const double* ksi_im) {
  bit_reverse_c(re, im, n);
  for (int len = 2; len <= n; len <<= 1) {
    const int half = len >> 1;
    const u64 lenq = (u64)len << 2, stride = m_order / lenq;
    for (int i = 0; i < n; i += len) {
      for (int j = 0; j < half; ++j) {
        const u64 k = (rot_group[j] % lenq) * stride;
        const double br = re[i + j + half], bi = im[i + j + half];
        const double wr = ksi_re[k], wi = ksi_im[k];
        const double p1 = br * wr, p2 = bi * wi, p3 = br * wi, p4 = bi * wr;
        const double vr = p1 - p2, vi = p3 + p4;
        const double ur = re[i + j], ui = im[i + j];
        re[i + j] = ur + vr; im[i + j] = ui + vi;
        re[i + j + half] = ur - vr; im[i + j + half] = ui - vi;
      }
    }
  }
}

/* Tables of the embedding: rot_group (N/2 words) and ksi (M doubles each). */
void orc_fft_tables(int log_n, u64* rot_group, double* ksi_re, double* ksi_im) {
  const u64 n = 1ULL << log_n, m = 2 * n;
  u64 r = 1;
  for (u64 j = 0; j < n / 2; ++j) { rot_group[j] = r; r = (r * 5) % m; }
  for (u64 k = 0; k < m; ++k) {
    const double angle = 2.0 * M_PI * (double)k / (double)m;
    ksi_re[k] = cos(angle);
    ksi_im[k] = sin(angle);
  }
}

/* Encode `slots` complex values at `scale` into N signed integer coefficients.  Returns 0, or -1
 * when a scaled value reaches 2^61 (the reference encoder's limit). */
int orc_encode(const double* z_re, const double* z_im, int slots, int log_n, double scale, const u64* rot_group,
               const double* ksi_re, const double* ksi_im, i64* coeffs) {
  const u64 n = 1ULL << log_n;
  double* re = (double*)malloc(sizeof(double) * slots);
  double* im = (double*)malloc(sizeof(double) * slots);
  memcpy(re, z_re, sizeof(double) * slots);
  memcpy(im, z_im, sizeof(double) * slots);
  orc_fft_special_inv(re, im, slots, 2 * n, rot_group, ksi_re, ksi_im);
  memset(coeffs, 0, sizeof(i64) * n);
  const u64 gap = n / (2 * (u64)slots);
  const double limit = 2305843009213693952.0; /* 2^61 */
  int rc = 0;
  for (int i = 0; i < slots; ++i) {
    const double vr = re[i] * scale, vi = im[i] * scale;
    if (!(fabs(vr) < limit) || !(fabs(vi) < limit)) { rc = -1; break; }
    coeffs[(u64)i * gap] = llround(vr);
    coeffs[(u64)i * gap + n / 2] = llround(vi);
  }
  free(re); free(im);
  return rc;
}

/* Decode N centred coefficients (as doubles) into `slots` complex values. */
void orc_decode(const double* coeffs, int slots, int log_n, double scale, const u64* rot_group, const double* ksi_re,
                const double* ksi_im, double* z_re, double* z_im) {
  const u64 n = 1ULL << log_n;
  const u64 gap = n / (2 * (u64)slots);
  for (int i = 0; i < slots; ++i) {
    z_re[i] = coeffs[(u64)i * gap] / scale;
    z_im[i] = coeffs[(u64)i * gap + n / 2] / scale;
  }
  orc_fft_special(z_re, z_im, slots, 2 * n, rot_group, ksi_re, ksi_im);
}

/* ------------------------------------------------------------------ ChaCha20 (RFC 8439) keyed sampler
 * key = (seed_lo, seed_hi, 0x6d6c6f68, 0x62323030, 0, 0, 0, 0); nonce = (domain, tag, word);
 * the block counter addresses 64-byte blocks of the stream. */
static inline uint32_t rotl32(uint32_t x, int r) { return (x << r) | (x >> (32 - r)); }
#define QR(a, b, c, d)                                   \
  a += b; d ^= a; d = rotl32(d, 16);                     \
  c += d; b ^= c; b = rotl32(b, 12);                     \
  a += b; d ^= a; d = rotl32(d, 8);                      \
  c += d; b ^= c; b = rotl32(b, 7);

void orc_chacha_block(u64 seed, uint32_t domain, uint32_t tag, uint32_t word, uint32_t counter, uint32_t out[16]) {
  uint32_t s[16] = {0x61707865u, 0x3320646eu, 0x79622d32u, 0x6b206574u,
                    (uint32_t)seed, (uint32_t)(seed >> 32), 0x6d6c6f68u, 0x62323030u, 0u, 0u, 0u, 0u,
                    counter, domain, tag, word};
  uint32_t x[16];
  memcpy(x, s, sizeof(x));
  for (int r = 0; r < 10; ++r) {
    QR(x[0], x[4], x[8], x[12]) QR(x[1], x[5], x[9], x[13]) QR(x[2], x[6], x[10], x[14]) QR(x[3], x[7], x[11], x[15])
    QR(x[0], x[5], x[10], x[15]) QR(x[1], x[6], x[11], x[12]) QR(x[2], x[7], x[8], x[13]) QR(x[3], x[4], x[9], x[14])
  }
  for (int i = 0; i < 16; ++i) out[i] = x[i] + s[i];
}

static inline u64 block_word(const uint32_t blk[16], int w) { return (u64)blk[2 * w] | ((u64)blk[2 * w + 1] << 32); }

/* Uniform residues mod q: coefficient i takes the 128-bit value (word 2(i&3)+1 : word 2(i&3)) of
 * block i/4 modulo q. */
void orc_sample_uniform(u64 seed, uint32_t domain, uint32_t tag, uint32_t word, u64 q, int log_n, u64* out) {
  const u64 n = 1ULL << log_n;
#pragma omp parallel for schedule(static)
  for (i64 b = 0; b < (i64)(n / 4); ++b) {
    uint32_t blk[16];
    orc_chacha_block(seed, domain, tag, word, (uint32_t)b, blk);
    for (int j = 0; j < 4; ++j) {
      const u64 lo = block_word(blk, 2 * j), hi = block_word(blk, 2 * j + 1);
      out[b * 4 + j] = (u64)((((u128)hi << 64) | lo) % q);
    }
  }
}

/* Centred binomial error (eta = 21): coefficient i = popcount(r & M21) - popcount((r >> 21) & M21) with
 * r word i&7 of block i/8. */
void orc_sample_cbd(u64 seed, uint32_t domain, uint32_t tag, uint32_t word, int log_n, i64* out) {
  const u64 n = 1ULL << log_n, m21 = (1ULL << 21) - 1;
  for (u64 b = 0; b < n / 8; ++b) {
    uint32_t blk[16];
    orc_chacha_block(seed, domain, tag, word, (uint32_t)b, blk);
    for (int j = 0; j < 8; ++j) {
      const u64 r = block_word(blk, j);
      out[b * 8 + j] = (i64)__builtin_popcountll(r & m21) - (i64)__builtin_popcountll((r >> 21) & m21);
    }
  }
}

/* Secret: hamming == 0 -> uniform ternary (r mod 3) - 1 from word i&7 of block i/8 (word field 0);
 * hamming > 0 -> exactly `hamming` nonzero +-1 coefficients placed by a partial Fisher-Yates shuffle:
 * step t draws r = word t&7 of block t/8 (word field 1), j = t + r mod (N - t), swaps idx[t], idx[j];
 * the sign of idx[t] is +1 when bit 0 of word t&7 of block t/8 (word field 2) is set, else -1. */
void orc_sample_secret(u64 seed, int log_n, int hamming, i64* out) {
  const u64 n = 1ULL << log_n;
  uint32_t blk[16];
  if (hamming <= 0) {
    for (u64 b = 0; b < n / 8; ++b) {
      orc_chacha_block(seed, 1, 0, 0, (uint32_t)b, blk);
      for (int j = 0; j < 8; ++j) out[b * 8 + j] = (i64)(block_word(blk, j) % 3) - 1;
    }
    return;
  }
  u64* idx = (u64*)malloc(sizeof(u64) * n);
  for (u64 i = 0; i < n; ++i) { idx[i] = i; out[i] = 0; }
  for (u64 t = 0; t < (u64)hamming; ++t) {
    orc_chacha_block(seed, 1, 0, 1, (uint32_t)(t / 8), blk);
    const u64 r = block_word(blk, (int)(t & 7));
    const u64 j = t + r % (n - t);
    const u64 tmp = idx[t]; idx[t] = idx[j]; idx[j] = tmp;
    orc_chacha_block(seed, 1, 0, 2, (uint32_t)(t / 8), blk);
    out[idx[t]] = (block_word(blk, (int)(t & 7)) & 1) ? 1 : -1;
  }
  free(idx);
}
