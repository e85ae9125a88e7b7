// Engine context construction: NTT-friendly primes, roots, CRT / Shoup tables, device upload.
//
// Parameters follow the reference's CKKS context (llama3fhe/config.py:15-25 SimulatorConfig;
// production values in llama3fhe/parallel/presets.py:63-127): one `first_mod`-bit prime, L-1
// `dcrt`-bit primes, and K special primes for the hybrid key switch with dnum digits of
// alpha = ceil(L / dnum) limbs.  Primes are q = 1 (mod 2N), largest first below 2^bits.
#include <cmath>
#include <cstring>
#include <vector>

#include "ctx.h"

namespace holmes {

typedef unsigned __int128 u128;

u64 host_mul_mod(u64 a, u64 b, u64 q) { return (u64)(((u128)a * b) % q); }
u64 host_pow_mod(u64 a, u64 e, u64 q) {
  u64 r = 1 % q;
  a %= q;
  while (e) {
    if (e & 1) r = host_mul_mod(r, a, q);
    a = host_mul_mod(a, a, q);
    e >>= 1;
  }
  return r;
}
u64 host_inv_mod(u64 a, u64 q) { return host_pow_mod(a % q, q - 2, q); }
Tw host_shoup(u64 w, u64 q) {
  Tw t;
  t.w = w;
  t.ws = (u64)(((u128)w << 64) / q);
  return t;
}
Mod host_mod(u64 q) {
  Mod m;
  int b = 63;
  while (!((q >> b) & 1)) --b;
  const int k = b + 63;
  m.q = q;
  m.mu = (u64)(((u128)1 << k) / q);
  m.shift = (u32)(k - 64);
  m.pad = 0;
  return m;
}

static bool probable_prime(u64 n) {
  if (n < 2) return false;
  static const u64 bases[] = {2, 3, 5, 7, 11, 13, 17, 19, 23, 29, 31, 37};
  u64 d = n - 1;
  int s = 0;
  while (!(d & 1)) { d >>= 1; ++s; }
  for (u64 a : bases) {
    if (n % a == 0) return n == a;
    u64 x = host_pow_mod(a, d, n);
    if (x == 1 || x == n - 1) continue;
    bool comp = true;
    for (int i = 1; i < s; ++i) {
      x = host_mul_mod(x, x, n);
      if (x == n - 1) { comp = false; break; }
    }
    if (comp) return false;
  }
  return true;
}

// Largest primes = 1 (mod 2N) below 2^bits, excluding those already chosen.
static bool pick_primes(int log_n, int bits, int count, std::vector<u64>& chosen) {
  const u64 m = 2ULL << log_n;
  u64 c = (((1ULL << bits) - 1) / m) * m + 1;
  if (c >= (1ULL << bits)) c -= m;
  int found = 0;
  while (found < count && c > m) {
    bool used = false;
    for (u64 v : chosen) used |= (v == c);
    if (!used && probable_prime(c)) { chosen.push_back(c); ++found; }
    c -= m;
  }
  return found == count;
}

static u64 find_psi(u64 q, int log_n) {
  const u64 two_n = 2ULL << log_n;
  for (u64 x = 2;; ++x) {
    const u64 psi = host_pow_mod(x, (q - 1) / two_n, q);
    if (host_pow_mod(psi, two_n >> 1, q) == q - 1) return psi;
  }
}

static u64 bitrev_host(u64 v, int bits) {
  u64 r = 0;
  for (int i = 0; i < bits; ++i) { r = (r << 1) | (v & 1); v >>= 1; }
  return r;
}

template <class T>
static int upload(HolmesCtx& c, T** dst, const std::vector<T>& src) {
  void* p = nullptr;
  const size_t bytes = src.size() * sizeof(T);
  HOLMES_CUDA_TRY(cudaMalloc(&p, bytes ? bytes : 16));
  if (bytes) HOLMES_CUDA_TRY(cudaMemcpy(p, src.data(), bytes, cudaMemcpyHostToDevice));
  c.owned.push_back(p);
  *dst = (T*)p;
  return 0;
}

// Fills every table; returns 0, a negative parameter error, or a cudaError_t.
int build_context(HolmesCtx& c, int log_n, int limbs, int dnum, int dcrt_bits, int first_mod_bits, int special_bits,
                  int special_limbs, int hamming, u64 seed) {
  if (log_n < 10 || log_n > 16) return -1;
  if (limbs < 1 || limbs > 128 || dnum < 1 || dnum > limbs) return -2;
  if (dcrt_bits < 20 || dcrt_bits > 60 || first_mod_bits < 20 || first_mod_bits > 60 || special_bits < 20 ||
      special_bits > 60)
    return -3;
  c.log_n = log_n;
  c.n = 1 << log_n;
  c.L = limbs;
  c.dnum = dnum;
  c.alpha = (limbs + dnum - 1) / dnum;
  c.K = special_limbs > 0 ? special_limbs : c.alpha;
  if (c.K > 128) return -2;
  c.T = c.L + c.K;
  c.beta_max = c.beta(c.L);
  c.hamming = hamming;
  c.seed = seed;
  HOLMES_CUDA_TRY(cudaGetDevice(&c.device));

  std::vector<u64> q;
  if (!pick_primes(log_n, first_mod_bits, 1, q)) return -4;
  if (!pick_primes(log_n, dcrt_bits, limbs - 1, q)) return -4;
  if (!pick_primes(log_n, special_bits, c.K, q)) return -4;
  c.q = q;
  c.psi.resize(c.T);
  const int N = c.n, T = c.T, L = c.L, K = c.K, A = c.alpha, B = c.beta_max;
  for (int i = 0; i < T; ++i) c.psi[i] = find_psi(q[i], log_n);

  std::vector<Mod> mods(T);
  std::vector<Tw> tw((size_t)T * N), itw((size_t)T * N), ninv(T), unit(T), unit_neg(T);
  for (int i = 0; i < T; ++i) {
    const u64 qi = q[i];
    mods[i] = host_mod(qi);
    const u64 psi = c.psi[i], ipsi = host_inv_mod(psi, qi);
    std::vector<u64> pw(N), ipw(N);
    pw[0] = ipw[0] = 1;
    for (int k = 1; k < N; ++k) { pw[k] = host_mul_mod(pw[k - 1], psi, qi); ipw[k] = host_mul_mod(ipw[k - 1], ipsi, qi); }
    for (int k = 0; k < N; ++k) {
      const u64 r = bitrev_host((u64)k, log_n);
      tw[(size_t)i * N + k] = host_shoup(pw[r], qi);
      itw[(size_t)i * N + k] = host_shoup(ipw[r], qi);
    }
    ninv[i] = host_shoup(host_inv_mod((u64)N % qi, qi), qi);
    const u64 u = host_pow_mod(psi, (u64)N / 2, qi);
    unit[i] = host_shoup(u, qi);
    unit_neg[i] = host_shoup(qi - u, qi);
  }

  // P mod q_i and P^-1 mod q_i (the ModDown factor, folded into the digits' Q rows)
  std::vector<u64> p_mod_q(L), p_inv(L);
  std::vector<Tw> md_pinv(L);
  for (int i = 0; i < L; ++i) {
    u64 P = 1;
    for (int k = 0; k < K; ++k) P = host_mul_mod(P, q[L + k] % q[i], q[i]);
    p_mod_q[i] = P;
    p_inv[i] = host_inv_mod(P, q[i]);
    md_pinv[i] = host_shoup(p_inv[i], q[i]);
  }
  // ModUp tables per level `cur` (1..L) and digit j: limbs [jA, min(jA + A, cur)).  The conversion constant of
  // a Q target carries P^-1 mod q_t.
  std::vector<Tw> mu_scale((size_t)(L + 1) * B * A, Tw{0, 0});
  std::vector<u64> mu_hat((size_t)(L + 1) * B * A * T, 0);
  for (int cur = 1; cur <= L; ++cur) {
    for (int j = 0; j * A < cur; ++j) {
      const int lo = j * A, hi = std::min(lo + A, cur);
      for (int k = lo; k < hi; ++k) {
        // Qhat_k = prod_{m in digit, m != k} q_m
        u64 hat_mod_k = 1;
        for (int mm = lo; mm < hi; ++mm)
          if (mm != k) hat_mod_k = host_mul_mod(hat_mod_k, q[mm] % q[k], q[k]);
        const u64 s = host_mul_mod(host_inv_mod(hat_mod_k, q[k]), ninv[k].w, q[k]);
        mu_scale[((size_t)cur * B + j) * A + (k - lo)] = host_shoup(s, q[k]);
        for (int t = 0; t < T; ++t) {
          u64 h = 1;
          for (int mm = lo; mm < hi; ++mm)
            if (mm != k) h = host_mul_mod(h, q[mm] % q[t], q[t]);
          mu_hat[(((size_t)cur * B + j) * A + (k - lo)) * T + t] = t < L ? host_mul_mod(h, p_inv[t], q[t]) : h;
        }
      }
    }
  }
  // ModDown tables: md_hat = (P / p_k) P^-1 = p_k^-1 mod q_i
  std::vector<Tw> md_scale(K);
  std::vector<u64> md_hat((size_t)K * L);
  for (int k = 0; k < K; ++k) {
    const u64 pk = q[L + k];
    u64 hk = 1;
    for (int m = 0; m < K; ++m)
      if (m != k) hk = host_mul_mod(hk, q[L + m] % pk, pk);
    md_scale[k] = host_shoup(host_mul_mod(host_inv_mod(hk, pk), ninv[L + k].w, pk), pk);
    for (int i = 0; i < L; ++i) md_hat[(size_t)k * L + i] = host_inv_mod(pk % q[i], q[i]);
  }
  // rescale: from `cur` limbs drop q_{cur-1}
  std::vector<Tw> rs((size_t)(L + 1) * L, Tw{0, 0});
  for (int cur = 2; cur <= L; ++cur)
    for (int i = 0; i < cur - 1; ++i) rs[(size_t)cur * L + i] = host_shoup(host_inv_mod(q[cur - 1] % q[i], q[i]), q[i]);
  // CKKS embedding tables
  std::vector<u64> rot(N / 2);
  std::vector<double> ksi((size_t)4 * N);
  {
    const u64 M = 2ULL * N;
    u64 r = 1;
    for (int j = 0; j < N / 2; ++j) { rot[j] = r; r = (r * 5) % M; }
    for (u64 k = 0; k < M; ++k) {
      const double angle = 2.0 * M_PI * (double)k / (double)M;
      ksi[2 * k] = cos(angle);
      ksi[2 * k + 1] = sin(angle);
    }
  }
  int rc;
  if ((rc = upload(c, &c.d_mod, mods))) return rc;
  if ((rc = upload(c, &c.d_tw, tw))) return rc;
  if ((rc = upload(c, &c.d_itw, itw))) return rc;
  if ((rc = upload(c, &c.d_ninv, ninv))) return rc;
  if ((rc = upload(c, &c.d_mu_scale, mu_scale))) return rc;
  if ((rc = upload(c, &c.d_mu_hat, mu_hat))) return rc;
  if ((rc = upload(c, &c.d_md_scale, md_scale))) return rc;
  if ((rc = upload(c, &c.d_md_hat, md_hat))) return rc;
  if ((rc = upload(c, &c.d_md_pinv, md_pinv))) return rc;
  if ((rc = upload(c, &c.d_rs_qinv, rs))) return rc;
  if ((rc = upload(c, &c.d_p_mod_q, p_mod_q))) return rc;
  {
    std::vector<Tw> pq(L);
    for (int i = 0; i < L; ++i) pq[i] = host_shoup(p_mod_q[i], q[i]);
    if ((rc = upload(c, &c.d_pmodq_tw, pq))) return rc;
  }
  if ((rc = upload(c, &c.d_unit, unit))) return rc;
  if ((rc = upload(c, &c.d_unit_neg, unit_neg))) return rc;
  if ((rc = upload(c, &c.d_rot_group, rot))) return rc;
  if ((rc = upload(c, &c.d_ksi, ksi))) return rc;
  {
    // root of butterfly j of special-FFT stage len: ksi[(4 len - rot[j] mod 4 len) M / (4 len)], gathered once
    // here so the FFT reads it in j order instead of through two dependent random lookups
    const u64 M = 2ULL * N;
    std::vector<double> ftw((size_t)N);  // (N/2 - 1) complex roots, padded to N doubles
    for (int len = 2; len <= N / 2; len <<= 1) {
      const u64 lenq = (u64)len << 2;
      for (int j = 0; j < len / 2; ++j) {
        const u64 k = (lenq - (rot[j] & (lenq - 1))) * (M / lenq);
        ftw[2 * ((size_t)len / 2 - 1 + j)] = ksi[2 * k];
        ftw[2 * ((size_t)len / 2 - 1 + j) + 1] = ksi[2 * k + 1];
      }
    }
    if ((rc = upload(c, &c.d_fft_tw, ftw))) return rc;
  }
  std::vector<u64> zeros((size_t)T * N, 0);
  if ((rc = upload(c, &c.d_secret, zeros))) return rc;
  return 0;
}

void free_context(HolmesCtx& c) {
  for (void* p : c.owned) cudaFree(p);
  c.owned.clear();
  if (c.side_ready) {
    for (cudaStream_t& s : c.side) cudaStreamDestroy(s);
    for (cudaEvent_t& e : c.ev) cudaEventDestroy(e);
    c.side_ready = false;
  }
}

int ensure_side(const HolmesCtx& c) {
  if (c.side_ready) return 0;
  int dev = 0;
  HOLMES_CUDA_TRY(cudaGetDevice(&dev));
  if (dev != c.device) HOLMES_CUDA_TRY(cudaSetDevice(c.device));
  for (cudaStream_t& s : c.side) HOLMES_CUDA_TRY(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking));
  for (cudaEvent_t& e : c.ev) HOLMES_CUDA_TRY(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
  if (dev != c.device) HOLMES_CUDA_TRY(cudaSetDevice(dev));
  c.side_ready = true;
  return 0;
}

// ------------------------------------------------------------------ ChaCha20 block (RFC 8439), host copy
static inline u32 rotl(u32 x, int r) { return (x << r) | (x >> (32 - r)); }
void host_chacha_block(u64 seed, u32 domain, u32 tag, u32 word, u32 counter, u32 out[16]) {
  u32 s[16] = {0x61707865u, 0x3320646eu, 0x79622d32u, 0x6b206574u, (u32)seed, (u32)(seed >> 32), 0x6d6c6f68u,
               0x62323030u, 0u, 0u, 0u, 0u, counter, domain, tag, word};
  u32 x[16];
  memcpy(x, s, sizeof(x));
#define HQR(a, b, c, d)                                           \
  x[a] += x[b]; x[d] ^= x[a]; x[d] = rotl(x[d], 16);               \
  x[c] += x[d]; x[b] ^= x[c]; x[b] = rotl(x[b], 12);               \
  x[a] += x[b]; x[d] ^= x[a]; x[d] = rotl(x[d], 8);                \
  x[c] += x[d]; x[b] ^= x[c]; x[b] = rotl(x[b], 7);
  for (int r = 0; r < 10; ++r) {
    HQR(0, 4, 8, 12) HQR(1, 5, 9, 13) HQR(2, 6, 10, 14) HQR(3, 7, 11, 15)
    HQR(0, 5, 10, 15) HQR(1, 6, 11, 12) HQR(2, 7, 8, 13) HQR(3, 4, 9, 14)
  }
#undef HQR
  for (int i = 0; i < 16; ++i) out[i] = x[i] + s[i];
}

// Secret coefficients in {-1, 0, 1}: uniform ternary (hamming 0) or exactly `hamming` nonzeros placed by a
// partial Fisher-Yates shuffle (domain 1; word field 0 ternary, 1 positions, 2 signs).
void host_secret_coeffs(const HolmesCtx& c, std::vector<i64>& s) {
  const u64 N = (u64)c.n;
  s.assign(N, 0);
  u32 blk[16] = {0};
  auto word = [&](int w) { return (u64)blk[2 * w] | ((u64)blk[2 * w + 1] << 32); };
  if (c.hamming <= 0) {
    for (u64 b = 0; b < N / 8; ++b) {
      host_chacha_block(c.seed, 1, 0, 0, (u32)b, blk);
      for (int j = 0; j < 8; ++j) s[b * 8 + j] = (i64)(word(j) % 3) - 1;
    }
    return;
  }
  std::vector<u64> idx(N);
  for (u64 i = 0; i < N; ++i) idx[i] = i;
  for (u64 t = 0; t < (u64)c.hamming && t < N; ++t) {
    host_chacha_block(c.seed, 1, 0, 1, (u32)(t / 8), blk);
    const u64 j = t + word((int)(t & 7)) % (N - t);
    std::swap(idx[t], idx[j]);
    host_chacha_block(c.seed, 1, 0, 2, (u32)(t / 8), blk);
    s[idx[t]] = (word((int)(t & 7)) & 1) ? 1 : -1;
  }
}

}  // namespace holmes
