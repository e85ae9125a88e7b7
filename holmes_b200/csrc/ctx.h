// Host-side engine context: RNS parameters and every device-resident table the kernels read.
#pragma once
#include <cstdint>
#include <vector>

#include "common.cuh"

namespace holmes {

struct HolmesCtx {
  int device = 0;
  int log_n = 0, n = 0;
  int L = 0;      // Q limbs at the top level
  int K = 0;      // special (P) limbs
  int alpha = 0;  // limbs per key-switch digit
  int dnum = 0;
  int T = 0;      // L + K moduli: Q limbs 0..L-1 then P limbs
  int beta_max = 0;
  int hamming = 0;
  u64 seed = 0;
  std::vector<u64> q, psi;

  // device tables
  Mod* d_mod = nullptr;          // [T]
  Tw* d_tw = nullptr;            // [T][N] forward twiddles psi^bitrev(k)
  Tw* d_itw = nullptr;           // [T][N] inverse twiddles psi^-bitrev(k)
  Tw* d_ninv = nullptr;          // [T] N^-1
  Tw* d_mu_scale = nullptr;      // [L+1][beta_max][alpha] N^-1 (Q_j/q_k)^-1 mod q_k (ModUp iNTT epilogue)
  u64* d_mu_hat = nullptr;       // [L+1][beta_max][alpha][T] (Q_j/q_k) mod m_t, times P^-1 for Q targets t < L
  Tw* d_md_scale = nullptr;      // [K] N^-1 (P/p_k)^-1 mod p_k (ModDown iNTT epilogue)
  u64* d_md_hat = nullptr;       // [K][L] (P/p_k) P^-1 = p_k^-1 mod q_i
  Tw* d_md_pinv = nullptr;       // [L] P^-1 mod q_i (scales the digits' own limbs in ModUp)
  Tw* d_rs_qinv = nullptr;       // [L+1][L] q_{l-1}^-1 mod q_i (rescale from l limbs)
  u64* d_p_mod_q = nullptr;      // [L] P mod q_i
  Tw* d_pmodq_tw = nullptr;      // [L] P mod q_i with its Shoup companion
  Tw* d_unit = nullptr;          // [T] psi^(N/2): X^(N/2) evaluated at the first half of the NTT words
  Tw* d_unit_neg = nullptr;      // [T] q - psi^(N/2)
  u64* d_rot_group = nullptr;    // [N/2] 5^j mod 2N
  double* d_ksi = nullptr;       // [2N][2] cos/sin(2 pi k / 2N)
  double* d_fft_tw = nullptr;    // [N/2 - 1][2] special-FFT roots by stage: stage len at len/2 - 1 + j
  u64* d_secret = nullptr;       // [T][N] secret key, NTT form (client side of the simulation context)
  std::vector<void*> owned;
  // side streams and events for independent chains inside one call (ModUp's digits), created on first use;
  // every call joins them back into its own stream before returning
  static constexpr int kSide = 3, kEvents = 17;
  mutable cudaStream_t side[kSide] = {};
  mutable cudaEvent_t ev[kEvents] = {};
  mutable bool side_ready = false;

  int beta(int cur) const { return (cur + alpha - 1) / alpha; }
  const Tw* mu_scale(int cur) const { return d_mu_scale + (size_t)cur * beta_max * alpha; }
  const u64* mu_hat(int cur) const { return d_mu_hat + (size_t)cur * beta_max * alpha * T; }
  const Tw* rs_qinv(int cur) const { return d_rs_qinv + (size_t)cur * L; }
};

// create the context's side streams and events (once; on the context's device)
int ensure_side(const HolmesCtx& c);

// host modular helpers shared by the C-ABI layer
u64 host_mul_mod(u64 a, u64 b, u64 q);
u64 host_pow_mod(u64 a, u64 e, u64 q);
u64 host_inv_mod(u64 a, u64 q);
Tw host_shoup(u64 w, u64 q);
Mod host_mod(u64 q);
void host_chacha_block(u64 seed, u32 domain, u32 tag, u32 word, u32 counter, u32 out[16]);

}  // namespace holmes
