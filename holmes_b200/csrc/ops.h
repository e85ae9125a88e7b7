// Host entry points of the kernel families (called by the C ABI in capi.cu).
// All return 0, a negative argument error, or a positive cudaError_t.
#pragma once
#include "ctx.h"

namespace holmes {

// Polynomial p of a batch [items][limbs][N] -> word offset and modulus index.
struct PolyMap {
  int limbs;               // polynomials per item
  long long item_stride;   // words between items
  long long limb_stride;   // words between limbs
  int mod_first;           // modulus of limb 0 (ext_cur == 0)
  int ext_cur;             // > 0: limb l < ext_cur is Q limb l, else special limb L + l - ext_cur
  int L;
  __host__ __device__ int mod(int p) const {
    const int l = p % limbs;
    return ext_cur > 0 ? (l < ext_cur ? l : L + l - ext_cur) : mod_first + l;
  }
  __host__ __device__ long long off(int p) const {
    return (long long)(p / limbs) * item_stride + (long long)(p % limbs) * limb_stride;
  }
};

inline PolyMap poly_map(int limbs, long long item_stride, long long limb_stride, int mod_first, int ext_cur = 0,
                        int L = 0) {
  PolyMap m;
  m.limbs = limbs;
  m.item_stride = item_stride;
  m.limb_stride = limb_stride;
  m.mod_first = mod_first;
  m.ext_cur = ext_cur;
  m.L = L;
  return m;
}

int ntt_plain(const HolmesCtx& c, const u64* src, u64* dst, PolyMap pm, int polys, bool inverse, cudaStream_t st);

// ModUp of `items` ciphertext components c1 [items][cur][N] (NTT, item stride c1_item) into digits
// [items][beta(cur)][cur + K][N] (NTT, item stride dig_item); scratch >= items * cur * N words.
int modup(const HolmesCtx& c, const u64* c1, long long c1_item, int cur, int items, u64* digits, long long dig_item,
          u64* scratch, cudaStream_t st);

// Inner product of digits (optionally read through the automorphism `galois`) with a switching key and
// ModDown, plus addends read through the same automorphism and plain addends:
//   out0 = perm(add0) + ModDown(sum_j perm(D_j) key_b[j]) + post0
//   out1 = perm(add1) + ModDown(sum_j perm(D_j) key_a[j]) + post1
// for `items` ciphertexts sharing the key (any addend may be null).  key [2][beta(cap)][cap + K][N]; scratch >= items * 2 * K * N words.
struct KsArgs {
  const u64* digits;
  long long dig_item;
  int cur;
  const u64* key;
  int key_cap;
  u64 galois;  // 1 (or 0) = no automorphism
  const u64* add0;
  const u64* add1;
  long long add_item;
  const u64* post0;
  const u64* post1;
  long long post_item;
  u64* out0;
  u64* out1;
  long long out_item;
  int items;
  u64* scratch;
};
int ks_apply(const HolmesCtx& c, const KsArgs& a, cudaStream_t st);
int ks_apply_ext(const HolmesCtx& c, const KsArgs& a, cudaStream_t st);
int moddown_ext(const HolmesCtx& c, const u64* in0, const u64* in1, long long in_item, int cur, u64* out0, u64* out1,
                long long out_item, int items, u64* scratch, cudaStream_t st);

// Rescale by the last limb: `comps` polynomials-of-limbs in [comps][cur] layout (stride in_stride / out_stride
// between components) -> [comps][cur - 1]; scratch >= comps * N words.  Optional post-operations on the
// rescaled words: doubled (dbl), minus sub[comp][limb] (component stride sub_stride, >= cur - 1 limbs), plus
// cst[limb].
int rescale(const HolmesCtx& c, const u64* in, long long in_stride, u64* out, long long out_stride, int cur, int comps,
            u64* scratch, cudaStream_t st, int dbl = 0, const u64* sub = nullptr, long long sub_stride = 0,
            const u64* cst = nullptr);

// Mod raise: [comps][1][N] modulo q0 (item stride in_stride) -> [comps][raise][N] (centred lift), scratch >= comps * N.
int modraise(const HolmesCtx& c, const u64* in, long long in_stride, u64* out, long long out_stride, int raise,
             int comps, u64* scratch, cudaStream_t st);

// out[item][l][n] = a[item][l][n] + consts[l] (a constant polynomial added in the NTT domain)
// scalar op with per-limb constants read from HOST memory (passed by value to the kernel)
constexpr int HOLMES_CONST_LIMBS = 64;
enum { CONST_ADD = 0, CONST_MUL = 1, CONST_AXPY = 2 };
int const_op(const HolmesCtx& c, int op, const u64* a, const u64* host_consts, u64* out, int items, int limbs,
             long long a_item, long long o_item, cudaStream_t st);
int add_const(const HolmesCtx& c, const u64* a, const u64* consts, u64* out, int items, int limbs, long long a_item,
              long long o_item, cudaStream_t st);

// Rows of slot vectors after the special inverse FFT ([rows][slots] complex, interleaved doubles) ->
// [rows][cur][N] NTT plaintexts at `scale`.  Out-of-range values set *flag = 1.
int encode_stage2(u64* out, const double* in, long long in_stride, int rows, double sf, int limbs, const u64* primes,
                  const u64* ratios, const u64* ks, const u64* roots, const u64* roots_shoup, int* flag,
                  cudaStream_t st);
int encode_rows(const HolmesCtx& c, const double* u, long long row_stride, int rows, int slots, double scale, int cur,
                u64* out, long long out_row_stride, int* flag, cudaStream_t st, int mod_first = 0);

int fft_special_inv(const HolmesCtx& c, double* z, long long row_stride, int rows, int slots, cudaStream_t st);

int pack_diagonals(const double* weight, int weight_complex, int dim, int lanes, int baby, int giant_base,
                   int giant_count, int lane_shift, int slots, double* out, long long row_stride, cudaStream_t st);
struct StructSources {
  const void* p[3];
  long long row_stride[3], col_stride[3];
  int count, fp32;
};
struct StructMaps {
  const long long *real_source, *real_row, *imag_source, *imag_row, *real_column, *imag_column;
  const double *real_scale, *imag_scale, *column_scale;
};
int pack_structured(const StructSources& S, const StructMaps& M, int dim, int lanes, int baby, int giant_base,
                    int giant_count, int lane_shift, int slots, double* out, long long row_stride, cudaStream_t st);

int decrypt_coef(const HolmesCtx& c, const u64* c0, const u64* c1, int cur, u64* out, cudaStream_t st);
int secret_ntt(HolmesCtx& c, cudaStream_t st);
int keygen(const HolmesCtx& c, u64 galois, int cap, u64* key, cudaStream_t st);
int encrypt(const HolmesCtx& c, const u64* m, int cur, u64 counter, u64* c0, u64* c1, cudaStream_t st);

enum EwOp { EW_ADD = 0, EW_SUB = 1, EW_MUL = 2, EW_NEG = 3 };
int tensor_product(const HolmesCtx& c, const u64* a0, const u64* a1, long long a_item, const u64* b0, const u64* b1,
                   long long b_item, u64* d0, u64* d1, u64* d2, long long d_item, int items, int limbs,
                   cudaStream_t st);
int elementwise(const HolmesCtx& c, int op, const u64* a, const u64* b, u64* out, int items, int limbs,
                long long a_item, long long b_item, long long o_item, cudaStream_t st);
int mul_i(const HolmesCtx& c, const u64* a, u64* out, int items, int limbs, long long a_item, long long o_item,
          cudaStream_t st);
int automorph(const HolmesCtx& c, const u64* a, u64* out, u64 galois, int items, int limbs, long long a_item,
              long long o_item, cudaStream_t st);
int weighted_acc(const HolmesCtx& c, const u64* a, long long a_item, int nk, const u64* w, u64* out, long long o_item,
                 int groups, int limbs, cudaStream_t st);
int mul_const(const HolmesCtx& c, const u64* a, const u64* consts, u64* out, int items, int limbs, long long a_item,
              long long o_item, cudaStream_t st);

// BSGS baby-step multiply-accumulate (see mac.cu)
// per-input baby pointers of the BSGS MAC (both components)
constexpr int kMaxInputs = 32;
struct InPtrs {
  const u64* c0[kMaxInputs];
  const u64* c1[kMaxInputs];
};
int mac_gather(ModSrc ms, u64* res, const u64* const* c0s, const u64* const* c1s, long long bstride, const int* idx,
               const int* prow, const int* seg, int inputs, int K, const u64* pts, long long pstride, int ti,
               int limbs, int log_n, cudaStream_t st);
// tensor-core MAC (mac_tc.cu): nb <= 128; returns -7 for shapes it does not take
int bsgs_mac_tc(ModSrc ms, u64* res, const InPtrs& in, long long bstride, int nb, int inputs, const u64* pts,
                long long pstride, int groups, int limbs, int log_n, cudaStream_t st);
// the tensor-core MAC's device error flag (a bounded wait ran out); reset clears it
int tc_error_flag(int reset, int* out);
int bsgs_mac(ModSrc ms, u64* res, const u64* const* c0s, const u64* const* c1s,
             long long bstride, int nb, int inputs, const u64* pts, long long pstride, int groups, int limbs, int n,
             cudaStream_t st);

// mod-q sum of `npeers` equally shaped [limbs][N] buffers (e.g. peer-mapped partials) into out
int modsum(const HolmesCtx& c, const u64* const* srcs, int nsrc, u64* out, int items, int limbs, long long item_stride,
           cudaStream_t st);

}  // namespace holmes
