// extern "C" entry points of libholmes_cuda (declared in include/holmes_cuda.h).
#include "../../include/holmes_cuda.h"
#include "ops.h"

using namespace holmes;

namespace holmes {
int build_context(HolmesCtx& c, int log_n, int limbs, int dnum, int dcrt_bits, int first_mod_bits, int special_bits,
                  int special_limbs, int hamming, u64 seed);
void free_context(HolmesCtx& c);
}  // namespace holmes

static inline cudaStream_t S(void* s) { return (cudaStream_t)s; }
static inline HolmesCtx* C(void* c) { return (HolmesCtx*)c; }

extern "C" {

int holmes_ctx_create(const holmes_params* p, void** ctx_out) {
  if (!p || !ctx_out) return -1;
  HolmesCtx* c = new HolmesCtx();
  int rc = build_context(*c, p->log_n, p->limbs, p->dnum, p->dcrt_bits, p->first_mod_bits, p->special_bits,
                         p->special_limbs, p->hamming, p->seed);
  if (!rc) rc = secret_ntt(*c, 0);
  if (rc) {
    free_context(*c);
    delete c;
    return rc;
  }
  *ctx_out = c;
  return 0;
}

int holmes_ctx_destroy(void* ctx) {
  if (!ctx) return -1;
  free_context(*C(ctx));
  delete C(ctx);
  return 0;
}

int holmes_ctx_moduli(void* ctx, uint64_t* out) {
  if (!ctx || !out) return -1;
  for (int i = 0; i < C(ctx)->T; ++i) out[i] = C(ctx)->q[i];
  return 0;
}

int holmes_ctx_dims(void* ctx, int* out) {
  if (!ctx || !out) return -1;
  const HolmesCtx& c = *C(ctx);
  out[0] = c.log_n;
  out[1] = c.L;
  out[2] = c.K;
  out[3] = c.alpha;
  out[4] = c.dnum;
  out[5] = c.beta_max;
  return 0;
}

int holmes_ctx_secret(void* ctx, void** out) {
  if (!ctx || !out) return -1;
  *out = C(ctx)->d_secret;
  return 0;
}

int holmes_galois(void* ctx, long long rotation, uint64_t* out) {
  if (!ctx || !out) return -1;
  const HolmesCtx& c = *C(ctx);
  const u64 m = 2ull * (u64)c.n;
  if (rotation == (long long)(m - 1)) {
    *out = m - 1;
    return 0;
  }
  const long long half = c.n / 2;
  long long r = rotation % half;
  if (r < 0) r += half;
  u64 g = 1;
  for (long long i = 0; i < r; ++i) g = (g * 5) % m;
  *out = g;
  return 0;
}

int holmes_key_words(void* ctx, int cap, long long* out) {
  if (!ctx || !out) return -1;
  const HolmesCtx& c = *C(ctx);
  if (cap < 1 || cap > c.L) return -2;
  *out = 2LL * c.beta(cap) * (cap + c.K) * (long long)c.n;
  return 0;
}

int holmes_keygen(void* ctx, uint64_t galois, int cap, uint64_t* key, void* stream) {
  if (!ctx || !key) return -1;
  if (galois != 0 && !(galois & 1)) return -3;
  return keygen(*C(ctx), galois, cap, key, S(stream));
}

int holmes_encrypt(void* ctx, const uint64_t* m, int cur, uint64_t counter, uint64_t* c0, uint64_t* c1, void* stream) {
  if (!ctx || !m || !c0 || !c1) return -1;
  return encrypt(*C(ctx), m, cur, counter, c0, c1, S(stream));
}

int holmes_decrypt(void* ctx, const uint64_t* c0, const uint64_t* c1, int cur, uint64_t* out, void* stream) {
  if (!ctx || !c0 || !c1 || !out) return -1;
  return decrypt_coef(*C(ctx), c0, c1, cur, out, S(stream));
}

int holmes_ntt(void* ctx, uint64_t* data, int items, int limbs, long long item_stride, int first_mod, int inverse,
               void* stream) {
  if (!ctx || !data) return -1;
  const HolmesCtx& c = *C(ctx);
  if (items < 1 || limbs < 1 || first_mod < 0 || first_mod + limbs > c.T) return -2;
  PolyMap pm = poly_map(limbs, item_stride, c.n, first_mod);
  return ntt_plain(c, data, data, pm, items * limbs, inverse != 0, S(stream));
}

int holmes_encode(void* ctx, double* z, long long row_stride, int rows, int slots, double scale, int cur, uint64_t* out,
                  long long out_row_stride, int* flag, void* stream) {
  if (!ctx || !z || !out || !flag) return -1;
  if (rows < 1) return 0;
  int rc = fft_special_inv(*C(ctx), z, row_stride, rows, slots, S(stream));
  if (rc) return rc;
  return encode_rows(*C(ctx), z, row_stride, rows, slots, scale, cur, out, out_row_stride, flag, S(stream));
}

int holmes_encode_stage2(void* out, const void* in, long long in_stride, int rows, double sf, int limbs,
                         const void* primes, const void* diffs, const void* ratios, const void* ks, const void* roots,
                         const void* roots_shoup, void* stream, int rows_per_launch, int parts, int limbs_per_block) {
  (void)diffs;             // negative values are reduced as signed integers directly
  (void)rows_per_launch;   // scheduling hints of the reference's kernels
  (void)limbs_per_block;
  if (!out || !in || !primes || !ratios || !ks || !roots || !roots_shoup) return -1;
  if ((parts & 3) == 0) return 0;
  return encode_stage2((u64*)out, (const double*)in, in_stride, rows, sf, limbs, (const u64*)primes,
                       (const u64*)ratios, (const u64*)ks, (const u64*)roots, (const u64*)roots_shoup, nullptr,
                       S(stream));
}

int holmes_fft_special_inv(void* ctx, double* z, long long row_stride, int rows, int slots, void* stream) {
  if (!ctx || !z) return -1;
  return fft_special_inv(*C(ctx), z, row_stride, rows, slots, S(stream));
}

int holmes_encode_fft(void* ctx, const double* u, long long row_stride, int rows, int slots, double scale, int cur,
                      uint64_t* out, long long out_row_stride, int* flag, void* stream) {
  if (!ctx || !u || !out || !flag) return -1;
  if (rows < 1) return 0;
  return encode_rows(*C(ctx), u, row_stride, rows, slots, scale, cur, out, out_row_stride, flag, S(stream));
}

int holmes_encode_fft_ext(void* ctx, const double* u, long long row_stride, int rows, int slots, double scale, int cur,
                          uint64_t* out, long long out_row_stride, int* flag, void* stream) {
  if (!ctx || !u || !out || !flag) return -1;
  if (rows < 1) return 0;
  const HolmesCtx& c = *C(ctx);
  if (cur < 1 || cur > c.L) return -2;
  if (out_row_stride < (long long)(cur + c.K) * c.n) return -4;
  const int e = encode_rows(c, u, row_stride, rows, slots, scale, cur, out, out_row_stride, flag, S(stream));
  if (e) return e;
  return encode_rows(c, u, row_stride, rows, slots, scale, c.K, out + (size_t)cur * c.n, out_row_stride, flag,
                     S(stream), c.L);
}

int holmes_pack_diagonals(const double* weight, int weight_complex, int dim, int lanes, int baby, int giant_base,
                          int giant_count, int lane_shift, int slots, double* out, long long row_stride, void* stream) {
  if (!weight || !out) return -1;
  return pack_diagonals(weight, weight_complex, dim, lanes, baby, giant_base, giant_count, lane_shift, slots, out,
                        row_stride, S(stream));
}

int holmes_pack_structured(const void* const* sources, const long long* row_strides, const long long* col_strides,
                           int source_count, int source_fp32, const long long* real_source, const long long* real_row,
                           const double* real_scale, const long long* imag_source, const long long* imag_row,
                           const double* imag_scale, const long long* real_column, const long long* imag_column,
                           const double* column_scale, int dim, int lanes, int baby, int giant_base, int giant_count,
                           int lane_shift, int slots, double* out, long long row_stride, void* stream) {
  if (!sources || !row_strides || !col_strides || !real_source || !real_row || !real_scale || !imag_source ||
      !imag_row || !imag_scale || !real_column || !imag_column || !column_scale || !out)
    return -1;
  if (source_count < 1 || source_count > 3) return -2;
  StructSources src{};
  for (int i = 0; i < 3; ++i) {
    const int k = i < source_count ? i : 0;
    if (!sources[k]) return -1;
    src.p[i] = sources[k];
    src.row_stride[i] = row_strides[k];
    src.col_stride[i] = col_strides[k];
  }
  src.count = source_count;
  src.fp32 = source_fp32 ? 1 : 0;
  StructMaps M{real_source, real_row, imag_source, imag_row, real_column, imag_column, real_scale, imag_scale,
               column_scale};
  return pack_structured(src, M, dim, lanes, baby, giant_base, giant_count, lane_shift, slots, out, row_stride,
                         S(stream));
}

int holmes_elementwise(void* ctx, int op, const uint64_t* a, const uint64_t* b, uint64_t* out, int items, int limbs,
                       long long a_item, long long b_item, long long out_item, void* stream) {
  if (!ctx || !a || !out || (op != EW_NEG && !b) || op < 0 || op > 3) return -1;
  return elementwise(*C(ctx), op, a, b, out, items, limbs, a_item, b_item, out_item, S(stream));
}

int holmes_tensor_product(void* ctx, const uint64_t* a0, const uint64_t* a1, long long a_item, const uint64_t* b0,
                          const uint64_t* b1, long long b_item, uint64_t* d0, uint64_t* d1, uint64_t* d2,
                          long long d_item, int items, int limbs, void* stream) {
  if (!ctx || !a0 || !a1 || !b0 || !b1 || !d0 || !d1 || !d2) return -1;
  return tensor_product(*C(ctx), a0, a1, a_item, b0, b1, b_item, d0, d1, d2, d_item, items, limbs, S(stream));
}

int holmes_mul_i(void* ctx, const uint64_t* a, uint64_t* out, int items, int limbs, long long a_item, long long out_item,
                 void* stream) {
  if (!ctx || !a || !out) return -1;
  return mul_i(*C(ctx), a, out, items, limbs, a_item, out_item, S(stream));
}

int holmes_automorph(void* ctx, const uint64_t* a, uint64_t* out, uint64_t galois, int items, int limbs,
                     long long a_item, long long out_item, void* stream) {
  if (!ctx || !a || !out) return -1;
  return automorph(*C(ctx), a, out, galois, items, limbs, a_item, out_item, S(stream));
}

int holmes_mul_const(void* ctx, const uint64_t* a, const uint64_t* consts, uint64_t* out, int items, int limbs,
                     long long a_item, long long out_item, void* stream) {
  if (!ctx || !a || !consts || !out) return -1;
  return mul_const(*C(ctx), a, consts, out, items, limbs, a_item, out_item, S(stream));
}

int holmes_weighted_acc(void* ctx, const uint64_t* a, long long a_item, int nk, const uint64_t* weights, uint64_t* out,
                        long long out_item, int groups, int limbs, void* stream) {
  if (!ctx || !a || !weights || !out) return -1;
  return weighted_acc(*C(ctx), a, a_item, nk, weights, out, out_item, groups, limbs, S(stream));
}

int holmes_rescale(void* ctx, const uint64_t* in, long long in_stride, uint64_t* out, long long out_stride, int cur,
                   int comps, uint64_t* scratch, void* stream) {
  if (!ctx || !in || !out || !scratch || comps < 1) return -1;
  return rescale(*C(ctx), in, in_stride, out, out_stride, cur, comps, scratch, S(stream));
}

int holmes_rescale_postop(void* ctx, const uint64_t* in, long long in_stride, uint64_t* out, long long out_stride,
                          int cur, int comps, uint64_t* scratch, int apply_double, const uint64_t* sub,
                          long long sub_stride, const uint64_t* consts, void* stream) {
  if (!ctx || !in || !out || !scratch || comps < 1) return -1;
  return rescale(*C(ctx), in, in_stride, out, out_stride, cur, comps, scratch, S(stream), apply_double ? 1 : 0, sub,
                 sub_stride, consts);
}

int holmes_modraise(void* ctx, const uint64_t* in, long long in_stride, uint64_t* out, long long out_stride, int raise,
                    int comps, uint64_t* scratch, void* stream) {
  if (!ctx || !in || !out || !scratch) return -1;
  return modraise(*C(ctx), in, in_stride, out, out_stride, raise, comps, scratch, S(stream));
}

int holmes_const_op(void* ctx, int op, const uint64_t* a, const uint64_t* host_consts, uint64_t* out, int items,
                    int limbs, long long a_item, long long out_item, void* stream) {
  if (!ctx || !a || !host_consts || !out) return -1;
  return const_op(*C(ctx), op, a, host_consts, out, items, limbs, a_item, out_item, S(stream));
}

int holmes_add_const(void* ctx, const uint64_t* a, const uint64_t* consts, uint64_t* out, int items, int limbs,
                     long long a_item, long long out_item, void* stream) {
  if (!ctx || !a || !consts || !out) return -1;
  return add_const(*C(ctx), a, consts, out, items, limbs, a_item, out_item, S(stream));
}

int holmes_modup(void* ctx, const uint64_t* c1, long long c1_item, int cur, int items, uint64_t* digits,
                 long long digit_item, uint64_t* scratch, void* stream) {
  if (!ctx || !c1 || !digits || !scratch) return -1;
  return modup(*C(ctx), c1, c1_item, cur, items, digits, digit_item, scratch, S(stream));
}

int holmes_keyswitch(void* ctx, const uint64_t* digits, long long digit_item, int cur, const uint64_t* key, int key_cap,
                     uint64_t galois, const uint64_t* add0, const uint64_t* add1, long long add_item,
                     const uint64_t* post0, const uint64_t* post1, long long post_item, uint64_t* out0, uint64_t* out1,
                     long long out_item, int items, uint64_t* scratch, void* stream) {
  if (!ctx || !digits || !key || !out0 || !out1 || !scratch) return -1;
  if (galois > 1 && !(galois & 1)) return -3;
  KsArgs a{digits, digit_item, cur,   key,  key_cap,  galois, add0,  add1,    add_item,
           post0,  post1,      post_item, out0, out1, out_item, items, scratch};
  return ks_apply(*C(ctx), a, S(stream));
}

int holmes_rotate_scratch_words(void* ctx, int cur, int items, long long* words) {
  if (!ctx || !words || cur < 1 || items < 1) return -1;
  const HolmesCtx& c = *C(ctx);
  if (cur > c.L) return -2;
  const long long n = c.n, rows = (long long)cur + c.K;
  const long long digits = (long long)items * c.beta(cur) * rows * n;
  const long long work = (long long)items * 2 * rows * n;  // >= the ModUp's items * cur * N as well
  *words = digits + work;
  return 0;
}

int holmes_scratch_words(void* ctx, int op, int cur, int items, long long* words) {
  long long base = 0;
  const int e = holmes_rotate_scratch_words(ctx, cur, items, &base);
  if (e) return e;
  const HolmesCtx& c = *C(ctx);
  const long long poly = (long long)items * cur * c.n;
  switch (op) {
    case HOLMES_OP_ROTATE: *words = base; return 0;
    case HOLMES_OP_GIANT_SUM: *words = base + 2 * poly; return 0;   // the ping-pong accumulator
    case HOLMES_OP_MUL_RELIN: *words = base + 4 * poly; return 0;   // d0, d1, d2 and one product
    default: return -4;
  }
}

int holmes_rotate(void* ctx, const uint64_t* c0, const uint64_t* c1, long long in_item, int cur, const uint64_t* key,
                  int key_cap, uint64_t galois, uint64_t* out0, uint64_t* out1, long long out_item, int items,
                  uint64_t* scratch, void* stream) {
  if (!ctx || !c0 || !c1 || !key || !out0 || !out1 || !scratch) return -1;
  if (cur < 1 || items < 1) return -2;
  if (galois <= 1 || !(galois & 1)) return -3;
  const HolmesCtx& c = *C(ctx);
  if (cur > c.L) return -2;
  const long long digit_item = (long long)c.beta(cur) * (cur + c.K) * c.n;
  uint64_t* digits = scratch;
  uint64_t* work = scratch + (size_t)items * digit_item;
  const int e = modup(c, c1, in_item, cur, items, digits, digit_item, work, S(stream));
  if (e) return e;
  KsArgs a{digits, digit_item, cur,     key,  key_cap, galois, c0,    nullptr, in_item,
           nullptr, nullptr,   0,       out0, out1,    out_item, items, work};
  return ks_apply(c, a, S(stream));
}

int holmes_hoisted_rotations(void* ctx, const uint64_t* c0, const uint64_t* c1, long long in_item, int cur, int items,
                             int count, const uint64_t* const* keys, const int* key_caps, const uint64_t* galois,
                             uint64_t* out0, uint64_t* out1, long long out_item, long long out_rot, uint64_t* scratch,
                             void* stream) {
  if (!ctx || !c0 || !c1 || !keys || !key_caps || !galois || !out0 || !out1 || !scratch) return -1;
  if (cur < 1 || items < 1 || count < 1) return -2;
  const HolmesCtx& c = *C(ctx);
  if (cur > c.L) return -2;
  const long long digit_item = (long long)c.beta(cur) * (cur + c.K) * c.n;
  uint64_t* digits = scratch;
  uint64_t* work = scratch + (size_t)items * digit_item;
  bool up = false;
  for (int r = 0; r < count; ++r) {
    uint64_t* o0 = out0 + (size_t)r * out_rot;
    uint64_t* o1 = out1 + (size_t)r * out_rot;
    if (galois[r] <= 1) {  // offset 0: the ciphertext itself
      for (int i = 0; i < items; ++i) {
        cudaError_t e = cudaMemcpyAsync(o0 + (size_t)i * out_item, c0 + (size_t)i * in_item,
                                        (size_t)cur * c.n * sizeof(uint64_t), cudaMemcpyDeviceToDevice, S(stream));
        if (e == cudaSuccess)
          e = cudaMemcpyAsync(o1 + (size_t)i * out_item, c1 + (size_t)i * in_item,
                              (size_t)cur * c.n * sizeof(uint64_t), cudaMemcpyDeviceToDevice, S(stream));
        if (e != cudaSuccess) return (int)e;
      }
      continue;
    }
    if (!(galois[r] & 1) || !keys[r]) return -3;
    if (!up) {
      const int e = modup(c, c1, in_item, cur, items, digits, digit_item, work, S(stream));
      if (e) return e;
      up = true;
    }
    KsArgs a{digits, digit_item, cur,  keys[r], key_caps[r], galois[r], c0,    nullptr, in_item,
             nullptr, nullptr,   0,    o0,      o1,          out_item,  items, work};
    const int e = ks_apply(c, a, S(stream));
    if (e) return e;
  }
  return 0;
}

int holmes_giant_sum(void* ctx, const uint64_t* p0, const uint64_t* p1, long long part_item, long long part_giant,
                     int cur, int items, int giants, const uint64_t* key, int key_cap, uint64_t galois, uint64_t* out0,
                     uint64_t* out1, long long out_item, uint64_t* scratch, void* stream) {
  if (!ctx || !p0 || !p1 || !key || !out0 || !out1 || !scratch) return -1;
  if (cur < 1 || items < 1 || giants < 1) return -2;
  if (galois <= 1 || !(galois & 1)) return -3;
  const HolmesCtx& c = *C(ctx);
  if (cur > c.L) return -2;
  const long long digit_item = (long long)c.beta(cur) * (cur + c.K) * c.n;
  const size_t poly = (size_t)cur * c.n;
  uint64_t* digits = scratch;
  uint64_t* work = digits + (size_t)items * digit_item;
  uint64_t* tmp0 = work + (size_t)items * 2 * (cur + c.K) * c.n;  // the other accumulator: [items][cur][N] x 2
  uint64_t* tmp1 = tmp0 + (size_t)items * poly;
  // acc = partial[G - 1]; acc = rot(acc) + partial[g] for g = G - 2 .. 0, ping-ponging so the last lands in out
  const uint64_t* a0 = p0 + (size_t)(giants - 1) * part_giant;
  const uint64_t* a1 = p1 + (size_t)(giants - 1) * part_giant;
  long long a_item = part_item;
  if (giants == 1) {
    for (int i = 0; i < items; ++i) {
      cudaError_t e = cudaMemcpyAsync(out0 + (size_t)i * out_item, a0 + (size_t)i * a_item, poly * sizeof(uint64_t),
                                      cudaMemcpyDeviceToDevice, S(stream));
      if (e == cudaSuccess)
        e = cudaMemcpyAsync(out1 + (size_t)i * out_item, a1 + (size_t)i * a_item, poly * sizeof(uint64_t),
                            cudaMemcpyDeviceToDevice, S(stream));
      if (e != cudaSuccess) return (int)e;
    }
    return 0;
  }
  for (int g = giants - 2; g >= 0; --g) {
    const bool to_out = ((giants - 2 - g) & 1) == ((giants - 2) & 1);  // the step g = 0 writes out
    uint64_t* d0 = to_out ? out0 : tmp0;
    uint64_t* d1 = to_out ? out1 : tmp1;
    const long long d_item = to_out ? out_item : (long long)poly;
    int e = modup(c, a1, a_item, cur, items, digits, digit_item, work, S(stream));
    if (e) return e;
    KsArgs ks{digits, digit_item, cur, key, key_cap, galois, a0, nullptr, a_item, p0 + (size_t)g * part_giant,
              p1 + (size_t)g * part_giant, part_item, d0, d1, d_item, items, work};
    e = ks_apply(c, ks, S(stream));
    if (e) return e;
    a0 = d0;
    a1 = d1;
    a_item = d_item;
  }
  return 0;
}

int holmes_mul_relin(void* ctx, const uint64_t* a0, const uint64_t* a1, const uint64_t* b0, const uint64_t* b1,
                     long long in_item, int cur, int items, const uint64_t* key, int key_cap, uint64_t* out0,
                     uint64_t* out1, long long out_item, uint64_t* scratch, void* stream) {
  if (!ctx || !a0 || !a1 || !b0 || !b1 || !key || !out0 || !out1 || !scratch) return -1;
  if (cur < 1 || items < 1) return -2;
  const HolmesCtx& c = *C(ctx);
  if (cur > c.L) return -2;
  const long long poly = (long long)cur * c.n;
  const long long digit_item = (long long)c.beta(cur) * (cur + c.K) * c.n;
  uint64_t* digits = scratch;
  uint64_t* work = digits + (size_t)items * digit_item;
  uint64_t* d0 = work + (size_t)items * 2 * (cur + c.K) * c.n;  // the tensor product, [items][cur][N] each
  uint64_t* d1 = d0 + (size_t)items * poly;
  uint64_t* d2 = d1 + (size_t)items * poly;
  uint64_t* t = d2 + (size_t)items * poly;
  int e = elementwise(c, EW_MUL, a0, b0, d0, items, cur, in_item, in_item, poly, S(stream));
  if (!e) e = elementwise(c, EW_MUL, a0, b1, d1, items, cur, in_item, in_item, poly, S(stream));
  if (!e) e = elementwise(c, EW_MUL, a1, b0, t, items, cur, in_item, in_item, poly, S(stream));
  if (!e) e = elementwise(c, EW_ADD, d1, t, d1, items, cur, poly, poly, poly, S(stream));
  if (!e) e = elementwise(c, EW_MUL, a1, b1, d2, items, cur, in_item, in_item, poly, S(stream));
  if (!e) e = modup(c, d2, poly, cur, items, digits, digit_item, work, S(stream));
  if (e) return e;
  KsArgs ks{digits, digit_item, cur, key, key_cap, 1, d0, d1, poly, nullptr, nullptr, 0, out0, out1, out_item, items,
            work};
  return ks_apply(c, ks, S(stream));
}

int holmes_encode_diag_rows(void* ctx, const double* weight, int weight_complex, int dim, int lanes, int baby,
                            int giant_base, int giant_count, int lane_shift, int slots, double scale, int cur,
                            uint64_t* out, long long out_row_stride, double* rows_scratch, int* flag, void* stream) {
  if (!ctx || !weight || !out || !rows_scratch || !flag) return -1;
  if (baby < 1 || giant_count < 1) return -2;
  const long long row_stride = 2LL * slots;
  int e = pack_diagonals(weight, weight_complex, dim, lanes, baby, giant_base, giant_count, lane_shift, slots,
                         rows_scratch, row_stride, S(stream));
  if (e) return e;
  e = fft_special_inv(*C(ctx), rows_scratch, row_stride, giant_count * baby, slots, S(stream));
  if (e) return e;
  return encode_rows(*C(ctx), rows_scratch, row_stride, giant_count * baby, slots, scale, cur, out, out_row_stride,
                     flag, S(stream));
}

int holmes_bsgs_mac(void* ctx, uint64_t* res, const uint64_t* const* c0s, const uint64_t* const* c1s, long long bstride,
                    int nb, int inputs, const uint64_t* pts, long long pstride, int groups, int limbs, void* stream) {
  if (!ctx || !res || !c0s || !c1s || !pts) return -1;
  const HolmesCtx& c = *C(ctx);
  if (limbs < 1 || limbs > c.L) return -2;
  ModSrc ms{c.d_mod, 0, nullptr, nullptr, nullptr};
  return bsgs_mac(ms, res, c0s, c1s, bstride, nb, inputs, pts, pstride, groups, limbs, c.n, S(stream));
}

int holmes_keyswitch_ext(void* ctx, const uint64_t* digits, long long digit_item, int cur, const uint64_t* key,
                         int key_cap, uint64_t galois, const uint64_t* add0, long long add_item, uint64_t* out0,
                         uint64_t* out1, long long out_item, int items, void* stream) {
  if (!ctx || !digits || !key || !out0 || !out1) return -1;
  if (galois > 1 && !(galois & 1)) return -3;
  KsArgs a{digits, digit_item, cur, key, key_cap, galois, add0, nullptr, add_item,
           nullptr, nullptr, 0, out0, out1, out_item, items, nullptr};
  return ks_apply_ext(*C(ctx), a, S(stream));
}

int holmes_moddown(void* ctx, const uint64_t* in0, const uint64_t* in1, long long in_item, int cur, uint64_t* out0,
                   uint64_t* out1, long long out_item, int items, uint64_t* scratch, void* stream) {
  if (!ctx || !in0 || !in1 || !out0 || !out1 || !scratch) return -1;
  return moddown_ext(*C(ctx), in0, in1, in_item, cur, out0, out1, out_item, items, scratch, S(stream));
}

int holmes_bsgs_mac_ext(void* ctx, uint64_t* res, const uint64_t* const* c0s, const uint64_t* const* c1s,
                        long long bstride, int nb, int inputs, const uint64_t* pts, long long pstride, int groups,
                        int cur, void* stream) {
  if (!ctx || !res || !c0s || !c1s || !pts) return -1;
  const HolmesCtx& c = *C(ctx);
  if (cur < 1 || cur > c.L) return -2;
  ModSrc ms{c.d_mod, 0, nullptr, nullptr, nullptr, cur, c.L};
  return bsgs_mac(ms, res, c0s, c1s, bstride, nb, inputs, pts, pstride, groups, cur + c.K, c.n, S(stream));
}

int holmes_modsum(void* ctx, const uint64_t* const* srcs, int nsrc, uint64_t* out, int items, int limbs,
                  long long item_stride, void* stream) {
  if (!ctx || !srcs || !out) return -1;
  return modsum(*C(ctx), srcs, nsrc, out, items, limbs, item_stride, S(stream));
}

int holmes_launch_count(unsigned long long* out) {
  if (!out) return -1;
  *out = launch_counter().load();
  return 0;
}

int holmes_device_error(int reset, int* flag_out) {
  if (!flag_out) return -1;
  return tc_error_flag(reset, flag_out);
}

int holmes_mac_gather(uint64_t* res, const uint64_t* const* c0s, const uint64_t* const* c1s, long long bstride,
                      const int* idx, const int* prow, const int* seg, int inputs, int K, const uint64_t* pts,
                      long long pstride, int ti, int limbs, const uint64_t* primes, const uint64_t* ratios,
                      const uint64_t* ks, void* stream_ptr) {
  if (!res || !c0s || !c1s || !idx || !prow || !seg || !pts || !primes || !ratios || !ks) return -1;
  ModSrc ms{nullptr, 0, primes, ratios, ks};
  return mac_gather(ms, res, c0s, c1s, bstride, idx, prow, seg, inputs, K, pts, pstride, ti, limbs, 16,
                    S(stream_ptr));
}

int holmes_mac_multi(uint64_t* res, const uint64_t* const* c0s, const uint64_t* const* c1s, long long bstride, int nb,
                     int inputs, const uint64_t* pts, long long pstride, int groups, int ti, int limbs,
                     const uint64_t* primes, const uint64_t* ratios, const uint64_t* ks, void* stream_ptr) {
  if (inputs < 1 || inputs > 32) return -1;
  if (nb < 1) return -2;
  if (groups < 1 || groups > 16) return -3;
  if (groups > 8 && ti != 10116) return -3;
  static const int valid[] = {1, 2, 4, 404, 408, 802, 804, 1601, 1602, 10108, 10116, 10204, 10208, 10402, 10404};
  bool ok = false;
  for (int v : valid) ok |= (v == ti);
  if (!ok) return -4;
  ModSrc ms{nullptr, 0, primes, ratios, ks};
  return bsgs_mac(ms, res, c0s, c1s, bstride, nb, inputs, pts, pstride, groups, limbs, 1 << 16, S(stream_ptr));
}

}  // extern "C"
