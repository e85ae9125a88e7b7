/*
 * holmes_cuda.h -- C ABI of libholmes_cuda, the B200 (sm_100a) RNS-CKKS engine under Holmes's
 * linear / key-switch hot path.
 *
 * Conventions (shared by every entry point):
 *   - every function returns 0 on success, a negative argument-error code, or a positive
 *     cudaError_t, like the reference's C ABIs (bench/cmp/kernels/holmes_mac.cu:359-402);
 *   - buffers are caller-owned device pointers; `stream` is a cudaStream_t (NULL = legacy stream);
 *   - residue arrays are uint64 words laid out [items][limbs][N] (limb stride N), the layout of
 *     EasyFHE's Cipher.cv components [batch][limbs_alloc][N] (llama3fhe/parallel/wire.py:81-120);
 *   - moduli are indexed 0..L-1 for the Q limbs and L..L+K-1 for the special limbs;
 *   - NTT-domain words use the reference's root order (bench/cmp/kernels/holmes_encode.cu:65-71).
 * No function allocates device memory except holmes_ctx_create (its tables) and
 * holmes_ctx_create's secret upload; scratch buffers are passed in.
 * A context is used by one host thread at a time: some calls (holmes_modup with one or two items)
 * run independent parts on side streams and events the context owns (created on first use), and
 * join them into `stream` before returning, so their work is ordered on `stream` as a whole.
 */
#ifndef HOLMES_CUDA_H
#define HOLMES_CUDA_H
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct holmes_params {
  int log_n;           /* ring degree 2^log_n, 10..16 */
  int limbs;           /* L: Q limbs at the top level (depth + 1) */
  int dnum;            /* key-switch digits; alpha = ceil(L / dnum) limbs per digit */
  int dcrt_bits;       /* bits of Q limbs 1..L-1 */
  int first_mod_bits;  /* bits of Q limb 0 */
  int special_bits;    /* bits of the special primes */
  int special_limbs;   /* K; 0 = alpha */
  int hamming;         /* secret hamming weight; 0 = uniform ternary */
  uint64_t seed;       /* key / encryption randomness seed */
} holmes_params;

/* ---- context: replaces EasyFHE's generate_client_context / CKKSContextSpec
 *      (llama3fhe/backend.py:556-596 create_sim_context) */
int holmes_ctx_create(const holmes_params* params, void** ctx_out);
int holmes_ctx_destroy(void* ctx);
/* moduli[L + K] (host) */
int holmes_ctx_moduli(void* ctx, uint64_t* moduli_out);
/* dims[6] = {log_n, L, K, alpha, dnum, beta_max} (host) */
int holmes_ctx_dims(void* ctx, int* dims_out);
/* device pointer of the secret key [L + K][N] (NTT form); simulation contexts hold the client key */
int holmes_ctx_secret(void* ctx, void** secret_out);
/* automorphism index of a slot rotation (negative r as N/2 + r, keys.py:91-102); M - 1 = conjugation */
int holmes_galois(void* ctx, long long rotation, uint64_t* galois_out);
/* words of one switching key holding Q limbs < cap: 2 * beta(cap) * (cap + K) * N (keys.py:105-118) */
int holmes_key_words(void* ctx, int cap, long long* words_out);

/* ---- keys and client (EasyFHE generate_client_context keygen, client.encrypt / decrypt,
 *      llama3fhe/backend.py:293-396) */
/* switching key for X -> X^galois (galois > 1) or relinearisation (galois == 0):
 * key[2][beta(cap)][cap + K][N] = (b, a) */
int holmes_keygen(void* ctx, uint64_t galois, int cap, uint64_t* key, void* stream);
/* secret-key encryption of the NTT plaintext m[cur][N]: c1 = a, c0 = e - a s + m */
int holmes_encrypt(void* ctx, const uint64_t* m, int cur, uint64_t counter, uint64_t* c0, uint64_t* c1, void* stream);
/* coefficients (not centred) of c0 + c1 s, [cur][N] */
int holmes_decrypt(void* ctx, const uint64_t* c0, const uint64_t* c1, int cur, uint64_t* coef_out, void* stream);

/* ---- transforms (EasyFHE NttImpl / encode; holmes_encode.cu:108-285) */
/* in-place forward (inverse = 0) or inverse NTT of [items][limbs][N], limb l with modulus first_mod + l */
int holmes_ntt(void* ctx, uint64_t* data, int items, int limbs, long long item_stride, int first_mod, int inverse,
               void* stream);
/* encode rows of `slots` complex values z[rows][slots][2] (overwritten by the inverse special FFT) at `scale`
 * into NTT plaintexts out[rows][cur][N]; *flag (device int) is set to 1 if a value reaches 2^61 */
int holmes_encode(void* ctx, double* z, long long row_stride, int rows, int slots, double scale, int cur, uint64_t* out,
                  long long out_row_stride, int* flag, void* stream);
/* the two halves of holmes_encode: the inverse special FFT in place (EasyFHE cv_pre_encode_stage1), and the
 * rounding / reduction / NTT of already transformed rows (cv_encode, holmes_encode.cu:115-226) */
int holmes_fft_special_inv(void* ctx, double* z, long long row_stride, int rows, int slots, void* stream);
/* The reference's in-tree encode ABI (bench/cmp/kernels/holmes_encode.cu:240-285, bound by
 * bench/cmp/holmes_fast_stage2.py:21-39), N = 2^16 full slots: in[rows][in_stride] interleaved stage-1 doubles ->
 * out[rows][limbs][N] NTT plaintexts at scale sf, from the caller's per-limb primes / Barrett ratios / exponents and
 * root tables (psi^bitrev(k) and Shoup companions, [limbs][N]; gathered once per table address and device).  diffs,
 * rows_per_launch and limbs_per_block are scheduling details of the reference's kernels and are not needed;
 * parts & 3 == 0 does nothing (the reference's single-kernel timing modes), any other value encodes. */
int holmes_encode_stage2(void* out, const void* in, long long in_stride, int rows, double sf, int limbs,
                         const void* primes, const void* diffs, const void* ratios, const void* ks, const void* roots,
                         const void* roots_shoup, void* stream, int rows_per_launch, int parts, int limbs_per_block);
int holmes_encode_fft(void* ctx, const double* u, long long row_stride, int rows, int slots, double scale, int cur,
                      uint64_t* out, long long out_row_stride, int* flag, void* stream);
/* holmes_encode_fft onto the extended basis: out[rows][cur + K][N], the Q limbs first, then the K special limbs
 * (plaintexts for holmes_bsgs_mac_ext; EasyFHE's is_ext constants) */
int holmes_encode_fft_ext(void* ctx, const double* u, long long row_stride, int rows, int slots, double scale, int cur,
                          uint64_t* out, long long out_row_stride, int* flag, void* stream);
/* one BSGS chunk's plaintexts from the weight page in one call (LinearWeight.plaintext, weight.py:471-582:
 * pack, special FFT, rounding, NTT): holmes_pack_diagonals into rows_scratch ([giant_count * baby][slots][2]
 * doubles), holmes_fft_special_inv on them in place, then holmes_encode_fft into out[giant_count * baby][cur][N] at
 * `scale` */
int holmes_encode_diag_rows(void* ctx, const double* weight, int weight_complex, int dim, int lanes, int baby,
                            int giant_base, int giant_count, int lane_shift, int slots, double scale, int cur,
                            uint64_t* out, long long out_row_stride, double* rows_scratch, int* flag, void* stream);
/* diagonal rows of one BSGS chunk (weight.py:122-154 _cpu_packer / gpu_packer.py:48-200):
 * out[giant_count * baby][slots][2] complex; weight [dim][dim] float64 (weight_complex = 0), complex128 (1) or
 * float32 (2, widened exactly) */
int holmes_pack_diagonals(const double* weight, int weight_complex, int dim, int lanes, int baby, int giant_base,
                          int giant_count, int lane_shift, int slots, double* out, long long row_stride, void* stream);
/* diagonal rows of one BSGS chunk from a structured weight, replacing the reference's Triton
 * pack_structured_token_lane_bsgs_weight_chunk_triton_gpu (llama3fhe/operators/linear/gpu_packer.py:201-476;
 * map semantics llama3fhe/operators/linear/structured_weight.py:52-140): one to three real source matrices (host
 * array of device pointers, element strides, float32 when source_fp32) and device maps of `dim` entries --
 * int64 real/imag source and row per physical row, int64 real/imag column per physical column (negative = zero),
 * float64 real/imag scale per row and column_scale per column; value = source * (row scale * column scale) */
int holmes_pack_structured(const void* const* sources, const long long* row_strides, const long long* col_strides,
                           int source_count, int source_fp32, const long long* real_source, const long long* real_row,
                           const double* real_scale, const long long* imag_source, const long long* imag_row,
                           const double* imag_scale, const long long* real_column, const long long* imag_column,
                           const double* column_scale, int dim, int lanes, int baby, int giant_base, int giant_count,
                           int lane_shift, int slots, double* out, long long row_stride, void* stream);

/* ---- ciphertext arithmetic (fhe.homo_add / homo_sub / homo_mul_pt / homo_mul_i / rescale,
 *      llama3fhe/operators/primitives.py:21-190) */
/* op: 0 add, 1 sub, 2 multiply, 3 negate (b unused); limb l uses modulus l */
int holmes_elementwise(void* ctx, int op, const uint64_t* a, const uint64_t* b, uint64_t* out, int items, int limbs,
                       long long a_item, long long b_item, long long out_item, void* stream);
/* tensor product before relinearisation (fhe.homo_mul without relin, primitives.py:21-37): d0 = a0 b0,
 * d1 = a0 b1 + a1 b0, d2 = a1 b1 (mod q_l), one launch; item strides even */
int holmes_tensor_product(void* ctx, const uint64_t* a0, const uint64_t* a1, long long a_item, const uint64_t* b0,
                          const uint64_t* b1, long long b_item, uint64_t* d0, uint64_t* d1, uint64_t* d2,
                          long long d_item, int items, int limbs, void* stream);
/* multiply by X^(N/2) (slot-wise i) */
int holmes_mul_i(void* ctx, const uint64_t* a, uint64_t* out, int items, int limbs, long long a_item, long long out_item,
                 void* stream);
/* NTT-domain automorphism X -> X^galois */
int holmes_automorph(void* ctx, const uint64_t* a, uint64_t* out, uint64_t galois, int items, int limbs,
                     long long a_item, long long out_item, void* stream);
/* out[g][l][n] = sum_k weights[g][k][l] * a[k][l][n] (mod q_l) for k < nk, canonical residues (one component;
 * EasyFHE grouped_scalar_weighted_acc, llama3fhe/operators/nonlinear/polynomial.py:255-300) */
int holmes_weighted_acc(void* ctx, const uint64_t* a, long long a_item, int nk, const uint64_t* weights, uint64_t* out,
                        long long out_item, int groups, int limbs, void* stream);
/* multiply limb l by consts[l] (device array of canonical residues) */
int holmes_mul_const(void* ctx, const uint64_t* a, const uint64_t* consts, uint64_t* out, int items, int limbs,
                     long long a_item, long long out_item, void* stream);
/* divide by the last limb with centred rounding: in[comps][cur][N] -> out[comps][cur - 1][N];
 * scratch >= comps * N words */
int holmes_rescale(void* ctx, const uint64_t* in, long long in_stride, uint64_t* out, long long out_stride, int cur,
                   int comps, uint64_t* scratch, void* stream);

/* holmes_rescale with the post-operations of EasyFHE's homo_mul_relin_rescale_postop fused into its store
 * (llama3fhe/operators/nonlinear/polynomial.py:139-193, the Chebyshev basis T_2j = 2 T_j^2 - 1 and
 * T_2j+1 = 2 T_j T_j+1 - T_1): every rescaled word is doubled when apply_double != 0, then sub[comp][limb][N]
 * (component stride sub_stride, at least cur - 1 limbs: a deeper ciphertext's modulus drop) is subtracted when
 * sub is not null, then consts[limb] (device, canonical residues) is added when consts is not null.  Pass sub
 * and consts for the components they apply to (a scalar to component 0 only). */
int holmes_rescale_postop(void* ctx, const uint64_t* in, long long in_stride, uint64_t* out, long long out_stride,
                          int cur, int comps, uint64_t* scratch, int apply_double, const uint64_t* sub,
                          long long sub_stride, const uint64_t* consts, void* stream);

/* bootstrapping's ModRaise (EasyFHE bs.openfhe raise_ciphertext, bench/cmp/holmes_batch_bs.py:65-90): in[comps][1][N]
 * modulo q0 (NTT) is read as centred integers and written modulo q_0..q_{raise-1}: out[comps][raise][N];
 * scratch >= comps * N words */
int holmes_modraise(void* ctx, const uint64_t* in, long long in_stride, uint64_t* out, long long out_stride, int raise,
                    int comps, uint64_t* scratch, void* stream);
/* add consts[l] (device, canonical residues) to every NTT word of limb l: a constant polynomial
 * (fhe.homo_add_scalar, operators/nonlinear/polynomial.py) */
int holmes_add_const(void* ctx, const uint64_t* a, const uint64_t* consts, uint64_t* out, int items, int limbs,
                     long long a_item, long long out_item, void* stream);
/* the same scalar arithmetic with the per-limb constants read from HOST memory at the call (copied into the
 * launch's parameters, so no device copy and no stream synchronisation): op 0 out = a + k, op 1 out = a * k,
 * op 2 out = out + a * k (mod q_l), k[l] canonical residues.  The scalar products and sums of EvalMod and of
 * the polynomial evaluators (fhe.homo_mul_scalar / homo_add_scalar, operators/nonlinear/polynomial.py).
 * limbs <= 64; a_item and out_item even.  Returns -2 on a bad op or size. */
int holmes_const_op(void* ctx, int op, const uint64_t* a, const uint64_t* host_consts, uint64_t* out, int items,
                    int limbs, long long a_item, long long out_item, void* stream);

/* holmes_rescale without caller scratch, for callers that cannot allocate device memory (a runtime that
 * owns the whole pool, or a loop where cudaMalloc's device synchronisation is unacceptable).  No
 * counterpart in the reference.  Scratch comes from a 2 MiB array compiled into the library (held by every
 * GPU that loads it): comps * N must not exceed 4 * 2^16 words (-6 otherwise), and the calling thread's
 * current device must be the context's (-7 otherwise).  The first call on a device looks up the array's
 * device address, so make it before any stream capture.  That address is kept for the rest of the process:
 * it assumes one primary-context lifetime per device, so do not call this after cudaDeviceReset (or any other
 * teardown and re-creation of the device's primary context) in the same process.  Calls that overlap on the
 * GPU race on the shared array; nothing needs clearing between calls. */
int holmes_rescale_noalloc(void* ctx, const uint64_t* in, long long in_stride, uint64_t* out, long long out_stride,
                           int cur, int comps, void* stream);

/* ---- hybrid key switch (EasyFHE cv_modup / cv_innerproduct / cv_moddown, bench/cmp/report.py:23-46;
 *      fhe.homo_rotate, prepare_hoisted_baby_rotations, homo_relinearize) */
/* digits[items][beta(cur)][cur + K][N] = ModUp(c1[items][cur][N]) (item strides c1_item / digit_item words),
 * with every Q row (limb i < cur) multiplied by P^-1 mod q_i: the ModDown factor, paid here once for all the key
 * switches of a hoisted set.  The digits are an opaque intermediate for holmes_keyswitch;
 * scratch >= items * cur * N words */
int holmes_modup(void* ctx, const uint64_t* c1, long long c1_item, int cur, int items, uint64_t* digits,
                 long long digit_item, uint64_t* scratch, void* stream);
/* homo_rotate of `items` ciphertexts sharing one key (fhe.homo_rotate, operator.py:447; qkv_kernel.py:832 for the
 * conjugation galois 2N - 1): holmes_modup then holmes_keyswitch with add0 = c0, in one call.  c0 and c1 share the
 * item stride in_item; galois must be odd and > 1 (holmes_galois); key / key_cap as holmes_keyswitch takes them;
 * scratch >= holmes_rotate_scratch_words(ctx, cur, items) words (the digits, then the ModUp's and the key switch's
 * work area). */
int holmes_rotate_scratch_words(void* ctx, int cur, int items, long long* words);
int holmes_rotate(void* ctx, const uint64_t* c0, const uint64_t* c1, long long in_item, int cur, const uint64_t* key,
                  int key_cap, uint64_t galois, uint64_t* out0, uint64_t* out1, long long out_item, int items,
                  uint64_t* scratch, void* stream);
/* prepare_hoisted_baby_rotations (operator.py:113-119) in one call: one ModUp of the `items` ciphertexts, then
 * rotation r < count by keys[r] / key_caps[r] / galois[r] (host arrays; galois <= 1 copies the input) into
 * out_c + r * out_rot (item stride out_item); scratch as holmes_rotate's */
int holmes_hoisted_rotations(void* ctx, const uint64_t* c0, const uint64_t* c1, long long in_item, int cur, int items,
                             int count, const uint64_t* const* keys, const int* key_caps, const uint64_t* galois,
                             uint64_t* out0, uint64_t* out1, long long out_item, long long out_rot, uint64_t* scratch,
                             void* stream);
/* the giant Horner chain of hoisted_mac_sum (bench/cmp/holmes_multi_mac.py:148-194) in one call: acc = partial[G-1];
 * acc = rot(acc, giant offset) + partial[g] for g = G-2 .. 0, partial g of item i at p_c + g * part_giant +
 * i * part_item, one key (galois of the giant offset); result in out_c; scratch >= holmes_rotate_scratch_words(ctx,
 * cur, items) + 2 * items * cur * N words */
int holmes_giant_sum(void* ctx, const uint64_t* p0, const uint64_t* p1, long long part_item, long long part_giant,
                     int cur, int items, int giants, const uint64_t* key, int key_cap, uint64_t galois, uint64_t* out0,
                     uint64_t* out1, long long out_item, uint64_t* scratch, void* stream);
/* homo_mul_relin (llama3fhe/operators/primitives.py:21-37) of `items` pairs in one call: the tensor product
 * (d0, d1, d2) = (a0 b0, a0 b1 + a1 b0, a1 b1), then the relinearisation key switch of d2 added to (d0, d1); key /
 * key_cap the relinearisation key (holmes_keygen with galois 0); the four inputs share the item stride in_item;
 * scratch >= holmes_rotate_scratch_words(ctx, cur, items) + 4 * items * cur * N words.  Not rescaled. */
int holmes_mul_relin(void* ctx, const uint64_t* a0, const uint64_t* a1, const uint64_t* b0, const uint64_t* b1,
                     long long in_item, int cur, int items, const uint64_t* key, int key_cap, uint64_t* out0,
                     uint64_t* out1, long long out_item, uint64_t* scratch, void* stream);
/* exact scratch words of a composed entry point for `items` ciphertexts at `cur` limbs:
 * op HOLMES_OP_ROTATE (holmes_rotate, holmes_hoisted_rotations), HOLMES_OP_GIANT_SUM (holmes_giant_sum),
 * HOLMES_OP_MUL_RELIN (holmes_mul_relin); -4 for an unknown op.  Same sizing rules as the comments above. */
#define HOLMES_OP_ROTATE 0
#define HOLMES_OP_GIANT_SUM 1
#define HOLMES_OP_MUL_RELIN 2
int holmes_scratch_words(void* ctx, int op, int cur, int items, long long* words);
/* for `items` ciphertexts sharing one key:
 *   out0 = perm(add0) + ModDown(sum_j perm(digit_j) key_b[j]) + post0
 *   out1 = perm(add1) + ModDown(sum_j perm(digit_j) key_a[j]) + post1
 * perm = automorphism X -> X^galois (galois <= 1: identity); every addend may be NULL;
 * scratch >= items * 2 * (K + cur) * N words */
int holmes_keyswitch(void* ctx, const uint64_t* digits, long long digit_item, int cur, const uint64_t* key, int key_cap,
                     uint64_t galois, const uint64_t* add0, const uint64_t* add1, long long add_item,
                     const uint64_t* post0, const uint64_t* post1, long long post_item, uint64_t* out0,
                     uint64_t* out1, long long out_item, int items, uint64_t* scratch, void* stream);

/* ---- extended basis Q u P (EasyFHE fast_rotate(output_ext=True) / grouped_pairwise_mac / moddown_from_ext,
 *      llama3fhe/operators/attention/prefill/input.py:1007-1031, 1198-1236).  Extended ciphertexts are
 *      [items][cur + K][N] with the Q limbs first. */
/* the key switch of holmes_keyswitch without its ModDown: out0 = P perm(add0) + sum_j perm(digit_j) key_b[j],
 * out1 = sum_j perm(digit_j) key_a[j], over all cur + K limbs (add0 may be NULL) */
int holmes_keyswitch_ext(void* ctx, const uint64_t* digits, long long digit_item, int cur, const uint64_t* key,
                         int key_cap, uint64_t galois, const uint64_t* add0, long long add_item, uint64_t* out0,
                         uint64_t* out1, long long out_item, int items, void* stream);
/* out_c [items][cur][N] = (in_c,Q - conv_{P->Q}(in_c,P)) P^-1, the ModDown; holmes_moddown(holmes_keyswitch_ext(x))
 * equals holmes_keyswitch(x) word for word; scratch >= items * 2 * (K + cur) * N words */
int holmes_moddown(void* ctx, const uint64_t* in0, const uint64_t* in1, long long in_item, int cur, uint64_t* out0,
                   uint64_t* out1, long long out_item, int items, uint64_t* scratch, void* stream);
/* holmes_bsgs_mac over the cur + K limbs of extended babies and plaintexts (limb l >= cur: special prime l - cur) */
int holmes_bsgs_mac_ext(void* ctx, uint64_t* res, const uint64_t* const* c0s, const uint64_t* const* c1s,
                        long long bstride, int nb, int inputs, const uint64_t* pts, long long pstride, int groups,
                        int cur, void* stream);

/* ---- BSGS plaintext multiply-accumulate (fhe.hoisted_mac_sum baby step, holmes_multi_mac.py:148-194):
 * res[2][groups][inputs][limbs][N] = sum_b pts[g * nb + b][limb] * baby_i[b][c][limb] (mod q_limb);
 * c0s / c1s: host arrays of `inputs` (<= 32) device pointers to baby bases [nb][>= limbs][N] (item stride bstride) */
int holmes_bsgs_mac(void* ctx, uint64_t* res, const uint64_t* const* c0s, const uint64_t* const* c1s, long long bstride,
                    int nb, int inputs, const uint64_t* pts, long long pstride, int groups, int limbs, void* stream);

/* ---- collectives: mod-q sum of nsrc (<= 16) equally shaped buffers (peer-mapped partials included);
 *      the owner-side reduce of parallel/decode/decode_collectives.py:59-195 and
 *      operators/attention/distributed/distributed_output.py:801-830 */
int holmes_modsum(void* ctx, const uint64_t* const* srcs, int nsrc, uint64_t* out, int items, int limbs,
                  long long item_stride, void* stream);

/* ---- modular reduce-scatter over peer memory (the modreduce_scatter export; replaces the reference's owner-side
 *      reduce of host-staged partials, parallel/prefill/stations.py:1565-1596, parallel/decode/decode_collectives.py:
 *      59-195, operators/linear/shard/mlp_feature_shard.py:536-575).  One process per GPU.
 * holmes_ipc_export: the 64-byte CUDA IPC handle of a device allocation, for the other ranks;
 * holmes_ipc_import: map a peer's handle into the CALLING device (make the reading device current first; peer access
 *   is enabled lazily); holmes_ipc_close: unmap. */
/* holmes_peer_alloc / holmes_peer_free: a zeroed device allocation of its own (an IPC handle names a whole
 * allocation, so buffers shared with peers are allocated here, not carved from a caching allocator's pool) */
int holmes_peer_alloc(unsigned long long bytes, void** ptr_out);
int holmes_peer_free(void* ptr);
int holmes_ipc_export(const void* dev_ptr, void* handle_out);
int holmes_ipc_import(const void* handle, void** ptr_out);
int holmes_ipc_close(void* ptr);
/* store `epoch` into each of `count` (<= 16) 64-bit flags (host array of device pointers, local or peer-mapped) after a
 * system-scope fence: every earlier write on `stream` is visible to the peers before the flag is */
int holmes_peer_signal(uint64_t* const* flags, int count, uint64_t epoch, void* stream);
/* wait on `stream` until every flag (host array of device pointers, local or peer-mapped) is >= epoch; a flag that
 * is still below after budget_cycles SM clocks makes the kernel write its index + 1 into *status (device int) and
 * return -- bounded, never a hang; the host reads *status after the stream's work */
int holmes_peer_wait(const uint64_t* const* flags, int count, uint64_t epoch, long long budget_cycles, int* status,
                     void* stream);
/* out = sum_k srcs[k] mod q over [items][limbs][N] (item stride item_stride words in every source and in out; srcs a
 * host array of nsrc <= 16 device pointers, this rank's own and peer-mapped ones, read with plain loads); does
 * nothing when *status is nonzero (a wait before it gave up) */
int holmes_modreduce_scatter(void* ctx, const uint64_t* const* srcs, int nsrc, uint64_t* out, int items, int limbs,
                             long long item_stride, const int* status, void* stream);

/* kernels launched by this library since it was loaded (all streams, all contexts) */
int holmes_launch_count(unsigned long long* count_out);

/* 1 when a tensor-core kernel's bounded wait ran out since the last reset (the kernel then stopped early and
 * its output is incomplete); reset != 0 clears the flag.  Synchronises with the device.  No reference
 * counterpart: EasyFHE kernels do not wait on hardware barriers. */
int holmes_device_error(int reset, int* flag_out);

/* The reference's gathered MAC for the attention sparse BSGS (bench/cmp/kernels/holmes_mac.cu:276-347, 404-428),
 * same signature and return codes (N = 2^16): res[c][k][i][l][n] = sum_{seg[k] <= r < seg[k+1]}
 * pts[prow[r]][l][n] * baby_i[idx[r]][c][l][n] (mod q_l), res [2][K][inputs][limbs][N]; c0s / c1s host arrays of
 * `inputs` (<= 32) device pointers to baby bases (item stride bstride); idx / prow [rows], seg [K + 1] (int32,
 * device); ti in {1, 2, 4}; moduli from the reference's primes / barret_ratio / barret_k arrays. */
int holmes_mac_gather(uint64_t* res, const uint64_t* const* c0s, const uint64_t* const* c1s, long long bstride,
                      const int* idx, const int* prow, const int* seg, int inputs, int K, const uint64_t* pts,
                      long long pstride, int ti, int limbs, const uint64_t* primes, const uint64_t* ratios,
                      const uint64_t* ks, void* stream_ptr);
/* ---- drop-in for the reference's own ctypes binding (bench/cmp/kernels/holmes_mac.cu:359-402, bound in
 *      bench/cmp/holmes_multi_mac.py:33-54): same signature, arguments and return codes; N = 2^16;
 *      `ti` is accepted from the reference's tile set and used only as a hint. */
int holmes_mac_multi(uint64_t* res, const uint64_t* const* c0s, const uint64_t* const* c1s, long long bstride, int nb,
                     int inputs, const uint64_t* pts, long long pstride, int groups, int ti, int limbs,
                     const uint64_t* primes, const uint64_t* ratios, const uint64_t* ks, void* stream_ptr);

#ifdef __cplusplus
}
#endif
#endif
