// BSGS plaintext multiply-accumulate on the 5th-generation tensor cores (tcgen05, kind::i8).
//
// res[c][g][i][l][n] = sum_b pt[g nb + b][l][n] * baby_i[b][c][l][n] mod q_l, the operation of k_bsgs_mac3,
// as byte-sliced integer matrix products.  For one coefficient n of limb l write every 64-bit residue as its
// eight little-endian bytes, x = sum_j x_j 256^j.  Then
//     D[(i, c, bb)][(g, a)] = sum_b baby_i[b][c]_bb * pt[g nb + b]_a          (u8 x u8 -> s32, exact)
//     res[c][g][i] = sum_{a, bb} 256^(a + bb) D[(i, c, bb)][(g, a)]  mod q_l,
// an M x N x K = (8 inputs x 2 components x 8 bytes) x (8 giants x 8 bytes) x (babies) product per M-tile.
// In MN-major operand layout the eight bytes of a residue are eight consecutive M (or N) entries, so the
// residues are copied into shared memory unchanged, one aligned 8-byte cp.async per word: no byte shuffling.
// Products are below 2^16 and K <= 128, so D < 2^23 and the recombined value V < 128 q^2 fits in 128 bits.
//
// Shared-memory operand layout (no swizzle, MN-major canonical form: 16 MN-bytes x 8 K-rows per 128-byte core
// matrix): A tile of one (coefficient, M-tile) per 32-baby stage = [K block 4][M block 8][8 rows][16 bytes],
// leading (K) byte offset 1024, stride (M) byte offset 128; B tile of one coefficient = [K block 4][N block 4]
// [8 rows][16 bytes], offsets 512 / 128.  The accumulator of one (coefficient, M-tile) is 128 TMEM lanes x 64
// columns (row m = lane m).
//
// Work: one persistent CTA per SM takes items of 4 coefficients x 8 inputs x 8 giants of one limb and runs them as
// one stream of 32-baby stages, with warps specialised by role:
//   * producers (4 warps) copy the stage's words into a 6-slot ring with 8-byte cp.async (thread p takes coefficient
//     p % 4 of baby p / 4 for every row group and giant, so 4 lanes read each 32-byte sector together) and arrive on
//     the slot's "full" mbarrier once their copies have landed (two stages in flight per thread);
//   * one thread issues the stage's MMAs into one of two TMEM accumulator buffers and commits them to the slot's
//     "empty" mbarrier (the producers may refill it) and, after an item's last stage, to the buffer's "full";
//   * the epilogue (8 warps, two per TMEM lane quadrant) reads the finished buffer, folds the 8 column bytes of each
//     giant, shifts by its own row byte, combines the 8 byte rows of each (input, component) in three butterfly
//     rounds over lanes ^4, ^2, ^1 (lane bb ends with giant bb), reduces mod q_l, stores, and arrives on the
//     buffer's "empty" so the MMAs of the item after next may overwrite it.
// Every wait is bounded and polls a shared abort flag; a wait that runs out sets g_tc_error and the flag, every
// role leaves its loop, and the CTA still waits (bounded) for its MMAs and copies and frees its TMEM.
#include "ops.h"

namespace holmes {

__device__ int g_tc_error;

namespace {

constexpr int kT = 4;    // coefficient positions per item (one 32-byte sector of every row)
constexpr int kKS = 32;  // babies per stage (the K of one MMA)
constexpr u32 kIdesc = (2u << 4)               // D: s32
                       | (0u << 7) | (0u << 10)  // A, B: u8
                       | (1u << 15) | (1u << 16) // A, B: MN-major
                       | ((64u >> 3) << 17)      // N = 64
                       | ((128u >> 4) << 24);    // M = 128
constexpr long long kWaitLimit = 1ll << 20;  // try_wait polls; a healthy wait ends within microseconds

// One item: kT coefficients x 8 inputs (one M-tile: 8 inputs x 2 components x 8 bytes) x 8 giants of one limb.
struct TcGeom {
  static constexpr int PRODUCERS = 128;  // warps 0-3
  static constexpr int MMA_WARP = 4;
  static constexpr int EPI_WARP0 = 5;    // warps 5-12: TMEM lane quadrant w % 4, coefficients 2 ((w - 5) / 4) .. +1
  static constexpr int EPILOGUE = 256;
  static constexpr int THREADS = PRODUCERS + 32 + EPILOGUE;
  static constexpr int A_BYTES = 128 * kKS;  // A tile of one coefficient per stage: 4 KB
  static constexpr int B_BYTES = 64 * kKS;   // B tile: 2 KB
  static constexpr int STAGE = kT * (A_BYTES + B_BYTES);
  static constexpr int NS = 6;               // ring slots
  static constexpr int LAG = 2;              // stages a producer keeps in flight before signalling one
  static constexpr int BAR = NS * STAGE;     // barrier area
  static constexpr int SMEM = NS * STAGE + 256;
  static constexpr int ACC = kT * 64;        // TMEM columns of one accumulator buffer
  static constexpr int TCOLS = 2 * ACC;      // 512: the whole TMEM, one CTA per SM
};

__device__ __forceinline__ u32 smem_u32(const void* p) { return (u32)__cvta_generic_to_shared(p); }
__device__ __forceinline__ u64 umma_desc(u32 addr, u32 lbo, u32 sbo) {
  return (u64)((addr >> 4) & 0x3FFF) | ((u64)((lbo >> 4) & 0x3FFF) << 16) | ((u64)((sbo >> 4) & 0x3FFF) << 32) |
         (1ull << 46);
}
__device__ __forceinline__ void cp_async8(u32 dst, const void* src, bool valid) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8, %2;\n" ::"r"(dst), "l"(src), "r"(valid ? 8 : 0));
}
__device__ __forceinline__ void mbar_arrive(u32 bar) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(bar) : "memory");
}
// bounded wait for the phase of parity `parity`; gives up early when another role raised the abort flag
__device__ __forceinline__ bool mbar_wait(u32 bar, u32 parity, const volatile int* abort_flag) {
  for (long long it = 0; it < kWaitLimit; ++it) {
    if ((it & 255) == 255 && *abort_flag) return false;
    u32 ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t"
        "}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    if (ok) return true;
  }
  return false;
}
__device__ __forceinline__ void tmem_ld16(u32 addr, u32 (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(addr));
}

// 128-bit values as four 32-bit words, least significant first
struct W4 {
  u32 w[4];
};
// x + y (mod 2^128), one carry chain
__device__ __forceinline__ W4 add4(const W4& x, const W4& y) {
  W4 r;
  asm("add.cc.u32 %0, %4, %8;\n\taddc.cc.u32 %1, %5, %9;\n\taddc.cc.u32 %2, %6, %10;\n\taddc.u32 %3, %7, %11;"
      : "=r"(r.w[0]), "=r"(r.w[1]), "=r"(r.w[2]), "=r"(r.w[3])
      : "r"(x.w[0]), "r"(x.w[1]), "r"(x.w[2]), "r"(x.w[3]), "r"(y.w[0]), "r"(y.w[1]), "r"(y.w[2]), "r"(y.w[3]));
  return r;
}
// sum_a c[a] 256^(a + bb) for the eight column bytes a of one giant (each c < 2^23) and this lane's byte bb:
// the words of sum_a c[a] 256^a (< 2^81) shifted by 8 (bb % 4) bits, then up one word when bb >= 4.  Every such
// term is at most the whole sum, which is below 2^128, so nothing is lost.
__device__ __forceinline__ W4 fold_shift(const u32* c, u32 sh, bool up) {
  const u32 p0 = c[0] + (c[1] << 8), p1 = c[2] + (c[3] << 8), p2 = c[4] + (c[5] << 8), p3 = c[6] + (c[7] << 8);
  const u64 q0 = (u64)p0 + ((u64)p1 << 16), q1 = (u64)p2 + ((u64)p3 << 16);  // < 2^49 each
  const u64 mid = (q0 >> 32) + (u32)q1;
  const u32 v0 = (u32)q0, v1 = (u32)mid, v2 = (u32)(q1 >> 32) + (u32)(mid >> 32);
  const u32 x0 = v0 << sh, x1 = __funnelshift_l(v0, v1, sh), x2 = __funnelshift_l(v1, v2, sh),
            x3 = __funnelshift_l(v2, 0u, sh);
  W4 r;
  r.w[0] = up ? 0u : x0;
  r.w[1] = up ? x0 : x1;
  r.w[2] = up ? x1 : x2;
  r.w[3] = up ? x2 : x3;
  return r;
}
// one butterfly round of the reduce-scatter over the 8 byte lanes: the lane with bit `hi` set keeps the upper
// half of its values, sends the lower half to lane ^ m and adds what it receives (branch-free selects)
__device__ __forceinline__ W4 exchange(const W4& lowv, const W4& highv, bool hi, int m) {
  W4 keep, send, recv;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    keep.w[k] = hi ? highv.w[k] : lowv.w[k];
    send.w[k] = hi ? lowv.w[k] : highv.w[k];
    recv.w[k] = __shfl_xor_sync(0xffffffffu, send.w[k], m);
  }
  return add4(keep, recv);
}

}  // namespace

template <int SPI>
__global__ void __launch_bounds__(TcGeom::THREADS, 1)
    k_bsgs_mac_tc(u64* __restrict__ res, InPtrs in, long long bstride, int nb, int inputs, int G,
                  const u64* __restrict__ pts, long long pstride, int limbs, ModSrc ms, int log_n) {
  using Geo = TcGeom;
  extern __shared__ __align__(1024) unsigned char tc_smem[];
  unsigned char* ring = tc_smem;
  u64* full = reinterpret_cast<u64*>(tc_smem + Geo::BAR);  // [NS]: producers -> MMA
  u64* empty = full + Geo::NS;                               // [NS]: MMA -> producers
  u64* afull = empty + Geo::NS;                              // [2]: MMA -> epilogue
  u64* aempty = afull + 2;                                   // [2]: epilogue -> MMA
  u32* tmem_slot = reinterpret_cast<u32*>(aempty + 2);
  int* abort_flag = reinterpret_cast<int*>(tmem_slot + 1);
  const volatile int* abort_v = abort_flag;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int N = 1 << log_n;
  const int nblocks = N / kT;
  const int ggroups = (G + 7) / 8;
  const int igroups = (inputs + 7) / 8;
  const int items = nblocks * limbs * ggroups * igroups;
  constexpr int spi = SPI;  // stages per item, (nb + 31) / 32
  const int my_items = (int)blockIdx.x < items ? (items - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
  const int stages = my_items * spi;

  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"((u32)Geo::TCOLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::);
  }
  if (tid == 0) {
    for (int b = 0; b < Geo::NS; ++b) {
      asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(full + b)), "r"((u32)Geo::PRODUCERS));
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_u32(empty + b)));
    }
    for (int b = 0; b < 2; ++b) {
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_u32(afull + b)));
      asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(aempty + b)), "r"((u32)Geo::EPILOGUE));
    }
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const u32 tmem = *tmem_slot;

  // item -> (input group, coefficient block, limb, giant group), input groups fastest so that the CTAs running
  // at one time share the plaintext words in L2 and read neighbouring words of the same rows
  struct Item {
    int limb, n0, g0, i0;
  };
  auto decode = [&](int it) {
    const int k = (int)blockIdx.x + it * (int)gridDim.x;
    Item x;
    x.i0 = (k % igroups) * 8;
    int r = k / igroups;
    x.n0 = (r % nblocks) * kT;
    r /= nblocks;
    x.limb = r % limbs;
    x.g0 = (r / limbs) * 8;
    return x;
  };
  auto fail = [&]() {
    *abort_flag = 1;
    atomicExch(&g_tc_error, 1);
  };

  int committed = -1;  // MMA thread: last stage whose MMAs were committed
  if (warp < Geo::PRODUCERS / 32) {
    // ------------------------------------------------------------------ producers
    // Thread p copies coefficient t = p % 4 of baby bl = p / 4 of the stage for all 16 row groups (A) and all 8
    // giants (B): the 4 lanes of a (row, baby) read one 32-byte sector together, 8 sectors per warp instruction.
    const int t = tid % kT, bl = tid / kT;
    const u32 a_off = (u32)(t * Geo::A_BYTES + (bl / 8) * 1024 + (bl % 8) * 16);
    const u32 b_off = (u32)(kT * Geo::A_BYTES + t * Geo::B_BYTES + (bl / 8) * 512 + (bl % 8) * 16);
    int ld_item = -1;
    Item x{0, 0, 0, 0};
    int k = 0;
    for (; k < stages; ++k) {
      const int slot = k % Geo::NS, use = k / Geo::NS;
      const bool ok = __all_sync(0xffffffffu, use == 0 || mbar_wait(smem_u32(empty + slot), (u32)((use - 1) & 1),
                                                                  abort_v));
      if (!ok) {
        if (lane == 0) fail();
        break;
      }
      const int it = k / spi, b = (k % spi) * kKS + bl;
      if (it != ld_item) {
        ld_item = it;
        x = decode(it);
      }
      const size_t lpos = ((size_t)x.limb << log_n) + x.n0 + t;
      const u32 base = smem_u32(ring + slot * Geo::STAGE);
      const bool bok = b < nb;
      const size_t boff = (size_t)b * bstride + lpos;
#pragma unroll
      for (int gm = 0; gm < 16; ++gm) {
        const int i = x.i0 + gm / 2;
        const bool ok2 = bok && i < inputs;
        const u64* src = ok2 ? (gm & 1 ? in.c1[i] : in.c0[i]) + boff : pts;
        cp_async8(base + a_off + (u32)((gm / 2) * 128 + 8 * (gm % 2)), src, ok2);
      }
#pragma unroll
      for (int g = 0; g < 8; ++g) {
        const bool ok2 = bok && x.g0 + g < G;
        const u64* src = ok2 ? pts + ((size_t)(x.g0 + g) * nb + b) * pstride + lpos : pts;
        cp_async8(base + b_off + (u32)((g / 2) * 128 + 8 * (g % 2)), src, ok2);
      }
      asm volatile("cp.async.commit_group;\n" ::);
      if (k >= Geo::LAG) {
        asm volatile("cp.async.wait_group %0;\n" ::"n"(Geo::LAG));
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        mbar_arrive(smem_u32(full + (k - Geo::LAG) % Geo::NS));
      }
    }
    asm volatile("cp.async.wait_all;\n" ::);
    if (k == stages) {  // the last LAG stages
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      for (int r = stages - Geo::LAG < 0 ? 0 : stages - Geo::LAG; r < stages; ++r) mbar_arrive(smem_u32(full + r % Geo::NS));
    }
  } else if (warp == Geo::MMA_WARP) {
    // ------------------------------------------------------------------ MMA issue (lane 0 issues; the warp waits
    // together so that every exit is warp-uniform)
    for (int it = 0; it < my_items; ++it) {
      const int buf = it & 1;
      bool ok = it < 2 || mbar_wait(smem_u32(aempty + buf), (u32)(((it >> 1) - 1) & 1), abort_v);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) {
        if (lane == 0) fail();
        break;
      }
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      for (int s2 = 0; s2 < spi && ok; ++s2) {
        const int k = it * spi + s2, slot = k % Geo::NS;
        ok = __all_sync(0xffffffffu, mbar_wait(smem_u32(full + slot), (u32)((k / Geo::NS) & 1), abort_v));
        if (!ok) break;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        if (lane == 0) {
          const u32 base = smem_u32(ring + slot * Geo::STAGE);
#pragma unroll
          for (int t = 0; t < kT; ++t) {
            const u64 da = umma_desc(base + t * Geo::A_BYTES, 1024, 128);
            const u64 db = umma_desc(base + kT * Geo::A_BYTES + t * Geo::B_BYTES, 512, 128);
            asm volatile(
                "{\n\t.reg .pred p;\n\t"
                "setp.ne.b32 p, %4, 0;\n\t"
                "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %5, %5, %5}, p;\n\t"
                "}" ::"r"(tmem + (u32)(buf * Geo::ACC + t * 64)),
                "l"(da), "l"(db), "r"(kIdesc), "r"((u32)(s2 > 0)), "r"(0u)
                : "memory");
          }
          asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                           smem_u32(empty + slot))
                       : "memory");
        }
        __syncwarp();
        committed = k;
      }
      if (!ok) {
        if (lane == 0) fail();
        break;
      }
      if (lane == 0)
        asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                         smem_u32(afull + buf))
                     : "memory");
      __syncwarp();
    }
  } else {
    // ------------------------------------------------------------------ epilogue
    const int quad = warp % 4, th = (warp - Geo::EPI_WARP0) / 4;
    const int row = quad * 32 + lane;  // TMEM lane = accumulator row (group, byte)
    const int gm = row / 8, bb = row % 8;
    const bool hi2 = bb & 4, hi1 = bb & 2, hi0 = bb & 1;
    const u32 sh = 8u * (u32)(bb & 3);
    for (int it = 0; it < my_items; ++it) {
      const int buf = it & 1;
      bool ok = mbar_wait(smem_u32(afull + buf), (u32)((it >> 1) & 1), abort_v);
      ok = __all_sync(0xffffffffu, ok);  // the TMEM loads below are warp-collective
      if (!ok) {
        if (lane == 0) fail();
        break;
      }
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const Item x = decode(it);
      const Mod m = ms.get(x.limb);
      u64 outv[2];
#pragma unroll
      for (int tt = 0; tt < 2; ++tt) {
        const int t = 2 * th + tt;
        const u32 col0 = tmem + ((u32)(quad * 32) << 16) + (u32)(buf * Geo::ACC + t * 64);
        u32 c[64];
        tmem_ld16(col0, *reinterpret_cast<u32(*)[16]>(c));
        tmem_ld16(col0 + 16u, *reinterpret_cast<u32(*)[16]>(c + 16));
        tmem_ld16(col0 + 32u, *reinterpret_cast<u32(*)[16]>(c + 32));
        tmem_ld16(col0 + 48u, *reinterpret_cast<u32(*)[16]>(c + 48));
        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
        W4 v[8];
#pragma unroll
        for (int g = 0; g < 8; ++g) v[g] = fold_shift(c + 8 * g, sh, hi2);
        W4 xr[4], y[2];
#pragma unroll
        for (int j = 0; j < 4; ++j) xr[j] = exchange(v[j], v[j + 4], hi2, 4);
#pragma unroll
        for (int j = 0; j < 2; ++j) y[j] = exchange(xr[j], xr[j + 2], hi1, 2);
        const W4 z = exchange(y[0], y[1], hi0, 1);
        outv[tt] = reduce128(((u64)z.w[3] << 32) | z.w[2], ((u64)z.w[1] << 32) | z.w[0], m);
      }
      // the accumulator buffer may be overwritten once every epilogue thread has read it
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      mbar_arrive(smem_u32(aempty + buf));
      // lane bb holds giant g0 + bb of (input i0 + gm / 2, component gm % 2) at coefficients n0 + 2 th, +1
      const int i = x.i0 + gm / 2, cc = gm % 2, g = x.g0 + bb;
      if (i < inputs && g < G) {
        const size_t is = (size_t)limbs << log_n, gs = (size_t)inputs * is;
        u64* dst = res + ((size_t)cc * G + g) * gs + (size_t)i * is + ((size_t)x.limb << log_n) + x.n0 + 2 * th;
        *reinterpret_cast<ulonglong2*>(dst) = make_ulonglong2(outv[0], outv[1]);
      }
    }
  }
  // let in-flight MMAs finish before the accumulators are released (bounded; immediate when all went well)
  if (warp == Geo::MMA_WARP && committed >= 0)
    mbar_wait(smem_u32(empty + committed % Geo::NS), (u32)((committed / Geo::NS) & 1), abort_v);
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 0)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"((u32)Geo::TCOLS));
}

int bsgs_mac_tc(ModSrc ms, u64* res, const InPtrs& in, long long bstride, int nb, int inputs, const u64* pts,
                long long pstride, int groups, int limbs, int log_n, cudaStream_t st) {
  // accumulated byte products stay exact and the recombined sum stays below 2^128 for up to 128 babies; the
  // item count stays an int
  if (nb < 1 || nb > 128 || inputs < 1 || inputs > kMaxInputs || log_n < 10) return -7;
  if ((long long)((1 << log_n) / kT) * limbs * ((groups + 7) / 8) * ((inputs + 7) / 8) >= (1ll << 31)) return -7;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int spi = (nb + kKS - 1) / kKS;
  auto go = [&](auto kernel) {
    cudaError_t e = set_smem_once((const void*)kernel, TcGeom::SMEM);
    if (e != cudaSuccess) return (int)e;
    count_launch();
    kernel<<<sms, TcGeom::THREADS, TcGeom::SMEM, st>>>(res, in, bstride, nb, inputs, groups, pts, pstride, limbs,
                                                        ms, log_n);
    return (int)cudaGetLastError();
  };
  switch (spi) {
    case 1: return go(k_bsgs_mac_tc<1>);
    case 2: return go(k_bsgs_mac_tc<2>);
    case 3: return go(k_bsgs_mac_tc<3>);
    default: return go(k_bsgs_mac_tc<4>);
  }
}

int tc_error_flag(int reset, int* out) {
  int v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, g_tc_error, sizeof(int));
  if (e != cudaSuccess) return (int)e;
  if (reset) {
    const int z = 0;
    e = cudaMemcpyToSymbol(g_tc_error, &z, sizeof(int));
    if (e != cudaSuccess) return (int)e;
  }
  *out = v;
  return 0;
}

}  // namespace holmes
