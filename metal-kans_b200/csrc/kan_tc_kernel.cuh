// kan_tc_kernel.cuh -- fused KAN layer on the 5th-generation tensor cores (tcgen05 + TMEM + TMA).
//
// Y[B, D_out] = bias + [Phi(x) | silu(x)] Wp^T is one dense contraction.  The weights are packed
// once (kan_tc_pack) into a feature-blocked layout: each 64-column K block holds F = 64 / KT whole
// input features of KT = K + has_base columns (the K basis terms of the feature, then its
// base-branch weight), zero padded.  One CTA computes a 128 x BN output tile over a range of K
// blocks:
//
//   warps 0-7  basis producers, two groups of four warps taking alternate pipeline stages; each
//              thread owns one row of the 128 x 64 A tile.  It prefetches the inputs of its next
//              block into registers, evaluates the K basis terms and SiLU of the block's F
//              features in registers (reference rounding points, see kan_device.cuh) and stores
//              the row as eight 16-byte chunks in the 128-byte-swizzled K-major layout the MMA
//              reads.  Phi never reaches HBM (the reference writes it to a scratch buffer and runs
//              MPS GEMMs on it, metal_kan_bridge.mm:503-523).  After the K loop these warps run
//              the epilogue: tcgen05.ld of the fp32 accumulator, + bias, round, store.
//   warp 8     TMA producer: one cp.async.bulk.tensor.2d per stage for the BN x 64 weight tile
//              (two 256-row boxes for BN = 512).
//   warp 9     TMEM allocator and MMA issuer: 4 x tcgen05.mma.cta_group::1.kind::f16
//              (M=128, N=BN, K=16) per stage into the TMEM accumulator -- for BN = 512 ("wide")
//              two N = 256 MMAs per K step into the two halves of TMEM, so each basis block the
//              producers build feeds twice the tensor work; tcgen05.commit frees the stage and
//              finally signals the epilogue.
//   warp 10    TMA producer of the input tiles (64 features x 128 rows per stage).
//
// The grid runs M tiles fastest: the CTAs resident at one time share a few weight panels in L2.
//
// Split-K (grid.z = S > 1, launched as clusters of S CTAs along z) serves grids too small to fill
// the 148 SMs without recomputing the basis per N tile: each CTA stages the other splits' column
// slices of its fp32 partial tile in its own shared memory and bulk-copies them to their owners
// (distributed shared memory, no multicast); CTA z sums column slice z over the S partials in
// split order (deterministic), adds the bias and stores Y -- in column rounds when the slots of
// whole slices do not fit.  No global scratch is involved.
//
// fuse_swiglu (GatedKAN): the packed weights interleave gate and up rows per 256 outputs and the
// epilogue writes silu(gate) * up of the wide tile's two halves.
//
// Every mbarrier wait is bounded (about one second of SM clocks); on expiry the kernel records
// the error in the device error word, skips its remaining work, still joins every CTA-wide and
// cluster-wide barrier and releases TMEM.
#pragma once

#include <cuda.h>

#include "kan_device.cuh"
#include "kan_launch.h"

namespace kan {
namespace tc {

constexpr int BM = 128;
constexpr int BK = 64;                 // 64 16-bit elements = one 128-byte swizzle row
constexpr int STAGES = 4;              // basis (A) tiles
constexpr int BSTAGES = 3;             // weight (B) tiles
constexpr int XSTAGES = 3;             // input tiles: 64 features x 128 rows, TMA-loaded
constexpr int A_STAGE_BYTES = BM * BK * 2;
constexpr int B_STAGE_BYTES = 256 * BK * 2;  // sized for the widest tile (BN = 256)
constexpr int X_STAGE_BYTES = BM * 64 * 2;
constexpr int NUM_PRODUCER_WARPS = 8;
constexpr int PRODUCER_THREADS = NUM_PRODUCER_WARPS * 32;
constexpr int TMA_WARP = 8;
constexpr int MMA_WARP = 9;
constexpr int XTMA_WARP = 10;
constexpr int THREADS = 352;
constexpr uint32_t TMEM_COLS = 256;
constexpr long long WAIT_LIMIT_CYCLES = 2000000000LL;  // ~1 s at the B200 boost clock
constexpr int MAX_SPLITS = 4;                          // split-K cluster size

constexpr int OFF_A = 0;
constexpr int OFF_B = OFF_A + STAGES * A_STAGE_BYTES;
constexpr int OFF_X = OFF_B + BSTAGES * B_STAGE_BYTES;
constexpr int OFF_BAR = OFF_X + XSTAGES * X_STAGE_BYTES;
// full/empty per A stage, per B stage and per x stage; accum; LayerNorm x tile; reduction
constexpr int NUM_BARS = 2 * STAGES + 2 * BSTAGES + 2 * XSTAGES + 3;
constexpr int OFF_TMEM = OFF_BAR + NUM_BARS * 8;
constexpr int OFF_FLAG = OFF_TMEM + 4;
constexpr int OFF_EPI = OFF_FLAG + 4;
constexpr int OFF_RED = OFF_EPI + 4;                       // split-K: a reduction wait expired
constexpr int OFF_STATS = (OFF_RED + 4 + 15) / 16 * 16;    // LayerNorm partial sums / stats
constexpr int SMEM_BYTES = OFF_STATS + 4 * BM * 4;
constexpr int SMEM_ALLOC = SMEM_BYTES + 1024;  // slack to align the base to 1024 B
// Split-K reduction buffers, over the (finished) pipeline buffers: (splits - 1) receive slots and
// (splits - 1) staging slots of [128][slice + 4] fp32 (slice = BN / splits columns).
__host__ __device__ constexpr int red_bytes(int splits, int slice) {
  return 2 * (splits - 1) * BM * (slice + 4) * 4;
}
static_assert(red_bytes(4, 64) <= OFF_BAR && red_bytes(2, 128) <= OFF_BAR,
              "split-K reduction slots must fit in the stage buffers");
// Rounds of the reduction: the slice in 1, 2 or 4 column chunks so that the slots fit in `avail`
// bytes of stage buffers (narrow tiles always take one round).
__host__ __device__ constexpr int red_rounds(int splits, int slice, int avail) {
  return red_bytes(splits, slice) <= avail ? 1 : (red_bytes(splits, slice / 2) <= avail ? 2 : 4);
}
static_assert(red_rounds(2, 256, 208 * 1024) == 2, "wide split-K reduction in two rounds");
// LayerNorm input tile (rows of <= 256 features) staged over the A stages before the first block
static_assert(BM * 256 * 2 <= STAGES * A_STAGE_BYTES, "x tile must fit in the A stages");

// Shared-memory layout of one kernel variant.  WIDE (BN = 512): two N = 256 accumulators (all 512
// TMEM columns) take every basis block, so each block the producers build feeds twice the MMA
// work.  Its weights stream through a ring of four 32 KB slots, one 256-row half of a block's
// 64 KB panel each, released half by half as the MMAs of that half complete: the load of a half
// is issued 1.5 blocks of MMA time before it is needed (a ring of two whole-block stages gave one
// block, and the weight loads then stalled the tensor pipe for ~20 % of the step).  This leaves
// room for 3 A and 2 input stages, no split-K slots and no staged LayerNorm tile.
template <bool WIDE>
struct Layout {
  static constexpr int kStages = WIDE ? 3 : STAGES;
  static constexpr int kBStages = WIDE ? 4 : BSTAGES;  // WIDE: half-block slots
  static constexpr int kXStages = WIDE ? 2 : XSTAGES;
  static constexpr int kBStageBytes = B_STAGE_BYTES;
  static constexpr uint32_t kTmemCols = WIDE ? 512u : TMEM_COLS;
  static constexpr int kOffB = OFF_A + kStages * A_STAGE_BYTES;
  static constexpr int kOffX = kOffB + kBStages * kBStageBytes;
  static constexpr int kOffBar = kOffX + kXStages * X_STAGE_BYTES;
  static constexpr int kNumBars = 2 * kStages + 2 * kBStages + 2 * kXStages + 3;
  static constexpr int kOffTmem = kOffBar + kNumBars * 8;
  static constexpr int kOffFlag = kOffTmem + 4;
  static constexpr int kOffEpi = kOffFlag + 4;
  static constexpr int kOffRed = kOffEpi + 4;
  static constexpr int kOffStats = (kOffRed + 4 + 15) / 16 * 16;
  static constexpr int kSmemAlloc = kOffStats + 4 * BM * 4 + 1024;
};
static_assert(Layout<false>::kSmemAlloc == SMEM_ALLOC, "narrow layout unchanged");
static_assert(Layout<true>::kSmemAlloc <= 227 * 1024, "wide layout fits the shared memory");

// ---------------------------------------------------------------------------------------------
// PTX wrappers
// ---------------------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(bar),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
// try_wait with a suspend-time hint: the thread is suspended in hardware until the phase
// completes or about `ns` nanoseconds pass, so a waiter neither spins on the issue slots the
// working warps need nor wakes late.
__device__ __forceinline__ bool mbar_try_wait_hint(uint32_t bar, uint32_t parity, uint32_t ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity), "r"(ns)
      : "memory");
  return ok != 0;
}
// Non-blocking probe of the phase.
__device__ __forceinline__ bool mbar_test_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait for the phase of `parity`; false when `limit` SM cycles passed first.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity,
                                          long long limit = WAIT_LIMIT_CYCLES) {
  if (limit < 40000LL) {
    // a short limit (the abort-path tests): poll without suspending, so that the limit and not
    // the hardware's own suspend window of try_wait decides when the wait gives up
    const long long t0 = clock64();
    while (!mbar_test_wait(bar, parity))
      if (clock64() - t0 > limit) return false;
    return true;
  }
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  while (!mbar_try_wait_hint(bar, parity, 20000u))
    if (clock64() - t0 > limit) return false;
  return true;
}
// Warp-wide bounded wait: lane 0 polls, the outcome is broadcast, each lane then takes the
// completed phase with one (immediately successful) try_wait for its own acquire ordering, and
// the warp leaves reconverged -- per-lane polling would let the lanes leave the loop at different
// iterations and run the following code (shuffles, the A-tile producer) diverged.
__device__ __forceinline__ bool mbar_wait_warp(uint32_t bar, uint32_t parity,
                                               long long limit = WAIT_LIMIT_CYCLES) {
  uint32_t ok = 0;
  if ((threadIdx.x & 31) == 0) ok = mbar_wait(bar, parity, limit) ? 1u : 0u;
  ok = __shfl_sync(0xffffffffu, ok, 0);
  if (ok) (void)mbar_try_wait(bar, parity);
  __syncwarp();
  return ok != 0;
}
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void named_bar(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;"
               ::: "memory");
}
__device__ __forceinline__ uint32_t map_to_rank(uint32_t local_addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local_addr), "r"(rank));
  return r;
}
// Shared -> shared copy into another CTA of the cluster, completing on that CTA's mbarrier.
__device__ __forceinline__ void bulk_s2cluster(uint32_t dst_cluster, uint32_t src_cta,
                                               uint32_t bytes, uint32_t bar_cluster) {
  asm volatile(
      "cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, "
      "[%3];" ::"r"(dst_cluster),
      "r"(src_cta), "r"(bytes), "r"(bar_cluster)
      : "memory");
}
// Contiguous global -> shared copy by the bulk-copy engine, completing on an mbarrier.
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes,
                                         uint32_t bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(dst),
      "l"(src), "r"(bytes), "r"(bar)
      : "memory");
}
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, uint32_t bar,
                                            int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
      "l"((uint64_t)map), "r"(bar), "r"(x), "r"(y)
      : "memory");
}
__device__ __forceinline__ void tmem_alloc(uint32_t slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(slot),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void mma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                        uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void mma_commit(uint32_t bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
      : "memory");
}
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&f)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) f[i] = __uint_as_float(r[i]);
}

// Shared-memory matrix descriptor: K-major operand, 128-byte swizzle, 8-row core groups 1024 B
// apart (SBO), LBO unused for swizzled K-major (encoded 1), descriptor version 1 (sm_100).
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t addr) {
  return (uint64_t)((addr >> 4) & 0x3FFF) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}
// Instruction descriptor, kind::f16: D fp32, A/B f16 (0) or bf16 (1), both K-major, N>>3, M>>4.
__device__ __forceinline__ uint32_t instr_desc(int ab_fmt, int n, int m) {
  return (1u << 4) | ((uint32_t)ab_fmt << 7) | ((uint32_t)ab_fmt << 10) |
         ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

// Round two fp32 values (RNE) into one 32-bit pair of the operand dtype, low half first.
template <int MODE>
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  if (MODE == MODE_F16) {
    __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
  } else {
    __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
  }
}

// Swizzled address of 16-byte chunk `chunk` of row `r` inside an A stage.
__device__ __forceinline__ uint32_t a_chunk_off(int r, int chunk) {
  return (uint32_t)(r * 128 + ((chunk ^ (r & 7)) << 4));
}

// ---------------------------------------------------------------------------------------------
// LayerNorm statistics: the two owner threads of a row (one per producer group) each sum one half
// of the row -- shifted by the row's first value, so that the one-pass variance keeps its
// precision when |mean| >> std -- and combine through shared memory.
// ---------------------------------------------------------------------------------------------
template <int MODE>
__device__ __forceinline__ void ln_partial(const typename Act<MODE>::T* xrow, bool valid,
                                           int D_in, int half, float& s, float& ss,
                                           float& pivot) {
  using T = typename Act<MODE>::T;
  s = 0.f;
  ss = 0.f;
  pivot = valid ? Act<MODE>::to_f(xrow[0]) : 0.f;
  if (!valid) return;
  const int lo = half ? D_in / 2 : 0, hi = half ? D_in : D_in / 2;
  const bool vec = ((D_in & 15) == 0) && ((((uintptr_t)xrow) & 15) == 0);
  if (vec) {
    // 16-byte loads, 8 in flight
    for (int c = lo; c < hi; c += 64) {
      uint4 raw[8];
#pragma unroll
      for (int u = 0; u < 8; ++u)
        raw[u] = (c + 8 * u < hi) ? *reinterpret_cast<const uint4*>(xrow + c + 8 * u)
                                  : make_uint4(0, 0, 0, 0);
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        if (c + 8 * u >= hi) continue;
        const T* e = reinterpret_cast<const T*>(&raw[u]);
#pragma unroll
        for (int t = 0; t < 8; ++t) {
          const float d = Act<MODE>::to_f(e[t]) - pivot;
          s += d;
          ss = fmaf(d, d, ss);
        }
      }
    }
  } else {
    for (int c = lo; c < hi; ++c) {
      const float d = Act<MODE>::to_f(xrow[c]) - pivot;
      s += d;
      ss = fmaf(d, d, ss);
    }
  }
}

// Rows of at most 256 features (D_in % 8 == 0, 16-byte aligned) are staged into shared memory by
// one bulk copy (the CTA's rows are contiguous in X).  The two owner threads of a row (one per
// producer group) then each sum one half of it -- 16-byte chunks visited in a per-row rotated
// order so that the 32 rows of a warp spread over the banks -- and combine through shared memory;
// mean and variance are two exact passes (no shuffles).
__device__ __forceinline__ bool ln_smem_ok(const LayerArgs& a) {
  return a.D_in <= 256 && (a.D_in % 16) == 0 && ((((uintptr_t)a.X) & 15) == 0);
}

template <int MODE>
__device__ __forceinline__ float ln_half_pass(const uint8_t* xrow_s, int nchunk, int c0, int r,
                                              float mean, bool second) {
  using T = typename Act<MODE>::T;
  float acc0 = 0.f, acc1 = 0.f;
#pragma unroll 4
  for (int i = 0; i < nchunk; ++i) {
    const int c = c0 + (i + r) % nchunk;
    const uint4 raw = *reinterpret_cast<const uint4*>(xrow_s + c * 16);
    const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
    for (int t = 0; t < 8; t += 2) {
      const float x0 = Act<MODE>::to_f(e[t]), x1 = Act<MODE>::to_f(e[t + 1]);
      if (second) {
        acc0 = fmaf(x0 - mean, x0 - mean, acc0);
        acc1 = fmaf(x1 - mean, x1 - mean, acc1);
      } else {
        acc0 += x0;
        acc1 += x1;
      }
    }
  }
  return acc0 + acc1;
}

// Statistics of row r (its two owner threads call this; `part` is [2][BM] floats of scratch).
template <int MODE>
__device__ __forceinline__ void ln_row_stats(const LayerArgs& a, const uint8_t* xtile, int r,
                                             int grp, bool valid, float* part, float& mean,
                                             float& rstd) {
  const int nchunk = a.D_in / 16;  // 16-byte chunks per half row
  const uint8_t* xrow_s = xtile + (size_t)r * a.D_in * 2;
  const float inv_n = 1.0f / (float)a.D_in;
  float s = valid ? ln_half_pass<MODE>(xrow_s, nchunk, grp * nchunk, r, 0.f, false) : 0.f;
  part[grp * BM + r] = s;
  named_bar(1, PRODUCER_THREADS);
  mean = (part[r] + part[BM + r]) * inv_n;
  named_bar(1, PRODUCER_THREADS);
  float ss = valid ? ln_half_pass<MODE>(xrow_s, nchunk, grp * nchunk, r, mean, true) : 0.f;
  part[grp * BM + r] = ss;
  named_bar(1, PRODUCER_THREADS);
  rstd = rsqrtf((part[r] + part[BM + r]) * inv_n + a.ln_eps);
}

// ---------------------------------------------------------------------------------------------
// inputs of a block from the input tiles (64 features x 128 rows, 128-byte swizzled)
// ---------------------------------------------------------------------------------------------
// 16-bit element e of a uint4 array (e < 8 * N, compile-time after unrolling)
template <int N>
__device__ __forceinline__ uint32_t half_bits(const uint4 (&ch)[N], int e) {
  const uint4 c = ch[e >> 3];
  const uint32_t w = ((e & 7) >> 1) == 0 ? c.x : ((e & 7) >> 1) == 1 ? c.y : ((e & 7) >> 1) == 2 ? c.z : c.w;
  return (e & 1) ? (w >> 16) : (w & 0xFFFFu);
}

// Features lo .. lo + F - 1 of row r.  Inside one tile: the 16-byte chunks covering them (one
// 16-byte load each, conflict-free across the warp thanks to the swizzle), the features picked
// out in registers; a block that straddles two tiles reads its features one by one.
template <int MODE, int F, int XSTAGES>
__device__ __forceinline__ void read_x_block(const uint8_t* xring, int lo, int xs_first, int r,
                                             float (&xs)[F]) {
  using T = typename Act<MODE>::T;
  const int e0 = lo & 63;
  if (e0 + F <= 64) {
    constexpr int NCH = (F + 7 + 7) / 8;  // chunks covering any start offset 0..7
    const uint8_t* row = xring + ((lo / 64 - xs_first) % XSTAGES) * X_STAGE_BYTES + r * 128;
    const int c0 = e0 >> 3, o = e0 & 7;
    uint4 ch[NCH];
#pragma unroll
    for (int k = 0; k < NCH; ++k) {
      const int c = c0 + k;
      ch[k] = c < 8 ? *reinterpret_cast<const uint4*>(row + ((c ^ (r & 7)) << 4))
                    : make_uint4(0, 0, 0, 0);
    }
    switch (o) {
#define KAN_X_CASE(O)                                                                  \
  case O:                                                                              \
    _Pragma("unroll") for (int f = 0; f < F; ++f) {                                    \
      const uint16_t b = (uint16_t)half_bits<NCH>(ch, O + f);                          \
      xs[f] = Act<MODE>::to_f(*reinterpret_cast<const T*>(&b));                        \
    }                                                                                  \
    break;
      KAN_X_CASE(0) KAN_X_CASE(1) KAN_X_CASE(2) KAN_X_CASE(3)
      KAN_X_CASE(4) KAN_X_CASE(5) KAN_X_CASE(6) KAN_X_CASE(7)
#undef KAN_X_CASE
    }
  } else {
#pragma unroll
    for (int f = 0; f < F; ++f) {
      const int i = lo + f;
      const int u = i / 64 - xs_first, c = i & 63;
      const uint8_t* xt = xring + (u % XSTAGES) * X_STAGE_BYTES;
      xs[f] = Act<MODE>::to_f(*reinterpret_cast<const T*>(
          xt + r * 128 + ((((c >> 3) ^ (r & 7))) << 4) + (c & 7) * 2));
    }
  }
}

// ---------------------------------------------------------------------------------------------
// A-tile producers: one row of one 64-column block
// ---------------------------------------------------------------------------------------------

// Compile-time K: the F inputs of the next block are prefetched into registers while the current
// block is evaluated; all 64 values live in registers and are rounded once, when packed.
template <int BASIS, int MODE, int K, bool HB>
struct RowProducer {
  static constexpr bool kXFromTiles = true;  // reads its inputs from the TMA input tiles
  static constexpr int KT = K + (HB ? 1 : 0);
  static constexpr int F = 64 / KT;
  using T = typename Act<MODE>::T;
  float g[K];                // RBF centres
  __half2 gh2[(K + 1) / 2];  // fp16 mode: centres as half pairs
  __half2 neg_inv2;          // fp16 mode: -inv_den as halves
  float xn[F];               // prefetched raw inputs of the next block

  __device__ __forceinline__ void setup(const LayerArgs& a) {
    if (BASIS == KAN_RBF) {
#pragma unroll
      for (int k = 0; k < K; ++k) g[k] = __ldg(a.grid + k);
      if (MODE == MODE_F16) {
#pragma unroll
        for (int j = 0; j < (K + 1) / 2; ++j)
          gh2[j] = __floats2half2_rn(g[2 * j], 2 * j + 1 < K ? g[2 * j + 1] : 0.f);
        neg_inv2 = __float2half2_rn(-a.inv_den);
      }
    }
  }

  // Inputs of features blk*F .. blk*F+F-1 (0 for rows >= B or features >= D_in: their packed
  // weights are zero and every basis value of 0 is finite, so they contribute nothing).
  __device__ __forceinline__ void prefetch(const T* xrow, bool valid, int blk, int D_in) {
#pragma unroll
    for (int f = 0; f < F; ++f) {
      const int i = blk * F + f;
      xn[f] = (valid && i < D_in) ? Act<MODE>::to_f(xrow[i]) : 0.f;
    }
  }

  __device__ __forceinline__ void produce(uint8_t* a_stage, int r, const float (&xs)[F],
                                          int blk, const LayerArgs& a, float mean, float rstd) {
    float xm[F];
    if (a.input_map == KAN_MAP_LAYERNORM) {
#pragma unroll
      for (int f = 0; f < F; ++f) xm[f] = Act<MODE>::round((xs[f] - mean) * rstd);
    } else if (a.input_map == KAN_MAP_TANH) {
#pragma unroll
      for (int f = 0; f < F; ++f) xm[f] = Act<MODE>::round(tanhf(xs[f]));
    } else {
#pragma unroll
      for (int f = 0; f < F; ++f) xm[f] = xs[f];
    }
    if constexpr (BASIS == KAN_BSPLINE && K == 8) produce_bspline8(a_stage, r, xm, a);
    else produce_terms(a_stage, r, xm, blk, a);
  }

  // Every basis: the row's 64 terms in fp32 registers, rounded and packed in pairs.
  __device__ __forceinline__ void produce_terms(uint8_t* a_stage, int r, const float (&xm)[F],
                                                int blk, const LayerArgs& a) {
    float v[64];
#pragma unroll
    for (int f = 0; f < F; ++f) {
      float* vf = v + f * KT;
      if (BASIS == KAN_CHEBY) {
        // T_k(clamp(x)) by the fp32 recurrence; the stored value is rounded at pack time
        const float xc = fminf(fmaxf(xm[f], -1.0f), 1.0f);
        const float x2 = 2.0f * xc;
        float t0 = 1.0f, t1 = xc;
        vf[0] = 1.0f;
        if (K > 1) vf[1] = xc;
#pragma unroll
        for (int k = 2; k < K; ++k) {
          const float t2 = fmaf(x2, t1, -t0);
          vf[k] = t2;
          t0 = t1;
          t1 = t2;
        }
      } else if (BASIS == KAN_RBF) {
        if (MODE == MODE_F16) {
          // reference half arithmetic two centres at a time: diff = x - c and
          // (-diff*diff) * inv_den (computed as (diff*diff) * -inv_den: the same rounded value),
          // then exp of the half argument in fp32
          const __half2 xh2 = __float2half2_rn(xm[f]);
#pragma unroll
          for (int j = 0; j < (K + 1) / 2; ++j) {
            const __half2 diff = __hsub2(xh2, gh2[j]);
            const __half2 t = __hmul2(__hmul2(diff, diff), neg_inv2);
            const float2 tf = __half22float2(t);
            vf[2 * j] = __expf(tf.x);
            if (2 * j + 1 < K) vf[2 * j + 1] = __expf(tf.y);
          }
        } else {
#pragma unroll
          for (int k = 0; k < K; ++k) {
            const float d = xm[f] - g[k];
            vf[k] = __expf(-(d * d) * a.inv_den);
          }
        }
      } else if (BASIS == KAN_BSPLINE) {
        BsplineGen<MODE> gen;
        gen.init(xm[f], 0, a);
#pragma unroll
        for (int k = 0; k < K; ++k) {
          const int d = k - gen.span;
          float val = 0.f;
          val = (d == 0) ? gen.b0 : val;
          val = (d == 1) ? gen.b1 : val;
          val = (d == 2) ? gen.b2 : val;
          val = (d == 3) ? gen.b3 : val;
          vf[k] = val;
        }
      } else {
        WaveletGen<MODE> gen;
        gen.init(xm[f], min(blk * F + f, a.D_in - 1), a);
#pragma unroll
        for (int k = 0; k < K; ++k) vf[k] = gen.next();
      }
      if (HB) vf[K] = silu_value<MODE>(xm[f]);
    }
#pragma unroll
    for (int c = F * KT; c < 64; ++c) v[c] = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      uint4 pk;
      pk.x = pack2<MODE>(v[8 * j + 0], v[8 * j + 1]);
      pk.y = pack2<MODE>(v[8 * j + 2], v[8 * j + 3]);
      pk.z = pack2<MODE>(v[8 * j + 4], v[8 * j + 5]);
      pk.w = pack2<MODE>(v[8 * j + 6], v[8 * j + 7]);
      *reinterpret_cast<uint4*>(a_stage + a_chunk_off(r, j)) = pk;
    }
  }

  // Cubic B-splines, K = 8: only the four terms at the span are nonzero.  They are rounded to the
  // operand dtype and packed as four 16-bit halves (the same values the generic path stores), moved
  // to their span by one 64-bit shift -- the feature's eight terms as four 32-bit words -- and
  // merged into the row's 32 words at the feature's column (odd columns by a 16-bit funnel shift).
  // No per-term selects and no fp32 staging of the row.
  __device__ __forceinline__ void produce_bspline8(uint8_t* a_stage, int r, const float (&xm)[F],
                                                   const LayerArgs& a) {
    uint32_t w[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) w[i] = 0u;
#pragma unroll
    for (int f = 0; f < F; ++f) {
      const int p = f * KT;  // first column of the feature
      float t0, t1, t2, t3;
      int span;
      BsplineGen<MODE>::terms(xm[f], a, t0, t1, t2, t3, span);
      const unsigned long long v =
          ((unsigned long long)pack2<MODE>(t2, t3) << 32) | (unsigned long long)pack2<MODE>(t0, t1);
      const int sh = 16 * span;
      unsigned long long lo = 0ull, hi = 0ull;
      if (sh < 0) {
        lo = sh > -64 ? v >> (-sh) : 0ull;
      } else if (sh < 64) {
        lo = v << sh;
        hi = sh ? v >> (64 - sh) : 0ull;
      } else if (sh < 128) {
        hi = v << (sh - 64);
      }
      const uint32_t q0 = (uint32_t)lo, q1 = (uint32_t)(lo >> 32);
      const uint32_t q2 = (uint32_t)hi, q3 = (uint32_t)(hi >> 32);
      if ((p & 1) == 0) {
        w[p / 2] |= q0;
        w[p / 2 + 1] |= q1;
        w[p / 2 + 2] |= q2;
        w[p / 2 + 3] |= q3;
      } else {
        const int b = p / 2;
        w[b] |= q0 << 16;
        w[b + 1] |= __funnelshift_l(q0, q1, 16);
        w[b + 2] |= __funnelshift_l(q1, q2, 16);
        w[b + 3] |= __funnelshift_l(q2, q3, 16);
        w[b + 4] |= q3 >> 16;
      }
      if (HB) {
        const uint32_t hs = pack2<MODE>(silu_value<MODE>(xm[f]), 0.f) & 0xFFFFu;
        const int ps = p + K;
        w[ps / 2] |= (ps & 1) ? (hs << 16) : hs;
      }
    }
#pragma unroll
    for (int j = 0; j < 8; ++j)
      *reinterpret_cast<uint4*>(a_stage + a_chunk_off(r, j)) =
          make_uint4(w[4 * j], w[4 * j + 1], w[4 * j + 2], w[4 * j + 3]);
  }
};

// Runtime K (any K + has_base <= 64): zero the row, then 2-byte stores of the computed terms.
template <int BASIS, int MODE>
struct RowProducerAnyK {
  static constexpr bool kXFromTiles = false;  // loads its inputs from global memory itself
  static constexpr int F = 1;
  using T = typename Act<MODE>::T;
  float xn[1];  // unused: this producer loads its inputs itself
  const T* xrow_;
  bool valid_;
  __device__ __forceinline__ void setup(const LayerArgs&) {}
  __device__ __forceinline__ void prefetch(const T* xrow, bool valid, int, int) {
    xrow_ = xrow;
    valid_ = valid;
  }
  __device__ __forceinline__ void produce(uint8_t* a_stage, int r, const float (&)[F], int blk,
                                          const LayerArgs& a, float mean, float rstd) {
    using Gen = typename GenFor<BASIS, MODE>::type;
    const int KT = a.K + (a.has_base ? 1 : 0);
    const int Fr = 64 / KT;
#pragma unroll
    for (int j = 0; j < 8; ++j)
      *reinterpret_cast<uint4*>(a_stage + a_chunk_off(r, j)) = make_uint4(0, 0, 0, 0);
    for (int f = 0; f < Fr; ++f) {
      const int i = blk * Fr + f;
      if (!valid_ || i >= a.D_in) break;
      const float xm = map_input<MODE>(Act<MODE>::to_f(xrow_[i]), a.input_map, mean, rstd);
      Gen gen;
      gen.init(xm, i, a);
      for (int k = 0; k < KT; ++k) {
        const float val = (k < a.K) ? gen.next() : silu_value<MODE>(xm);
        const int c = f * KT + k;
        *reinterpret_cast<T*>(a_stage + a_chunk_off(r, c >> 3) + (c & 7) * 2) =
            Act<MODE>::from_f(val);
      }
    }
  }
};

// ---------------------------------------------------------------------------------------------
// the kernel
// ---------------------------------------------------------------------------------------------
template <int BASIS, int MODE, class Producer, bool WIDE>
__global__ void __launch_bounds__(THREADS, 1)
    kan_tc_kernel(const __grid_constant__ CUtensorMap tmap_w,
                  const __grid_constant__ CUtensorMap tmap_x, LayerArgs a, int BN, int nb_total,
                  int splits, int x_tma) {
  using T = typename Act<MODE>::T;
  // this variant's layout (the names shadow the narrow defaults)
  using LY = Layout<WIDE>;
  constexpr int STAGES = LY::kStages, BSTAGES = LY::kBStages, XSTAGES = LY::kXStages;
  constexpr int B_STAGE_BYTES = LY::kBStageBytes;
  constexpr uint32_t TMEM_COLS = LY::kTmemCols;
  constexpr int OFF_B = LY::kOffB, OFF_X = LY::kOffX, OFF_BAR = LY::kOffBar;
  constexpr int OFF_TMEM = LY::kOffTmem, OFF_FLAG = LY::kOffFlag, OFF_EPI = LY::kOffEpi;
  constexpr int OFF_RED = LY::kOffRed;
  constexpr int OFF_STATS = LY::kOffStats;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  const uint32_t s_base = smem_u32(smem);
  const uint32_t bar_full_a = s_base + OFF_BAR;
  const uint32_t bar_empty = bar_full_a + STAGES * 8;     // A stage consumed by the MMA
  const uint32_t bar_full_b = bar_empty + STAGES * 8;
  const uint32_t bar_empty_b = bar_full_b + BSTAGES * 8;  // B stage consumed by the MMA
  const uint32_t bar_full_x = bar_empty_b + BSTAGES * 8;
  const uint32_t bar_empty_x = bar_full_x + XSTAGES * 8;  // x stage released by every producer
  const uint32_t bar_accum = bar_empty_x + XSTAGES * 8;
  const uint32_t bar_x = bar_accum + 8;     // LayerNorm x tile landed
  const uint32_t bar_red = bar_x + 8;       // split-K slices from the other CTAs landed
  volatile uint32_t* tmem_slot = reinterpret_cast<volatile uint32_t*>(smem + OFF_TMEM);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + OFF_FLAG);
  volatile int* epi_flag = reinterpret_cast<volatile int*>(smem + OFF_EPI);
  volatile int* red_expired = reinterpret_cast<volatile int*>(smem + OFF_RED);
  float* s_stats = reinterpret_cast<float*>(smem + OFF_STATS);  // [4][BM]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // M tiles vary fastest in the grid: the CTAs resident at one time share a few weight panels
  // (read from HBM about once, then from L2) instead of every panel at once
  const int m0 = blockIdx.x * BM, n0 = blockIdx.y * BN;
  const int z = blockIdx.z;
  // this split's K blocks: [kb0, kb1)
  const int kb0 = (int)((long long)nb_total * z / splits);
  const int kb1 = (int)((long long)nb_total * (z + 1) / splits);
  const int nj = kb1 - kb0;
  const bool ln_staged = !WIDE && a.input_map == KAN_MAP_LAYERNORM && ln_smem_ok(a);
  const int rows_valid = min(BM, a.B - m0);
  const int slice = BN / splits;  // split-K: columns of the tile this CTA finishes
  // Pipeline waits (a stage filled or freed by another role) take the call's limit; waits for
  // copies or MMAs this CTA already has in flight (bar_x, the TMA drains, bar_accum, bar_red)
  // always take the full limit, so that nothing still targets this CTA's shared memory or TMEM
  // when it aborts and exits.
  const long long plim = a.wait_cycles > 0 ? a.wait_cycles : WAIT_LIMIT_CYCLES;

  // input stages of this split: 64-feature tiles covering features [F*kb0, F*kb1)
  const TcBlocking blocking = tc_blocking(a.D_in, a.K, a.has_base);
  const int xs_first = (blocking.F * kb0) / 64;
  const int xs_last = nj > 0 ? (blocking.F * kb1 - 1) / 64 : xs_first - 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(bar_full_a + 8 * s, NUM_PRODUCER_WARPS / 2);
      mbar_init(bar_empty + 8 * s, 1);
    }
    for (int s = 0; s < BSTAGES; ++s) {
      mbar_init(bar_full_b + 8 * s, 1);
      mbar_init(bar_empty_b + 8 * s, 1);
    }
    for (int s = 0; s < XSTAGES; ++s) {
      mbar_init(bar_full_x + 8 * s, 1);
      mbar_init(bar_empty_x + 8 * s, NUM_PRODUCER_WARPS);
    }
    mbar_init(bar_accum, 1);
    mbar_init(bar_x, 1);
    mbar_init(bar_red, 1);
    *abort_flag = 0;
    *epi_flag = 0;
    *red_expired = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    if (ln_staged) {
      // the CTA's input rows are one contiguous block of X
      const uint32_t bytes = (uint32_t)(rows_valid * a.D_in * 2);
      mbar_arrive_expect_tx(bar_x, bytes);
      bulk_g2s(s_base + OFF_A, (const T*)a.X + (size_t)m0 * a.D_in, bytes, bar_x);
    }
    // the other splits' slices arrive after the first cluster barrier, i.e. after this point
    if (splits > 1) {
      const int chunk0 = slice / red_rounds(splits, slice, OFF_BAR);
      mbar_arrive_expect_tx(bar_red, (uint32_t)((splits - 1) * BM * (chunk0 + 4) * 4));
    }
  }
  if (warp == MMA_WARP) tmem_alloc(s_base + OFF_TMEM, TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_d = *tmem_slot;
  bool producer_aborted = true;  // set by the epilogue threads (the producer warps)

  if (warp < NUM_PRODUCER_WARPS) {
    // ------------------------------------------------------------------ basis producers
    const int q = warp & 3, grp = warp >> 2;
    const int r = q * 32 + lane;
    const int row = m0 + r;
    const bool valid = row < a.B;
    const T* xrow = (const T*)a.X + (size_t)(valid ? row : 0) * a.D_in;

    Producer prod;
    prod.setup(a);
    if (!x_tma && grp < nj) prod.prefetch(xrow, valid, kb0 + grp, a.D_in);
    int xs_rel = xs_first;  // next input stage this warp has to release
    auto release_x_until = [&](int stage_end) {  // release stages < stage_end
      for (; xs_rel < stage_end && xs_rel <= xs_last; ++xs_rel) {
        __syncwarp();
        if (lane == 0) mbar_arrive(bar_empty_x + 8 * ((xs_rel - xs_first) % XSTAGES));
      }
    };

    float mean = 0.f, rstd = 1.f;
    if (ln_staged) {
      if (!mbar_wait_warp(bar_x, 0)) {
        raise_device_error(a.err, DEVERR_TIMEOUT_FULL_A);
        *abort_flag = 1;
      }
      ln_row_stats<MODE>(a, smem + OFF_A, r, grp, valid, s_stats, mean, rstd);
      // every thread is done with the x tile before the A stages are overwritten
      named_bar(1, PRODUCER_THREADS);
    } else if (a.input_map == KAN_MAP_LAYERNORM) {
      float s, ss, pv;
      ln_partial<MODE>(xrow, valid, a.D_in, grp, s, ss, pv);
      s_stats[grp * BM + r] = s;
      s_stats[(2 + grp) * BM + r] = ss;
      named_bar(1, PRODUCER_THREADS);
      const float st = s_stats[r] + s_stats[BM + r];
      const float sst = s_stats[2 * BM + r] + s_stats[3 * BM + r];
      const float md = st / (float)a.D_in;
      mean = pv + md;
      rstd = rsqrtf(fmaxf(sst / (float)a.D_in - md * md, 0.f) + a.ln_eps);
    }

    for (int j = grp; j < nj; j += 2) {
      const int s = j % STAGES;
      const uint32_t it = (uint32_t)(j / STAGES);
      float xs[Producer::F];
      if (x_tma) {
        // this block's inputs from the TMA-loaded input tiles (rows >= B and features >= D_in
        // read as zero)
        const int lo = (kb0 + j) * Producer::F;
        const int st_lo = lo / 64, st_hi = (lo + Producer::F - 1) / 64;
        release_x_until(st_lo);
        bool ok = true;
        for (int st = st_lo; st <= st_hi && ok; ++st) {
          const int u = st - xs_first;
          ok = mbar_wait_warp(bar_full_x + 8 * (u % XSTAGES), (uint32_t)(u / XSTAGES) & 1u,
                              plim);
        }
        if (!ok) {
          raise_device_error(a.err, DEVERR_TIMEOUT_FULL_A);
          *abort_flag = 1;
          break;
        }
        read_x_block<MODE, Producer::F, XSTAGES>(smem + OFF_X, lo, xs_first, r, xs);
      } else {
#pragma unroll
        for (int f = 0; f < Producer::F; ++f) xs[f] = prod.xn[f];
        if (j + 2 < nj) prod.prefetch(xrow, valid, kb0 + j + 2, a.D_in);
      }
      if (!mbar_wait_warp(bar_empty + 8 * s, (it & 1u) ^ 1u, plim)) {
        raise_device_error(a.err, DEVERR_TIMEOUT_EMPTY);
        *abort_flag = 1;
        break;
      }
      if (*abort_flag) break;
      prod.produce(smem + OFF_A + s * A_STAGE_BYTES, r, xs, kb0 + j, a, mean, rstd);
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar_full_a + 8 * s);
    }
    // After an abort the input stages this warp did not get to are not released: a load may
    // still be landing in them, and a release would let the input TMA warp reuse the slot with
    // the earlier load in flight.  That warp's own wait then expires and it drains its loads.
    const bool aborted_here = __shfl_sync(0xffffffffu, *abort_flag, 0) != 0;
    if (x_tma && !aborted_here) release_x_until(xs_last + 1);

    // ------------------------------------------------------------------ epilogue
    if (!mbar_wait_warp(bar_accum, 0)) {
      raise_device_error(a.err, DEVERR_TIMEOUT_ACCUM);
      *abort_flag = 1;
    }
    tc_fence_after();
    // all epilogue threads must agree on the abort decision before the barriers below
    named_bar(3, PRODUCER_THREADS);
    if (threadIdx.x == 0) *epi_flag = *abort_flag ? 1 : 0;
    named_bar(3, PRODUCER_THREADS);
    const bool aborted = (*epi_flag != 0) || nj <= 0;

    const int h = grp;  // column half of the tile
    const int HALF = BN >> 1;
    T* Y = (T*)a.Y;
    const T* bias = (const T*)a.bias;
    const bool vec_ok = (a.D_out % 8) == 0;
    auto store_chunk = [&](float (&out)[32], int col0) {
#pragma unroll
      for (int jj = 0; jj < 32; ++jj)
        out[jj] += (a.has_bias && col0 + jj < a.D_out) ? Act<MODE>::to_f(bias[col0 + jj]) : 0.f;
      T* yrow = Y + (size_t)row * a.D_out;
      if (vec_ok && col0 + 32 <= a.D_out) {
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) {
          uint4 pk;
          pk.x = pack2<MODE>(out[8 * jj + 0], out[8 * jj + 1]);
          pk.y = pack2<MODE>(out[8 * jj + 2], out[8 * jj + 3]);
          pk.z = pack2<MODE>(out[8 * jj + 4], out[8 * jj + 5]);
          pk.w = pack2<MODE>(out[8 * jj + 6], out[8 * jj + 7]);
          *reinterpret_cast<uint4*>(yrow + col0 + 8 * jj) = pk;
        }
      } else {
#pragma unroll
        for (int jj = 0; jj < 32; ++jj)
          if (col0 + jj < a.D_out) yrow[col0 + jj] = Act<MODE>::from_f(out[jj]);
      }
    };

    if (splits == 1 && a.fuse_swiglu) {
      // gate + up pair (wide tile, BN = 512): tile columns [0, 256) are gate rows, [256, 512) up
      // rows of the same 256 outputs; group h finishes outputs [128 h, 128 h + 128).  Each layer's output
      // is rounded to the act dtype (bias first), then silu(gate) * up with the SiLU argument
      // clamped to +-20, as a separate SwiGLU pass over the two stored outputs computes it.
      if (!aborted) {
        const int QUART = BN >> 2;
        T* Hout = (T*)a.Y;
        const T* bg = (const T*)a.bias;
        const T* bu = (const T*)a.bias2;
        const int hbase = n0 >> 1;  // first output column of this tile
        const bool hvec = (a.h_cols % 8) == 0;
#pragma unroll 1
        for (int cc = 0; cc < QUART; cc += 32) {
          const int oc = h * QUART + cc;
          uint32_t ag[32], au[32];
          tmem_ld32(tmem_d + ((uint32_t)(q * 32) << 16) + (uint32_t)oc, ag);
          tmem_ld32(tmem_d + ((uint32_t)(q * 32) << 16) + (uint32_t)(HALF + oc), au);
          const int col0 = hbase + oc;
          if (!valid || col0 >= a.h_cols) continue;
          float out[32];
#pragma unroll
          for (int jj = 0; jj < 32; ++jj) {
            const int col = col0 + jj;
            const bool in = col < a.h_cols;
            const float g = Act<MODE>::round(__uint_as_float(ag[jj]) +
                                             ((a.has_bias && in) ? Act<MODE>::to_f(bg[col]) : 0.f));
            const float u = Act<MODE>::round(__uint_as_float(au[jj]) +
                                             ((a.has_bias2 && in) ? Act<MODE>::to_f(bu[col]) : 0.f));
            const float sig = 1.0f / (1.0f + expf(-fminf(fmaxf(g, -20.0f), 20.0f)));
            out[jj] = (g * sig) * u;
          }
          T* hrow = Hout + (size_t)row * a.h_cols;
          if (hvec && col0 + 32 <= a.h_cols) {
#pragma unroll
            for (int jj = 0; jj < 4; ++jj) {
              uint4 pk;
              pk.x = pack2<MODE>(out[8 * jj + 0], out[8 * jj + 1]);
              pk.y = pack2<MODE>(out[8 * jj + 2], out[8 * jj + 3]);
              pk.z = pack2<MODE>(out[8 * jj + 4], out[8 * jj + 5]);
              pk.w = pack2<MODE>(out[8 * jj + 6], out[8 * jj + 7]);
              *reinterpret_cast<uint4*>(hrow + col0 + 8 * jj) = pk;
            }
          } else {
#pragma unroll
            for (int jj = 0; jj < 32; ++jj)
              if (col0 + jj < a.h_cols) hrow[col0 + jj] = Act<MODE>::from_f(out[jj]);
          }
        }
      }
    } else if (splits == 1) {
      if (!aborted) {
#pragma unroll 1
        for (int cc = 0; cc < HALF; cc += 32) {
          uint32_t acc[32];
          const int ct = h * HALF + cc;
          tmem_ld32(tmem_d + ((uint32_t)(q * 32) << 16) + (uint32_t)ct, acc);
          const int col0 = n0 + ct;
          if (!valid || col0 >= a.D_out) continue;
          float out[32];
#pragma unroll
          for (int jj = 0; jj < 32; ++jj) out[jj] = __uint_as_float(acc[jj]);
          store_chunk(out, col0);
        }
      }
    }
    producer_aborted = aborted;
  } else if (warp == TMA_WARP) {
    // ------------------------------------------------------------------ weight TMA
    if (lane == 0) {
      // a wide tile's block is two slots (weight rows 0..255, 256..511: one box each)
      constexpr int H = WIDE ? 2 : 1;
      const uint32_t bytes = (uint32_t)(WIDE ? 256 : BN) * BK * 2;
      int issued = 0;
      for (int t = 0; t < nj * H; ++t) {
        const int j = t / H, h = t % H;
        const int s = t % BSTAGES;
        const uint32_t it = (uint32_t)(t / BSTAGES);
        if (!mbar_wait(bar_empty_b + 8 * s, (it & 1u) ^ 1u, plim)) {
          raise_device_error(a.err, DEVERR_TIMEOUT_EMPTY);
          *abort_flag = 1;
          break;
        }
        if (*abort_flag) break;
        mbar_arrive_expect_tx(bar_full_b + 8 * s, bytes);
        tma_load_2d(s_base + OFF_B + s * B_STAGE_BYTES, &tmap_w, bar_full_b + 8 * s,
                    (kb0 + j) * BK, n0 + 256 * h);
        ++issued;
      }
      // drain: wait (bounded) for the copies still landing in shared memory
      for (int j = issued - 1; j >= 0 && j >= issued - BSTAGES; --j)
        (void)mbar_wait(bar_full_b + 8 * (j % BSTAGES), (uint32_t)(j / BSTAGES) & 1u);
    }
    __syncwarp();
  } else if (warp == MMA_WARP) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc = instr_desc(MODE == MODE_BF16 ? 1 : 0, WIDE ? 256 : BN, BM);
      constexpr int H = WIDE ? 2 : 1;  // weight slots (accumulator halves) per block
      bool stop = false;
      for (int j = 0; j < nj && !stop; ++j) {
        const int s = j % STAGES;
        const uint32_t par = (uint32_t)(j / STAGES) & 1u;
        if (!mbar_wait(bar_full_a + 8 * s, par, plim)) {
          raise_device_error(a.err, DEVERR_TIMEOUT_FULL_A);
          *abort_flag = 1;
          break;
        }
        const uint32_t a_addr = s_base + OFF_A + s * A_STAGE_BYTES;
#pragma unroll
        for (int h = 0; h < H; ++h) {
          const int t = j * H + h, sb = t % BSTAGES;
          if (!mbar_wait(bar_full_b + 8 * sb, (uint32_t)(t / BSTAGES) & 1u, plim)) {
            raise_device_error(a.err, DEVERR_TIMEOUT_FULL_B);
            *abort_flag = 1;
          }
          if (*abort_flag) {
            stop = true;
            break;
          }
          tc_fence_after();
          const uint32_t b_addr = s_base + OFF_B + sb * B_STAGE_BYTES;
          // wide tile: half h takes weight rows / accumulator columns 256 h .. 256 h + 255
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk)
            mma_f16(tmem_d + 256u * (uint32_t)h, smem_desc_sw128(a_addr + kk * 32),
                    smem_desc_sw128(b_addr + kk * 32), idesc, (j > 0 || kk > 0) ? 1u : 0u);
          mma_commit(bar_empty_b + 8 * sb);  // this half's weight slot is free once it is read
        }
        if (stop) break;
        mma_commit(bar_empty + 8 * s);
      }
      // signal the epilogue (also on abort, so that it does not wait out its own limit)
      mma_commit(bar_accum);
    }
    __syncwarp();
  } else if (warp == XTMA_WARP) {
    // ------------------------------------------------------------------ input tile TMA
    if (lane == 0 && x_tma) {
      int issued = 0;
      for (int st = xs_first; st <= xs_last; ++st) {
        const int u = st - xs_first, slot = u % XSTAGES;
        if (!mbar_wait(bar_empty_x + 8 * slot, ((uint32_t)(u / XSTAGES) & 1u) ^ 1u, plim)) {
          raise_device_error(a.err, DEVERR_TIMEOUT_EMPTY);
          *abort_flag = 1;
          break;
        }
        if (*abort_flag) break;
        mbar_arrive_expect_tx(bar_full_x + 8 * slot, (uint32_t)X_STAGE_BYTES);
        tma_load_2d(s_base + OFF_X + slot * X_STAGE_BYTES, &tmap_x, bar_full_x + 8 * slot,
                    st * 64, m0);
        ++issued;
      }
      for (int u = issued - 1; u >= 0 && u >= issued - XSTAGES; --u)
        (void)mbar_wait(bar_full_x + 8 * (u % XSTAGES), (uint32_t)(u / XSTAGES) & 1u);
    }
    __syncwarp();
  }

  if (splits > 1) {
    // Split-K reduction.  Slot k of a CTA's receive area [0, (S-1) slots) holds the slice sent by
    // the k-th other split; its staging area (the next S-1 slots) holds the slices it sends.
    // When the slots of whole slices do not fit (wide tiles), the slice goes in `rounds` column
    // chunks, each staged, copied, summed and stored before the next reuses the slots.
    const int rounds = red_rounds(splits, slice, OFF_BAR);
    const int chunk = slice / rounds;
    const int pitch = chunk + 4;  // slot row pitch in floats
    const int slot_bytes = BM * pitch * 4;
    auto other = [&](int zz, int self) { return zz < self ? zz : zz - 1; };
    const int half = chunk >> 1;  // chunk columns per producer warp (host: chunk % 32 == 0)
    bool ok = !producer_aborted && nj > 0;
    for (int rd = 0; rd < rounds; ++rd) {
    const int c0 = rd * chunk;  // first slice column of this round
    // A reduction wait that expired (a slice did not land within the limit) leaves bar_red's
    // phase incomplete: it is then neither re-armed nor waited on again, and this CTA stops
    // staging and summing; it still sends its copies (their contents then meaningless, the error
    // word set) and joins every cluster barrier, so that the other CTAs of the cluster complete
    // their rounds.  The flag is read after the cluster barrier that ends the previous round.
    // This wait always has the full limit: it waits for copies already in flight.
    const bool red_live = *red_expired == 0;
    if (!red_live) ok = false;
    if (rd > 0 && threadIdx.x == 0 && red_live)
      mbar_arrive_expect_tx(bar_red, (uint32_t)((splits - 1) * slot_bytes));
    if (warp < NUM_PRODUCER_WARPS) {
      // 1. stage this CTA's slices of the other splits' columns (TMEM -> shared)
      const int q = warp & 3, h = warp >> 2;
      const int r = q * 32 + lane;
      const uint32_t taddr0 = tmem_d + ((uint32_t)(q * 32) << 16);
      if (ok) {
        for (int zz = 0; zz < splits; ++zz) {
          if (zz == z) continue;
          float* stage = reinterpret_cast<float*>(smem + OFF_A + (splits - 1 + other(zz, z)) *
                                                                   slot_bytes) + r * pitch;
#pragma unroll 1
          for (int cc = 0; cc < half; cc += 16) {
            const int cs = h * half + cc;  // column within the slice
            float v[16];
            tmem_ld16(taddr0 + (uint32_t)(zz * slice + c0 + cs), v);
#pragma unroll
            for (int u = 0; u < 4; ++u)
              *reinterpret_cast<float4*>(stage + cs + 4 * u) =
                  make_float4(v[4 * u], v[4 * u + 1], v[4 * u + 2], v[4 * u + 3]);
          }
        }
      }
      fence_proxy_async_smem();  // the staged slices are read by the bulk-copy engine
    }
    __syncwarp();
    // every CTA has finished its main loop (its receive area is free) and staged its slices
    cluster_sync_all();
    // 2. one bulk copy per other split: staging slot -> that CTA's receive slot for this split.
    //    Sent even after an abort (the data is then meaningless, the error word is set), so that
    //    every receiver's phase of bar_red completes before it is armed for the next round.
    if (threadIdx.x == 0) {
      for (int zz = 0; zz < splits; ++zz) {
        if (zz == z) continue;
        bulk_s2cluster(map_to_rank(s_base + OFF_A + other(z, zz) * slot_bytes, (uint32_t)zz),
                       s_base + OFF_A + (splits - 1 + other(zz, z)) * slot_bytes,
                       (uint32_t)slot_bytes, map_to_rank(bar_red, (uint32_t)zz));
      }
    }
    if (warp < NUM_PRODUCER_WARPS) {
      const int q = warp & 3, h = warp >> 2;
      const int r = q * 32 + lane;
      const int row = m0 + r;
      const uint32_t taddr0 = tmem_d + ((uint32_t)(q * 32) << 16);
      // 3. the other splits' slices of this CTA's own columns have landed (always waited for:
      //    no copy may still target this CTA's shared memory when it exits)
      if (red_live && !mbar_wait_warp(bar_red, (uint32_t)rd & 1u)) {
        raise_device_error(a.err, DEVERR_TIMEOUT_ACCUM);
        *red_expired = 1;
        ok = false;
      }
      // 4. sum in split order (deterministic), bias, store 16 outputs at a time
      if (ok) {
        T* Y = (T*)a.Y;
        const T* bias = (const T*)a.bias;
        const bool vec = (a.D_out % 8) == 0;
        const float* recv = reinterpret_cast<const float*>(smem + OFF_A);
#pragma unroll 1
        for (int cc = 0; cc < half; cc += 16) {
          const int cs = h * half + cc;
          float own[16];
          tmem_ld16(taddr0 + (uint32_t)(z * slice + c0 + cs), own);  // warp-collective
          float sum[16];
#pragma unroll
          for (int t = 0; t < 16; ++t) sum[t] = 0.f;
          for (int zz = 0; zz < splits; ++zz) {
            if (zz == z) {
#pragma unroll
              for (int t = 0; t < 16; ++t) sum[t] += own[t];
            } else {
              const float4* src = reinterpret_cast<const float4*>(
                  recv + (other(zz, z) * BM + r) * pitch + cs);
#pragma unroll
              for (int u = 0; u < 4; ++u) {
                const float4 p = src[u];
                sum[4 * u] += p.x;
                sum[4 * u + 1] += p.y;
                sum[4 * u + 2] += p.z;
                sum[4 * u + 3] += p.w;
              }
            }
          }
          const int col0 = n0 + z * slice + c0 + cs;
          if (row >= a.B || col0 >= a.D_out) continue;
          if (vec && col0 + 16 <= a.D_out) {
            if (a.has_bias) {
              const uint4 b0 = *reinterpret_cast<const uint4*>(bias + col0);
              const uint4 b1 = *reinterpret_cast<const uint4*>(bias + col0 + 8);
              const T* bb0 = reinterpret_cast<const T*>(&b0);
              const T* bb1 = reinterpret_cast<const T*>(&b1);
#pragma unroll
              for (int t = 0; t < 8; ++t) {
                sum[t] += Act<MODE>::to_f(bb0[t]);
                sum[8 + t] += Act<MODE>::to_f(bb1[t]);
              }
            }
            uint4 o0, o1;
            o0.x = pack2<MODE>(sum[0], sum[1]);
            o0.y = pack2<MODE>(sum[2], sum[3]);
            o0.z = pack2<MODE>(sum[4], sum[5]);
            o0.w = pack2<MODE>(sum[6], sum[7]);
            o1.x = pack2<MODE>(sum[8], sum[9]);
            o1.y = pack2<MODE>(sum[10], sum[11]);
            o1.z = pack2<MODE>(sum[12], sum[13]);
            o1.w = pack2<MODE>(sum[14], sum[15]);
            uint4* dst = reinterpret_cast<uint4*>(Y + (size_t)row * a.D_out + col0);
            dst[0] = o0;
            dst[1] = o1;
          } else {
#pragma unroll
            for (int t = 0; t < 16; ++t) {
              const int col = col0 + t;
              if (col < a.D_out) {
                const float b = a.has_bias ? Act<MODE>::to_f(bias[col]) : 0.f;
                Y[(size_t)row * a.D_out + col] = Act<MODE>::from_f(sum[t] + b);
              }
            }
          }
        }
      }
    }
    // every copy out of this CTA's staging slots has landed (its receiver waited for it), so
    // the next round may overwrite them, or the CTA may exit
    __syncwarp();
    cluster_sync_all();
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == MMA_WARP) {
    tc_fence_after();
    tmem_dealloc(tmem_d, TMEM_COLS);
  }
}

template <int BASIS, int MODE, class Producer, bool WIDE>
static cudaError_t launch_kernel(const CUtensorMap& tw, const CUtensorMap& tx, int x_tma,
                                 const LayerArgs& a, int BN, int nb, int splits, dim3 grid,
                                 cudaStream_t s) {
  auto kern = kan_tc_kernel<BASIS, MODE, Producer, WIDE>;
  constexpr int smem = Layout<WIDE>::kSmemAlloc;
  static std::atomic<unsigned long long> configured{0};  // per device, one per template instance
  cudaError_t e = ensure_smem_attr(kern, smem, configured);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(THREADS, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = (unsigned)splits;
  cfg.attrs = attr;
  cfg.numAttrs = splits > 1 ? 1 : 0;
  const int use_x = (x_tma && Producer::kXFromTiles) ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, tw, tx, a, BN, nb, splits, use_x);
}

// BN = 512 runs the wide variant (K split at most in two: its reduction slots fit in two rounds)
template <int BASIS, int MODE, class Producer>
static cudaError_t launch_bn(const CUtensorMap& tw, const CUtensorMap& tx, int x_tma,
                             const LayerArgs& a, int BN, int nb, int splits, dim3 grid,
                             cudaStream_t s) {
  if (BN == 512) {
    if (splits > 2) return cudaErrorInvalidValue;
    return launch_kernel<BASIS, MODE, Producer, true>(tw, tx, x_tma, a, BN, nb, splits, grid, s);
  }
  return launch_kernel<BASIS, MODE, Producer, false>(tw, tx, x_tma, a, BN, nb, splits, grid, s);
}

// Compile-time-K producers for the shapes the BASELINE configs and common layers use; any other
// K runs the runtime-K producer.
template <int BASIS, int MODE>
static cudaError_t dispatch_k(const CUtensorMap& tw, const CUtensorMap& tx, int x_tma,
                              const LayerArgs& a, int BN, int nb, int splits, dim3 grid,
                              cudaStream_t s) {
#define KAN_TC_CASE(KK, HBV)                                                              \
  if (a.K == KK && (a.has_base != 0) == HBV)                                              \
    return launch_bn<BASIS, MODE, RowProducer<BASIS, MODE, KK, HBV>>(tw, tx, x_tma, a, BN, nb,  \
                                                                     splits, grid, s);
  if (BASIS == KAN_CHEBY) {
    KAN_TC_CASE(4, true) KAN_TC_CASE(4, false) KAN_TC_CASE(5, true) KAN_TC_CASE(5, false)
    KAN_TC_CASE(8, true) KAN_TC_CASE(8, false) KAN_TC_CASE(9, true) KAN_TC_CASE(9, false)
  } else if (BASIS == KAN_RBF) {
    KAN_TC_CASE(8, true) KAN_TC_CASE(8, false)
  } else if (BASIS == KAN_BSPLINE) {
    KAN_TC_CASE(8, true) KAN_TC_CASE(8, false)
  } else if (BASIS == KAN_WAVELET) {
    KAN_TC_CASE(6, true) KAN_TC_CASE(6, false) KAN_TC_CASE(8, true) KAN_TC_CASE(8, false)
  }
#undef KAN_TC_CASE
  return launch_bn<BASIS, MODE, RowProducerAnyK<BASIS, MODE>>(tw, tx, x_tma, a, BN, nb, splits,
                                                               grid, s);
}

}  // namespace tc
}  // namespace kan
