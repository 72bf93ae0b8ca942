// kan_gemv_i8.cuh -- small-batch path (5 <= B <= 16) for ternary weights on the tensor cores in
// 8-bit integers.
//
// At B = 5..16 a CUDA-core dot product costs too many dp4a per weight, and 16-bit operands cost
// the decoders two bytes of TMEM traffic and a lookup table per weight.  Here the ternary codes
// become signed bytes (-1, 0, +1: the reference's dequantiser without the scale) and the basis
// the fixed-point hi / lo bytes of the CUDA-core small-batch path (v = 128 hi + lo, v =
// rint(phi * 2^13), kan_gemv_cc.cuh), so that tcgen05.mma.kind::i8 computes exact integer sums;
// the group's scale is applied afterwards, per group and row, in fp32.
//
//   swap-AB: the weights are the MMA's A operand (M = 128 output rows per CTA) and the basis its
//   B operand, N = 2 * NP (NP = 8 or 16 padded batch rows: NP hi rows, then NP lo rows).
//
//   warp 0      TMA: per task (128 rows x one window of 512 codes), the 128-byte code rows
//               (128-byte swizzle), the window's scales, the four [2 NP x 128] basis tiles
//               (128-byte swizzle) and, in the base segment, the chunk exponents.
//   warps 1, 2  MMA issuers, taking alternate quantisation groups: per 64-code unit two
//               tcgen05.mma.cta_group::1.kind::i8 (K = 32) with A from TMEM, into the group's own
//               accumulator slot (int32, N columns), committed to the epilogue when the group is
//               complete.  In the base segment the basis changes exponent every 64 features, so
//               there every 64-code unit is a group of its own (sharing its 128-code group's scale).
//   warps 3-10  decoders (two per TMEM lane quarter, taking alternate units): a thread owns an
//               output row; per unit one 16-byte shared load of 64 codes, a byte-permute table per
//               16 codes, one tcgen05.st of 16 columns into the A ring.
//   warps 11-18 epilogue (two per lane quarter, each half of the batch rows): per group one
//               tcgen05.ld of its hi and lo columns, the exact total 128 H + L converted once and
//               multiplied by the group's scale (rounded to the operand dtype: the reference's
//               dequantised weight exactly) and the basis's 2^-E, accumulated per row in fp32.
//
// Work: the (row block, window) tasks, row-block major, are cut into one contiguous range per CTA
// (grid = SMs); a row block's partial sums from several CTAs are added by the last contributor in
// contributor order (deterministic), with the per-row-block counters of the lanes-along-K kernel
// (kan_gemv_kl.cuh).  The basis matrix comes from the CUDA-core path's pre-pass (table byte order,
// cc_phi_kernel), launched as this kernel's programmatic dependency.
//
// Every wait is bounded; on expiry a role records the device error word and stops; the TMA warp
// waits (full limit) for the loads it issued, each MMA issuer for its last MMAs, and TMEM is freed
// after every role is done.
#pragma once

#include <cuda.h>

#include "kan_gemv_kl.cuh"

namespace kan {
namespace i8 {

using tc::mbar_arrive;
using tc::mbar_arrive_expect_tx;
using tc::mbar_init;
using tc::mbar_wait;
using tc::mbar_wait_warp;
using tc::mma_commit;
using tc::named_bar;
using tc::smem_desc_sw128;
using tc::smem_u32;
using tc::tc_fence_after;
using tc::tc_fence_before;
using tc::tma_load_2d;

constexpr int ROWS = 128;                 // output rows per CTA (the MMA's M)
constexpr int UNIT = 64;                  // codes of one decoder step (two MMAs of K = 32)
constexpr int STAGE_UNITS = 8;            // one window: 512 codes, 128 code bytes per row
constexpr int WIN_CODES = UNIT * STAGE_UNITS;
constexpr int CODE_TILE = ROWS * 128;     // 16 KB
constexpr int STAGES = 4;
constexpr int ASLOTS = 8;                 // TMEM A ring, in units
constexpr int A_COLS = UNIT / 4;          // TMEM columns of one unit (4 bytes per column)
constexpr int ACC_SLOTS = 8;              // per-group accumulators in TMEM
constexpr int ACC_COL = ASLOTS * A_COLS;  // accumulators follow the A ring
constexpr uint32_t TMEM_COLS = 512;
constexpr int WARP_TMA = 0, WARP_MMA0 = 1, NISS = 2, WARP_DEC0 = 3, NDEC = 8,
              WARP_EPI0 = WARP_DEC0 + NDEC, NEPI = 8;
constexpr int THREADS = (WARP_EPI0 + NEPI) * 32;  // 608
constexpr int EPI_THREADS = NEPI * 32;
constexpr int BAR_EPI = 1;                // named barrier of the epilogue warps
constexpr int PHI_E = cc::PHI_E;
static_assert(ACC_COL + ACC_SLOTS * 32 <= (int)TMEM_COLS, "TMEM budget at NP = 16");

struct Params {
  int W, Ww;                 // windows per row: all, basis segment
  int gpu;                   // units per quantisation group (1: 64 codes, 2: 128 codes)
  int sfl;                   // scale floats per row and window (512 / group size)
  int units_w, units_b;      // 16-code units per row of the basis matrix, per segment
  int stage_bytes, off_phi, off_scale, off_p2b;  // one stage and its parts
  int off_bar, smem;
  int rowblocks;
  long long tasks;
  int G;                     // CTAs
  int maxc;                  // most contributors of one row block
  unsigned epoch;
  const float* p2b;          // [B][units_b]: 2^-E of each base unit (pre-pass)
  float* part;               // [rowblocks][maxc][NP][ROWS]
  unsigned long long* counters;  // [rowblocks]
};

__device__ __forceinline__ uint32_t idesc_i8(int n, int m) {
  // D s32 (2), A and B signed 8-bit (1), both K-major, N >> 3, M >> 4
  return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) |
         ((uint32_t)(m >> 4) << 24);
}

// D[tmem] (+)= A[tmem] * B[smem]^T, 8-bit integers, int32 accumulate
__device__ __forceinline__ void mma_i8_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc,
                                          uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], [%1], %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15])
      : "memory");
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// NC (4 or 8) consecutive 32-bit TMEM columns of this warp's lane quarter (no wait).
template <int NC>
__device__ __forceinline__ void tmem_ld_cols(uint32_t taddr, uint32_t (&r)[NC]) {
  if constexpr (NC == 8) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7])
        : "r"(taddr));
  } else {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(taddr));
  }
}

__device__ __forceinline__ bool warp_aborted(volatile int* flag) {
  return __shfl_sync(0xffffffffu, *flag, 0) != 0;
}

template <int MODE, int NP>
__global__ void __launch_bounds__(THREADS, 1)
    kan_gemv_i8_kernel(const __grid_constant__ CUtensorMap tm_cw,
                       const __grid_constant__ CUtensorMap tm_sw,
                       const __grid_constant__ CUtensorMap tm_cb,
                       const __grid_constant__ CUtensorMap tm_sb,
                       const __grid_constant__ CUtensorMap tm_hi,
                       const __grid_constant__ CUtensorMap tm_lo,
                       const __grid_constant__ LayerArgs a, const __grid_constant__ Params p) {
  using A = Act<MODE>;
  using T = typename A::T;
  constexpr int N = 2 * NP;        // MMA N: NP hi rows, then NP lo rows of the basis
  constexpr int BTILE = N * 128;   // one 128-code basis tile
  constexpr int HN = NP / 2;       // batch rows per epilogue warp
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  const uint32_t s_base = smem_u32(smem);
  const uint32_t bar_full = s_base + p.off_bar;           // [STAGES] task's tiles landed
  const uint32_t bar_empty = bar_full + 8 * STAGES;       // [STAGES] every role done with them
  const uint32_t bar_afull = bar_empty + 8 * STAGES;      // [ASLOTS] unit decoded into TMEM
  const uint32_t bar_aempty = bar_afull + 8 * ASLOTS;     // [ASLOTS] unit's MMAs complete
  const uint32_t bar_cfull = bar_aempty + 8 * ASLOTS;     // [ACC_SLOTS] group's sums complete
  const uint32_t bar_cempty = bar_cfull + 8 * ACC_SLOTS;  // [ACC_SLOTS] group's sums read
  const uint32_t bar_done = bar_cempty + 8 * ACC_SLOTS;   // [NISS] an issuer's last MMAs
  constexpr int NBARS = 2 * STAGES + 2 * ASLOTS + 2 * ACC_SLOTS + NISS;
  volatile uint32_t* tmem_slot = reinterpret_cast<volatile uint32_t*>(smem + p.off_bar + NBARS * 8);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + p.off_bar + NBARS * 8 + 4);
  volatile int* decision = abort_flag + 1;
  const long long plim = a.wait_cycles > 0 ? a.wait_cycles : tc::WAIT_LIMIT_CYCLES;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long t0 = p.tasks * blockIdx.x / p.G;
  const long long t1 = p.tasks * (blockIdx.x + 1) / p.G;
  const int ntask = (int)(t1 - t0);
  if (ntask <= 0) return;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(bar_full + 8 * s, 1);
      mbar_init(bar_empty + 8 * s, NDEC + NEPI + NISS);
    }
    for (int s = 0; s < ASLOTS; ++s) {
      mbar_init(bar_afull + 8 * s, 4);  // the unit's four decoder warps (one per lane quarter)
      mbar_init(bar_aempty + 8 * s, 1);
    }
    for (int s = 0; s < ACC_SLOTS; ++s) {
      mbar_init(bar_cfull + 8 * s, 1);
      mbar_init(bar_cempty + 8 * s, NEPI);
    }
    for (int e = 0; e < NISS; ++e) mbar_init(bar_done + 8 * e, 1);
    *abort_flag = 0;
    *decision = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == WARP_MMA0) tc::tmem_alloc(s_base + p.off_bar + NBARS * 8, TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == WARP_TMA) {
    // ------------------------------------------------------------------ TMA
    if (lane == 0) {
      auto task_bytes = [&](bool seg) {
        return (uint32_t)(CODE_TILE + 4 * BTILE + ROWS * p.sfl * 4 + (seg ? a.B * 128 : 0));
      };
      // the basis tiles (and base exponents) of task i: written by the pre-pass this launch
      // depends on, so requested only after griddepcontrol.wait
      auto issue_basis = [&](int i) {
        const int s = i % STAGES;
        const long long t = t0 + i;
        const int w = (int)(t % p.W);
        const bool seg = w >= p.Ww;
        const int col = seg ? p.units_w * 16 + (w - p.Ww) * WIN_CODES : w * WIN_CODES;
        const uint32_t st = s_base + s * p.stage_bytes;
#pragma unroll
        for (int b = 0; b < 4; ++b) {
          tma_load_2d(st + p.off_phi + b * BTILE, &tm_hi, bar_full + 8 * s, col + 128 * b, 0);
          tma_load_2d(st + p.off_phi + b * BTILE + NP * 128, &tm_lo, bar_full + 8 * s,
                      col + 128 * b, 0);
        }
        if (seg)
          for (int n = 0; n < a.B; ++n)
            tc::bulk_g2s(st + p.off_p2b + n * 128,
                         p.p2b + (size_t)n * p.units_b + (size_t)(w - p.Ww) * (WIN_CODES / 16),
                         128u, bar_full + 8 * s);
      };
      const int first = ntask < STAGES ? ntask : STAGES;
      int issued = 0, basis_issued = 0;
      for (int i = 0; i < ntask; ++i) {
        const int s = i % STAGES;
        if (!mbar_wait(bar_empty + 8 * s, ((uint32_t)(i / STAGES) & 1u) ^ 1u, plim)) {
          raise_device_error(a.err, DEVERR_TIMEOUT_EMPTY);
          *abort_flag = 1;
          break;
        }
        if (*abort_flag) break;
        const long long t = t0 + i;
        const int w = (int)(t % p.W), rb = (int)(t / p.W);
        const bool seg = w >= p.Ww;
        const int wl = seg ? w - p.Ww : w;
        const uint32_t st = s_base + s * p.stage_bytes;
        mbar_arrive_expect_tx(bar_full + 8 * s, task_bytes(seg));
        tma_load_2d(st, seg ? &tm_cb : &tm_cw, bar_full + 8 * s, wl * 128, rb * ROWS);
        tma_load_2d(st + p.off_scale, seg ? &tm_sb : &tm_sw, bar_full + 8 * s, wl * p.sfl,
                    rb * ROWS);
        ++issued;
        if (i + 1 == first) {
          asm volatile("griddepcontrol.wait;" ::: "memory");
          for (; basis_issued <= i; ++basis_issued) issue_basis(basis_issued);
        } else if (i >= first) {
          issue_basis(i);
          basis_issued = i + 1;
        }
      }
      // a task whose basis was deferred still gets it, so that every issued stage completes
      if (basis_issued < issued) {
        asm volatile("griddepcontrol.wait;" ::: "memory");
        for (; basis_issued < issued; ++basis_issued) issue_basis(basis_issued);
      }
      // every load issued lands before the CTA may exit
      for (int i = issued - 1; i >= 0 && i >= issued - STAGES; --i)
        (void)mbar_wait(bar_full + 8 * (i % STAGES), (uint32_t)(i / STAGES) & 1u);
    }
    __syncwarp();
  } else if (warp < WARP_MMA0 + NISS) {
    // ------------------------------------------------------------------ MMA issuers
    if (lane == 0) {
      const int e = warp - WARP_MMA0;
      const uint32_t idesc = idesc_i8(N, ROWS);
      // groups in CTA order; a task's groups are its quantisation groups in the basis segment
      // and its 64-code units in the base segment (the basis's exponent changes every 64
      // features there, so a 128-code group is summed as two)
      int g = 0;
      bool stop = false;
      for (int i = 0; i < ntask && !stop; ++i) {
        const bool seg = (int)((t0 + i) % p.W) >= p.Ww;
        const int upg = seg ? 1 : p.gpu, gpt = STAGE_UNITS / upg;
        const int s = i % STAGES;
        bool waited = false;
        for (int gl = 0; gl < gpt && !stop; ++gl, ++g) {
          if (g % NISS != e) continue;
          if (!waited) {
            if (!mbar_wait(bar_full + 8 * s, (uint32_t)(i / STAGES) & 1u, plim)) {
              raise_device_error(a.err, DEVERR_TIMEOUT_FULL_B);
              *abort_flag = 1;
              stop = true;
              break;
            }
            waited = true;
          }
          const int cs = g % ACC_SLOTS;
          // the slot's previous group has been read by the epilogue
          if (!mbar_wait(bar_cempty + 8 * cs, ((uint32_t)(g / ACC_SLOTS) & 1u) ^ 1u, plim)) {
            raise_device_error(a.err, DEVERR_TIMEOUT_EMPTY);
            *abort_flag = 1;
            stop = true;
            break;
          }
          const uint32_t dacc = tmem + ACC_COL + (uint32_t)(cs * N);
          for (int uu = 0; uu < upg; ++uu) {
            const int j = gl * upg + uu, u = i * STAGE_UNITS + j, as = u % ASLOTS;
            if (!mbar_wait(bar_afull + 8 * as, (uint32_t)(u / ASLOTS) & 1u, plim)) {
              raise_device_error(a.err, DEVERR_TIMEOUT_FULL_A);
              *abort_flag = 1;
              stop = true;
              break;
            }
            if (*abort_flag) {
              stop = true;
              break;
            }
            tc_fence_after();
            const uint32_t btile =
                s_base + s * p.stage_bytes + p.off_phi + (j >> 1) * BTILE + (j & 1) * 64;
            const uint32_t aaddr = tmem + (uint32_t)(as * A_COLS);
#pragma unroll
            for (int kk = 0; kk < 2; ++kk)
              mma_i8_ts(dacc, aaddr + (uint32_t)(kk * 8), smem_desc_sw128(btile + kk * 32), idesc,
                        (uu > 0 || kk > 0) ? 1u : 0u);
            mma_commit(bar_aempty + 8 * as);  // the unit's A slot is free once these complete
          }
          if (stop) break;
          mma_commit(bar_cfull + 8 * cs);
        }
        // done with this task's basis tiles once these MMAs complete (every issuer has groups in
        // every task: a task holds at least four groups)
        if (!stop) mma_commit(bar_empty + 8 * s);
      }
      // every MMA of this issuer completes before TMEM may be freed
      mma_commit(bar_done + 8 * e);
      (void)mbar_wait(bar_done + 8 * e, 0u);
    }
    __syncwarp();
  } else if (warp < WARP_EPI0) {
    // ------------------------------------------------------------------ decoders
    const int q = warp & 3;                    // TMEM lane quarter this warp may access
    const int h = (warp - WARP_DEC0) >> 2;     // this warp takes units j = h, h + 2, ...
    const int r = q * 32 + lane;
    const uint32_t lane_base = (uint32_t)(q * 32) << 16;
    for (int i = 0; i < ntask && !warp_aborted(abort_flag); ++i) {
      const int s = i % STAGES;
      if (!mbar_wait_warp(bar_full + 8 * s, (uint32_t)(i / STAGES) & 1u, plim)) {
        raise_device_error(a.err, DEVERR_TIMEOUT_FULL_B);
        *abort_flag = 1;
        break;
      }
      const uint8_t* crow = smem + s * p.stage_bytes + r * 128;
      uint4 cw[STAGE_UNITS / 2];
#pragma unroll
      for (int jj = 0; jj < STAGE_UNITS / 2; ++jj) {
        const int j = 2 * jj + h;
        cw[jj] = *reinterpret_cast<const uint4*>(crow + ((j ^ (r & 7)) << 4));
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(bar_empty + 8 * s);
#pragma unroll
      for (int jj = 0; jj < STAGE_UNITS / 2; ++jj) {
        const int u = i * STAGE_UNITS + 2 * jj + h, as = u % ASLOTS;
        if (!mbar_wait_warp(bar_aempty + 8 * as, ((uint32_t)(u / ASLOTS) & 1u) ^ 1u, plim)) {
          raise_device_error(a.err, DEVERR_TIMEOUT_EMPTY);
          *abort_flag = 1;
          break;
        }
        // 64 codes -> 64 signed bytes (-1, 0, +1) in the K order of the basis (cc::unit_pos)
        uint32_t op[16];
        uint32_t d[4];
        kl::decode16<false>(cw[jj].x, d);
        op[0] = d[0], op[1] = d[1], op[2] = d[2], op[3] = d[3];
        kl::decode16<false>(cw[jj].y, d);
        op[4] = d[0], op[5] = d[1], op[6] = d[2], op[7] = d[3];
        kl::decode16<false>(cw[jj].z, d);
        op[8] = d[0], op[9] = d[1], op[10] = d[2], op[11] = d[3];
        kl::decode16<false>(cw[jj].w, d);
        op[12] = d[0], op[13] = d[1], op[14] = d[2], op[15] = d[3];
        tmem_st16(tmem + lane_base + (uint32_t)(as * A_COLS), op);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar_afull + 8 * as);
      }
    }
  } else {
    // ------------------------------------------------------------------ epilogue
    const int ew = warp - WARP_EPI0;
    const int q = warp & 3, h = ew >> 2;  // lane quarter, half of the batch rows
    const int r = q * 32 + lane;
    const uint32_t lane_base = (uint32_t)(q * 32) << 16;
    T* Y = (T*)a.Y;
    const T* bias = (const T*)a.bias;
    float out[HN];
#pragma unroll
    for (int n = 0; n < HN; ++n) out[n] = 0.f;
    int g = 0;
    for (int i = 0; i < ntask; ++i) {
      const long long t = t0 + i;
      const int w = (int)(t % p.W), rb = (int)(t / p.W);
      const bool seg = w >= p.Ww;
      const int s = i % STAGES;
      bool live = !warp_aborted(abort_flag);
      if (live && !mbar_wait_warp(bar_full + 8 * s, (uint32_t)(i / STAGES) & 1u, plim)) {
        raise_device_error(a.err, DEVERR_TIMEOUT_FULL_B);
        *abort_flag = 1;
        live = false;
      }
      // the task's groups as the issuers count them (base segment: one per 64-code unit)
      const int upg = seg ? 1 : p.gpu, gps = STAGE_UNITS / upg;
      if (live) {
        const float* srow =
            reinterpret_cast<const float*>(smem + s * p.stage_bytes + p.off_scale) + r * p.sfl;
        const float* p2b = reinterpret_cast<const float*>(smem + s * p.stage_bytes + p.off_p2b);
        for (int gg = 0; gg < gps; ++gg, ++g) {
          const int cs = g % ACC_SLOTS;
          if (!mbar_wait_warp(bar_cfull + 8 * cs, (uint32_t)(g / ACC_SLOTS) & 1u, plim)) {
            raise_device_error(a.err, DEVERR_TIMEOUT_ACCUM);
            *abort_flag = 1;
            live = false;
            break;
          }
          tc_fence_after();
          uint32_t hv[HN], lv[HN];
          const uint32_t col = tmem + lane_base + ACC_COL + (uint32_t)(cs * N + h * HN);
          tmem_ld_cols<HN>(col, hv);
          tmem_ld_cols<HN>(col + NP, lv);
          asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(bar_cempty + 8 * cs);
          // act(scale): the dequantised weight is +-sa; the group's first unit is gg * upg
          const float sa = A::round(srow[gg * upg / p.gpu]);
          if (!seg) {
            const float f = sa * (1.0f / (float)(1 << PHI_E));
#pragma unroll
            for (int n = 0; n < HN; ++n)
              out[n] = fmaf((float)((int)hv[n] * 128 + (int)lv[n]), f, out[n]);
          } else {
            // base segment: each batch row's chunk exponent (unit gg = sixteen-code units
            // 4 gg .. 4 gg + 3, one 64-feature chunk)
#pragma unroll
            for (int n = 0; n < HN; ++n)
              out[n] = fmaf((float)((int)hv[n] * 128 + (int)lv[n]),
                            sa * p2b[(h * HN + n) * 32 + gg * 4], out[n]);
          }
        }
        __syncwarp();
        if (lane == 0 && live) mbar_arrive(bar_empty + 8 * s);
      }

      // -------------------------------------------------------------- row block done here
      if (((t + 1) % p.W) != 0 && i + 1 != ntask) continue;
      const int first = kl::owner((long long)rb * p.W, p.tasks, p.G);
      const int count = kl::owner((long long)rb * p.W + p.W - 1, p.tasks, p.G) - first + 1;
      const int slot = (int)blockIdx.x - first;
      const int row = rb * ROWS + r;
      const bool writer = *abort_flag == 0;
      if (count == 1) {
        if (writer && row < a.D_out) {
          const float bv = a.has_bias ? A::to_f(bias[row]) : 0.f;
#pragma unroll
          for (int n = 0; n < HN; ++n)
            if (h * HN + n < a.B) Y[(size_t)(h * HN + n) * a.D_out + row] = A::from_f(out[n] + bv);
        }
      } else {
        if (writer)
#pragma unroll
          for (int n = 0; n < HN; ++n)
            p.part[((size_t)(rb * p.maxc + slot) * NP + h * HN + n) * ROWS + r] = out[n];
        __threadfence();
        named_bar(BAR_EPI, EPI_THREADS);
        if (ew == 0 && lane == 0) {
          int last = 0;
          if (*abort_flag == 0) {
            unsigned long long* c = p.counters + rb;
            unsigned long long old = *reinterpret_cast<volatile unsigned long long*>(c), nv = 0;
            bool done = false;
            for (int it = 0; it < (1 << 20) && !done; ++it) {
              nv = ((unsigned)(old >> 32) == p.epoch)
                       ? old + 1
                       : (((unsigned long long)p.epoch << 32) | 1ull);
              const unsigned long long prev = atomicCAS(c, old, nv);
              done = prev == old;
              old = prev;
            }
            if (!done) {
              raise_device_error(a.err, DEVERR_TIMEOUT_ACCUM);
              *abort_flag = 1;
            }
            last = done && (int)(unsigned)nv == count;
          }
          *decision = last;
        }
        named_bar(BAR_EPI, EPI_THREADS);
        if (*decision) {
          // the last contributor: partials in contributor order, bias, round, store
          __threadfence();
          for (int idx = ew * 32 + lane; idx < ROWS * NP; idx += EPI_THREADS) {
            const int n = idx / ROWS, rr = idx % ROWS, rw = rb * ROWS + rr;
            if (n >= a.B || rw >= a.D_out) continue;
            float sum = 0.f;
            for (int z = 0; z < count; ++z)
              sum += __ldcg(p.part + ((size_t)(rb * p.maxc + z) * NP + n) * ROWS + rr);
            const float bv = a.has_bias ? A::to_f(bias[rw]) : 0.f;
            Y[(size_t)n * a.D_out + rw] = A::from_f(sum + bv);
          }
          if (ew == 0 && lane == 0) atomicExch(p.counters + rb, 0ull);
        }
      }
#pragma unroll
      for (int n = 0; n < HN; ++n) out[n] = 0.f;
    }
  }

  // every role is done (the issuers waited for their last MMAs): free TMEM
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == WARP_MMA0) tc::tmem_dealloc(tmem, TMEM_COLS);
}

}  // namespace i8
}  // namespace kan
