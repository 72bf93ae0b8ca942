// kan_gemv.cu -- small-batch path (B <= 64) for 2-bit packed weights (ternary / INT2 codebook).
//
// At small batch the layer is a weight stream: Y[B, D_out] = [Phi(x) | silu(x)] W^T reads every
// packed weight once and does only B multiply-adds with it.  The kernel therefore runs the
// contraction "swapped": the weights are the MMA's M operand (128 output rows per CTA) and the
// batch is N (B rounded up to 16), so tcgen05 does the arithmetic while
// the CUDA cores only decode.  The packed codes are never expanded in HBM:
//
//   warp 0      TMA producer: per stage, a 128-row x 32-word (512 codes) tile of the packed codes
//               (128-byte swizzle) and the matching per-(row, group) fp32 scales.
//   warps 1, 19 TMEM allocator (1) and MMA issuers, taking alternate units (a unit = two 64-code
//               chunks): per chunk 4 tcgen05.mma.cta_group::1.kind::f16 with A read from TMEM
//               (the decoded weights), B from shared memory (the basis tile), fp32 accumulators
//               in TMEM (one per issuer, summed in the epilogue).
//   warp 2      basis TMA: per unit, the two [B x 64] tiles of the basis matrix (below).
//   warps 3-18  decoders, four groups of four warps (one per TMEM lane quarter); group h decodes
//               unit h of every code stage.  A thread owns one output row: two 16-byte shared
//               loads of its eight code words, per-group lookup tables (two registers: low and
//               high bytes of the four dequantised values act(code_value * scale)), then per code
//               pair one byte permute (prmt) -> a bf16x2 / f16x2 operand pair; tcgen05.st of the
//               64 columns into the TMEM A ring (6 units deep, to cover the MMA round trip).
//               After the K loop group 0 reads the accumulators.
//
// The decoded operand equals the reference's dequantised weight rounded once to the operand
// dtype (metal_kan_bridge.mm:5073-5146, fused_kan.metal:2392-2441; code 3 of ternary -> 0).
// The code pairs come out permuted inside each 16-code word.
//
// The basis matrix Phi[B_pad][cols] (every basis term T_k(x_i) and silu(x_i) of the batch, in the
// operand dtype with the reference rounding points, kan_device.cuh) is written once per call by
// a small pre-pass kernel, in the same permuted order inside each 16-code word (perm_pos), to an
// L2-resident scratch buffer (B = 16: 1.3 MB for the 4096 x 9 + 4096 codes of a 4096-wide layer);
// the main kernel is launched as its programmatic dependent, so the code stream starts while the
// pre-pass runs, and only the basis TMA waits for it (griddepcontrol.wait).
//
// K is split over the S CTAs of a cluster (1 x 1 x S, S picked on the host from the number of
// clusters the GPU can hold at once, so that the grid runs in one wave): CTA z owns input features
// [z * FS, (z + 1) * FS) (FS a multiple of 64, so basis and base chunks both start on 64-code
// boundaries).  Partials are reduced through distributed shared memory in split order
// (deterministic); CTA z finishes batch rows n = z, z + S, ...
//
// Every wait is bounded (~1 s); on expiry the kernel records the error word, skips its remaining
// work, still joins every barrier and releases TMEM.
#include <cuda.h>

#include <algorithm>
#include <mutex>

#include "kan_tc_kernel.cuh"

namespace kan {
namespace sb {

using tc::bulk_g2s;
using tc::cluster_sync_all;
using tc::fence_proxy_async_smem;
using tc::instr_desc;
using tc::map_to_rank;
using tc::mbar_arrive;
using tc::mbar_arrive_expect_tx;
using tc::mbar_init;
using tc::mbar_wait;
using tc::mbar_wait_warp;
using tc::mma_commit;
using tc::smem_desc_sw128;
using tc::smem_u32;
using tc::tc_fence_after;
using tc::tc_fence_before;
using tc::tma_load_2d;
using tc::tmem_alloc;
using tc::tmem_dealloc;

constexpr int ROWS = 128;              // output rows per CTA (the MMA's M)
constexpr int CHUNK = 64;              // codes of one basis tile (4 words, 4 MMAs of K = 16)
constexpr int UNIT = 2;                // chunks per pipeline unit (one decoder step, 8 MMAs)
constexpr int STAGE_CHUNKS = 8;        // TMA stage: 32 words (128 B) per row
constexpr int UNITS_PER_STAGE = STAGE_CHUNKS / UNIT;
constexpr int CODE_STAGES = 4;
constexpr int SLOTS = 6;               // TMEM A ring and shared basis ring, in units
constexpr int MAXN = 64;               // largest (padded) batch
constexpr int MAX_SPLITS = 8;
constexpr int DEC_GROUPS = UNITS_PER_STAGE;  // decoder group h decodes unit h of every stage
constexpr int NUM_ISSUERS = 2;         // MMA-issuing threads (lane 0 of warp 1 and of the last warp)
constexpr int WARP_TMA = 0, WARP_MMA = 1, WARP_PHI = 2, WARP_DEC0 = 3,
              NUM_DEC_WARPS = 4 * DEC_GROUPS, WARP_MMA2 = WARP_DEC0 + NUM_DEC_WARPS;
constexpr int THREADS = (WARP_MMA2 + NUM_ISSUERS - 1) * 32;  // 640
constexpr uint32_t TMEM_COLS = 512;
constexpr int A_COLS = 32;             // TMEM columns of one chunk (64 16-bit values per lane)
constexpr int ACC_COL = SLOTS * UNIT * A_COLS;  // accumulators after the A ring (384)
// Several MMA issuers (issuer i takes the units u with u % NUM_ISSUERS == i), one accumulator
// each: at N = 16 the issue of tcgen05.mma, not the tensor pipe, bounds the rate, so more issuing
// threads raise it.  The accumulators are summed in the epilogue.
constexpr int NACC = NUM_ISSUERS;
constexpr int CODE_STAGE_BYTES = ROWS * 128;
static_assert(UNITS_PER_STAGE % NUM_ISSUERS == 0, "an issuer takes fixed unit positions");

// Shared memory: code stages, scale stages (sized by the group size), the basis ring (sized by the
// padded batch), the CTA's input slice when it fits, barriers.  Offsets are planned on the host.
constexpr int OFF_CODE = 0;
constexpr int OFF_SCALE = OFF_CODE + CODE_STAGES * CODE_STAGE_BYTES;
// code full/empty per stage; unit full (decoded A + basis tiles), slot empty per unit slot;
// accumulators ready
constexpr int NUM_BARS = 2 * CODE_STAGES + 2 * SLOTS + 1;
constexpr int SMEM_LIMIT = 227 * 1024;
static_assert(ROWS * MAXN * 4 <= CODE_STAGES * CODE_STAGE_BYTES, "partials fit the code stages");
static_assert(ACC_COL + NACC * MAXN <= (int)TMEM_COLS, "TMEM budget");

// Kernel-side view of the launch plan (host: plan()).
struct GemvParams {
  int S;         // K splits (cluster size along z)
  int FS;        // features per split (multiple of 64)
  int npad;      // batch rounded up to 16
  int gs;        // group size (32, 64 or 128)
  int gs_log2;
  int scale_pitch;  // floats per row of a scale stage: 512 / gs + 4
  int words_w, words_b;  // code words per row of W (D_in*K codes) and of Wb (D_in codes)
  int off_phi, off_bar, smem_alloc;  // shared-memory layout
  int kb_cols;   // basis columns of the basis matrix (D_in*K rounded up to 64); base columns follow
  int kpad;      // columns of the basis matrix
  uint32_t mul17;  // 0x11, passed at run time so that the selector products stay multiplies
};

// Position inside a 16-code word of the MMA K index that code u lands on (see decode_word).
__device__ __forceinline__ int perm_pos(int u) {
  return 2 * ((u & 3) + 4 * (u >> 3)) + ((u >> 2) & 1);
}

// Byte offset of element (n, k) (k < 64) in a K-major 128-byte-swizzled basis tile.
__device__ __forceinline__ uint32_t phi_off(int n, int k) {
  return (uint32_t)((n >> 3) * 1024 + (n & 7) * 128 + ((((k >> 3) ^ (n & 7)) << 4)) +
                    (k & 7) * 2);
}

// 16 codes of one word -> 8 operand pairs.  Column j (0..3) holds codes (j, j+4), column 4+j holds
// codes (j+8, j+12): byte t of a_j is code 4t+j; the selector byte 17*c + 64 = nibbles (c, c+4)
// picks the low byte of value c from tlo and its high byte from thi.  The selector of the upper
// code pair is the high word of a_j * (17 << 16) (a multiply-high, on the FMA pipe like the
// lower one, which leaves the integer pipe to the masks and byte permutes).
__device__ __forceinline__ void decode_word(uint32_t w, uint32_t tlo, uint32_t thi, uint32_t m17,
                                            uint32_t m17h, uint32_t* out) {
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint32_t aj = (w >> (2 * j)) & 0x03030303u;
    out[j] = __byte_perm(tlo, thi, aj * m17 + 0x40404040u);
    out[4 + j] = __byte_perm(tlo, thi, __umulhi(aj, m17h) + 0x4040u);
  }
}

// 16-bit pattern of act(v) (RNE), in the low half.
template <int MODE>
__device__ __forceinline__ uint32_t act_bits(float v) {
  if (MODE == MODE_F16) return (uint32_t)__half_as_ushort(__float2half_rn(v));
  return (uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(v));
}

// Lookup table of the four dequantised values of a group with scale s: tlo = their low bytes,
// thi = their high bytes (byte c = value of code c).
template <int MODE, int FMT>
__device__ __forceinline__ void make_table(float s, const float* cb, uint32_t& tlo,
                                           uint32_t& thi) {
  if (FMT == KAN_W_TERNARY) {
    // codes 0, 1, 2, 3 -> -s, 0, +s, 0 (the product by -1 / +1 is exact: act(-s) = -act(s))
    const uint32_t S = act_bits<MODE>(s);
    tlo = (S & 0xFFu) * 0x00010001u;
    thi = ((S >> 8) ^ 0x80u) | ((S >> 8) << 16);
  } else {
    const uint32_t p01 = act_bits<MODE>(__fmul_rn(cb[0], s)) |
                         (act_bits<MODE>(__fmul_rn(cb[1], s)) << 16);
    const uint32_t p23 = act_bits<MODE>(__fmul_rn(cb[2], s)) |
                         (act_bits<MODE>(__fmul_rn(cb[3], s)) << 16);
    tlo = __byte_perm(p01, p23, 0x6420);
    thi = __byte_perm(p01, p23, 0x7531);
  }
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]),
      "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]),
      "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
__device__ __forceinline__ void tmem_st_wait() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}
// D[tmem] (+)= A[tmem] * B[smem]^T
__device__ __forceinline__ void mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc,
                                       uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// The abort flag as one value for the whole warp (lanes must not split around warp-wide steps).
__device__ __forceinline__ bool warp_aborted(volatile int* flag) {
  return __shfl_sync(0xffffffffu, *flag, 0) != 0;
}
__device__ __forceinline__ float ld_cluster_f32(uint32_t addr) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
  return v;
}

// The CTA's work: the basis chunks [cb0, cb0 + nb_ch) of W, then the base chunks
// [cB0, cB0 + nB_ch) of Wb, in code stages of 8 chunks (a part's last stage may be short; the base
// part starts a new stage).  Unit u = 4 * stage + h covers chunks 2h, 2h + 1 of its stage; units
// past the end of a short stage are empty but still pass through every ring (so that all roles
// count units alike).
struct Plan {
  int cb0, cB0, nb_ch, nB_ch, nst_b, nst;
  __device__ __forceinline__ bool base(int st) const { return st >= nst_b; }
  __device__ __forceinline__ int first_cid(int st) const {
    return st < nst_b ? cb0 + st * STAGE_CHUNKS : cB0 + (st - nst_b) * STAGE_CHUNKS;
  }
  __device__ __forceinline__ int stage_chunks(int st) const {
    return st < nst_b ? min(STAGE_CHUNKS, nb_ch - st * STAGE_CHUNKS)
                      : min(STAGE_CHUNKS, nB_ch - (st - nst_b) * STAGE_CHUNKS);
  }
  // chunks in unit u (0, 1 or 2)
  __device__ __forceinline__ int unit_chunks(int u) const {
    const int h = u % UNITS_PER_STAGE;
    return max(0, min(UNIT, stage_chunks(u / UNITS_PER_STAGE) - UNIT * h));
  }
};

template <int MODE, int FMT, bool HALF_GROUPS>
__global__ void __launch_bounds__(THREADS, 1)
    kan_gemv_kernel(const __grid_constant__ CUtensorMap tm_wc,
                    const __grid_constant__ CUtensorMap tm_ws,
                    const __grid_constant__ CUtensorMap tm_bc,
                    const __grid_constant__ CUtensorMap tm_bs,
                    const __grid_constant__ CUtensorMap tm_phi, LayerArgs a, GemvParams p) {
  using T = typename Act<MODE>::T;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  const uint32_t s_base = smem_u32(smem);
  const uint32_t bar_cfull = s_base + p.off_bar;
  const uint32_t bar_cempty = bar_cfull + CODE_STAGES * 8;
  const uint32_t bar_afull = bar_cempty + CODE_STAGES * 8;  // decoders + basis TMA
  const uint32_t bar_sempty = bar_afull + SLOTS * 8;
  const uint32_t bar_acc = bar_sempty + SLOTS * 8;
  volatile uint32_t* tmem_slot =
      reinterpret_cast<volatile uint32_t*>(smem + p.off_bar + NUM_BARS * 8);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + p.off_bar + NUM_BARS * 8 + 4);
  const int tile_bytes = p.npad * 128;            // one chunk's basis tile
  const int phi_slot_bytes = UNIT * tile_bytes;   // one unit's
  const int scale_stage_bytes = ROWS * p.scale_pitch * 4;  // a multiple of 1024

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row0 = blockIdx.x * ROWS;
  const int z = blockIdx.z;
  const int B = a.B, K = a.K;
  // this split's input features and the chunk ranges they cover
  const int f0 = z * p.FS, f1 = min(a.D_in, f0 + p.FS);
  Plan pl;
  pl.cb0 = (f0 * K) / CHUNK;
  pl.cB0 = f0 / CHUNK;
  const int cb1 = (f1 * K + CHUNK - 1) / CHUNK;
  const int cB1 = a.has_base ? (f1 + CHUNK - 1) / CHUNK : pl.cB0;
  pl.nb_ch = max(0, cb1 - pl.cb0);
  pl.nB_ch = max(0, cB1 - pl.cB0);
  pl.nst_b = (pl.nb_ch + STAGE_CHUNKS - 1) / STAGE_CHUNKS;
  pl.nst = pl.nst_b + (pl.nB_ch + STAGE_CHUNKS - 1) / STAGE_CHUNKS;
  const int nst = pl.nst, nunits = nst * UNITS_PER_STAGE;

  if (threadIdx.x == 0) {
    for (int s = 0; s < CODE_STAGES; ++s) {
      mbar_init(bar_cfull + 8 * s, 1);
      mbar_init(bar_cempty + 8 * s, NUM_DEC_WARPS);
    }
    for (int s = 0; s < SLOTS; ++s) {
      // the four warps of the unit's decoder group + the basis TMA's arrival (with its bytes)
      mbar_init(bar_afull + 8 * s, 5);
      mbar_init(bar_sempty + 8 * s, 1);
    }
    mbar_init(bar_acc, NUM_ISSUERS);  // one commit per MMA issuer
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == WARP_MMA) tmem_alloc(s_base + p.off_bar + NUM_BARS * 8, TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == WARP_TMA) {
    // ------------------------------------------------------------------ code / scale TMA
    if (lane == 0) {
      const uint32_t bytes = (uint32_t)(CODE_STAGE_BYTES + ROWS * p.scale_pitch * 4);
      int issued = 0;
      for (int st = 0; st < nst; ++st) {
        const int slot = st % CODE_STAGES;
        if (!mbar_wait(bar_cempty + 8 * slot, ((uint32_t)(st / CODE_STAGES) & 1u) ^ 1u)) {
          raise_device_error(a.err, DEVERR_TIMEOUT_EMPTY);
          *abort_flag = 1;
          break;
        }
        if (*abort_flag) break;
        const bool base = pl.base(st);
        const int first_cid = pl.first_cid(st);
        const int g0 = first_cid * CHUNK / p.gs;
        mbar_arrive_expect_tx(bar_cfull + 8 * slot, bytes);
        tma_load_2d(s_base + OFF_CODE + slot * CODE_STAGE_BYTES, base ? &tm_bc : &tm_wc,
                    bar_cfull + 8 * slot, first_cid * 4, row0);
        tma_load_2d(s_base + OFF_SCALE + slot * scale_stage_bytes, base ? &tm_bs : &tm_ws,
                    bar_cfull + 8 * slot, g0 & ~3, row0);
        ++issued;
      }
      for (int st = issued - 1; st >= 0 && st >= issued - CODE_STAGES; --st)
        (void)mbar_wait(bar_cfull + 8 * (st % CODE_STAGES),
                        (uint32_t)(st / CODE_STAGES) & 1u);
    }
    __syncwarp();
  } else if (warp == WARP_MMA || warp >= WARP_MMA2) {
    // ------------------------------------------------------------------ MMA issuers
    if (lane == 0) {
      const int iss = warp == WARP_MMA ? 0 : 1 + warp - WARP_MMA2;
      const uint32_t idesc = instr_desc(MODE == MODE_BF16 ? 1 : 0, p.npad, 128);
      const uint32_t dacc = tmem + ACC_COL + (uint32_t)(iss * p.npad);
      // descriptor of slot 0's first basis tile; slot s, chunk c, K step kk add
      // (s * phi_slot_bytes + c * tile_bytes + 32 * kk) >> 4 to its address field
      const uint64_t bdesc0 = smem_desc_sw128(s_base + p.off_phi);
      uint32_t acc_flag = 0u;  // the issuer's first MMA overwrites its accumulator
      int s = iss % SLOTS;
      uint32_t par = (uint32_t)(iss / SLOTS) & 1u;
      for (int u = iss; u < nunits; u += NUM_ISSUERS) {
        if (!mbar_wait(bar_afull + 8 * s, par)) {
          raise_device_error(a.err, DEVERR_TIMEOUT_FULL_A);
          *abort_flag = 1;
          break;
        }
        if (*abort_flag) break;
        tc_fence_after();
        const int nv = pl.unit_chunks(u);
        const uint64_t bd = bdesc0 + (uint64_t)((s * phi_slot_bytes) >> 4);
        const uint32_t ad = tmem + (uint32_t)(s * UNIT * A_COLS);
        if (nv > 0) {
#pragma unroll
          for (int kk = 0; kk < CHUNK / 16; ++kk) {
            mma_ts(dacc, ad + (uint32_t)(kk * 8), bd + (uint64_t)(2 * kk), idesc, acc_flag);
            acc_flag = 1u;
          }
        }
        if (nv > 1) {
          const uint64_t bd1 = bd + (uint64_t)(tile_bytes >> 4);
#pragma unroll
          for (int kk = 0; kk < CHUNK / 16; ++kk)
            mma_ts(dacc, ad + (uint32_t)(A_COLS + kk * 8), bd1 + (uint64_t)(2 * kk), idesc, 1u);
        }
        mma_commit(bar_sempty + 8 * s);
        s += NUM_ISSUERS;
        if (s >= SLOTS) {
          s -= SLOTS;
          par ^= 1u;
        }
      }
      mma_commit(bar_acc);
    }
    __syncwarp();
  } else if (warp == WARP_PHI) {
    // ------------------------------------------------------------------ basis tile TMA
    if (lane == 0) {
      // the basis matrix is written by the pre-pass kernel this launch depends on
      asm volatile("griddepcontrol.wait;" ::: "memory");
      int issued = 0;
      for (int u = 0; u < nunits; ++u) {
        const int s = u % SLOTS;
        if (!mbar_wait(bar_sempty + 8 * s, ((uint32_t)(u / SLOTS) & 1u) ^ 1u)) {
          raise_device_error(a.err, DEVERR_TIMEOUT_EMPTY);
          *abort_flag = 1;
          break;
        }
        if (*abort_flag) break;
        const int nv = pl.unit_chunks(u);
        const int st = u / UNITS_PER_STAGE, h = u % UNITS_PER_STAGE;
        if (nv == 0) {
          mbar_arrive(bar_afull + 8 * s);
        } else {
          const int col = (pl.base(st) ? p.kb_cols : 0) + (pl.first_cid(st) + UNIT * h) * CHUNK;
          mbar_arrive_expect_tx(bar_afull + 8 * s, (uint32_t)(nv * tile_bytes));
          for (int c = 0; c < nv; ++c)
            tma_load_2d(s_base + p.off_phi + s * phi_slot_bytes + c * tile_bytes, &tm_phi,
                        bar_afull + 8 * s, col + c * CHUNK, 0);
        }
        ++issued;
      }
      // drain: the last copies land before the CTA may exit (the issuer waited for them unless
      // it aborted)
      for (int u = issued - 1; u >= 0 && u >= issued - SLOTS; --u)
        (void)mbar_wait(bar_afull + 8 * (u % SLOTS), (uint32_t)(u / SLOTS) & 1u);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------------ decoders + epilogue
    const int dw = warp - WARP_DEC0;
    const int q = warp & 3;           // TMEM lane quarter this warp may access
    const int h = dw >> 2;            // this warp's group decodes unit h of every stage
    const int r = q * 32 + lane;      // row within the CTA tile
    const uint32_t lane_base = (uint32_t)(q * 32) << 16;
    const uint32_t m17 = p.mul17, m17h = p.mul17 << 16;
    float cbw[4] = {0.f, 0.f, 0.f, 0.f}, cbb[4] = {0.f, 0.f, 0.f, 0.f};
    if (FMT == KAN_W_INT2) {
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        cbw[c] = __ldg(a.w.codebook + c);
        cbb[c] = a.has_base ? __ldg(a.wb.codebook + c) : 0.f;
      }
    }
    // Per stage: wait for the codes, take this group's unit (two 16-byte loads per row and the
    // scales of its groups), release the stage, decode into the TMEM A ring, publish the unit.
    uint32_t op[32];
    for (int st = 0; st < nst && !warp_aborted(abort_flag); ++st) {
      const int slot = st % CODE_STAGES;
      if (!mbar_wait_warp(bar_cfull + 8 * slot, (uint32_t)(st / CODE_STAGES) & 1u)) {
        raise_device_error(a.err, DEVERR_TIMEOUT_FULL_B);
        *abort_flag = 1;
        break;
      }
      const int u = st * UNITS_PER_STAGE + h;
      const int s = u % SLOTS;
      const int nv = pl.unit_chunks(u);
      const bool base = pl.base(st);
      const int first_cid = pl.first_cid(st);
      const int gbase = ((first_cid * CHUNK) >> p.gs_log2) & ~3;
      const int cid0 = first_cid + UNIT * h;
      const uint8_t* cst = smem + OFF_CODE + slot * CODE_STAGE_BYTES + r * 128;
      const float* sst = reinterpret_cast<const float*>(smem + OFF_SCALE +
                                                        slot * scale_stage_bytes) +
                         r * p.scale_pitch;
      uint4 wv0 = make_uint4(0u, 0u, 0u, 0u), wv1 = wv0;
      // lookup tables of the unit's four 32-code quarters (a group covers whole quarters)
      uint32_t tlo[4], thi[4];
      if (nv > 0) {
        wv0 = *reinterpret_cast<const uint4*>(cst + (((UNIT * h) ^ (r & 7)) << 4));
        if (nv > 1) wv1 = *reinterpret_cast<const uint4*>(cst + (((UNIT * h + 1) ^ (r & 7)) << 4));
        const float* cb = base ? cbb : cbw;
        if (HALF_GROUPS) {
#pragma unroll
          for (int j = 0; j < 4; ++j)
            make_table<MODE, FMT>(sst[((cid0 * CHUNK + 32 * j) >> p.gs_log2) - gbase], cb, tlo[j],
                                  thi[j]);
        } else {
          // groups of 64 or 128 codes: one table per chunk
#pragma unroll
          for (int c = 0; c < UNIT; ++c) {
            make_table<MODE, FMT>(sst[(((cid0 + c) * CHUNK) >> p.gs_log2) - gbase], cb,
                                  tlo[2 * c], thi[2 * c]);
            tlo[2 * c + 1] = tlo[2 * c];
            thi[2 * c + 1] = thi[2 * c];
          }
        }
      }
      // every code word and scale of this stage this warp needs is in registers
      __syncwarp();
      if (lane == 0) mbar_arrive(bar_cempty + 8 * slot);
      if (!mbar_wait_warp(bar_sempty + 8 * s, ((uint32_t)(u / SLOTS) & 1u) ^ 1u)) {
        raise_device_error(a.err, DEVERR_TIMEOUT_EMPTY);
        *abort_flag = 1;
        break;
      }
      if (nv > 0) {
        const uint32_t ta = tmem + lane_base + (uint32_t)(s * UNIT * A_COLS);
        decode_word(wv0.x, tlo[0], thi[0], m17, m17h, op);
        decode_word(wv0.y, tlo[0], thi[0], m17, m17h, op + 8);
        decode_word(wv0.z, tlo[1], thi[1], m17, m17h, op + 16);
        decode_word(wv0.w, tlo[1], thi[1], m17, m17h, op + 24);
        tmem_st32(ta, op);
        if (nv > 1) {
          decode_word(wv1.x, tlo[2], thi[2], m17, m17h, op);
          decode_word(wv1.y, tlo[2], thi[2], m17, m17h, op + 8);
          decode_word(wv1.z, tlo[3], thi[3], m17, m17h, op + 16);
          decode_word(wv1.w, tlo[3], thi[3], m17, m17h, op + 24);
          tmem_st32(ta + (uint32_t)A_COLS, op);
        }
        tmem_st_wait();
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar_afull + 8 * s);
    }

    // ------------------------------------------------------------------ epilogue
    if (!mbar_wait_warp(bar_acc, 0)) {
      raise_device_error(a.err, DEVERR_TIMEOUT_ACCUM);
      *abort_flag = 1;
    }
    tc_fence_after();
    // the warps of decoder group 0 read the accumulators (16 columns at a time, summed over the
    // issuers in a fixed order) into the partials [n][ROWS] over the finished code stages
    const bool reader = h == 0;
    float* part = reinterpret_cast<float*>(smem + OFF_CODE);
    // issuer u takes the units whose position in the stage is u mod 2: it had an MMA iff some
    // stage holds more than 2u chunks
    const int maxc = max(min(STAGE_CHUNKS, pl.nb_ch), min(STAGE_CHUNKS, pl.nB_ch));
    for (int c = 0; c < p.npad; c += 16) {
      if (!reader) break;
      float acc[16];
#pragma unroll
      for (int t = 0; t < 16; ++t) acc[t] = 0.f;
#pragma unroll
      for (int u = 0; u < NACC; ++u) {
        if (maxc <= UNIT * u) continue;  // issuer u had no chunk
        float v[16];
        tc::tmem_ld16(tmem + lane_base + (uint32_t)(ACC_COL + u * p.npad + c), v);
#pragma unroll
        for (int t = 0; t < 16; ++t) acc[t] += v[t];
      }
#pragma unroll
      for (int t = 0; t < 16; ++t)
        if (c + t < B) part[(c + t) * ROWS + r] = acc[t];
    }
    // keep the partials of every CTA alive until the whole cluster has read them
    asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
    asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
    const int row = row0 + r;
    const bool ab = warp_aborted(abort_flag);
    if (reader && row < a.D_out && !ab) {
      T* Y = (T*)a.Y;
      const float b = a.has_bias ? Act<MODE>::to_f(((const T*)a.bias)[row]) : 0.f;
      const uint32_t part_addr = smem_u32(part);
      for (int n = z; n < B; n += p.S) {
        float sum = 0.f;
        for (int zz = 0; zz < p.S; ++zz)
          sum += ld_cluster_f32(map_to_rank(part_addr, (uint32_t)zz) +
                                (uint32_t)((n * ROWS + r) * 4));
        Y[(size_t)n * a.D_out + row] = Act<MODE>::from_f(sum + b);
      }
    }
  }

  if (warp < WARP_DEC0 || warp >= WARP_MMA2) {
    // the other warps join the two cluster barriers of the epilogue
    __syncwarp();
    asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
    asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
  }
  __syncwarp();
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");

  tc_fence_before();
  __syncthreads();
  if (warp == WARP_MMA) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

// Basis matrix pre-pass: Phi[n][c] for n < npad, c < kpad.  Column c < kb_cols is basis code c
// (term c % K of feature c / K), column kb_cols + i is silu of feature i; rows >= B and the
// padding columns are zero.  Inside each 16-column word the value of code u sits at perm_pos(u).
// One thread per (row, feature): one input load, the Chebyshev recurrence (ChebyGen's values),
// K + 1 two-byte stores; threads past D_in zero the padding columns.
__device__ __forceinline__ int phi_col(int c) { return (c & ~15) + perm_pos(c & 15); }

template <int MODE>
__global__ void __launch_bounds__(256) gemv_phi_kernel(LayerArgs a, typename Act<MODE>::T* phi,
                                                       int npad, int kb_cols, int kpad) {
  // let the dependent main kernel start its prologue and code stream now
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  using T = typename Act<MODE>::T;
  const int n = blockIdx.y;  // batch row
  const bool valid = n < a.B;
  const T* xrow = (const T*)a.X + (size_t)n * a.D_in;
  T* prow = phi + (size_t)n * kpad;
  const int K = a.K, kdim = a.D_in * K;
  const T zero = Act<MODE>::from_f(0.f);
  for (int f = blockIdx.x * blockDim.x + threadIdx.x; f < a.D_in + CHUNK;
       f += gridDim.x * blockDim.x) {
    if (f < a.D_in) {
      const float xm =
          valid ? map_input<MODE>(Act<MODE>::to_f(xrow[f]), a.input_map, 0.f, 1.f) : 0.f;
      ChebyGen<MODE> gen;
      gen.init(xm, f, a);
      for (int k = 0; k < K; ++k) {
        const float v = gen.next();
        prow[phi_col(f * K + k)] = valid ? Act<MODE>::from_f(v) : zero;
      }
      if (a.has_base) prow[phi_col(kb_cols + f)] = valid ? Act<MODE>::from_f(silu_value<MODE>(xm)) : zero;
    } else {
      const int e = f - a.D_in;  // 0..63: padding columns
      if (kdim + e < kb_cols) prow[phi_col(kdim + e)] = zero;
      if (a.has_base && kb_cols + a.D_in + e < kpad) prow[phi_col(kb_cols + a.D_in + e)] = zero;
    }
  }
}

// ---------------------------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------------------------
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn get_encode() {
  static EncodeTiledFn fn = nullptr;
  static bool tried = false;
  if (!tried) {
    tried = true;
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = (EncodeTiledFn)ptr;
  }
  return fn;
}

// [rows][cols] 32-bit matrix, box = box_cols x ROWS, zero fill outside.
static bool make_map32(CUtensorMap* m, const void* base, int rows, int cols, int box_cols,
                       bool codes) {
  EncodeTiledFn enc = get_encode();
  if (!enc || ((uintptr_t)base & 15) || (cols % 4)) return false;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)cols * 4};
  cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)ROWS};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(m, codes ? CU_TENSOR_MAP_DATA_TYPE_UINT32 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2,
                   const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE,
                   codes ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// Basis matrix [npad][kpad] of the operand dtype: box = 64 columns x npad rows, 128-byte swizzle.
static bool make_map_phi(CUtensorMap* m, const void* base, int npad, int kpad, bool bf16) {
  EncodeTiledFn enc = get_encode();
  if (!enc || ((uintptr_t)base & 15)) return false;
  cuuint64_t dims[2] = {(cuuint64_t)kpad, (cuuint64_t)npad};
  cuuint64_t strides[1] = {(cuuint64_t)kpad * 2};
  cuuint32_t box[2] = {(cuuint32_t)CHUNK, (cuuint32_t)npad};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(m, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
                   const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// K split of a row block: S CTAs of FS features each (FS a multiple of 64).
static void set_split(GemvParams& p, int D_in, int S) {
  const int f64 = (D_in + 63) / 64;
  S = std::max(1, std::min(S, f64));
  p.FS = ((f64 + S - 1) / S) * 64;
  p.S = (D_in + p.FS - 1) / p.FS;
}

static GemvParams plan(const LayerArgs& a) {
  GemvParams p = {};
  const int R = (a.D_out + ROWS - 1) / ROWS;
  set_split(p, a.D_in, std::max(1, std::min(MAX_SPLITS, 148 / std::max(1, R))));
  p.npad = (a.B + 15) / 16 * 16;
  p.gs = a.w.group_size;
  p.gs_log2 = p.gs == 32 ? 5 : (p.gs == 64 ? 6 : 7);
  p.scale_pitch = STAGE_CHUNKS * CHUNK / p.gs + 4;
  p.words_w = (a.D_in * a.K + 15) / 16;
  p.words_b = (a.D_in + 15) / 16;
  const int scale_end = OFF_SCALE + CODE_STAGES * ROWS * p.scale_pitch * 4;
  p.off_phi = (scale_end + 1023) / 1024 * 1024;
  p.off_bar = p.off_phi + SLOTS * UNIT * p.npad * 128;
  p.smem_alloc = p.off_bar + NUM_BARS * 8 + 16 + 1024;  // + slack to align the base to 1024 B
  p.kb_cols = (a.D_in * a.K + CHUNK - 1) / CHUNK * CHUNK;
  p.kpad = p.kb_cols + (a.has_base ? (a.D_in + CHUNK - 1) / CHUNK * CHUNK : 0);
  p.mul17 = 0x11u;
  return p;
}

}  // namespace sb

bool gemv_supported(const LayerArgs& a, int act_dtype) {
  using namespace sb;
  if (act_dtype != KAN_F16 && act_dtype != KAN_BF16) return false;
  if (a.basis != KAN_CHEBY) return false;
  if (a.B < 1 || a.B > MAXN) return false;
  if (a.input_map == KAN_MAP_LAYERNORM) return false;
  if (a.w.format != KAN_W_TERNARY && a.w.format != KAN_W_INT2) return false;
  const int gs = a.w.group_size;
  if (gs != 32 && gs != 64 && gs != 128) return false;
  if (a.has_base && (a.wb.format != a.w.format || a.wb.group_size != gs)) return false;
  if (a.D_out < ROWS || a.D_in < 512 || a.K < 1) return false;
  const int words_w = (a.D_in * a.K + 15) / 16, words_b = (a.D_in + 15) / 16;
  const int groups_w = (a.D_in * a.K + gs - 1) / gs, groups_b = (a.D_in + gs - 1) / gs;
  const int pitch = STAGE_CHUNKS * CHUNK / gs + 4;
  if (words_w % 4 || groups_w % 4 || groups_w < pitch) return false;
  if (a.has_base && (words_b % 4 || groups_b % 4 || groups_b < pitch || words_b < 32))
    return false;
  auto al = [](const void* ptr) { return ((uintptr_t)ptr & 15) == 0; };
  if (!al(a.w.data) || !al(a.w.scales) || (a.has_base && (!al(a.wb.data) || !al(a.wb.scales))))
    return false;
  return true;
}

size_t gemv_phi_bytes(const LayerArgs& a) {
  const sb::GemvParams p = sb::plan(a);
  return (size_t)p.npad * p.kpad * 2;
}

// cudaOccupancyMaxActiveClusters, cached per (kernel instance, cluster size, shared memory).
template <class Kern>
static int max_clusters(Kern kern, int ki, const cudaLaunchConfig_t& q) {
  struct Entry {
    int ki, S, smem, clusters;
  };
  static Entry cache[32];
  static int used = 0;
  static std::mutex mu;
  std::lock_guard<std::mutex> lk(mu);
  const int S = (int)q.attrs[0].val.clusterDim.z, smem = (int)q.dynamicSmemBytes;
  for (int i = 0; i < used; ++i)
    if (cache[i].ki == ki && cache[i].S == S && cache[i].smem == smem) return cache[i].clusters;
  int clusters = 0;
  if (cudaOccupancyMaxActiveClusters(&clusters, kern, &q) != cudaSuccess) {
    (void)cudaGetLastError();
    clusters = 0;
  }
  if (used < 32) cache[used++] = {ki, S, smem, clusters};
  return clusters;
}

cudaError_t launch_gemv(const LayerArgs& a, int act_dtype, void* phi, cudaStream_t s) {
  using namespace sb;
  const GemvParams p = plan(a);
  const bool bf = act_dtype == KAN_BF16;
  CUtensorMap tphi;
  if (!make_map_phi(&tphi, phi, p.npad, p.kpad, bf)) return cudaErrorInvalidValue;
  const int groups_w = (a.D_in * a.K + p.gs - 1) / p.gs, groups_b = (a.D_in + p.gs - 1) / p.gs;
  CUtensorMap wc, ws, bc, bs;
  if (!make_map32(&wc, a.w.data, a.D_out, p.words_w, 32, true) ||
      !make_map32(&ws, a.w.scales, a.D_out, groups_w, p.scale_pitch, false))
    return cudaErrorInvalidValue;
  if (a.has_base) {
    if (!make_map32(&bc, a.wb.data, a.D_out, p.words_b, 32, true) ||
        !make_map32(&bs, a.wb.scales, a.D_out, groups_b, p.scale_pitch, false))
      return cudaErrorInvalidValue;
  } else {
    bc = wc;
    bs = ws;
  }
  const bool tern = a.w.format == KAN_W_TERNARY;
  {
    // one wave (every block reaches launch_dependents at once): grid (x, row), grid-stride in x
    const int bx = std::max(1, std::min((a.D_in + CHUNK + 255) / 256, 148 * 4 / p.npad));
    const dim3 grid((unsigned)bx, (unsigned)p.npad);
    if (bf)
      gemv_phi_kernel<MODE_BF16><<<grid, 256, 0, s>>>(a, (__nv_bfloat16*)phi, p.npad, p.kb_cols,
                                                      p.kpad);
    else
      gemv_phi_kernel<MODE_F16><<<grid, 256, 0, s>>>(a, (__half*)phi, p.npad, p.kb_cols, p.kpad);
    note_launch();
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
  }
  using KernFn = void (*)(const CUtensorMap, const CUtensorMap, const CUtensorMap,
                          const CUtensorMap, const CUtensorMap, LayerArgs, GemvParams);
  // [bf16][int2][32-code groups]
  static const KernFn kerns[8] = {
      kan_gemv_kernel<MODE_F16, KAN_W_TERNARY, false>, kan_gemv_kernel<MODE_F16, KAN_W_TERNARY, true>,
      kan_gemv_kernel<MODE_F16, KAN_W_INT2, false>, kan_gemv_kernel<MODE_F16, KAN_W_INT2, true>,
      kan_gemv_kernel<MODE_BF16, KAN_W_TERNARY, false>, kan_gemv_kernel<MODE_BF16, KAN_W_TERNARY, true>,
      kan_gemv_kernel<MODE_BF16, KAN_W_INT2, false>, kan_gemv_kernel<MODE_BF16, KAN_W_INT2, true>};
  const int ki = (bf ? 4 : 0) + (tern ? 0 : 2) + (p.gs == 32 ? 1 : 0);
  const KernFn kern = kerns[ki];
  static std::atomic<unsigned long long> configured[8];  // per device, one per instance
  {
    cudaError_t e = ensure_smem_attr(kern, SMEM_LIMIT, configured[ki]);
    if (e != cudaSuccess) return e;
  }
  // K splits: the largest power of two (<= the plan's) whose whole grid of clusters the GPU holds
  // at once (clusters must fit inside one GPC; a second wave would double the time)
  const int R = (a.D_out + ROWS - 1) / ROWS;
  GemvParams pl = p;
  for (int S = p.S; S >= 1; S = (S > 1 ? S / 2 : 0)) {
    set_split(pl, a.D_in, S);
    if (pl.S == 1) break;
    cudaLaunchConfig_t q = {};
    q.gridDim = dim3((unsigned)R, 1, (unsigned)pl.S);
    q.blockDim = dim3(THREADS, 1, 1);
    q.dynamicSmemBytes = (size_t)pl.smem_alloc;
    cudaLaunchAttribute qa[1];
    qa[0].id = cudaLaunchAttributeClusterDimension;
    qa[0].val.clusterDim.x = 1;
    qa[0].val.clusterDim.y = 1;
    qa[0].val.clusterDim.z = (unsigned)pl.S;
    q.attrs = qa;
    q.numAttrs = 1;
    if (max_clusters(kern, ki, q) >= R) break;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)R, 1, (unsigned)pl.S);
  cfg.blockDim = dim3(THREADS, 1, 1);
  cfg.dynamicSmemBytes = (size_t)pl.smem_alloc;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = (unsigned)pl.S;
  // programmatic dependent launch: starts while the basis pre-pass runs (see griddepcontrol)
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  note_launch();
  return cudaLaunchKernelEx(&cfg, kern, wc, ws, bc, bs, tphi, a, pl);
}

}  // namespace kan
