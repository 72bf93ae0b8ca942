// kan_gemv_cc.cuh -- small-batch path on the CUDA cores (B <= 4): ternary, INT8 and INT4 weights.
//
// With a handful of rows the layer is a stream of packed weights: each weight is read once and
// meets only B basis values.  The tensor cores cannot help there (an MMA needs N >= 16 batch
// columns, so 15/16 of it would be padding), and expanding the codes to 16-bit operands costs more
// CUDA-core work than the dot products themselves.  This path keeps the codes packed all the way:
//
//   * a pre-pass (one warp per 64 input features, launched as the main kernel's programmatic
//     dependency) evaluates every basis term phi and silu(x) of the batch with the reference
//     rounding points (kan_device.cuh), then writes each value in fixed point, v = rint(phi * 2^E)
//     with |v| <= 8192, as two signed bytes v = 128 * hi + lo (hi in [-64, 64], lo in [-64, 63]).
//     Basis terms are bounded by 1 in magnitude (Chebyshev on the clamped input, Gaussians,
//     cubic B-splines, the three wavelets, tents, sines and cosines), so their E is 13: every
//     operand-dtype value of magnitude >= 2^-6 is represented exactly, smaller ones to within
//     2^-14.  silu(x) is not bounded, so each 64-feature chunk of the base branch gets its own E
//     from its largest value.
//   * the main kernel streams [32 rows x 256 code bytes] stages of the packed weights (two TMA
//     boxes of 128 bytes, 128-byte swizzle) and their per-group scales / minima into a 4-stage
//     ring; one lane per output row reads its 16-byte chunks (conflict-free), turns each 16-code
//     unit into four words of bytes and accumulates dp4a products against the hi and lo bytes of
//     the basis in eight independent int32 chains per batch row (one per word and half).  Once per
//     quantisation group (or per 16-byte chunk, whichever is smaller) the chains are combined into
//     the exact integer sum 128 * H + L, converted once and scaled by the group's fp32 scale
//     (ternary: rounded to the operand dtype, which makes the product the reference's dequantised
//     weight rounded to the operand dtype, exactly); INT8/INT4 add the group minimum times the
//     (exact) basis sum of the group's codes.
//   * ternary decode: with KAN_WFLAG_TERNARY_NO3 (no code 3) a word x of 16 codes gives its four
//     byte words as x & (0x03030303 << 2f) -- code c in place, times 4^f -- so the chains hold
//     4^f * sum(c v), rescaled when combined, and value c - 1 is obtained by subtracting the unit
//     sums of v.  Without the flag a byte-permute table maps 0, 1, 2, 3 to -1, 0, +1, 0.
//   * K is split over S CTAs per 32-row block (S from the occupancy, so the whole grid is resident
//     at once); each split stores its fp32 partials, and the last CTA of a row block to finish
//     (atomic counter) sums them in split order -- deterministic -- adds the bias, rounds, stores.
//
// A unit's basis bytes are stored in the order its decoder produces codes: unit_pos below.
//
// Every wait is bounded; on expiry the kernel records the device error word, stops consuming,
// and the TMA warp still waits (full limit) for each load it issued before the CTA exits.
#pragma once

#include <cuda.h>

#include "kan_tc_kernel.cuh"

namespace kan {
namespace cc {

using tc::mbar_arrive;
using tc::mbar_arrive_expect_tx;
using tc::mbar_init;
using tc::mbar_wait;
using tc::mbar_wait_warp;
using tc::smem_u32;
using tc::tma_load_2d;

constexpr int ROWS = 32;                      // output rows per CTA: one per lane
constexpr int BOX_BYTES = 128;                // code bytes of one row in one TMA box
constexpr int BOXES = 2;                      // boxes per stage
constexpr int ROW_BYTES = BOX_BYTES * BOXES;  // code bytes of one row per stage
constexpr int BOX_TILE = ROWS * BOX_BYTES;    // 4 KB
constexpr int CODE_TILE = ROWS * ROW_BYTES;   // 8 KB
constexpr int NWARPS = 4;                     // compute warps
constexpr int CHUNKS_PER_WARP = ROW_BYTES / 16 / NWARPS;
constexpr int WARP_TMA = NWARPS;
constexpr int THREADS = (NWARPS + 1) * 32;
constexpr int STAGES = 4;
constexpr int MAXB = 4;
constexpr int PHI_E = 13;                     // fixed-point exponent of the basis terms
constexpr int PRE_THREADS = 64;               // pre-pass: one thread per input feature,
constexpr int PRE_FEATURES = 64;              // 64 features (one base exponent chunk) per CTA

struct Params {
  int fmt;                   // KAN_W_TERNARY / KAN_W_INT8 / KAN_W_INT4
  int fast;                  // ternary without code 3: in-place decode
  int fu;                    // 16-code units per flush of the integer chains
  int cpb;                   // codes per byte: 4, 1, 2
  int stages_w, stages_b;    // stages of the basis / base segment
  int nst;                   // stages_w + stages_b
  int S;                     // K splits (grid.y)
  int gs;                    // group size in codes (a power of two, >= 16)
  int lg;                    // log2(gs / 16): 16-code units per group
  int groups_w, groups_b;    // scale groups of one row, per segment
  int sbox_w, sbox_b;        // floats per row of a scale (and minimum) tile, per segment
  int sbox_max;
  int units_w, units_b;      // 16-code units per batch row of the basis matrix, per segment
  int phi_pitch;             // bytes of one batch row of the hi (or lo) matrix
  int ups;                   // 16-code units per stage
  int tile_bytes;            // one ring stage: codes, scales (, minima), basis slice, unit data
  int off_phi, off_aux;      // offsets inside a stage of the basis slice and the unit data
  int off_red, off_bar, smem;
  int rowblocks;
  // scratch (device pointers into one buffer)
  int8_t* phi_hi;
  int8_t* phi_lo;
  float* sumphi;             // [B][units_w + units_b]: basis sum of each unit (INT8/INT4: real
                             // value; in-place ternary: fixed-point integer)
  float* p2b;                // [B][units_b]: 2^-E of each base unit
  float* part;               // [S][B][D_out] split partials
  int* counters;             // [rowblocks]
};

// Position of code j (0..15) of a unit in its decoder's byte order: four words of four bytes.
// Table decoders (ternary with code 3, INT8, INT4): [0 2 4 6 | 1 3 5 7 | 8 10 12 14 | 9 11 13 15];
// in-place ternary: word f holds codes f, 4+f, 8+f, 12+f.
__host__ __device__ __forceinline__ int unit_pos(int j, bool fast) {
  return fast ? (((j & 3) << 2) | (j >> 2)) : ((j & 8) | ((j & 1) << 2) | ((j & 7) >> 1));
}

__device__ __forceinline__ int dp4a_ss(uint32_t a, uint32_t b, int c) {
  int d;
  asm("dp4a.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
__device__ __forceinline__ int dp4a_us(uint32_t a, uint32_t b, int c) {
  int d;
  asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

// ---------------------------------------------------------------------------------------------
// pre-pass: fixed-point basis matrix (hi / lo bytes), unit sums, base-chunk exponents
// ---------------------------------------------------------------------------------------------
__device__ __forceinline__ void put_fixed(int8_t* hi, int8_t* lo, int code, int q, bool fast) {
  const int h = (q + 64) >> 7;
  const int pos = (code & ~15) | unit_pos(code & 15, fast);
  hi[pos] = (int8_t)h;
  lo[pos] = (int8_t)(q - (h << 7));
}

// Exponent E <= 13 with max_abs * 2^E <= 8191 (so |rint(v * 2^E)| <= 8191).
__device__ __forceinline__ int fixed_exponent(float max_abs) {
  if (!(max_abs > 0.f)) return PHI_E;
  int e = min(PHI_E, (int)floorf(log2f(8191.f / max_abs)));
  while (max_abs * exp2f((float)e) > 8191.f) --e;
  return e;
}

template <int MODE, int BASIS>
__global__ void __launch_bounds__(PRE_THREADS) cc_phi_kernel(LayerArgs a, Params p) {
  // the dependent main kernel may start streaming weights now
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  using T = typename Act<MODE>::T;
  using Gen = typename GenFor<BASIS, MODE>::type;
  const int n = blockIdx.y;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const bool fast = p.fast != 0;
  const T* xrow = (const T*)a.X + (size_t)n * a.D_in;
  int8_t* hi = p.phi_hi + (size_t)n * p.phi_pitch;
  int8_t* lo = p.phi_lo + (size_t)n * p.phi_pitch;
  const int units = p.units_w + p.units_b;
  float* sum = p.sumphi + (size_t)n * units;
  const int K = a.K, kdim = a.D_in * K;
  const bool need_sums = p.fmt != KAN_W_TERNARY || fast;

  if (blockIdx.x == 0 && n == 0)
    for (int i = tid; i < p.rowblocks; i += PRE_THREADS) p.counters[i] = 0;

  // LayerNorm statistics of the row (each CTA of the row computes them; rows are short here)
  __shared__ float red[PRE_THREADS / 32];
  float mean = 0.f, rstd = 1.f;
  if (a.input_map == KAN_MAP_LAYERNORM) {
    float s = 0.f;
    for (int i = tid; i < a.D_in; i += PRE_THREADS) s += Act<MODE>::to_f(xrow[i]);
    for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (lane == 0) red[warp] = s;
    __syncthreads();
    s = 0.f;
    for (int w = 0; w < PRE_THREADS / 32; ++w) s += red[w];
    mean = s / (float)a.D_in;
    __syncthreads();
    float v = 0.f;
    for (int i = tid; i < a.D_in; i += PRE_THREADS) {
      const float d = Act<MODE>::to_f(xrow[i]) - mean;
      v = fmaf(d, d, v);
    }
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (lane == 0) red[warp] = v;
    __syncthreads();
    v = 0.f;
    for (int w = 0; w < PRE_THREADS / 32; ++w) v += red[w];
    rstd = rsqrtf(v / (float)a.D_in + a.ln_eps);
  }

  // padding codes of both segments (whole stages are streamed) are zero; block 0 of the row
  // clears them every call, since the scratch is shared with other layers
  if (blockIdx.x == 0) {
    for (int c = kdim + tid; c < p.units_w * 16; c += PRE_THREADS) put_fixed(hi, lo, c, 0, fast);
    for (int c = a.D_in + tid; c < p.units_b * 16; c += PRE_THREADS)
      put_fixed(hi + p.units_w * 16, lo + p.units_w * 16, c, 0, fast);
    for (int u = (kdim + 15) / 16 + tid; u < p.units_w; u += PRE_THREADS) sum[u] = 0.f;
    for (int u = (a.D_in + 15) / 16 + tid; u < p.units_b; u += PRE_THREADS) {
      sum[p.units_w + u] = 0.f;
      p.p2b[(size_t)n * p.units_b + u] = 0.f;
    }
  }

  // this CTA's 64 features, one per thread: the basis terms (E = 13) and silu (E of the chunk)
  // are put in fixed point into shared memory in the main kernel's byte order, then copied out
  // with 16-byte stores and summed per unit there -- no read-back of scattered global bytes
  extern __shared__ __align__(16) int8_t pre_smem[];
  const int wcodes = PRE_FEATURES * K;  // this CTA's basis codes: a whole number of 64-code groups
  int8_t* s_hi = pre_smem;
  int8_t* s_lo = pre_smem + wcodes + PRE_FEATURES;
  __shared__ float s_max[PRE_THREADS / 32];
  const int f0 = blockIdx.x * PRE_FEATURES, f = f0 + tid;
  const bool valid = f < a.D_in;
  float xm = 0.f;
  if (valid) xm = map_input<MODE>(Act<MODE>::to_f(xrow[f]), a.input_map, mean, rstd);
  {
    Gen gen;
    if (valid) gen.init(xm, f, a);
    for (int k = 0; k < K; ++k) {
      const int q = valid ? __float2int_rn(gen.next() * (float)(1 << PHI_E)) : 0;
      put_fixed(s_hi, s_lo, tid * K + k, q, fast);
    }
  }
  const float sv = (valid && a.has_base) ? silu_value<MODE>(xm) : 0.f;
  float smax = fabsf(sv);
  for (int o = 16; o; o >>= 1) smax = fmaxf(smax, __shfl_xor_sync(0xffffffffu, smax, o));
  if (lane == 0) s_max[warp] = smax;
  __syncthreads();
  smax = 0.f;
  for (int w = 0; w < PRE_THREADS / 32; ++w) smax = fmaxf(smax, s_max[w]);
  const int e = fixed_exponent(smax);
  put_fixed(s_hi + wcodes, s_lo + wcodes, tid, __float2int_rn(sv * exp2f((float)e)), fast);
  __syncthreads();

  // basis units [f0 K / 16, + 4 K) (clamped to the row's units) and the 4 base units
  const int u_lo = f0 * K / 16, nunits = wcodes / 16;
  for (int i = tid; i < nunits; i += PRE_THREADS) {
    const int u = u_lo + i;
    if (u >= p.units_w) break;
    reinterpret_cast<uint4*>(hi)[u] = reinterpret_cast<const uint4*>(s_hi)[i];
    reinterpret_cast<uint4*>(lo)[u] = reinterpret_cast<const uint4*>(s_lo)[i];
  }
  const int ub = f0 / 16 + tid;  // base units of this CTA (tid < 4)
  if (a.has_base && tid < PRE_FEATURES / 16 && ub < p.units_b) {
    reinterpret_cast<uint4*>(hi + p.units_w * 16)[ub] = reinterpret_cast<const uint4*>(s_hi + wcodes)[tid];
    reinterpret_cast<uint4*>(lo + p.units_w * 16)[ub] = reinterpret_cast<const uint4*>(s_lo + wcodes)[tid];
    p.p2b[(size_t)n * p.units_b + ub] = exp2f((float)-e);
  }
  if (!need_sums) return;
  // basis sum of each flush group (p.fu units, the codes the main kernel converts at once),
  // stored at the group's first unit.  Shared memory holds zeros for features past D_in, so
  // every unit sums all 16 positions.  INT8/INT4 keep the real value (times the minimum of the
  // group), in-place ternary the fixed-point integer (subtracted from the integer sum: value
  // c - 1).  A group is fu consecutive threads (fu divides 4; a CTA's range is whole groups).
  const int fu = p.fu;
  auto unit_sum = [&](const int8_t* h8, const int8_t* l8, int i) {
    const uint4 h = reinterpret_cast<const uint4*>(h8)[i];
    const uint4 l = reinterpret_cast<const uint4*>(l8)[i];
    const uint32_t one = 0x01010101u;
    const int sh = dp4a_ss(h.x, one, dp4a_ss(h.y, one, dp4a_ss(h.z, one, dp4a_ss(h.w, one, 0))));
    const int sl = dp4a_ss(l.x, one, dp4a_ss(l.y, one, dp4a_ss(l.z, one, dp4a_ss(l.w, one, 0))));
    return 128 * sh + sl;
  };
  for (int i0 = 0; i0 < nunits; i0 += PRE_THREADS) {
    const int i = i0 + tid, u = u_lo + i;
    int acc = i < nunits ? unit_sum(s_hi, s_lo, i) : 0;
    for (int o = 1; o < fu; o <<= 1) acc += __shfl_down_sync(0xffffffffu, acc, o, fu);
    if (i < nunits && u < p.units_w && u % fu == 0)
      sum[u] = fast ? (float)acc : (float)acc * (1.0f / (float)(1 << PHI_E));
  }
  if (a.has_base) {
    int acc = tid < PRE_FEATURES / 16 ? unit_sum(s_hi + wcodes, s_lo + wcodes, tid) : 0;
    for (int o = 1; o < fu; o <<= 1) acc += __shfl_down_sync(0xffffffffu, acc, o, fu);
    if (tid < PRE_FEATURES / 16 && ub < p.units_b && ub % fu == 0)
      sum[p.units_w + ub] = fast ? (float)acc : (float)acc * exp2f((float)-e);
  }
}

// Dynamic shared memory of the pre-pass: hi and lo bytes of 64 features' K terms and silu.
__host__ __device__ inline int pre_smem_bytes(int K) { return 2 * (PRE_FEATURES * K + PRE_FEATURES); }

// ---------------------------------------------------------------------------------------------
// main kernel
// ---------------------------------------------------------------------------------------------
// 32-bit word i (compile-time) of a 16-byte chunk.
template <int I>
__device__ __forceinline__ uint32_t word_of(const uint4& q) {
  return I == 0 ? q.x : (I == 1 ? q.y : (I == 2 ? q.z : q.w));
}

// Unit J (16 codes) of a 16-byte chunk -> four words of bytes in unit_pos order.
template <int FMT, bool FAST, int J>
__device__ __forceinline__ void decode_unit(const uint4& q, uint32_t (&d)[4]) {
  if (FMT == KAN_W_TERNARY && FAST) {
    // code c of field f in place: byte = c * 4^f (0..192), value c - 1 restored by the unit sums
    const uint32_t x = word_of<J>(q);
    d[0] = x & 0x03030303u;
    d[1] = x & 0x0C0C0C0Cu;
    d[2] = x & 0x30303030u;
    d[3] = x & 0xC0C0C0C0u;
  } else if (FMT == KAN_W_TERNARY) {
    // byte value per code: 0 -> -1, 1 -> 0, 2 -> +1, 3 -> 0 (the reference's dequantiser)
    const uint32_t lut = 0x000100FFu;
    const uint32_t x = word_of<J>(q);
    d[0] = __byte_perm(lut, 0u, x & 0x3333u);
    d[1] = __byte_perm(lut, 0u, (x >> 2) & 0x3333u);
    d[2] = __byte_perm(lut, 0u, (x >> 16) & 0x3333u);
    d[3] = __byte_perm(lut, 0u, (x >> 18) & 0x3333u);
  } else if (FMT == KAN_W_INT4) {
    // byte = q[2i] | q[2i+1] << 4
    const uint32_t w0 = word_of<2 * J>(q), w1 = word_of<2 * J + 1>(q);
    d[0] = w0 & 0x0F0F0F0Fu;
    d[1] = (w0 >> 4) & 0x0F0F0F0Fu;
    d[2] = w1 & 0x0F0F0F0Fu;
    d[3] = (w1 >> 4) & 0x0F0F0F0Fu;
  } else {
    d[0] = __byte_perm(q.x, q.y, 0x6420);
    d[1] = __byte_perm(q.x, q.y, 0x7531);
    d[2] = __byte_perm(q.z, q.w, 0x6420);
    d[3] = __byte_perm(q.z, q.w, 0x7531);
  }
}

// Runtime unit index that is a constant after unrolling -> the compile-time decoder.
template <int FMT, bool FAST, int UPC>
__device__ __forceinline__ void decode_at(const uint4& q, int j, uint32_t (&d)[4]) {
  if (j == 0) decode_unit<FMT, FAST, 0>(q, d);
  else if (j == 1) decode_unit<FMT, FAST, (UPC > 1 ? 1 : 0)>(q, d);
  else if (j == 2) decode_unit<FMT, FAST, (UPC > 2 ? 2 : 0)>(q, d);
  else decode_unit<FMT, FAST, (UPC > 3 ? 3 : 0)>(q, d);
}

template <bool SIGNED>
__device__ __forceinline__ int dp4(uint32_t a, uint32_t b, int c) {
  return SIGNED ? dp4a_ss(a, b, c) : dp4a_us(a, b, c);
}

// NB: batch rows (the launch's B); FU: 16-code units per flush (divides the units per chunk).
template <int MODE, int FMT, bool FAST, int FU, int NB>
__global__ void __launch_bounds__(THREADS) kan_gemv_cc_kernel(
    const __grid_constant__ CUtensorMap tm_cw, const __grid_constant__ CUtensorMap tm_sw,
    const __grid_constant__ CUtensorMap tm_mw, const __grid_constant__ CUtensorMap tm_cb,
    const __grid_constant__ CUtensorMap tm_sb, const __grid_constant__ CUtensorMap tm_mb,
    LayerArgs a, Params p) {
  using T = typename Act<MODE>::T;
  constexpr bool AFFINE = FMT != KAN_W_TERNARY;
  constexpr bool SUMS = AFFINE || FAST;                // unit sums of the basis are used
  constexpr bool SIGNED = FMT == KAN_W_TERNARY && !FAST;  // decoded bytes are signed
  constexpr int UPC = FMT == KAN_W_TERNARY ? 4 : (FMT == KAN_W_INT4 ? 2 : 1);  // units/chunk
  constexpr int ups = ROW_BYTES / 16 * UPC;  // units per stage
  static_assert(UPC % FU == 0, "a flush covers whole units of one chunk");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  const uint32_t s_base = smem_u32(smem);
  const uint32_t bar_full = s_base + p.off_bar;
  const uint32_t bar_empty = bar_full + STAGES * 8;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + p.off_bar + 2 * STAGES * 8);
  float* red = reinterpret_cast<float*>(smem + p.off_red);  // [NWARPS][NB][ROWS]
  const long long plim = a.wait_cycles > 0 ? a.wait_cycles : tc::WAIT_LIMIT_CYCLES;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rb = blockIdx.x, z = blockIdx.y;
  const int st0 = (int)((long long)p.nst * z / p.S), st1 = (int)((long long)p.nst * (z + 1) / p.S);
  const int nmine = st1 - st0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(bar_full + 8 * s, 1);
      mbar_init(bar_empty + 8 * s, NWARPS);
    }
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();

  // Scale-tile origin of stage-in-segment `sis`: 4-aligned, clamped so the box stays in the row.
  auto scale_origin = [&](bool seg, int sis) {
    const int groups = seg ? p.groups_b : p.groups_w, sbox = seg ? p.sbox_b : p.sbox_w;
    return min(((sis * ups) >> p.lg) & ~3, groups - sbox);
  };

  if (warp == WARP_TMA) {
    // ------------------------------------------------------------------ weight TMA
    if (lane == 0) {
      const int units = p.units_w + p.units_b;
      // A stage is the weight tiles (independent of the pre-pass, so the first ring's worth is
      // requested before waiting for it) plus the stage's slice of the basis matrix and unit data
      // (written by the pre-pass: requested once it has completed).
      auto stage_bytes = [&](bool seg) {
        const int sbox = seg ? p.sbox_b : p.sbox_w;
        return (uint32_t)(CODE_TILE + ROWS * sbox * 4 * (AFFINE ? 2 : 1) +
                          NB * (2 * ups * 16 + ((SUMS ? 1 : 0) + (seg ? 1 : 0)) * ups * 4));
      };
      auto issue_basis = [&](int i) {
        const int gst = st0 + i, slot = i % STAGES;
        const bool seg = gst >= p.stages_w;
        const int u0 = (seg ? p.units_w + (gst - p.stages_w) * ups : gst * ups);
        const uint32_t bar = bar_full + 8 * slot;
        const uint32_t dst = s_base + slot * p.tile_bytes;
#pragma unroll
        for (int n = 0; n < NB; ++n) {
          tc::bulk_g2s(dst + p.off_phi + (2 * n) * ups * 16,
                       p.phi_hi + (size_t)n * p.phi_pitch + (size_t)u0 * 16, ups * 16, bar);
          tc::bulk_g2s(dst + p.off_phi + (2 * n + 1) * ups * 16,
                       p.phi_lo + (size_t)n * p.phi_pitch + (size_t)u0 * 16, ups * 16, bar);
          if (SUMS)
            tc::bulk_g2s(dst + p.off_aux + (2 * n) * ups * 4, p.sumphi + (size_t)n * units + u0,
                         ups * 4, bar);
          if (seg)
            tc::bulk_g2s(dst + p.off_aux + (2 * n + 1) * ups * 4,
                         p.p2b + (size_t)n * p.units_b + (u0 - p.units_w), ups * 4, bar);
        }
      };
      const int first = nmine < STAGES ? nmine : STAGES;
      int issued = 0, basis_issued = 0;
      for (int i = 0; i < nmine; ++i) {
        const int slot = i % STAGES;
        if (!mbar_wait(bar_empty + 8 * slot, ((uint32_t)(i / STAGES) & 1u) ^ 1u, plim)) {
          raise_device_error(a.err, DEVERR_TIMEOUT_EMPTY);
          *abort_flag = 1;
          break;
        }
        if (*abort_flag) break;
        const int gst = st0 + i;
        const bool seg = gst >= p.stages_w;
        const int sis = seg ? gst - p.stages_w : gst;
        const int gal = scale_origin(seg, sis);
        const int sbox = seg ? p.sbox_b : p.sbox_w;
        const uint32_t dst = s_base + slot * p.tile_bytes;
        const uint32_t bar = bar_full + 8 * slot;
        const CUtensorMap* cm = seg ? &tm_cb : &tm_cw;
        mbar_arrive_expect_tx(bar, stage_bytes(seg));
#pragma unroll
        for (int bx = 0; bx < BOXES; ++bx)
          tma_load_2d(dst + bx * BOX_TILE, cm, bar, sis * ROW_BYTES + bx * BOX_BYTES, rb * ROWS);
        tma_load_2d(dst + CODE_TILE, seg ? &tm_sb : &tm_sw, bar, gal, rb * ROWS);
        if (AFFINE)
          tma_load_2d(dst + CODE_TILE + ROWS * sbox * 4, seg ? &tm_mb : &tm_mw, bar, gal,
                      rb * ROWS);
        ++issued;
        if (i + 1 == first) {
          // the basis matrix is written by the pre-pass kernel this launch depends on
          asm volatile("griddepcontrol.wait;" ::: "memory");
          for (; basis_issued <= i; ++basis_issued) issue_basis(basis_issued);
        } else if (i >= first) {
          issue_basis(i);
          basis_issued = i + 1;
        }
      }
      // stages whose basis slice was deferred still get it, so that every issued stage completes
      if (basis_issued < issued) {
        asm volatile("griddepcontrol.wait;" ::: "memory");
        for (; basis_issued < issued; ++basis_issued) issue_basis(basis_issued);
      }
      // every load issued lands before the CTA may exit (the consumers waited for all of them
      // unless they aborted)
      for (int i = issued - 1; i >= 0 && i >= issued - STAGES; --i)
        (void)mbar_wait(bar_full + 8 * (i % STAGES), (uint32_t)(i / STAGES) & 1u);
    }
    __syncwarp();
    return;
  }

  // ------------------------------------------------------------------ compute warps
  const int r = lane;
  float acc[NB];
#pragma unroll
  for (int n = 0; n < NB; ++n) acc[n] = 0.f;

  for (int i = 0; i < nmine; ++i) {
    const int slot = i % STAGES;
    if (!mbar_wait_warp(bar_full + 8 * slot, (uint32_t)(i / STAGES) & 1u, plim)) {
      raise_device_error(a.err, DEVERR_TIMEOUT_FULL_B);
      *abort_flag = 1;
      break;
    }
    const int gst = st0 + i;
    const bool seg = gst >= p.stages_w;
    const int sis = seg ? gst - p.stages_w : gst;
    const int gal = scale_origin(seg, sis);
    const int sbox = seg ? p.sbox_b : p.sbox_w;
    const uint8_t* tile = smem + slot * p.tile_bytes;
    const float* stile = reinterpret_cast<const float*>(tile + CODE_TILE) + r * sbox;
    const float* mtile = stile + ROWS * sbox;
    const uint8_t* ptile = tile + p.off_phi;                                  // [NB][hi, lo][ups][16]
    const float* atile = reinterpret_cast<const float*>(tile + p.off_aux);  // [NB][sum, p2b][ups]
    const int ubase = sis * ups;
#pragma unroll
    for (int cc = 0; cc < CHUNKS_PER_WARP; ++cc) {
      const int c = warp * CHUNKS_PER_WARP + cc;
      const uint8_t* box = tile + (c / (BOX_BYTES / 16)) * BOX_TILE;
      const int cb = c % (BOX_BYTES / 16);
      const uint4 q = *reinterpret_cast<const uint4*>(box + r * BOX_BYTES + ((cb ^ (r & 7)) << 4));
#pragma unroll
      for (int j0 = 0; j0 < UPC; j0 += FU) {
        int ch[NB][8];
#pragma unroll
        for (int n = 0; n < NB; ++n)
#pragma unroll
          for (int k = 0; k < 8; ++k) ch[n][k] = 0;
#pragma unroll
        for (int jj = 0; jj < FU; ++jj) {
          uint32_t d[4];
          decode_at<FMT, FAST, UPC>(q, j0 + jj, d);
          const int ul = c * UPC + j0 + jj;  // unit within the stage
#pragma unroll
          for (int n = 0; n < NB; ++n) {
            const uint4 h = *reinterpret_cast<const uint4*>(ptile + ((2 * n) * ups + ul) * 16);
            const uint4 l = *reinterpret_cast<const uint4*>(ptile + ((2 * n + 1) * ups + ul) * 16);
            ch[n][0] = dp4<SIGNED>(d[0], h.x, ch[n][0]);
            ch[n][1] = dp4<SIGNED>(d[1], h.y, ch[n][1]);
            ch[n][2] = dp4<SIGNED>(d[2], h.z, ch[n][2]);
            ch[n][3] = dp4<SIGNED>(d[3], h.w, ch[n][3]);
            ch[n][4] = dp4<SIGNED>(d[0], l.x, ch[n][4]);
            ch[n][5] = dp4<SIGNED>(d[1], l.y, ch[n][5]);
            ch[n][6] = dp4<SIGNED>(d[2], l.z, ch[n][6]);
            ch[n][7] = dp4<SIGNED>(d[3], l.w, ch[n][7]);
          }
        }
        // flush: the FU units lie in one group (and, in the base segment, one exponent chunk)
        const int ul0 = c * UPC + j0;
        const int g = min(((ubase + ul0) >> p.lg) - gal, sbox - 1);  // past the row: padding
        float s = stile[g];
        if (!AFFINE) s = Act<MODE>::round(s);  // act(+-s) = +-act(s): the dequantised weight
        const float mn = AFFINE ? mtile[g] : 0.f;
#pragma unroll
        for (int n = 0; n < NB; ++n) {
          int H, L;
          if (FAST) {  // chain f holds 4^f * sum(c v): H = 64 * sum over the four chains
            H = (ch[n][0] * 4 + ch[n][1]) * 16 + (ch[n][2] * 4 + ch[n][3]);
            L = (ch[n][4] * 4 + ch[n][5]) * 16 + (ch[n][6] * 4 + ch[n][7]);
          } else {
            H = (ch[n][0] + ch[n][1]) + (ch[n][2] + ch[n][3]);
            L = (ch[n][4] + ch[n][5]) + (ch[n][6] + ch[n][7]);
          }
          int tot = H * 128 + L;
          if (FAST) tot >>= 6;  // exact: a multiple of 64
          float v = (float)tot;
          // the basis sum of the FU units (pre-summed by the pre-pass at the first unit)
          const float sp = SUMS ? atile[(2 * n) * ups + ul0] : 0.f;
          if (FAST) v -= sp;  // value c - 1
          const float sc = seg ? s * atile[(2 * n + 1) * ups + ul0] : s * (1.0f / (1 << PHI_E));
          acc[n] = fmaf(v, sc, acc[n]);
          if (AFFINE) acc[n] = fmaf(mn, sp, acc[n]);
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(bar_empty + 8 * slot);
  }

  // ------------------------------------------------------------------ reduction and store
#pragma unroll
  for (int n = 0; n < NB; ++n) red[(warp * NB + n) * ROWS + r] = acc[n];
  asm volatile("bar.sync 1, %0;" ::"r"(NWARPS * 32) : "memory");
  if (warp != 0) return;
  const int row = rb * ROWS + r;
  float v[NB];
#pragma unroll
  for (int n = 0; n < NB; ++n) {
    v[n] = 0.f;
#pragma unroll
    for (int w = 0; w < NWARPS; ++w) v[n] += red[(w * NB + n) * ROWS + r];
  }
  T* Y = (T*)a.Y;
  const float b = (a.has_bias && row < a.D_out) ? Act<MODE>::to_f(((const T*)a.bias)[row]) : 0.f;
  if (p.S == 1) {
#pragma unroll
    for (int n = 0; n < NB; ++n)
      if (row < a.D_out) Y[(size_t)n * a.D_out + row] = Act<MODE>::from_f(v[n] + b);
    return;
  }
#pragma unroll
  for (int n = 0; n < NB; ++n)
    if (row < a.D_out) p.part[((size_t)z * NB + n) * a.D_out + row] = v[n];
  __threadfence();
  __syncwarp();
  // the counters are reset by the pre-pass (long finished: its basis matrix has been consumed)
  asm volatile("griddepcontrol.wait;" ::: "memory");
  int prev = 0;
  if (lane == 0) prev = atomicAdd(p.counters + rb, 1);
  prev = __shfl_sync(0xffffffffu, prev, 0);
  if (prev != p.S - 1) return;
  // the last split of this row block: sum the partials in split order (deterministic)
  __threadfence();
  if (row < a.D_out) {
#pragma unroll
    for (int n = 0; n < NB; ++n) {
      float sum = 0.f;
      for (int zz = 0; zz < p.S; ++zz) sum += __ldcg(p.part + ((size_t)zz * NB + n) * a.D_out + row);
      Y[(size_t)n * a.D_out + row] = Act<MODE>::from_f(sum + b);
    }
  }
  if (lane == 0) p.counters[rb] = 0;
}

using MainFn = void (*)(const CUtensorMap, const CUtensorMap, const CUtensorMap,
                        const CUtensorMap, const CUtensorMap, const CUtensorMap, LayerArgs,
                        Params);

// The main-kernel instance of (format, in-place ternary, units per flush) for a dtype and batch
// size (explicitly instantiated in kan_gemv_cc_inst.cu, one translation unit per pair).
template <int MODE, int NB>
MainFn select_main(int fmt, bool fast, int fu);

}  // namespace cc
}  // namespace kan

namespace kan {
namespace cc {
#define KAN_CC_DECLARE(M, N) template <> MainFn select_main<M, N>(int fmt, bool fast, int fu);
KAN_CC_DECLARE(MODE_F16, 1)
KAN_CC_DECLARE(MODE_F16, 2)
KAN_CC_DECLARE(MODE_F16, 3)
KAN_CC_DECLARE(MODE_F16, 4)
KAN_CC_DECLARE(MODE_BF16, 1)
KAN_CC_DECLARE(MODE_BF16, 2)
KAN_CC_DECLARE(MODE_BF16, 3)
KAN_CC_DECLARE(MODE_BF16, 4)
#undef KAN_CC_DECLARE
}  // namespace cc
}  // namespace kan
