// kan_gemv_cc.cu -- small-batch path on the CUDA cores (B <= 4): ternary, INT8 and INT4 weights.
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
//     cubic B-splines, the three wavelets), so their E is 13: every operand-dtype value of
//     magnitude >= 2^-6 is represented exactly, smaller ones to within 2^-14.  silu(x) is not
//     bounded, so each 64-feature chunk of the base branch gets its own E from its largest value.
//   * the main kernel streams [32 rows x 128 code bytes] tiles of the packed weights (and their
//     per-group scales / minima) with TMA into a 4-stage ring; one lane per output row reads its
//     16-byte chunks (128-byte swizzle: conflict-free), turns 16 codes into four words of signed
//     (ternary: -1/0/+1, code 3 -> 0) or unsigned (INT8/INT4: q) bytes with byte permutes and
//     masks, and accumulates 8 dp4a per batch row (4 against the hi bytes, 4 against the lo bytes)
//     into an exact int32 sum 128 * H + L.  That sum is converted once per 16 codes and scaled by
//     the group's fp32 scale (ternary: rounded to the operand dtype, which makes the product the
//     reference's dequantised weight rounded to the operand dtype, exactly); INT8/INT4 add the
//     group minimum times the (exact) basis sum of the 16 codes.
//   * K is split over S CTAs per 32-row block (S from the occupancy, so the whole grid is resident
//     at once); each split stores its fp32 partials, and the last CTA of a row block to finish
//     (atomic counter) sums them in split order -- deterministic -- adds the bias, rounds, stores.
//
// The basis matrix keeps each 16-code unit in the order the decoder produces bytes in:
// [0 2 4 6 | 1 3 5 7 | 8 10 12 14 | 9 11 13 15] (perm16 below), the same for all three formats.
//
// Every wait is bounded; on expiry the kernel records the device error word, stops consuming,
// and the TMA warp still waits (full limit) for each load it issued before the CTA exits.
#include <cuda.h>

#include <algorithm>
#include <mutex>

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
constexpr int ROW_BYTES = 128;                // code bytes of one row per stage
constexpr int CODE_TILE = ROWS * ROW_BYTES;   // 4 KB
constexpr int NWARPS = 4;                     // compute warps
constexpr int CHUNKS_PER_WARP = ROW_BYTES / 16 / NWARPS;
constexpr int WARP_TMA = NWARPS;
constexpr int THREADS = (NWARPS + 1) * 32;
constexpr int STAGES = 4;
constexpr int MAXB = 4;
constexpr int PHI_E = 13;                     // fixed-point exponent of the basis terms
constexpr int PRE_THREADS = 128;              // pre-pass: 4 warps x 64 features
constexpr int PRE_FEATURES = 256;

struct Params {
  int fmt;                   // KAN_W_TERNARY / KAN_W_INT8 / KAN_W_INT4
  int cpb;                   // codes per byte: 4, 1, 2
  int stages_w, stages_b;    // stages of the basis / base segment
  int nst;                   // stages_w + stages_b
  int S;                     // K splits (grid.y)
  int gs;                    // group size in codes (multiple of 16)
  int sbox;                  // floats per row of a scale (and minimum) tile
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
  float* sumphi;             // [B][units_w + units_b]: exact basis sum of each unit (INT8/INT4)
  float* p2b;                // [B][units_b]: 2^-E of each base unit
  float* part;               // [S][B][D_out] split partials
  int* counters;             // [rowblocks]
};

// Position of code j (0..15) of a unit in the decoder's byte order.
__host__ __device__ __forceinline__ int perm16(int j) {
  return (j & 8) | ((j & 1) << 2) | ((j & 7) >> 1);
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
__device__ __forceinline__ void put_fixed(int8_t* hi, int8_t* lo, int code, int q) {
  const int h = (q + 64) >> 7;
  const int pos = (code & ~15) | perm16(code & 15);
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
  const T* xrow = (const T*)a.X + (size_t)n * a.D_in;
  int8_t* hi = p.phi_hi + (size_t)n * p.phi_pitch;
  int8_t* lo = p.phi_lo + (size_t)n * p.phi_pitch;
  const int units = p.units_w + p.units_b;
  float* sum = p.sumphi + (size_t)n * units;
  const int K = a.K, kdim = a.D_in * K;
  const bool need_sums = p.fmt != KAN_W_TERNARY;

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
    for (int c = kdim + tid; c < p.units_w * 16; c += PRE_THREADS) put_fixed(hi, lo, c, 0);
    for (int c = a.D_in + tid; c < p.units_b * 16; c += PRE_THREADS)
      put_fixed(hi + p.units_w * 16, lo + p.units_w * 16, c, 0);
    for (int u = (kdim + 15) / 16 + tid; u < p.units_w; u += PRE_THREADS) sum[u] = 0.f;
    for (int u = (a.D_in + 15) / 16 + tid; u < p.units_b; u += PRE_THREADS) {
      sum[p.units_w + u] = 0.f;
      p.p2b[(size_t)n * p.units_b + u] = 0.f;
    }
  }

  // this warp's 64 features: basis terms (E = 13) and silu (E of the chunk)
  const int f0 = blockIdx.x * PRE_FEATURES + warp * 64;
  float sv[2];
  float smax = 0.f;
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int f = f0 + h * 32 + lane;
    sv[h] = 0.f;
    if (f < a.D_in) {
      const float xm = map_input<MODE>(Act<MODE>::to_f(xrow[f]), a.input_map, mean, rstd);
      Gen gen;
      gen.init(xm, f, a);
      for (int k = 0; k < K; ++k)
        put_fixed(hi, lo, f * K + k, __float2int_rn(gen.next() * (float)(1 << PHI_E)));
      if (a.has_base) sv[h] = silu_value<MODE>(xm);
      smax = fmaxf(smax, fabsf(sv[h]));
    }
  }
  if (a.has_base && f0 < a.D_in) {
    for (int o = 16; o; o >>= 1) smax = fmaxf(smax, __shfl_xor_sync(0xffffffffu, smax, o));
    const int e = fixed_exponent(smax);
    const float sc = exp2f((float)e);
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int f = f0 + h * 32 + lane;
      if (f < a.D_in)
        put_fixed(hi + p.units_w * 16, lo + p.units_w * 16, f, __float2int_rn(sv[h] * sc));
    }
    if (lane < 4 && f0 / 16 + lane < p.units_b)
      p.p2b[(size_t)n * p.units_b + f0 / 16 + lane] = exp2f((float)-e);
  }
  if (!need_sums || f0 >= a.D_in) return;
  // exact basis sum of each unit this warp wrote (its own global writes, ordered by the warp
  // barrier); codes past the real ones are skipped, whatever the padding holds
  __syncwarp();
  const int ulo = f0 * K / 16, uhi = min((f0 + 64) * K, kdim + 15) / 16;
  for (int u = ulo + lane; u < uhi && u < p.units_w; u += 32) {
    int acc = 0;
    for (int j = 0; j < 16; ++j) {
      const int c = u * 16 + j;
      if (c >= kdim) break;
      const int pos = u * 16 + perm16(j);
      acc += 128 * (int)hi[pos] + (int)lo[pos];
    }
    sum[u] = (float)acc * (1.0f / (float)(1 << PHI_E));
  }
  if (a.has_base && lane < 4) {
    const int u = f0 / 16 + lane;
    if (u < p.units_b && u * 16 < a.D_in) {
      int acc = 0;
      for (int j = 0; j < 16 && u * 16 + j < a.D_in; ++j) {
        const int pos = p.units_w * 16 + u * 16 + perm16(j);
        acc += 128 * (int)hi[pos] + (int)lo[pos];
      }
      sum[p.units_w + u] = (float)acc * p.p2b[(size_t)n * p.units_b + u];
    }
  }
}

// ---------------------------------------------------------------------------------------------
// main kernel
// ---------------------------------------------------------------------------------------------
// 32-bit word i (compile-time) of a 16-byte chunk.
template <int I>
__device__ __forceinline__ uint32_t word_of(const uint4& q) {
  return I == 0 ? q.x : (I == 1 ? q.y : (I == 2 ? q.z : q.w));
}

// Unit J (16 codes) of a 16-byte chunk -> four words of bytes in perm16 order.
template <int FMT, int J>
__device__ __forceinline__ void decode_unit(const uint4& q, uint32_t (&d)[4]) {
  if (FMT == KAN_W_TERNARY) {
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

template <int MODE, int FMT>
__global__ void __launch_bounds__(THREADS) kan_gemv_cc_kernel(
    const __grid_constant__ CUtensorMap tm_cw, const __grid_constant__ CUtensorMap tm_sw,
    const __grid_constant__ CUtensorMap tm_mw, const __grid_constant__ CUtensorMap tm_cb,
    const __grid_constant__ CUtensorMap tm_sb, const __grid_constant__ CUtensorMap tm_mb,
    LayerArgs a, Params p) {
  using T = typename Act<MODE>::T;
  constexpr bool AFFINE = FMT != KAN_W_TERNARY;
  constexpr int UPC = FMT == KAN_W_TERNARY ? 4 : (FMT == KAN_W_INT4 ? 2 : 1);  // units/chunk
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  const uint32_t s_base = smem_u32(smem);
  const uint32_t bar_full = s_base + p.off_bar;
  const uint32_t bar_empty = bar_full + STAGES * 8;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + p.off_bar + 2 * STAGES * 8);
  float* red = reinterpret_cast<float*>(smem + p.off_red);  // [NWARPS][MAXB][ROWS]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rb = blockIdx.x, z = blockIdx.y;
  const int st0 = (int)((long long)p.nst * z / p.S), st1 = (int)((long long)p.nst * (z + 1) / p.S);
  const int nmine = st1 - st0;
  const int B = a.B;
  const int scale_floats = ROWS * p.sbox;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(bar_full + 8 * s, 1);
      mbar_init(bar_empty + 8 * s, NWARPS);
    }
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();

  if (warp == WARP_TMA) {
    // ------------------------------------------------------------------ weight TMA
    if (lane == 0) {
      const int ups = p.ups, units = p.units_w + p.units_b;
      // A stage is the weight tiles (independent of the pre-pass, so the first ring's worth is
      // requested before waiting for it) plus the stage's slice of the basis matrix and unit data
      // (written by the pre-pass: requested once it has completed).
      auto stage_bytes = [&](bool seg) {
        return (uint32_t)(CODE_TILE + scale_floats * 4 * (AFFINE ? 2 : 1) +
                          B * (2 * ups * 16 + ((AFFINE ? 1 : 0) + (seg ? 1 : 0)) * ups * 4));
      };
      auto issue_basis = [&](int i) {
        const int gst = st0 + i, slot = i % STAGES;
        const bool seg = gst >= p.stages_w;
        const int u0 = (seg ? p.units_w + (gst - p.stages_w) * ups : gst * ups);
        const uint32_t bar = bar_full + 8 * slot;
        const uint32_t dst = s_base + slot * p.tile_bytes;
        for (int n = 0; n < B; ++n) {
          tc::bulk_g2s(dst + p.off_phi + (2 * n) * ups * 16,
                       p.phi_hi + (size_t)n * p.phi_pitch + (size_t)u0 * 16, ups * 16, bar);
          tc::bulk_g2s(dst + p.off_phi + (2 * n + 1) * ups * 16,
                       p.phi_lo + (size_t)n * p.phi_pitch + (size_t)u0 * 16, ups * 16, bar);
          if (AFFINE)
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
        if (!mbar_wait(bar_empty + 8 * slot, ((uint32_t)(i / STAGES) & 1u) ^ 1u)) {
          raise_device_error(a.err, DEVERR_TIMEOUT_EMPTY);
          *abort_flag = 1;
          break;
        }
        if (*abort_flag) break;
        const int gst = st0 + i;
        const bool seg = gst >= p.stages_w;
        const int sis = seg ? gst - p.stages_w : gst;
        const int gal = ((sis * ROW_BYTES * p.cpb) / p.gs) & ~3;
        const uint32_t dst = s_base + slot * p.tile_bytes;
        mbar_arrive_expect_tx(bar_full + 8 * slot, stage_bytes(seg));
        tma_load_2d(dst, seg ? &tm_cb : &tm_cw, bar_full + 8 * slot, sis * ROW_BYTES, rb * ROWS);
        tma_load_2d(dst + CODE_TILE, seg ? &tm_sb : &tm_sw, bar_full + 8 * slot, gal, rb * ROWS);
        if (AFFINE)
          tma_load_2d(dst + CODE_TILE + scale_floats * 4, seg ? &tm_mb : &tm_mw,
                      bar_full + 8 * slot, gal, rb * ROWS);
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
  const int ups = p.ups;
  float accw[MAXB], accr[MAXB];
#pragma unroll
  for (int n = 0; n < MAXB; ++n) accw[n] = accr[n] = 0.f;

  for (int i = 0; i < nmine; ++i) {
    const int slot = i % STAGES;
    if (!mbar_wait_warp(bar_full + 8 * slot, (uint32_t)(i / STAGES) & 1u)) {
      raise_device_error(a.err, DEVERR_TIMEOUT_FULL_B);
      *abort_flag = 1;
      break;
    }
    const int gst = st0 + i;
    const bool seg = gst >= p.stages_w;
    const int sis = seg ? gst - p.stages_w : gst;
    const int gal = ((sis * ROW_BYTES * p.cpb) / p.gs) & ~3;
    const uint8_t* tile = smem + slot * p.tile_bytes;
    const float* stile = reinterpret_cast<const float*>(tile + CODE_TILE) + r * p.sbox;
    const float* mtile = stile + scale_floats;
    const uint8_t* ptile = tile + p.off_phi;                                  // [B][hi, lo][ups][16]
    const float* atile = reinterpret_cast<const float*>(tile + p.off_aux);  // [B][sum, p2b][ups]
#pragma unroll
    for (int cc = 0; cc < CHUNKS_PER_WARP; ++cc) {
      const int c = warp * CHUNKS_PER_WARP + cc;
      const uint4 q = *reinterpret_cast<const uint4*>(tile + r * ROW_BYTES + ((c ^ (r & 7)) << 4));
#pragma unroll
      for (int j = 0; j < UPC; ++j) {
        uint32_t d[4];
        if (j == 0) decode_unit<FMT, 0>(q, d);
        else if (j == 1) decode_unit<FMT, (UPC > 1 ? 1 : 0)>(q, d);
        else if (j == 2) decode_unit<FMT, (UPC > 2 ? 2 : 0)>(q, d);
        else decode_unit<FMT, (UPC > 3 ? 3 : 0)>(q, d);
        const int code0 = (sis * ROW_BYTES + c * 16) * p.cpb + j * 16;  // within the segment
        const int ul = c * UPC + j;                                      // unit within the stage
        const int g = code0 / p.gs - gal;
        float s = stile[g];
        if (!AFFINE) s = Act<MODE>::round(s);  // act(+-s) = +-act(s): the dequantised weight
        const float mn = AFFINE ? mtile[g] : 0.f;
#pragma unroll
        for (int n = 0; n < MAXB; ++n) {
          if (n >= B) break;
          const uint4 h = *reinterpret_cast<const uint4*>(ptile + ((2 * n) * ups + ul) * 16);
          const uint4 l = *reinterpret_cast<const uint4*>(ptile + ((2 * n + 1) * ups + ul) * 16);
          int t;
          if (AFFINE) {
            t = dp4a_us(d[0], h.x, 0);
            t = dp4a_us(d[1], h.y, t);
            t = dp4a_us(d[2], h.z, t);
            t = dp4a_us(d[3], h.w, t);
            t <<= 7;
            t = dp4a_us(d[0], l.x, t);
            t = dp4a_us(d[1], l.y, t);
            t = dp4a_us(d[2], l.z, t);
            t = dp4a_us(d[3], l.w, t);
          } else {
            t = dp4a_ss(d[0], h.x, 0);
            t = dp4a_ss(d[1], h.y, t);
            t = dp4a_ss(d[2], h.z, t);
            t = dp4a_ss(d[3], h.w, t);
            t <<= 7;
            t = dp4a_ss(d[0], l.x, t);
            t = dp4a_ss(d[1], l.y, t);
            t = dp4a_ss(d[2], l.z, t);
            t = dp4a_ss(d[3], l.w, t);
          }
          if (!seg) {
            accw[n] = fmaf((float)t, s, accw[n]);
          } else {
            accr[n] = fmaf((float)t, s * atile[(2 * n + 1) * ups + ul], accr[n]);
          }
          if (AFFINE) accr[n] = fmaf(mn, atile[(2 * n) * ups + ul], accr[n]);
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(bar_empty + 8 * slot);
  }

  // ------------------------------------------------------------------ reduction and store
#pragma unroll
  for (int n = 0; n < MAXB; ++n)
    red[(warp * MAXB + n) * ROWS + r] = accw[n] * (1.0f / (float)(1 << PHI_E)) + accr[n];
  asm volatile("bar.sync 1, %0;" ::"r"(NWARPS * 32) : "memory");
  if (warp != 0) return;
  const int row = rb * ROWS + r;
  float v[MAXB];
#pragma unroll
  for (int n = 0; n < MAXB; ++n) {
    v[n] = 0.f;
    for (int w = 0; w < NWARPS; ++w) v[n] += red[(w * MAXB + n) * ROWS + r];
  }
  T* Y = (T*)a.Y;
  const float b = (a.has_bias && row < a.D_out) ? Act<MODE>::to_f(((const T*)a.bias)[row]) : 0.f;
  if (p.S == 1) {
#pragma unroll
    for (int n = 0; n < MAXB; ++n)
      if (n < B && row < a.D_out) Y[(size_t)n * a.D_out + row] = Act<MODE>::from_f(v[n] + b);
    return;
  }
#pragma unroll
  for (int n = 0; n < MAXB; ++n)
    if (n < B && row < a.D_out) p.part[((size_t)z * B + n) * a.D_out + row] = v[n];
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
    for (int n = 0; n < B; ++n) {
      float sum = 0.f;
      for (int zz = 0; zz < p.S; ++zz) sum += __ldcg(p.part + ((size_t)zz * B + n) * a.D_out + row);
      Y[(size_t)n * a.D_out + row] = Act<MODE>::from_f(sum + b);
    }
  }
  if (lane == 0) p.counters[rb] = 0;
}

// ---------------------------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------------------------
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// [rows][cols] matrix of `esz`-byte elements, box = box_cols x ROWS, zero fill outside.
static bool make_map(CUtensorMap* m, const void* base, int rows, long long cols, int box_cols,
                     bool codes) {
  EncodeTiledFn enc = (EncodeTiledFn)tensor_map_encoder();
  const int esz = codes ? 1 : 4;
  if (!enc || ((uintptr_t)base & 15) || ((cols * esz) % 16)) return false;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(cols * esz)};
  cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)ROWS};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(m, codes ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2,
                   const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE,
                   codes ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// Code bytes and groups of one row of a packed weight with `cols` logical columns.
struct RowShape {
  long long bytes;
  int groups;
};
static RowShape row_shape(const kan_weight& w, int cols) {
  RowShape s = {0, 0};
  if (w.format == KAN_W_TERNARY || w.format == KAN_W_INT2) {
    s.bytes = (long long)((cols + 15) / 16) * 4;
    s.groups = (cols + w.group_size - 1) / w.group_size;
  } else if (w.format == KAN_W_INT8 || w.format == KAN_W_INT4) {
    s.bytes = w.format == KAN_W_INT8 ? w.padded_cols : w.padded_cols / 2;
    s.groups = w.group_size > 0 ? w.padded_cols / w.group_size : 0;
  }
  return s;
}

static int sm_count() {
  static int n[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (!n[dev]) {
    int v = 0;
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v <= 0)
      v = 148;
    n[dev] = v;
  }
  return n[dev];
}

using MainFn = void (*)(const CUtensorMap, const CUtensorMap, const CUtensorMap,
                        const CUtensorMap, const CUtensorMap, const CUtensorMap, LayerArgs,
                        Params);
static MainFn main_kernel(int mode, int fmt) {
  if (mode == MODE_F16) {
    if (fmt == KAN_W_TERNARY) return kan_gemv_cc_kernel<MODE_F16, KAN_W_TERNARY>;
    if (fmt == KAN_W_INT8) return kan_gemv_cc_kernel<MODE_F16, KAN_W_INT8>;
    return kan_gemv_cc_kernel<MODE_F16, KAN_W_INT4>;
  }
  if (fmt == KAN_W_TERNARY) return kan_gemv_cc_kernel<MODE_BF16, KAN_W_TERNARY>;
  if (fmt == KAN_W_INT8) return kan_gemv_cc_kernel<MODE_BF16, KAN_W_INT8>;
  return kan_gemv_cc_kernel<MODE_BF16, KAN_W_INT4>;
}

static std::atomic<unsigned long long> g_configured[6];  // per device: shared-memory limit set
// The dynamic shared-memory limit every instance is given (once per device): the CTA maximum,
// so that a launch of any batch size (the stage size grows with B) stays within it.
constexpr int SMEM_MAX = 227 * 1024;

// Resident CTAs per SM of a main-kernel instance (cached per device and instance); raises the
// instance's dynamic shared-memory limit on this device first.
static int occupancy(MainFn k, int ki, int smem) {
  if (ensure_smem_attr(k, SMEM_MAX, g_configured[ki]) != cudaSuccess) {
    (void)cudaGetLastError();
    return 1;
  }
  static int cache[64][6] = {};
  static std::mutex mu;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) dev = 0;
  std::lock_guard<std::mutex> lk(mu);
  if (!cache[dev][ki]) {
    int v = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&v, k, THREADS, smem) != cudaSuccess ||
        v <= 0) {
      (void)cudaGetLastError();
      v = 1;
    }
    cache[dev][ki] = v;
  }
  return cache[dev][ki];
}

static size_t align256(size_t v) { return (v + 255) & ~size_t(255); }

// The launch plan; `scratch` (may be null) fills the scratch pointers.  Returns the scratch
// bytes needed.
static size_t plan(const LayerArgs& a, int act_dtype, Params& p, void* scratch) {
  p = Params{};
  p.fmt = a.w.format;
  p.cpb = p.fmt == KAN_W_TERNARY ? 4 : (p.fmt == KAN_W_INT4 ? 2 : 1);
  p.gs = a.w.group_size;
  const RowShape rw = row_shape(a.w, a.D_in * a.K);
  const RowShape rbs = a.has_base ? row_shape(a.wb, a.D_in) : RowShape{0, 0};
  p.stages_w = (int)((rw.bytes + ROW_BYTES - 1) / ROW_BYTES);
  p.stages_b = (int)((rbs.bytes + ROW_BYTES - 1) / ROW_BYTES);
  p.nst = p.stages_w + p.stages_b;
  const int ups = ROW_BYTES * p.cpb / 16;  // units per stage
  p.units_w = p.stages_w * ups;
  p.units_b = p.stages_b * ups;
  p.phi_pitch = (p.units_w + p.units_b) * 16;
  const int gps = std::max(1, ROW_BYTES * p.cpb / std::max(1, p.gs));  // groups per stage
  p.sbox = (gps + 3) / 4 * 4 + 4;
  const bool affine = p.fmt != KAN_W_TERNARY;
  p.ups = ups;
  const int Bs = std::max(1, a.B);
  p.off_phi = CODE_TILE + ROWS * p.sbox * 4 * (affine ? 2 : 1);            // multiple of 128
  p.off_aux = p.off_phi + Bs * 2 * ups * 16;
  p.tile_bytes = p.off_aux + Bs * 2 * ups * 4;
  p.tile_bytes = (p.tile_bytes + 1023) / 1024 * 1024;  // 128-byte swizzle: 1 KB aligned stages
  p.off_red = STAGES * p.tile_bytes;
  p.off_bar = p.off_red + NWARPS * MAXB * ROWS * 4;
  p.smem = p.off_bar + 2 * STAGES * 8 + 16 + 1024;
  p.rowblocks = (a.D_out + ROWS - 1) / ROWS;
  const int mode = act_dtype == KAN_F16 ? MODE_F16 : MODE_BF16;
  const int ki = (mode == MODE_F16 ? 0 : 3) + (p.fmt == KAN_W_TERNARY ? 0 : (p.fmt == KAN_W_INT8 ? 1 : 2));
  const int occ = occupancy(main_kernel(mode, p.fmt), ki, p.smem);
  // as many K splits as keep the whole grid resident at once (one wave), at least 2 stages each
  int S = std::max(1, sm_count() * occ / std::max(1, p.rowblocks));
  S = std::min(S, std::max(1, p.nst / 2));
  p.S = S;
  const int Bn = std::max(1, a.B);
  size_t off = 0;
  const size_t o_hi = off;
  off = align256(off + (size_t)Bn * p.phi_pitch);
  const size_t o_lo = off;
  off = align256(off + (size_t)Bn * p.phi_pitch);
  const size_t o_sum = off;
  off = align256(off + (size_t)Bn * (p.units_w + p.units_b) * 4);
  const size_t o_p2b = off;
  off = align256(off + (size_t)Bn * std::max(1, p.units_b) * 4);
  const size_t o_part = off;
  off = align256(off + (size_t)S * Bn * a.D_out * 4);
  const size_t o_cnt = off;
  off = align256(off + (size_t)p.rowblocks * 4);
  if (scratch) {
    uint8_t* base = (uint8_t*)scratch;
    p.phi_hi = (int8_t*)(base + o_hi);
    p.phi_lo = (int8_t*)(base + o_lo);
    p.sumphi = (float*)(base + o_sum);
    p.p2b = (float*)(base + o_p2b);
    p.part = (float*)(base + o_part);
    p.counters = (int*)(base + o_cnt);
  }
  return off;
}

}  // namespace cc

bool gemv_cc_supported(const LayerArgs& a, int act_dtype) {
  using namespace cc;
  if (act_dtype != KAN_F16 && act_dtype != KAN_BF16) return false;
  if (a.B < 1 || a.B > MAXB || a.D_in < 1 || a.D_out < 1 || a.K < 1) return false;
  const int fmt = a.w.format;
  if (fmt != KAN_W_TERNARY && fmt != KAN_W_INT8 && fmt != KAN_W_INT4) return false;
  const int gs = a.w.group_size;
  if (gs < 16 || gs % 16 || gs > 4096) return false;
  if (a.has_base && (a.wb.format != fmt || a.wb.group_size != gs)) return false;
  // TMA: rows of 16-byte multiples, at least one full stage and one scale tile wide
  const int cpb = fmt == KAN_W_TERNARY ? 4 : (fmt == KAN_W_INT4 ? 2 : 1);
  const int sbox = (std::max(1, ROW_BYTES * cpb / gs) + 3) / 4 * 4 + 4;
  auto fits = [&](const RowShape& s) {
    return s.bytes % 16 == 0 && s.bytes >= ROW_BYTES && s.groups % 4 == 0 && s.groups >= sbox;
  };
  if (!fits(row_shape(a.w, a.D_in * a.K))) return false;
  if (a.has_base && !fits(row_shape(a.wb, a.D_in))) return false;
  if (fmt != KAN_W_TERNARY) {
    // the padded row holds whole groups: codes of a row start at row * padded_cols
    if (a.w.padded_cols % gs || a.w.padded_cols < a.D_in * a.K) return false;
    if (a.has_base && (a.wb.padded_cols % gs || a.wb.padded_cols < a.D_in)) return false;
  }
  auto al = [](const void* ptr) { return ((uintptr_t)ptr & 15) == 0; };
  if (!al(a.w.data) || !al(a.w.scales) || (fmt != KAN_W_TERNARY && !al(a.w.biases))) return false;
  if (a.has_base &&
      (!al(a.wb.data) || !al(a.wb.scales) || (fmt != KAN_W_TERNARY && !al(a.wb.biases))))
    return false;
  return tensor_map_encoder() != nullptr;
}

size_t gemv_cc_scratch_bytes(const LayerArgs& a) {
  cc::Params p;
  return cc::plan(a, a.act_dtype, p, nullptr);
}

int gemv_cc_splits(const LayerArgs& a) {
  cc::Params p;
  cc::plan(a, a.act_dtype, p, nullptr);
  return p.S;
}

template <int MODE>
static void launch_phi(const LayerArgs& a, const cc::Params& p, cudaStream_t s) {
  const dim3 grid((unsigned)((a.D_in + cc::PRE_FEATURES - 1) / cc::PRE_FEATURES), (unsigned)a.B);
  switch (a.basis) {
    case KAN_CHEBY: cc::cc_phi_kernel<MODE, KAN_CHEBY><<<grid, cc::PRE_THREADS, 0, s>>>(a, p); break;
    case KAN_RBF: cc::cc_phi_kernel<MODE, KAN_RBF><<<grid, cc::PRE_THREADS, 0, s>>>(a, p); break;
    case KAN_BSPLINE:
      cc::cc_phi_kernel<MODE, KAN_BSPLINE><<<grid, cc::PRE_THREADS, 0, s>>>(a, p);
      break;
    default: cc::cc_phi_kernel<MODE, KAN_WAVELET><<<grid, cc::PRE_THREADS, 0, s>>>(a, p); break;
  }
}

cudaError_t launch_gemv_cc(const LayerArgs& a, int act_dtype, void* scratch, cudaStream_t s) {
  using namespace cc;
  Params p;
  plan(a, act_dtype, p, scratch);
  const int mode = act_dtype == KAN_F16 ? MODE_F16 : MODE_BF16;
  const int fmt = p.fmt;
  CUtensorMap cw, sw, mw, cb, sb, mb;
  const RowShape rw = row_shape(a.w, a.D_in * a.K);
  if (!make_map(&cw, a.w.data, a.D_out, rw.bytes, ROW_BYTES, true) ||
      !make_map(&sw, a.w.scales, a.D_out, rw.groups, p.sbox, false))
    return cudaErrorInvalidValue;
  mw = sw;
  if (fmt != KAN_W_TERNARY && !make_map(&mw, a.w.biases, a.D_out, rw.groups, p.sbox, false))
    return cudaErrorInvalidValue;
  cb = cw;
  sb = sw;
  mb = mw;
  if (a.has_base) {
    const RowShape rbs = row_shape(a.wb, a.D_in);
    if (!make_map(&cb, a.wb.data, a.D_out, rbs.bytes, ROW_BYTES, true) ||
        !make_map(&sb, a.wb.scales, a.D_out, rbs.groups, p.sbox, false))
      return cudaErrorInvalidValue;
    if (fmt != KAN_W_TERNARY && !make_map(&mb, a.wb.biases, a.D_out, rbs.groups, p.sbox, false))
      return cudaErrorInvalidValue;
  }
  if (mode == MODE_F16) launch_phi<MODE_F16>(a, p, s);
  else launch_phi<MODE_BF16>(a, p, s);
  note_launch();
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;

  const MainFn kern = main_kernel(mode, fmt);
  const int ki = (mode == MODE_F16 ? 0 : 3) + (fmt == KAN_W_TERNARY ? 0 : (fmt == KAN_W_INT8 ? 1 : 2));
  if ((e = ensure_smem_attr(kern, SMEM_MAX, g_configured[ki])) != cudaSuccess) return e;
  if (p.smem > SMEM_MAX) return cudaErrorInvalidValue;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)p.rowblocks, (unsigned)p.S, 1);
  cfg.blockDim = dim3(THREADS, 1, 1);
  cfg.dynamicSmemBytes = (size_t)p.smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  // programmatic dependent launch: the weight stream starts while the pre-pass runs
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  note_launch();
  return cudaLaunchKernelEx(&cfg, kern, cw, sw, mw, cb, sb, mb, a, p);
}

}  // namespace kan
