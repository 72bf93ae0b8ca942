// kan_gemv_kl.cuh -- small-batch path on the CUDA cores for ternary weights, lanes along K
// (B <= 4, f16/bf16 layers, group sizes 32..256).
//
// The layer at B <= 4 is a stream of 2-bit codes: every weight is read once and meets B basis
// values, so the work per weight must stay at about one instruction for the stream to run at the
// HBM rate.  This kernel puts the 32 lanes of a warp side by side along K: lane l owns 32
// consecutive codes (8 bytes) of every row of a 1024-code window, and its 32 basis values per
// batch row sit in registers for all the rows the warp visits in that window.  Per row and lane
// the work is one 8-byte shared load of codes, the decode into four words of bytes per 16 codes,
// 16 dp4a per batch row against the hi and lo bytes of the fixed-point basis, and one fp32 FMA
// with the group's scale.  The basis is never broadcast from shared memory per row, and no
// pre-pass runs: the CTA evaluates each window's basis itself, double-buffered one window ahead.
//
//   * work: a CTA is 8 compute warps x 16 rows = 128 output rows and one TMA warp.  The
//     (row block, window) tasks of the layer, row-block major, are cut into one contiguous range
//     per CTA (grid = SMs, ranges within one window of each other); a CTA accumulates the windows
//     of one row block in registers and, when its range leaves the row block, hands the row
//     block's partial sums on: the last of the row block's contributors (a per-row-block counter
//     tagged with the call's epoch) adds the partials in contributor order -- deterministic --
//     adds the bias, rounds and stores.
//   * stages: [128 rows x 256 code bytes] of the packed weights and the [128 rows x 1024/gs]
//     scales of each task stream by TMA into a ring of 2-4 stages.  There is no copy warp (eight
//     warps keep the per-scheduler register budget at 255): the first stages are requested at the
//     start, and the last warp to finish with a stage (a shared counter) requests the task that
//     refills it.
//   * basis: the same fixed point as the small-batch pre-pass (kan_gemv_cc.cuh): basis terms
//     (|phi| <= 1) as rint(phi * 2^13) split into signed hi / lo bytes, v = 128 hi + lo; silu of
//     the base branch with one exponent per 64-feature chunk.  Byte order inside 16 codes follows
//     the decoder (cc::unit_pos), and the window's 64 units are stored [unit & 1][lane] so that a
//     lane's 16-byte loads are conflict-free.
//   * ternary decode: without code 3 (KAN_WFLAG_TERNARY_NO3) field f of a word is shifted down and
//     masked, giving code c in 0..2 per byte; the lane's chain starts from minus its basis sum, so
//     the integer total is sum((c - 1) v).  With code 3 a byte-permute table maps 0..3 to -1, 0,
//     +1, 0 (the reference's dequantiser) and signed dp4a take it.
//   * scale: per row and lane, the group's fp32 scale rounded to the activation dtype (so that the
//     product is the reference's dequantised weight rounded to the operand dtype, exactly), times
//     the exact integer total converted once.
//
// Every wait is bounded; on expiry the kernel records the device error word and stops consuming
// (a stage a warp did not wait for is never counted as consumed, so it is not refilled while a
// load may still be landing); before exit one thread waits (full limit) for the last load issued
// into every stage.  All warps pass the same barriers whatever happens, so an expired wait never
// strands a barrier.
#pragma once

#include <cuda.h>

#include "kan_gemv_cc.cuh"

namespace kan {
namespace kl {

using tc::mbar_arrive;
using tc::mbar_arrive_expect_tx;
using tc::mbar_init;
using tc::mbar_wait;
using tc::mbar_wait_warp;
using tc::named_bar;
using tc::smem_u32;
using tc::tma_load_2d;

constexpr int WARPS = 8;                    // compute warps
constexpr int RW = 16;                      // rows per compute warp
constexpr int ROWS = WARPS * RW;            // rows per CTA
constexpr int LANE_BYTES = 8;               // code bytes per lane, row and window (32 codes)
constexpr int WIN_BYTES = 32 * LANE_BYTES;  // code bytes of a row in one window
constexpr int WIN_CODES = WIN_BYTES * 4;    // 1024 codes
constexpr int CTHREADS = WARPS * 32;
constexpr int THREADS = CTHREADS;           // no copy warp: the last consumer of a stage refills it
constexpr int MAXB = 4;
constexpr int PHI_E = cc::PHI_E;
constexpr int PHI_BUF = 2 * WIN_CODES;      // hi and lo bytes of one batch row's window
constexpr int CODE_TILE = ROWS * WIN_BYTES; // 32 KB
constexpr int BAR_ID = 1;                   // named barrier of the compute warps
constexpr int MAX_STAGES = 4;
// misc area: [NB][mean, rstd] stats, [WARPS][NB] reduction scratch, abort flag, decision, per
// stage the consumption count and the number of loads issued
constexpr int MISC_BYTES = (2 * MAXB + WARPS * MAXB) * 4 + 16 + 2 * MAX_STAGES * 4;

struct Params {
  int W, Ww;                 // windows per row: all, basis segment (the rest: base segment)
  int lgs;                   // log2(group size)
  int sfl;                   // scale floats per row and window (WIN_CODES / gs)
  int stages;
  int stage_bytes;           // codes + scales of one stage (1 KB multiple)
  int off_x, off_phi, off_fac, off_misc, off_bar, smem;
  int rowblocks;
  long long tasks;           // rowblocks * W
  int G;                     // CTAs
  int maxc;                  // most contributors of one row block
  unsigned epoch;            // nonzero, new for every launch
  float* part;               // [rowblocks][maxc][NB][ROWS]
  unsigned long long* counters;  // [rowblocks]: epoch << 32 | contributions so far
};

// CTA whose task range holds task x (ranges: [T i / G, T (i + 1) / G)).
__host__ __device__ __forceinline__ int owner(long long x, long long T, int G) {
  return (int)(((x + 1) * (long long)G - 1) / T);
}

// Epoch of a launch of a kernel with per-row-block counters (this one and the 8-bit tensor-core
// small-batch kernel): one process-wide sequence, never 0, so that a counter left behind by any
// earlier launch (an aborted one, or another layer sharing the scratch) never carries the
// current epoch (kan_gemv_cc.cu).
unsigned next_epoch();

// Position of code c (0..1023) of a window in the basis buffer: unit u = c / 16 of lane u / 2,
// slot [u & 1][lane], byte cc::unit_pos inside the unit.
__device__ __forceinline__ int phi_pos(int c, bool fast) {
  return ((((c >> 4) & 1) * 32 + (c >> 5)) << 4) | cc::unit_pos(c & 15, fast);
}

__device__ __forceinline__ void put_q(int8_t* buf, int c, int q, bool fast) {
  const int h = (q + 64) >> 7;
  const int pos = phi_pos(c, fast);
  buf[pos] = (int8_t)h;
  buf[WIN_CODES + pos] = (int8_t)(q - (h << 7));
}

template <class Gen>
__device__ __forceinline__ void put_terms(int8_t* buf, float xm, int f, int c_lo,
                                          const LayerArgs& a, bool fast) {
  Gen gen;
  gen.init(xm, f, a);
  const int c0 = f * a.K - c_lo;
  for (int k = 0; k < a.K; ++k) {
    const float v = gen.next();
    const int c = c0 + k;
    if ((unsigned)c < (unsigned)WIN_CODES)
      put_q(buf, c, __float2int_rn(v * (float)(1 << PHI_E)), fast);
  }
}

// The basis of window w for the NB batch rows into `buf` ([NB][hi, lo][1024]) and, for a window
// of the base segment, the factor 2^(13 - E) of each 64-feature chunk into `fac` ([NB][16]).
// Called by all compute threads; `tid` (0..255) spreads the basis segment's features over the
// warps.
template <int MODE, bool FAST, int NB>
__device__ __noinline__ void produce_window(const LayerArgs& a, const Params& p, int w,
                                            int8_t* buf, float* fac,
                                            const typename Act<MODE>::T* xs, const float* stats,
                                            int tid) {
  using A = Act<MODE>;
  if (w < p.Ww) {
    const int c_lo = w * WIN_CODES;
    const int kdim = a.D_in * a.K;
    const int f_lo = c_lo / a.K;
    const int f_hi = min(a.D_in - 1, (c_lo + WIN_CODES - 1) / a.K);
    for (int f = f_lo + tid; f <= f_hi; f += CTHREADS) {
#pragma unroll
      for (int n = 0; n < NB; ++n) {
        const float xm = map_input<MODE>(A::to_f(xs[n * a.D_in + f]), a.input_map,
                                         stats[2 * n], stats[2 * n + 1]);
        int8_t* bn = buf + n * PHI_BUF;
        switch (a.basis) {
          case KAN_CHEBY: put_terms<ChebyGen<MODE>>(bn, xm, f, c_lo, a, FAST); break;
          case KAN_RBF: put_terms<RbfGen<MODE>>(bn, xm, f, c_lo, a, FAST); break;
          case KAN_BSPLINE: put_terms<BsplineGen<MODE>>(bn, xm, f, c_lo, a, FAST); break;
          case KAN_WAVELET: put_terms<WaveletGen<MODE>>(bn, xm, f, c_lo, a, FAST); break;
          case KAN_RELU: put_terms<ReluGen<MODE>>(bn, xm, f, c_lo, a, FAST); break;
          default: put_terms<FourierGen<MODE>>(bn, xm, f, c_lo, a, FAST); break;
        }
      }
    }
    // codes of the window past the row's end read zero basis values
    const int inside = kdim - c_lo;
    if (inside < WIN_CODES)
      for (int c = max(inside, 0) + tid; c < WIN_CODES; c += CTHREADS)
#pragma unroll
        for (int n = 0; n < NB; ++n) put_q(buf + n * PHI_BUF, c, 0, FAST);
  } else {
    // base segment: features [fb0, fb0 + 1024), four consecutive ones per thread (in thread
    // order, not the spread order of `tid`), so that the 64 features of an exponent chunk are the
    // 16 threads of a half warp
    const int fb0 = (w - p.Ww) * WIN_CODES;
    tid = (int)threadIdx.x;
#pragma unroll
    for (int n = 0; n < NB; ++n) {
      float sv[4];
      float m = 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int f = fb0 + 4 * tid + j;
        sv[j] = 0.f;
        if (f < a.D_in)
          sv[j] = silu_value<MODE>(map_input<MODE>(A::to_f(xs[n * a.D_in + f]), a.input_map,
                                                   stats[2 * n], stats[2 * n + 1]));
        m = fmaxf(m, fabsf(sv[j]));
      }
#pragma unroll
      for (int o = 8; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
      const int e = cc::fixed_exponent(m);
      const float sc = exp2f((float)e);
#pragma unroll
      for (int j = 0; j < 4; ++j) put_q(buf + n * PHI_BUF, 4 * tid + j, __float2int_rn(sv[j] * sc), FAST);
      if ((tid & 15) == 0) fac[n * 16 + (tid >> 4)] = exp2f((float)(PHI_E - e));
    }
  }
}

// 16 codes (one word) -> four words of bytes in cc::unit_pos order.
template <bool FAST>
__device__ __forceinline__ void decode16(uint32_t x, uint32_t (&d)[4]) {
  if (FAST) {
    const uint32_t y = x >> 2;
    d[0] = x & 0x03030303u;
    d[1] = y & 0x03030303u;
    d[2] = (x >> 4) & 0x03030303u;
    d[3] = (y >> 4) & 0x03030303u;
  } else {
    const uint32_t lut = 0x000100FFu;  // 0 -> -1, 1 -> 0, 2 -> +1, 3 -> 0
    d[0] = __byte_perm(lut, 0u, x & 0x3333u);
    d[1] = __byte_perm(lut, 0u, (x >> 2) & 0x3333u);
    d[2] = __byte_perm(lut, 0u, (x >> 16) & 0x3333u);
    d[3] = __byte_perm(lut, 0u, (x >> 18) & 0x3333u);
  }
}

template <bool FAST>
__device__ __forceinline__ int dp4(uint32_t a, uint32_t b, int c) {
  return FAST ? cc::dp4a_us(a, b, c) : cc::dp4a_ss(a, b, c);
}

// Sum of the lanes' partials of 8 rows per batch row: after the exchange lane l holds row
// (l >> 2) & 7 (the four lanes of a row agree).
__device__ __forceinline__ float reduce8(float (&v)[8], int lane) {
  const bool b4 = lane & 16, b3 = lane & 8, b2 = lane & 4;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float send = b4 ? v[j] : v[j + 4];
    const float keep = b4 ? v[j + 4] : v[j];
    v[j] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
  }
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    const float send = b3 ? v[j] : v[j + 2];
    const float keep = b3 ? v[j + 2] : v[j];
    v[j] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
  }
  {
    const float send = b2 ? v[0] : v[1];
    const float keep = b2 ? v[1] : v[0];
    v[0] = keep + __shfl_xor_sync(0xffffffffu, send, 4);
  }
  v[0] += __shfl_xor_sync(0xffffffffu, v[0], 2);
  v[0] += __shfl_xor_sync(0xffffffffu, v[0], 1);
  return v[0];
}

// The warp's rows of one stage for a window of the basis (SEG = false) or base (true) segment:
// acc[r][n] += scale * (integer total of row r, batch row n) [* base factor].
template <int MODE, bool FAST, int NB, bool SEG>
__device__ __forceinline__ void stage_rows(float (&acc)[RW][NB], const uint8_t* tile, int sfl,
                                           int lgs, int warp, int lane, const uint4 (&bh)[NB][2],
                                           const uint4 (&bl)[NB][2], const int (&l0)[NB],
                                           const float (&fn)[NB]) {
  using A = Act<MODE>;
  const float* stile = reinterpret_cast<const float*>(tile + CODE_TILE);
  const int gl = (lane * 32) >> lgs;  // the lane's scale group within the window
#pragma unroll
  for (int r = 0; r < RW; ++r) {
    const int row = warp * RW + r;
    const uint2 cw = *reinterpret_cast<const uint2*>(tile + row * WIN_BYTES + lane * LANE_BYTES);
    const float sc = A::round(stile[row * sfl + gl]);
    uint32_t d0[4], d1[4];
    decode16<FAST>(cw.x, d0);
    decode16<FAST>(cw.y, d1);
#pragma unroll
    for (int n = 0; n < NB; ++n) {
      int H = 0, L = l0[n];
      H = dp4<FAST>(d0[0], bh[n][0].x, H);
      L = dp4<FAST>(d0[0], bl[n][0].x, L);
      H = dp4<FAST>(d0[1], bh[n][0].y, H);
      L = dp4<FAST>(d0[1], bl[n][0].y, L);
      H = dp4<FAST>(d0[2], bh[n][0].z, H);
      L = dp4<FAST>(d0[2], bl[n][0].z, L);
      H = dp4<FAST>(d0[3], bh[n][0].w, H);
      L = dp4<FAST>(d0[3], bl[n][0].w, L);
      H = dp4<FAST>(d1[0], bh[n][1].x, H);
      L = dp4<FAST>(d1[0], bl[n][1].x, L);
      H = dp4<FAST>(d1[1], bh[n][1].y, H);
      L = dp4<FAST>(d1[1], bl[n][1].y, L);
      H = dp4<FAST>(d1[2], bh[n][1].z, H);
      L = dp4<FAST>(d1[2], bl[n][1].z, L);
      H = dp4<FAST>(d1[3], bh[n][1].w, H);
      L = dp4<FAST>(d1[3], bl[n][1].w, L);
      float v = (float)(H * 128 + L);  // exact: |total| < 2^24
      if (SEG) v *= fn[n];
      acc[r][n] = fmaf(v, sc, acc[r][n]);
    }
  }
}

template <int MODE, bool FAST, int NB>
__global__ void __launch_bounds__(THREADS, 1)
    kan_gemv_kl_kernel(const __grid_constant__ CUtensorMap tm_cw,
                       const __grid_constant__ CUtensorMap tm_sw,
                       const __grid_constant__ CUtensorMap tm_cb,
                       const __grid_constant__ CUtensorMap tm_sb,
                       const __grid_constant__ LayerArgs a, const __grid_constant__ Params p) {
  using A = Act<MODE>;
  using T = typename A::T;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  const uint32_t s_base = smem_u32(smem);
  const uint32_t bar_full = s_base + p.off_bar;
  const uint32_t bar_phi = bar_full + 8 * p.stages;  // [2]: a window's basis is in place
  const uint32_t bar_never = bar_phi + 16;            // completed by nothing (abort-path tests)
  T* xs = reinterpret_cast<T*>(smem + p.off_x);                  // [NB][D_in]
  int8_t* phi = reinterpret_cast<int8_t*>(smem + p.off_phi);     // [2][NB][hi, lo][1024]
  float* fac = reinterpret_cast<float*>(smem + p.off_fac);       // [2][NB][16]
  float* stats = reinterpret_cast<float*>(smem + p.off_misc);    // [NB][mean, rstd]
  float* red = stats + 2 * MAXB;                                 // [WARPS][NB]
  volatile int* abort_flag = reinterpret_cast<volatile int*>(red + WARPS * MAXB);
  volatile int* decision = abort_flag + 1;
  int* consumed = const_cast<int*>(decision + 3);  // [MAX_STAGES] warps done with the stage
  int* issued = consumed + MAX_STAGES;             // [MAX_STAGES] loads requested into the stage
  const long long plim = a.wait_cycles > 0 ? a.wait_cycles : tc::WAIT_LIMIT_CYCLES;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const long long t0 = p.tasks * blockIdx.x / p.G;
  const long long t1 = p.tasks * (blockIdx.x + 1) / p.G;
  const int ntask = (int)(t1 - t0);
  if (ntask <= 0) return;

  const uint32_t stage_tx = (uint32_t)(CODE_TILE + ROWS * p.sfl * 4);
  // request task i's codes and scales into its stage (one thread)
  auto request = [&](int i) {
    const int s = i % p.stages;
    const long long t = t0 + i;
    const int w = (int)(t % p.W), rb = (int)(t / p.W);
    const bool seg = w >= p.Ww;
    const int wl = seg ? w - p.Ww : w;
    const uint32_t dst = s_base + s * p.stage_bytes;
    mbar_arrive_expect_tx(bar_full + 8 * s, stage_tx);
    tma_load_2d(dst, seg ? &tm_cb : &tm_cw, bar_full + 8 * s, wl * WIN_BYTES, rb * ROWS);
    tma_load_2d(dst + CODE_TILE, seg ? &tm_sb : &tm_sw, bar_full + 8 * s, wl * p.sfl, rb * ROWS);
    issued[s] += 1;
  };

  if (tid == 0) {
    for (int s = 0; s < p.stages; ++s) {
      mbar_init(bar_full + 8 * s, 1);
      consumed[s] = 0;
      issued[s] = 0;
    }
    mbar_init(bar_phi, WARPS);
    mbar_init(bar_phi + 8, WARPS);
    mbar_init(bar_never, 1);
    *abort_flag = 0;
    *decision = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    for (int i = 0; i < ntask && i < p.stages; ++i) request(i);
  }
  __syncthreads();

  // -------------------------------------------------------------------- compute warps
  // the batch rows' inputs into shared memory
  {
    const int n_el = NB * a.D_in;
    const T* X = (const T*)a.X;
    if ((((uintptr_t)X) & 15) == 0 && (n_el & 7) == 0) {
      for (int i = tid; i < n_el / 8; i += CTHREADS)
        reinterpret_cast<uint4*>(xs)[i] = __ldg(reinterpret_cast<const uint4*>(X) + i);
    } else {
      for (int i = tid; i < n_el; i += CTHREADS) xs[i] = X[i];
    }
  }
  if (tid < NB) {
    stats[2 * tid] = 0.f;
    stats[2 * tid + 1] = 1.f;
  }
  named_bar(BAR_ID, CTHREADS);
  if (a.input_map == KAN_MAP_LAYERNORM) {
    // mean, then the mean square deviation (two passes, as the pre-pass computes them)
    for (int pass = 0; pass < 2; ++pass) {
      float s[NB];
#pragma unroll
      for (int n = 0; n < NB; ++n) {
        s[n] = 0.f;
        const float mu = pass ? stats[2 * n] : 0.f;
        for (int i = tid; i < a.D_in; i += CTHREADS) {
          const float d = A::to_f(xs[n * a.D_in + i]) - mu;
          s[n] = pass ? fmaf(d, d, s[n]) : s[n] + d;
        }
#pragma unroll
        for (int o = 16; o; o >>= 1) s[n] += __shfl_xor_sync(0xffffffffu, s[n], o);
        if (lane == 0) red[warp * MAXB + n] = s[n];
      }
      named_bar(BAR_ID, CTHREADS);
      if (tid < NB) {
        float t = 0.f;
        for (int w = 0; w < WARPS; ++w) t += red[w * MAXB + tid];
        if (pass == 0) stats[2 * tid] = t / (float)a.D_in;
        else stats[2 * tid + 1] = rsqrtf(t / (float)a.D_in + a.ln_eps);
      }
      named_bar(BAR_ID, CTHREADS);
    }
  }

  // basis producers: features spread over the warps first, so that no warp carries a window's
  // whole basis evaluation
  const int ptid = lane * WARPS + warp;
  produce_window<MODE, FAST, NB>(a, p, (int)(t0 % p.W), phi, fac, xs, stats, ptid);
  __syncwarp();
  if (lane == 0) mbar_arrive(bar_phi);

  float acc[RW][NB];
#pragma unroll
  for (int r = 0; r < RW; ++r)
#pragma unroll
    for (int n = 0; n < NB; ++n) acc[r][n] = 0.f;


  T* Y = (T*)a.Y;
  const T* bias = (const T*)a.bias;
  for (int i = 0; i < ntask; ++i) {
    const long long t = t0 + i;
    const int w = (int)(t % p.W), rb = (int)(t / p.W);
    const bool seg = w >= p.Ww;
    const int pb = i & 1;
    bool live = __shfl_sync(0xffffffffu, *abort_flag, 0) == 0;
    // this window's basis (produced one window ahead by all warps).  The kernel's waits are short
    // (stages land while the warps build the basis, and the warps reach each basis barrier
    // together), so a limit below 16 cycles -- the abort-path tests -- makes the first of them wait
    // on a barrier that nothing completes: the abort path then runs whatever the timing.
    const bool never = i == 0 && a.wait_cycles > 0 && a.wait_cycles < 16;
    if (live && !mbar_wait_warp(never ? bar_never : bar_phi + 8 * pb, (uint32_t)(i >> 1) & 1u,
                                plim)) {
      raise_device_error(a.err, DEVERR_TIMEOUT_FULL_A);
      *abort_flag = 1;
      live = false;
    }
    uint4 bh[NB][2], bl[NB][2];
    int l0[NB];
    float fn[NB];
#pragma unroll
    for (int n = 0; n < NB; ++n) {
      const int8_t* bn = phi + (pb * NB + n) * PHI_BUF;
      bh[n][0] = *reinterpret_cast<const uint4*>(bn + lane * 16);
      bh[n][1] = *reinterpret_cast<const uint4*>(bn + (32 + lane) * 16);
      bl[n][0] = *reinterpret_cast<const uint4*>(bn + WIN_CODES + lane * 16);
      bl[n][1] = *reinterpret_cast<const uint4*>(bn + WIN_CODES + (32 + lane) * 16);
      l0[n] = 0;
      if (FAST) {  // minus the lane's basis sum: the chains then total sum((c - 1) v)
        const uint32_t one = 0x01010101u;
        int sh = 0, sl = 0;
        sh = cc::dp4a_ss(bh[n][0].x, one, sh);
        sh = cc::dp4a_ss(bh[n][0].y, one, sh);
        sh = cc::dp4a_ss(bh[n][0].z, one, sh);
        sh = cc::dp4a_ss(bh[n][0].w, one, sh);
        sh = cc::dp4a_ss(bh[n][1].x, one, sh);
        sh = cc::dp4a_ss(bh[n][1].y, one, sh);
        sh = cc::dp4a_ss(bh[n][1].z, one, sh);
        sh = cc::dp4a_ss(bh[n][1].w, one, sh);
        sl = cc::dp4a_ss(bl[n][0].x, one, sl);
        sl = cc::dp4a_ss(bl[n][0].y, one, sl);
        sl = cc::dp4a_ss(bl[n][0].z, one, sl);
        sl = cc::dp4a_ss(bl[n][0].w, one, sl);
        sl = cc::dp4a_ss(bl[n][1].x, one, sl);
        sl = cc::dp4a_ss(bl[n][1].y, one, sl);
        sl = cc::dp4a_ss(bl[n][1].z, one, sl);
        sl = cc::dp4a_ss(bl[n][1].w, one, sl);
        l0[n] = -(sh * 128 + sl);
      }
      fn[n] = seg ? fac[(pb * NB + n) * 16 + (lane >> 1)] : 1.f;
    }
    // the next window's basis into the other buffer: every warp read that buffer (the window
    // before this one) before it arrived for this window's, which this warp has waited for
    if (i + 1 < ntask) {
      if (live)
        produce_window<MODE, FAST, NB>(a, p, (int)((t + 1) % p.W), phi + (pb ^ 1) * NB * PHI_BUF,
                                       fac + (pb ^ 1) * NB * 16, xs, stats, ptid);
      __syncwarp();
      if (lane == 0) mbar_arrive(bar_phi + 8 * (pb ^ 1));
    }
    // this task's stage
    const int s = i % p.stages;
    if (live && !mbar_wait_warp(bar_full + 8 * s, (uint32_t)(i / p.stages) & 1u, plim)) {
      raise_device_error(a.err, DEVERR_TIMEOUT_FULL_B);
      *abort_flag = 1;
      live = false;
    }
    if (live) {
      const uint8_t* tile = smem + s * p.stage_bytes;
      if (seg)
        stage_rows<MODE, FAST, NB, true>(acc, tile, p.sfl, p.lgs, warp, lane, bh, bl, l0, fn);
      else
        stage_rows<MODE, FAST, NB, false>(acc, tile, p.sfl, p.lgs, warp, lane, bh, bl, l0, fn);
      // done with the stage (counted only after this warp's wait completed: a stage whose load
      // may still be landing is never refilled); the last warp requests the task that refills it
      __syncwarp();
      if (lane == 0) {
        __threadfence_block();
        if (atomicAdd(consumed + s, 1) == WARPS - 1) {
          atomicExch(consumed + s, 0);
          if (i + p.stages < ntask && *abort_flag == 0) {
            // this CTA's reads of the stage (generic proxy) before the copy's writes (async)
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            request(i + p.stages);
          }
        }
      }
    }

    // ---------------------------------------------------------------- row block done here
    if (((t + 1) % p.W) != 0 && i + 1 != ntask) continue;
    const int first = owner((long long)rb * p.W, p.tasks, p.G);
    const int count = owner((long long)rb * p.W + p.W - 1, p.tasks, p.G) - first + 1;
    const int slot = (int)blockIdx.x - first;
    float out[RW / 8][NB];
#pragma unroll
    for (int b = 0; b < RW / 8; ++b)
#pragma unroll
      for (int n = 0; n < NB; ++n) {
        float v[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] = acc[8 * b + j][n];
        out[b][n] = reduce8(v, lane) * (1.0f / (float)(1 << PHI_E));
      }
#pragma unroll
    for (int r = 0; r < RW; ++r)
#pragma unroll
      for (int n = 0; n < NB; ++n) acc[r][n] = 0.f;
    const bool writer = (lane & 3) == 0 && *abort_flag == 0;
    if (count == 1) {
      if (writer)
#pragma unroll
        for (int b = 0; b < RW / 8; ++b) {
          const int row = rb * ROWS + warp * RW + 8 * b + (lane >> 2);
          if (row >= a.D_out) continue;
          const float bv = a.has_bias ? A::to_f(bias[row]) : 0.f;
#pragma unroll
          for (int n = 0; n < NB; ++n) Y[(size_t)n * a.D_out + row] = A::from_f(out[b][n] + bv);
        }
      continue;
    }
    if (writer)
#pragma unroll
      for (int b = 0; b < RW / 8; ++b)
#pragma unroll
        for (int n = 0; n < NB; ++n)
          p.part[((size_t)(rb * p.maxc + slot) * NB + n) * ROWS + warp * RW + 8 * b + (lane >> 2)] =
              out[b][n];
    __threadfence();
    named_bar(BAR_ID, CTHREADS);
    if (tid == 0) {
      int last = 0;
      if (*abort_flag == 0) {
        // count this contribution; a counter left by another call carries another epoch
        unsigned long long* c = p.counters + rb;
        unsigned long long old = *reinterpret_cast<volatile unsigned long long*>(c), nv = 0;
        bool done = false;
        for (int it = 0; it < (1 << 20) && !done; ++it) {
          nv = ((unsigned)(old >> 32) == p.epoch) ? old + 1
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
    named_bar(BAR_ID, CTHREADS);
    if (*decision) {
      // the last contributor: sum the partials in contributor order, bias, round, store
      __threadfence();
      for (int idx = tid; idx < ROWS * NB; idx += CTHREADS) {
        const int n = idx / ROWS, r = idx % ROWS, row = rb * ROWS + r;
        if (row >= a.D_out) continue;
        float sum = 0.f;
        for (int z = 0; z < count; ++z)
          sum += __ldcg(p.part + ((size_t)(rb * p.maxc + z) * NB + n) * ROWS + r);
        const float bv = a.has_bias ? A::to_f(bias[row]) : 0.f;
        Y[(size_t)n * a.D_out + row] = A::from_f(sum + bv);
      }
      if (tid == 0) atomicExch(p.counters + rb, 0ull);
    }
  }
  // every load requested lands before the CTA exits (after an abort some may still be in flight)
  named_bar(BAR_ID, CTHREADS);
  if (tid == 0)
    for (int s = 0; s < p.stages; ++s)
      if (issued[s] > 0) (void)mbar_wait(bar_full + 8 * s, (uint32_t)(issued[s] - 1) & 1u);
}

using KlFn = void (*)(const CUtensorMap, const CUtensorMap, const CUtensorMap, const CUtensorMap,
                      LayerArgs, Params);

// The instance for (dtype, batch size): in-place ternary decode or the table decoder (explicitly
// instantiated in kan_gemv_kl_inst.cu, one translation unit per pair).
template <int MODE, int NB>
KlFn select_kl(bool fast);

#define KAN_KL_DECLARE(M, N) template <> KlFn select_kl<M, N>(bool fast);
KAN_KL_DECLARE(MODE_F16, 1)
KAN_KL_DECLARE(MODE_F16, 2)
KAN_KL_DECLARE(MODE_F16, 3)
KAN_KL_DECLARE(MODE_F16, 4)
KAN_KL_DECLARE(MODE_BF16, 1)
KAN_KL_DECLARE(MODE_BF16, 2)
KAN_KL_DECLARE(MODE_BF16, 3)
KAN_KL_DECLARE(MODE_BF16, 4)
#undef KAN_KL_DECLARE

}  // namespace kl
}  // namespace kan
