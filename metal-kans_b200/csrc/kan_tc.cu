// kan_tc.cu -- fused KAN layer on the 5th-generation tensor cores (tcgen05 + TMEM + TMA), sm_100a.
//
// Y[B, D_out] = bias + [Phi(x) | silu(x)] Wp^T is one dense contraction.  The weights are first
// packed (kan_tc_pack / pack_kernel below) into a feature-blocked layout: each 64-column K block
// holds F = 64 / KT whole input features of KT = K + has_base columns (the K basis terms of the
// feature, then its base-branch weight), zero padded.  One CTA computes a 128 x BN output tile
// over a range of K blocks:
//
//   warps 0-7  basis producers, two groups of four warps taking alternate pipeline stages; each
//              thread owns one row of the 128 x 64 A tile: it loads the F inputs of its row,
//              evaluates their K basis terms and SiLU in registers (the generators of
//              kan_device.cuh, with the reference's rounding points), and writes the row straight
//              into shared memory in the 128-byte-swizzled K-major layout the MMA reads.  Phi is
//              never written to HBM (the reference stores it to a scratch buffer and runs MPS
//              GEMMs on it, metal_kan_bridge.mm:503-523).  After the K loop these warps are the
//              epilogue: tcgen05.ld of the fp32 accumulator, + bias, round, store.
//   warp 8     TMA producer: one cp.async.bulk.tensor.2d per stage for the BN x 64 weight tile.
//   warp 9     TMEM allocator and MMA issuer: 4 x tcgen05.mma.cta_group::1.kind::f16
//              (M=128, N=BN, K=16) per stage into the TMEM accumulator; tcgen05.commit frees the
//              stage and finally signals the epilogue.
//
// Split-K (grid.z > 1) serves grids too small to fill the 148 SMs without recomputing the basis
// for several N tiles: every split writes its fp32 partial tile to scratch, and the CTA that
// completes a tile (per-tile arrival counter) sums the partials in split order -- deterministic --
// adds the bias, stores Y and resets the counter.
//
// Every mbarrier wait is bounded (about one second of SM clocks); on expiry the kernel records
// the error in the device error word, skips its remaining work and still releases TMEM.
#include <cuda.h>

#include "kan_device.cuh"
#include "kan_launch.h"

namespace kan {
namespace tc {

constexpr int BM = 128;
constexpr int BK = 64;                 // 64 16-bit elements = one 128-byte swizzle row
constexpr int STAGES = 4;              // even: producer group g owns stages g, g+2
constexpr int A_STAGE_BYTES = BM * BK * 2;
constexpr int B_STAGE_BYTES = 256 * BK * 2;  // sized for the widest tile (BN = 256)
constexpr int NUM_PRODUCER_WARPS = 8;
constexpr int PRODUCER_THREADS = NUM_PRODUCER_WARPS * 32;
constexpr int TMA_WARP = 8;
constexpr int MMA_WARP = 9;
constexpr int THREADS = 320;
constexpr uint32_t TMEM_COLS = 256;
constexpr long long WAIT_LIMIT_CYCLES = 2000000000LL;  // ~1 s at the B200 boost clock

constexpr int OFF_A = 0;
constexpr int OFF_B = OFF_A + STAGES * A_STAGE_BYTES;
constexpr int OFF_BAR = OFF_B + STAGES * B_STAGE_BYTES;
constexpr int NUM_BARS = 3 * STAGES + 1;
constexpr int OFF_TMEM = OFF_BAR + NUM_BARS * 8;
constexpr int OFF_FLAG = OFF_TMEM + 4;
constexpr int OFF_LAST = OFF_FLAG + 4;
constexpr int OFF_STATS = (OFF_LAST + 4 + 15) / 16 * 16;
constexpr int SMEM_BYTES = OFF_STATS + 2 * BM * 4;
constexpr int SMEM_ALLOC = SMEM_BYTES + 1024;  // slack to align the base to 1024 B

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
// Bounded wait for the phase of `parity`; false when the limit expired.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (clock64() - t0 > WAIT_LIMIT_CYCLES) return false;
  }
  return true;
}
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void named_bar(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
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
// A-tile producers: one row of one 64-column block
// ---------------------------------------------------------------------------------------------

// Compile-time K: all 64 values live in registers and are stored as 8 swizzled 16-byte chunks.
template <int BASIS, int MODE, int K, bool HB>
struct RowProducer {
  static constexpr int KT = K + (HB ? 1 : 0);
  static constexpr int F = 64 / KT;
  using T = typename Act<MODE>::T;
  float g[K];  // RBF centres (registers)

  __device__ __forceinline__ void setup(const LayerArgs& a) {
    if (BASIS == KAN_RBF) {
#pragma unroll
      for (int k = 0; k < K; ++k) g[k] = __ldg(a.grid + k);
    }
  }

  __device__ __forceinline__ void produce(uint8_t* a_stage, int r, const T* xrow, bool valid,
                                          int blk, const LayerArgs& a, float mean, float rstd) {
    float v[64];
    float xs[F];
#pragma unroll
    for (int f = 0; f < F; ++f) {
      const int i = blk * F + f;
      xs[f] = (valid && i < a.D_in) ? Act<MODE>::to_f(xrow[i]) : 0.f;
    }
#pragma unroll
    for (int f = 0; f < F; ++f) {
      const int i = blk * F + f;
      const bool live = valid && i < a.D_in;
      const float xm = map_input<MODE>(xs[f], a.input_map, mean, rstd);
      if (BASIS == KAN_CHEBY) {
        ChebyGen<MODE> gen;
        gen.init(xm, i, a);
#pragma unroll
        for (int k = 0; k < K; ++k) v[f * KT + k] = gen.next();
      } else if (BASIS == KAN_RBF) {
        if (MODE == MODE_F16) {
          const __half xh = __float2half_rn(xm);
          const __half ih = __float2half_rn(a.inv_den);
#pragma unroll
          for (int k = 0; k < K; ++k) {
            __half diff = __hsub(xh, __float2half_rn(g[k]));
            __half t = __hmul(__hmul(__hneg(diff), diff), ih);
            v[f * KT + k] = __half2float(__float2half_rn(__expf(__half2float(t))));
          }
        } else {
#pragma unroll
          for (int k = 0; k < K; ++k) {
            float d = xm - g[k];
            v[f * KT + k] = Act<MODE>::round(__expf(-(d * d) * a.inv_den));
          }
        }
      } else if (BASIS == KAN_BSPLINE) {
        BsplineGen<MODE> gen;
        gen.init(xm, i, a);
#pragma unroll
        for (int k = 0; k < K; ++k) {
          const int d = k - gen.span;
          float val = 0.f;
          val = (d == 0) ? gen.b0 : val;
          val = (d == 1) ? gen.b1 : val;
          val = (d == 2) ? gen.b2 : val;
          val = (d == 3) ? gen.b3 : val;
          v[f * KT + k] = val;
        }
      } else {
        WaveletGen<MODE> gen;
        gen.init(xm, live ? i : 0, a);
#pragma unroll
        for (int k = 0; k < K; ++k) v[f * KT + k] = gen.next();
      }
      if (HB) v[f * KT + K] = silu_value<MODE>(xm);
      if (!live) {
#pragma unroll
        for (int k = 0; k < KT; ++k) v[f * KT + k] = 0.f;
      }
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
};

// Runtime K (any K + has_base <= 64): zero the row, then 2-byte stores of the computed terms.
template <int BASIS, int MODE>
struct RowProducerAnyK {
  using T = typename Act<MODE>::T;
  __device__ __forceinline__ void setup(const LayerArgs&) {}
  __device__ __forceinline__ void produce(uint8_t* a_stage, int r, const T* xrow, bool valid,
                                          int blk, const LayerArgs& a, float mean, float rstd) {
    using Gen = typename GenFor<BASIS, MODE>::type;
    const int KT = a.K + (a.has_base ? 1 : 0);
    const int F = 64 / KT;
#pragma unroll
    for (int j = 0; j < 8; ++j)
      *reinterpret_cast<uint4*>(a_stage + a_chunk_off(r, j)) = make_uint4(0, 0, 0, 0);
    for (int f = 0; f < F; ++f) {
      const int i = blk * F + f;
      if (!valid || i >= a.D_in) break;
      const float xm = map_input<MODE>(Act<MODE>::to_f(xrow[i]), a.input_map, mean, rstd);
      Gen gen;
      gen.init(xm, i, a);
      for (int k = 0; k < KT; ++k) {
        const float val = (k < a.K) ? gen.next() : silu_value<MODE>(xm);
        const int c = f * KT + k;
        T tv = Act<MODE>::from_f(val);
        *reinterpret_cast<T*>(a_stage + a_chunk_off(r, c >> 3) + (c & 7) * 2) = tv;
      }
    }
  }
};

// ---------------------------------------------------------------------------------------------
// the kernel
// ---------------------------------------------------------------------------------------------
template <int BASIS, int MODE, class Producer>
__global__ void __launch_bounds__(THREADS, 1)
    kan_tc_kernel(const __grid_constant__ CUtensorMap tmap_w, LayerArgs a, int BN, int nb_total,
                  int splits) {
  using T = typename Act<MODE>::T;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  const uint32_t s_base = smem_u32(smem);
  const uint32_t bar_full_a = s_base + OFF_BAR;
  const uint32_t bar_full_b = bar_full_a + STAGES * 8;
  const uint32_t bar_empty = bar_full_b + STAGES * 8;
  const uint32_t bar_accum = bar_empty + STAGES * 8;
  volatile uint32_t* tmem_slot = reinterpret_cast<volatile uint32_t*>(smem + OFF_TMEM);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + OFF_FLAG);
  volatile int* last_flag = reinterpret_cast<volatile int*>(smem + OFF_LAST);
  float* s_mean = reinterpret_cast<float*>(smem + OFF_STATS);
  float* s_rstd = s_mean + BM;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
  const int z = blockIdx.z;
  // this split's K blocks: [kb0, kb1)
  const int kb0 = (int)((long long)nb_total * z / splits);
  const int kb1 = (int)((long long)nb_total * (z + 1) / splits);
  const int nj = kb1 - kb0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(bar_full_a + 8 * s, NUM_PRODUCER_WARPS / 2);
      mbar_init(bar_full_b + 8 * s, 1);
      mbar_init(bar_empty + 8 * s, 1);
    }
    mbar_init(bar_accum, 1);
    *abort_flag = 0;
    *last_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == MMA_WARP) tmem_alloc(s_base + OFF_TMEM, TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_d = *tmem_slot;

  if (warp < NUM_PRODUCER_WARPS) {
    // ------------------------------------------------------------------ basis producers
    const int q = warp & 3, grp = warp >> 2;
    const int r = q * 32 + lane;
    const int row = m0 + r;
    const bool valid = row < a.B;
    const T* X = (const T*)a.X;
    const T* xrow = X + (size_t)(valid ? row : 0) * a.D_in;

    if (a.input_map == KAN_MAP_LAYERNORM) {
      // 16 rows per producer warp, two-pass fp32 statistics
      for (int rr = warp * 16; rr < warp * 16 + 16; ++rr) {
        const int grow = m0 + rr;
        float mean = 0.f, rstd = 1.f;
        if (grow < a.B) {
          const T* xr = X + (size_t)grow * a.D_in;
          float sum = 0.f;
          for (int i = lane; i < a.D_in; i += 32) sum += Act<MODE>::to_f(xr[i]);
#pragma unroll
          for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
          mean = sum / (float)a.D_in;
          float var = 0.f;
          for (int i = lane; i < a.D_in; i += 32) {
            float d = Act<MODE>::to_f(xr[i]) - mean;
            var += d * d;
          }
#pragma unroll
          for (int o = 16; o; o >>= 1) var += __shfl_xor_sync(0xffffffffu, var, o);
          rstd = rsqrtf(var / (float)a.D_in + a.ln_eps);
        }
        if (lane == 0) {
          s_mean[rr] = mean;
          s_rstd[rr] = rstd;
        }
      }
      named_bar(1, PRODUCER_THREADS);
    }
    const float mean = (a.input_map == KAN_MAP_LAYERNORM) ? s_mean[r] : 0.f;
    const float rstd = (a.input_map == KAN_MAP_LAYERNORM) ? s_rstd[r] : 1.f;
    Producer prod;
    prod.setup(a);

    for (int j = grp; j < nj; j += 2) {
      const int s = j % STAGES;
      const uint32_t it = (uint32_t)(j / STAGES);
      if (!mbar_wait(bar_empty + 8 * s, (it & 1u) ^ 1u)) {
        raise_device_error(a.err, DEVERR_TIMEOUT_EMPTY);
        *abort_flag = 1;
        break;
      }
      if (*abort_flag) break;
      prod.produce(smem + OFF_A + s * A_STAGE_BYTES, r, xrow, valid, kb0 + j, a, mean, rstd);
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar_full_a + 8 * s);
    }

    // ------------------------------------------------------------------ epilogue
    if (!mbar_wait(bar_accum, 0)) {
      raise_device_error(a.err, DEVERR_TIMEOUT_ACCUM);
      *abort_flag = 1;
    }
    tc_fence_after();
    // all epilogue threads must agree on the abort decision before the named barriers below
    named_bar(3, PRODUCER_THREADS);
    if (threadIdx.x == 0) *last_flag = *abort_flag ? 2 : 0;
    named_bar(3, PRODUCER_THREADS);
    const bool aborted = (*last_flag == 2);
    named_bar(3, PRODUCER_THREADS);
    if (threadIdx.x == 0) *last_flag = 0;
    named_bar(3, PRODUCER_THREADS);
    const int h = grp;  // column half of the tile
    const int HALF = BN >> 1;
    T* Y = (T*)a.Y;
    const T* bias = (const T*)a.bias;
    const bool vec_ok = (a.D_out % 8) == 0;
    const int tile = blockIdx.y * gridDim.x + blockIdx.x;
    float* part = a.partials + (size_t)tile * splits * BM * BN;  // [split][row][col]

    // Store (or accumulate into) Y one 32-column chunk at a time.
    auto finish_chunk = [&](const float (&out)[32], int col0) {
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
    auto bias_of = [&](int col) -> float {
      return (a.has_bias && col < a.D_out) ? Act<MODE>::to_f(bias[col]) : 0.f;
    };

    if (!aborted && nj > 0) {
      if (splits == 1) {
#pragma unroll 1
        for (int cc = 0; cc < HALF; cc += 32) {
          uint32_t acc[32];
          const int ct = h * HALF + cc;
          tmem_ld32(tmem_d + ((uint32_t)(q * 32) << 16) + (uint32_t)ct, acc);
          const int col0 = n0 + ct;
          if (!valid || col0 >= a.D_out) continue;
          float out[32];
#pragma unroll
          for (int jj = 0; jj < 32; ++jj) out[jj] = __uint_as_float(acc[jj]) + bias_of(col0 + jj);
          finish_chunk(out, col0);
        }
      } else {
        // phase 1: this split's partial tile -> scratch
#pragma unroll 1
        for (int cc = 0; cc < HALF; cc += 32) {
          uint32_t acc[32];
          const int ct = h * HALF + cc;
          tmem_ld32(tmem_d + ((uint32_t)(q * 32) << 16) + (uint32_t)ct, acc);
          float4* dst = reinterpret_cast<float4*>(part + ((size_t)z * BM + r) * BN + ct);
#pragma unroll
          for (int jj = 0; jj < 8; ++jj)
            dst[jj] = make_float4(__uint_as_float(acc[4 * jj]), __uint_as_float(acc[4 * jj + 1]),
                                  __uint_as_float(acc[4 * jj + 2]),
                                  __uint_as_float(acc[4 * jj + 3]));
        }
        __threadfence();
        named_bar(2, PRODUCER_THREADS);
        if (threadIdx.x == 0) {
          const int prev = atomicAdd(a.counters + tile, 1);
          *last_flag = (prev == splits - 1) ? 1 : 0;
        }
        named_bar(2, PRODUCER_THREADS);
        if (*last_flag) {
          __threadfence();
          // phase 2 (last split to arrive): sum the partials in split order, bias, store
#pragma unroll 1
          for (int cc = 0; cc < HALF; cc += 32) {
            uint32_t acc[32];
            const int ct = h * HALF + cc;
            tmem_ld32(tmem_d + ((uint32_t)(q * 32) << 16) + (uint32_t)ct, acc);
            const int col0 = n0 + ct;
            if (!valid || col0 >= a.D_out) continue;
            float out[32];
#pragma unroll
            for (int jj = 0; jj < 32; ++jj) out[jj] = 0.f;
            for (int zz = 0; zz < splits; ++zz) {
              if (zz == z) {
#pragma unroll
                for (int jj = 0; jj < 32; ++jj) out[jj] += __uint_as_float(acc[jj]);
              } else {
                const float4* src =
                    reinterpret_cast<const float4*>(part + ((size_t)zz * BM + r) * BN + ct);
#pragma unroll
                for (int jj = 0; jj < 8; ++jj) {
                  const float4 p4 = __ldcg(src + jj);
                  out[4 * jj] += p4.x;
                  out[4 * jj + 1] += p4.y;
                  out[4 * jj + 2] += p4.z;
                  out[4 * jj + 3] += p4.w;
                }
              }
            }
#pragma unroll
            for (int jj = 0; jj < 32; ++jj) out[jj] += bias_of(col0 + jj);
            finish_chunk(out, col0);
          }
          if (threadIdx.x == 0) a.counters[tile] = 0;  // ready for the next launch
        }
      }
    }
  } else if (warp == TMA_WARP) {
    // ------------------------------------------------------------------ weight TMA
    if (lane == 0) {
      const uint32_t bytes = (uint32_t)BN * BK * 2;
      int issued = 0;
      for (int j = 0; j < nj; ++j) {
        const int s = j % STAGES;
        const uint32_t it = (uint32_t)(j / STAGES);
        if (!mbar_wait(bar_empty + 8 * s, (it & 1u) ^ 1u)) {
          raise_device_error(a.err, DEVERR_TIMEOUT_EMPTY);
          *abort_flag = 1;
          break;
        }
        if (*abort_flag) break;
        mbar_arrive_expect_tx(bar_full_b + 8 * s, bytes);
        tma_load_2d(s_base + OFF_B + s * B_STAGE_BYTES, &tmap_w, bar_full_b + 8 * s,
                    (kb0 + j) * BK, n0);
        ++issued;
      }
      // drain: wait (bounded) for the copies still landing in shared memory
      for (int j = issued - 1; j >= 0 && j >= issued - STAGES; --j)
        (void)mbar_wait(bar_full_b + 8 * (j % STAGES), (uint32_t)(j / STAGES) & 1u);
    }
  } else {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc = instr_desc(MODE == MODE_BF16 ? 1 : 0, BN, BM);
      for (int j = 0; j < nj; ++j) {
        const int s = j % STAGES;
        const uint32_t par = (uint32_t)(j / STAGES) & 1u;
        bool ok = mbar_wait(bar_full_a + 8 * s, par);
        if (!ok) raise_device_error(a.err, DEVERR_TIMEOUT_FULL_A);
        if (ok && !mbar_wait(bar_full_b + 8 * s, par)) {
          raise_device_error(a.err, DEVERR_TIMEOUT_FULL_B);
          ok = false;
        }
        if (!ok || *abort_flag) {
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        const uint32_t a_addr = s_base + OFF_A + s * A_STAGE_BYTES;
        const uint32_t b_addr = s_base + OFF_B + s * B_STAGE_BYTES;
#pragma unroll
        for (int kk = 0; kk < BK / 16; ++kk)
          mma_f16(tmem_d, smem_desc_sw128(a_addr + kk * 32), smem_desc_sw128(b_addr + kk * 32),
                  idesc, (j > 0 || kk > 0) ? 1u : 0u);
        mma_commit(bar_empty + 8 * s);
      }
      // signal the epilogue (also on abort, so that it does not wait out its own limit)
      mma_commit(bar_accum);
    }
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == MMA_WARP) {
    tc_fence_after();
    tmem_dealloc(tmem_d, TMEM_COLS);
  }
}

// ---------------------------------------------------------------------------------------------
// weight packing into the feature-blocked tensor-core layout
// ---------------------------------------------------------------------------------------------
template <int MODE>
__global__ void pack_kernel(LayerArgs a, typename Act<MODE>::T* out, int KT, int F, int NB) {
  const long long cols = (long long)NB * BK;
  const long long total = cols * a.D_out;
  const int Kdim = a.D_in * a.K;
  for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < total;
       e += (long long)gridDim.x * blockDim.x) {
    const int o = (int)(e / cols);
    const int c = (int)(e - (long long)o * cols);
    const int b = c / BK, jj = c - b * BK;
    const int f = jj / KT, t = jj - f * KT;
    const int i = b * F + f;
    float v = 0.f;
    if (f < F && i < a.D_in) {
      v = (t < a.K) ? weight_value<MODE>(a.w, o, i * a.K + t, Kdim)
                    : weight_value<MODE>(a.wb, o, i, a.D_in);
    }
    out[e] = Act<MODE>::from_f(v);
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
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = (EncodeTiledFn)p;
  }
  return fn;
}

// 2-D tensor map over the packed [rows][cols] 16-bit matrix, box = 64 columns x box_rows,
// 128-byte swizzle, zero fill out of range (rows beyond D_out).
static bool make_tmap(CUtensorMap* m, const void* base, int rows, long long cols, int box_rows,
                      int mode) {
  EncodeTiledFn enc = get_encode();
  if (!enc || ((uintptr_t)base & 15)) return false;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
  cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(m, mode == MODE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                        : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                   2, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

template <int BASIS, int MODE, class Producer>
static cudaError_t launch_kernel(const CUtensorMap& tw, const LayerArgs& a, int BN, int nb,
                                 int splits, dim3 grid, cudaStream_t s) {
  auto kern = kan_tc_kernel<BASIS, MODE, Producer>;
  static bool configured = false;  // one per template instance
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         SMEM_ALLOC);
    if (e != cudaSuccess) return e;
    configured = true;
  }
  kern<<<grid, THREADS, SMEM_ALLOC, s>>>(tw, a, BN, nb, splits);
  return cudaGetLastError();
}

// Compile-time-K producers for the shapes the BASELINE configs and common layers use; any other
// K runs the runtime-K producer.
template <int BASIS, int MODE>
static cudaError_t dispatch_k(const CUtensorMap& tw, const LayerArgs& a, int BN, int nb,
                              int splits, dim3 grid, cudaStream_t s) {
#define KAN_TC_CASE(KK, HBV)                                                                 \
  if (a.K == KK && (a.has_base != 0) == HBV)                                                 \
    return launch_kernel<BASIS, MODE, RowProducer<BASIS, MODE, KK, HBV>>(tw, a, BN, nb, splits, \
                                                                         grid, s);
  if (BASIS == KAN_CHEBY) {
    KAN_TC_CASE(4, true) KAN_TC_CASE(4, false) KAN_TC_CASE(5, true) KAN_TC_CASE(5, false)
    KAN_TC_CASE(8, true) KAN_TC_CASE(8, false) KAN_TC_CASE(9, true) KAN_TC_CASE(9, false)
  } else if (BASIS == KAN_RBF) {
    KAN_TC_CASE(8, true) KAN_TC_CASE(8, false)
  } else if (BASIS == KAN_BSPLINE) {
    KAN_TC_CASE(8, true) KAN_TC_CASE(8, false)
  } else {
    KAN_TC_CASE(6, true) KAN_TC_CASE(6, false) KAN_TC_CASE(8, true) KAN_TC_CASE(8, false)
  }
#undef KAN_TC_CASE
  return launch_kernel<BASIS, MODE, RowProducerAnyK<BASIS, MODE>>(tw, a, BN, nb, splits, grid, s);
}

template <int MODE>
static cudaError_t dispatch_basis(const CUtensorMap& tw, const LayerArgs& a, int BN, int nb,
                                  int splits, dim3 grid, cudaStream_t s) {
  switch (a.basis) {
    case KAN_CHEBY: return dispatch_k<KAN_CHEBY, MODE>(tw, a, BN, nb, splits, grid, s);
    case KAN_RBF: return dispatch_k<KAN_RBF, MODE>(tw, a, BN, nb, splits, grid, s);
    case KAN_BSPLINE: return dispatch_k<KAN_BSPLINE, MODE>(tw, a, BN, nb, splits, grid, s);
    default: return dispatch_k<KAN_WAVELET, MODE>(tw, a, BN, nb, splits, grid, s);
  }
}

}  // namespace tc

bool tc_supported(const LayerArgs& a, int act_dtype) {
  if (act_dtype != KAN_F16 && act_dtype != KAN_BF16) return false;
  if (a.B <= 0 || a.D_in <= 0 || a.D_out <= 0 || a.K <= 0) return false;
  if (a.K + (a.has_base ? 1 : 0) > 64) return false;
  return tc::get_encode() != nullptr;
}

TcPlan tc_plan(const LayerArgs& a) {
  TcPlan p;
  p.BN = a.D_out > 128 ? 256 : (a.D_out > 64 ? 128 : 64);
  const TcBlocking bl = tc_blocking(a.D_in, a.K, a.has_base);
  p.nb = bl.NB;
  p.mtiles = (a.B + tc::BM - 1) / tc::BM;
  p.ntiles = (a.D_out + p.BN - 1) / p.BN;
  const long long tiles = (long long)p.mtiles * p.ntiles;
  int splits = 1;
  if (tiles < 120) {
    splits = (int)(148 / tiles);
    splits = splits > 8 ? 8 : splits;
    const int max_by_k = p.nb / 4;  // keep >= 4 K blocks per split
    splits = splits > max_by_k ? max_by_k : splits;
    splits = splits < 1 ? 1 : splits;
  }
  p.splits = splits;
  p.partial_floats = splits > 1 ? (size_t)tiles * splits * tc::BM * p.BN : 0;
  p.counters = splits > 1 ? (size_t)tiles : 0;
  return p;
}

cudaError_t launch_tc(const LayerArgs& a, int act_dtype, const TcPlan& p, cudaStream_t s) {
  if (!tc_supported(a, act_dtype) || !a.tc_weights) return cudaErrorNotSupported;
  if (p.splits > 1 && (!a.partials || !a.counters)) return cudaErrorInvalidValue;
  const int mode = act_dtype == KAN_F16 ? MODE_F16 : MODE_BF16;
  CUtensorMap tw;
  if (!tc::make_tmap(&tw, a.tc_weights, a.D_out, (long long)p.nb * tc::BK, p.BN, mode))
    return cudaErrorInvalidValue;
  note_launch();
  dim3 grid(p.ntiles, p.mtiles, p.splits);
  if (mode == MODE_F16) return tc::dispatch_basis<MODE_F16>(tw, a, p.BN, p.nb, p.splits, grid, s);
  return tc::dispatch_basis<MODE_BF16>(tw, a, p.BN, p.nb, p.splits, grid, s);
}

cudaError_t launch_tc_pack(const LayerArgs& a, int act_dtype, void* out, cudaStream_t s) {
  const TcBlocking bl = tc_blocking(a.D_in, a.K, a.has_base);
  if (bl.F <= 0) return cudaErrorInvalidValue;
  note_launch();
  const long long total = (long long)bl.NB * tc::BK * a.D_out;
  long long blocks = (total + 255) / 256;
  if (blocks > 148LL * 16) blocks = 148LL * 16;
  if (blocks < 1) blocks = 1;
  if (act_dtype == KAN_F16)
    tc::pack_kernel<MODE_F16><<<(int)blocks, 256, 0, s>>>(a, (__half*)out, bl.KT, bl.F, bl.NB);
  else
    tc::pack_kernel<MODE_BF16><<<(int)blocks, 256, 0, s>>>(a, (__nv_bfloat16*)out, bl.KT, bl.F,
                                                          bl.NB);
  return cudaGetLastError();
}

}  // namespace kan
