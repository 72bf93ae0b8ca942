// kan_tc.cu -- fused KAN layer on the 5th-generation tensor cores (tcgen05 + TMEM + TMA), sm_100a.
//
// Y[B, D_out] = bias + Phi(x) W^T + silu(x) Wb^T is one dense contraction over
// K_total = D_in*K (+ D_in for the base branch).  One CTA computes a 128 x BN output tile:
//
//   warps 0-7  basis producers: evaluate the basis of their rows in registers (the generators of
//              kan_device.cuh, reference rounding points) and write the 128 x 64 A tile of each
//              pipeline stage straight into shared memory in the 128-byte-swizzled K-major layout
//              the MMA reads -- Phi never exists in HBM (the reference writes it to a scratch
//              buffer and runs MPS GEMMs on it, metal_kan_bridge.mm:503-523).  After the K loop
//              the same warps are the epilogue: tcgen05.ld of the fp32 accumulator, + bias,
//              round to the act dtype, store.
//   warp 8     TMA producer: one cp.async.bulk.tensor.2d per stage for the BN x 64 weight tile
//              (W for the basis blocks, W_base for the base blocks), out-of-range rows/columns
//              zero-filled by the tensor map.
//   warp 9     TMEM allocator and MMA issuer: 4 x tcgen05.mma.cta_group::1.kind::f16
//              (M=128, N=BN, K=16) per stage into a TMEM fp32 accumulator; tcgen05.commit frees
//              the stage and finally signals the epilogue.
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
constexpr int A_STAGE_BYTES = BM * BK * 2;
constexpr int NUM_PRODUCER_WARPS = 8;
constexpr int PRODUCER_THREADS = NUM_PRODUCER_WARPS * 32;
constexpr int TMA_WARP = 8;
constexpr int MMA_WARP = 9;
constexpr int THREADS = 320;
constexpr long long WAIT_LIMIT_CYCLES = 2000000000LL;  // ~1 s at the B200 boost clock

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
__host__ __device__ constexpr uint32_t instr_desc(int ab_fmt, int n, int m) {
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

template <int BN, int STAGES>
struct Layout {
  static constexpr int B_STAGE_BYTES = BN * BK * 2;
  static constexpr int OFF_A = 0;
  static constexpr int OFF_B = OFF_A + STAGES * A_STAGE_BYTES;
  static constexpr int OFF_BAR = OFF_B + STAGES * B_STAGE_BYTES;
  static constexpr int NUM_BARS = 3 * STAGES + 1;
  static constexpr int OFF_TMEM = OFF_BAR + NUM_BARS * 8;
  static constexpr int OFF_FLAG = OFF_TMEM + 4;
  static constexpr int OFF_STATS = (OFF_FLAG + 4 + 15) / 16 * 16;
  static constexpr int BYTES = OFF_STATS + 2 * BM * 4;
  static constexpr int ALLOC = BYTES + 1024;  // slack to align the base to 1024 B
  static constexpr uint32_t TMEM_COLS = BN < 32 ? 32 : BN;
};

// ---------------------------------------------------------------------------------------------
// the kernel
// ---------------------------------------------------------------------------------------------
template <int BASIS, int MODE, int BN, int STAGES>
__global__ void __launch_bounds__(THREADS, 1)
    kan_tc_kernel(const __grid_constant__ CUtensorMap tmap_w,
                  const __grid_constant__ CUtensorMap tmap_wb, LayerArgs a, int n_kb_basis,
                  int n_kb_base) {
  using L = Layout<BN, STAGES>;
  using T = typename Act<MODE>::T;
  using Gen = typename GenFor<BASIS, MODE>::type;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  const uint32_t s_base = smem_u32(smem);
  const uint32_t bar_full_a = s_base + L::OFF_BAR;
  const uint32_t bar_full_b = bar_full_a + STAGES * 8;
  const uint32_t bar_empty = bar_full_b + STAGES * 8;
  const uint32_t bar_accum = bar_empty + STAGES * 8;
  volatile uint32_t* tmem_slot = reinterpret_cast<volatile uint32_t*>(smem + L::OFF_TMEM);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::OFF_FLAG);
  float* s_mean = reinterpret_cast<float*>(smem + L::OFF_STATS);
  float* s_rstd = s_mean + BM;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
  const int n_kb = n_kb_basis + n_kb_base;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(bar_full_a + 8 * s, PRODUCER_THREADS);
      mbar_init(bar_full_b + 8 * s, 1);
      mbar_init(bar_empty + 8 * s, 1);
    }
    mbar_init(bar_accum, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == MMA_WARP) tmem_alloc(s_base + L::OFF_TMEM, L::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_d = *tmem_slot;

  if (warp < NUM_PRODUCER_WARPS) {
    // ------------------------------------------------------------------ basis producers
    const int q = warp & 3, h = warp >> 2;
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
      asm volatile("bar.sync 1, %0;" ::"r"(PRODUCER_THREADS) : "memory");
    }
    const float mean = (a.input_map == KAN_MAP_LAYERNORM) ? s_mean[r] : 0.f;
    const float rstd = (a.input_map == KAN_MAP_LAYERNORM) ? s_rstd[r] : 1.f;
    const int Kdim = a.D_in * a.K;

    bool ok = true;
    for (int kb = 0; kb < n_kb && ok; ++kb) {
      const int s = kb % STAGES;
      const uint32_t it = (uint32_t)(kb / STAGES);
      if (!mbar_wait(bar_empty + 8 * s, (it & 1u) ^ 1u)) {
        raise_device_error(a.err, DEVERR_TIMEOUT_EMPTY);
        *abort_flag = 1;
        ok = false;
        break;
      }
      if (*abort_flag) {
        ok = false;
        break;
      }
      float v[32];
      if (kb < n_kb_basis) {
        // warp-uniform walk over columns c_start .. c_start+31 of Phi (column = i*K + k)
        const int c_start = kb * BK + h * 32;
        int i = c_start / a.K;
        int k = c_start - i * a.K;
        Gen g;
        bool live = valid && i < a.D_in;
        {
          float x = live ? Act<MODE>::to_f(xrow[i]) : 0.f;
          g.init(map_input<MODE>(x, a.input_map, mean, rstd), i, a);
          for (int t = 0; t < k; ++t) (void)g.next();
        }
#pragma unroll
        for (int c = 0; c < 32; ++c) {
          v[c] = (live && c_start + c < Kdim) ? g.next() : 0.f;
          if (++k == a.K) {
            k = 0;
            ++i;
            live = valid && i < a.D_in;
            float x = live ? Act<MODE>::to_f(xrow[i]) : 0.f;
            g.init(map_input<MODE>(x, a.input_map, mean, rstd), i, a);
          }
        }
      } else {
        const int f_start = (kb - n_kb_basis) * BK + h * 32;
#pragma unroll
        for (int c = 0; c < 32; ++c) {
          const int f = f_start + c;
          float val = 0.f;
          if (valid && f < a.D_in) {
            float x = Act<MODE>::to_f(xrow[f]);
            val = silu_value<MODE>(map_input<MODE>(x, a.input_map, mean, rstd));
          }
          v[c] = val;
        }
      }
      // 4 x 16-byte chunks into the swizzled K-major A tile (chunk ^= row % 8)
      uint8_t* a_row = smem + L::OFF_A + s * A_STAGE_BYTES + r * 128;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int chunk = h * 4 + j;
        uint4 pk;
        pk.x = pack2<MODE>(v[8 * j + 0], v[8 * j + 1]);
        pk.y = pack2<MODE>(v[8 * j + 2], v[8 * j + 3]);
        pk.z = pack2<MODE>(v[8 * j + 4], v[8 * j + 5]);
        pk.w = pack2<MODE>(v[8 * j + 6], v[8 * j + 7]);
        *reinterpret_cast<uint4*>(a_row + ((chunk ^ (r & 7)) << 4)) = pk;
      }
      fence_proxy_async_smem();
      mbar_arrive(bar_full_a + 8 * s);
    }

    // ------------------------------------------------------------------ epilogue
    if (!mbar_wait(bar_accum, 0)) {
      raise_device_error(a.err, DEVERR_TIMEOUT_ACCUM);
      *abort_flag = 1;
    }
    tc_fence_after();
    if (!*abort_flag && n_kb > 0) {
      T* Y = (T*)a.Y;
      const T* bias = (const T*)a.bias;
      const bool vec_ok = (a.D_out % 8) == 0;
      constexpr int HALF = BN / 2;
#pragma unroll 1
      for (int cc = 0; cc < HALF; cc += 32) {
        uint32_t acc[32];
        const int col_in_tile = h * HALF + cc;
        tmem_ld32(tmem_d + ((uint32_t)(q * 32) << 16) + (uint32_t)col_in_tile, acc);
        const int col0 = n0 + col_in_tile;
        if (!valid || col0 >= a.D_out) continue;
        float out[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          float b = 0.f;
          if (a.has_bias && col0 + j < a.D_out) b = Act<MODE>::to_f(bias[col0 + j]);
          out[j] = __uint_as_float(acc[j]) + b;
        }
        T* yrow = Y + (size_t)row * a.D_out;
        if (vec_ok && col0 + 32 <= a.D_out) {
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            uint4 pk;
            pk.x = pack2<MODE>(out[8 * j + 0], out[8 * j + 1]);
            pk.y = pack2<MODE>(out[8 * j + 2], out[8 * j + 3]);
            pk.z = pack2<MODE>(out[8 * j + 4], out[8 * j + 5]);
            pk.w = pack2<MODE>(out[8 * j + 6], out[8 * j + 7]);
            *reinterpret_cast<uint4*>(yrow + col0 + 8 * j) = pk;
          }
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (col0 + j < a.D_out) yrow[col0 + j] = Act<MODE>::from_f(out[j]);
        }
      }
    }
  } else if (warp == TMA_WARP) {
    // ------------------------------------------------------------------ weight TMA
    if (lane == 0) {
      int issued = 0;
      for (int kb = 0; kb < n_kb; ++kb) {
        const int s = kb % STAGES;
        const uint32_t it = (uint32_t)(kb / STAGES);
        if (!mbar_wait(bar_empty + 8 * s, (it & 1u) ^ 1u)) {
          raise_device_error(a.err, DEVERR_TIMEOUT_EMPTY);
          *abort_flag = 1;
          break;
        }
        if (*abort_flag) break;
        const uint32_t dst = s_base + L::OFF_B + s * L::B_STAGE_BYTES;
        mbar_arrive_expect_tx(bar_full_b + 8 * s, L::B_STAGE_BYTES);
        if (kb < n_kb_basis) tma_load_2d(dst, &tmap_w, bar_full_b + 8 * s, kb * BK, n0);
        else tma_load_2d(dst, &tmap_wb, bar_full_b + 8 * s, (kb - n_kb_basis) * BK, n0);
        ++issued;
      }
      // drain: wait (bounded) for the copies still landing in shared memory
      for (int kb = issued - 1; kb >= 0 && kb >= issued - STAGES; --kb) {
        const int s = kb % STAGES;
        (void)mbar_wait(bar_full_b + 8 * s, (uint32_t)(kb / STAGES) & 1u);
      }
    }
  } else {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc = instr_desc(MODE == MODE_BF16 ? 1 : 0, BN, BM);
      bool ok = true;
      for (int kb = 0; kb < n_kb; ++kb) {
        const int s = kb % STAGES;
        const uint32_t par = (uint32_t)(kb / STAGES) & 1u;
        if (!mbar_wait(bar_full_a + 8 * s, par)) {
          raise_device_error(a.err, DEVERR_TIMEOUT_FULL_A);
          ok = false;
        } else if (!mbar_wait(bar_full_b + 8 * s, par)) {
          raise_device_error(a.err, DEVERR_TIMEOUT_FULL_B);
          ok = false;
        }
        if (!ok || *abort_flag) {
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        const uint32_t a_addr = s_base + L::OFF_A + s * A_STAGE_BYTES;
        const uint32_t b_addr = s_base + L::OFF_B + s * L::B_STAGE_BYTES;
#pragma unroll
        for (int kk = 0; kk < BK / 16; ++kk) {
          mma_f16(tmem_d, smem_desc_sw128(a_addr + kk * 32), smem_desc_sw128(b_addr + kk * 32),
                  idesc, (kb > 0 || kk > 0) ? 1u : 0u);
        }
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
    tmem_dealloc(tmem_d, L::TMEM_COLS);
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

// 2-D tensor map over a row-major [rows][cols] 16-bit matrix, box = 64 columns x box_rows,
// 128-byte swizzle, zero fill out of range.
static bool make_tmap(CUtensorMap* m, const void* base, int rows, int cols, int box_rows,
                      int mode) {
  EncodeTiledFn enc = get_encode();
  if (!enc) return false;
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

static const void* tc_weight_ptr(const kan_weight& w) {
  if (w.format == KAN_W_DENSE) return w.data;
  return w.dense;
}

bool tc_supported(const LayerArgs& a, int act_dtype) {
  if (act_dtype != KAN_F16 && act_dtype != KAN_BF16) return false;
  if (a.B <= 0 || a.D_in <= 0 || a.D_out <= 0 || a.K <= 0 || a.K > 64) return false;
  const void* w = tc_weight_ptr(a.w);
  if (!w || ((uintptr_t)w & 15)) return false;
  if (((long long)a.D_in * a.K) % 8 != 0) return false;
  if (a.has_base) {
    const void* wb = tc_weight_ptr(a.wb);
    if (!wb || ((uintptr_t)wb & 15) || (a.D_in % 8) != 0) return false;
  }
  if (!get_encode()) return false;
  return true;
}

template <int BASIS, int MODE, int BN, int STAGES>
static cudaError_t launch_cfg(const CUtensorMap& tw, const CUtensorMap& twb, const LayerArgs& a,
                              int nkb, int nkb_base, cudaStream_t s) {
  using L = Layout<BN, STAGES>;
  auto kern = kan_tc_kernel<BASIS, MODE, BN, STAGES>;
  static bool configured = false;  // per template instance
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         L::ALLOC);
    if (e != cudaSuccess) return e;
    configured = true;
  }
  dim3 grid((a.D_out + BN - 1) / BN, (a.B + BM - 1) / BM);
  kern<<<grid, THREADS, L::ALLOC, s>>>(tw, twb, a, nkb, nkb_base);
  return cudaGetLastError();
}

template <int BASIS, int MODE>
static cudaError_t launch_basis(const LayerArgs& a, cudaStream_t s) {
  const int Kdim = a.D_in * a.K;
  const int nkb = (Kdim + BK - 1) / BK;
  const int nkb_base = a.has_base ? (a.D_in + BK - 1) / BK : 0;
  // Tile width: the widest N whose grid still covers the 148 SMs, else the smallest.
  const int mt = (a.B + BM - 1) / BM;
  int bn = 256;
  if ((long long)mt * ((a.D_out + 255) / 256) < 148 || a.D_out <= 128) bn = 128;
  if (bn == 128 && ((long long)mt * ((a.D_out + 127) / 128) < 148 || a.D_out <= 64)) bn = 64;
  CUtensorMap tw, twb;
  if (!make_tmap(&tw, tc_weight_ptr(a.w), a.D_out, Kdim, bn, MODE)) return cudaErrorInvalidValue;
  if (a.has_base) {
    if (!make_tmap(&twb, tc_weight_ptr(a.wb), a.D_out, a.D_in, bn, MODE))
      return cudaErrorInvalidValue;
  } else {
    twb = tw;
  }
  if (bn == 256) return launch_cfg<BASIS, MODE, 256, 4>(tw, twb, a, nkb, nkb_base, s);
  if (bn == 128) return launch_cfg<BASIS, MODE, 128, 6>(tw, twb, a, nkb, nkb_base, s);
  return launch_cfg<BASIS, MODE, 64, 8>(tw, twb, a, nkb, nkb_base, s);
}

template <int MODE>
static cudaError_t launch_mode(const LayerArgs& a, cudaStream_t s) {
  switch (a.basis) {
    case KAN_CHEBY: return launch_basis<KAN_CHEBY, MODE>(a, s);
    case KAN_RBF: return launch_basis<KAN_RBF, MODE>(a, s);
    case KAN_BSPLINE: return launch_basis<KAN_BSPLINE, MODE>(a, s);
    default: return launch_basis<KAN_WAVELET, MODE>(a, s);
  }
}

}  // namespace tc

bool tc_supported(const LayerArgs& a, int act_dtype) { return tc::tc_supported(a, act_dtype); }

cudaError_t launch_tc(const LayerArgs& a, int act_dtype, cudaStream_t s) {
  if (!tc::tc_supported(a, act_dtype)) return cudaErrorNotSupported;
  note_launch();
  if (act_dtype == KAN_F16) return tc::launch_mode<MODE_F16>(a, s);
  return tc::launch_mode<MODE_BF16>(a, s);
}

}  // namespace kan
