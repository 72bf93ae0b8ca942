// kan_simt.cu -- fused KAN layer on the CUDA cores (FFMA), fp32 accumulation.
//
// This is the engine's exact path: the fp32 layers (tolerance 1e-5 against the reference's fp32
// kernels) and the fallback for shapes the tensor-core kernel does not take.  The basis values of
// a feature chunk are generated straight into a shared-memory A tile (never written to HBM,
// unlike the reference's eval_*_basis + MPS GEMM pair, metal_kan_bridge.mm:443-530), the base
// branch is folded in as one extra column per feature (silu(x) against W_base), and the bias is
// added in the epilogue.  Packed weights are decoded on the way into shared memory.
//
// Tile: BM rows x 64 output columns per CTA, 256 threads; BM = 32 (2 x 4 outputs per thread), or
// BM = 8 (1 x 2 outputs per thread) for grids too small to fill the GPU; the K loop walks FC
// features at a time (FC * (K + has_base) <= 72 columns).
#include "kan_device.cuh"
#include "kan_launch.h"

namespace kan {

constexpr int SIMT_BM = 32;     // rows per CTA of the wide tile
constexpr int SIMT_BM_SMALL = 8;  // rows per CTA of the narrow tile
constexpr int SIMT_BN = 64;
constexpr int SIMT_KCAP = 72;  // max columns per chunk (K + base <= 65 is enforced by the host)
constexpr int SIMT_THREADS = 256;

// Per-row LayerNorm statistics (two-pass, fp32) for rows [row0, row0 + n) into smem.
template <int MODE>
__device__ void row_stats(const LayerArgs& a, int row0, int n, float* s_mean, float* s_rstd) {
  using T = typename Act<MODE>::T;
  const T* X = (const T*)a.X;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  for (int r = warp; r < n; r += nw) {
    int row = row0 + r;
    float mean = 0.f, rstd = 1.f;
    if (row < a.B) {
      const T* xr = X + (size_t)row * a.D_in;
      float s = 0.f;
      for (int i = lane; i < a.D_in; i += 32) s += Act<MODE>::to_f(xr[i]);
#pragma unroll
      for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
      mean = s / (float)a.D_in;
      float v = 0.f;
      for (int i = lane; i < a.D_in; i += 32) {
        float d = Act<MODE>::to_f(xr[i]) - mean;
        v += d * d;
      }
#pragma unroll
      for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
      rstd = rsqrtf(v / (float)a.D_in + a.ln_eps);
    }
    if (lane == 0) {
      s_mean[r] = mean;
      s_rstd[r] = rstd;
    }
  }
}

template <int BASIS, int MODE, int BM>
__global__ void __launch_bounds__(SIMT_THREADS) kan_simt_kernel(LayerArgs a) {
  using T = typename Act<MODE>::T;
  using Gen = typename GenFor<BASIS, MODE>::type;
  constexpr int RPT = BM / 16 > 0 ? BM / 16 : 1;    // rows per thread (2 or 1)
  constexpr int TY = BM / RPT;                        // thread rows (16 or 8)
  constexpr int TX = SIMT_THREADS / TY;               // thread columns (16 or 32)
  constexpr int CPT = SIMT_BN / TX;                   // columns per thread (4 or 2)
  __shared__ float As[BM][SIMT_KCAP + 1];
  __shared__ float Ws[SIMT_BN][SIMT_KCAP + 1];
  __shared__ float s_mean[BM], s_rstd[BM];

  const int tid = threadIdx.x, tx = tid % TX, ty = tid / TX;
  const int row0 = blockIdx.y * BM, col0 = blockIdx.x * SIMT_BN;
  const int KT = a.K + (a.has_base ? 1 : 0);
  const int FC = max(1, SIMT_KCAP / KT);
  const int Kdim = a.D_in * a.K;
  const T* X = (const T*)a.X;
  const bool dense = a.w.format == KAN_W_DENSE && (!a.has_base || a.wb.format == KAN_W_DENSE);

  if (a.input_map == KAN_MAP_LAYERNORM) row_stats<MODE>(a, row0, BM, s_mean, s_rstd);
  __syncthreads();

  float acc[RPT][CPT];
#pragma unroll
  for (int r = 0; r < RPT; ++r)
#pragma unroll
    for (int c = 0; c < CPT; ++c) acc[r][c] = 0.f;

  for (int f0 = 0; f0 < a.D_in; f0 += FC) {
    const int nf = min(FC, a.D_in - f0);
    const int kc = nf * KT;
    // A tile: basis (+ silu) of (row, feature) pairs
    for (int p = tid; p < BM * FC; p += SIMT_THREADS) {
      const int r = p / FC, f = p - r * FC;
      const int row = row0 + r;
      if (f >= nf) continue;
      float* dst = &As[r][f * KT];
      if (row < a.B) {
        float x = Act<MODE>::to_f(X[(size_t)row * a.D_in + f0 + f]);
        float xm = map_input<MODE>(x, a.input_map, s_mean[r], s_rstd[r]);
        Gen g;
        g.init(xm, f0 + f, a);
        for (int k = 0; k < a.K; ++k) dst[k] = g.next();
        if (a.has_base) dst[a.K] = silu_value<MODE>(xm);
      } else {
        for (int k = 0; k < KT; ++k) dst[k] = 0.f;
      }
    }
    // W tile: decoded weights, rounded to the operand dtype.  Dense weights (already in the act
    // dtype): row segments copied with coalesced loads, no per-element decode.
    if (dense) {
      const T* W = (const T*)a.w.data;
      const int cb = nf * a.K;
#pragma unroll 6
      for (int q = tid; q < SIMT_BN * cb; q += SIMT_THREADS) {
        const int n = q / cb, c = q - n * cb;
        const int j = col0 + n;
        const float v = j < a.D_out ? Act<MODE>::to_f(W[(size_t)j * Kdim + f0 * a.K + c]) : 0.f;
        if (a.has_base) {
          const int f = c / a.K;
          Ws[n][f * KT + (c - f * a.K)] = v;
        } else {
          Ws[n][c] = v;
        }
      }
      if (a.has_base) {
        const T* Wb = (const T*)a.wb.data;
        for (int q = tid; q < SIMT_BN * nf; q += SIMT_THREADS) {
          const int n = q / nf, f = q - n * nf;
          const int j = col0 + n;
          Ws[n][f * KT + a.K] =
              j < a.D_out ? Act<MODE>::to_f(Wb[(size_t)j * a.D_in + f0 + f]) : 0.f;
        }
      }
    } else
    for (int q = tid; q < SIMT_BN * kc; q += SIMT_THREADS) {
      const int n = q / kc, c = q - n * kc;
      const int f = c / KT, k = c - f * KT;
      const int j = col0 + n;
      float v = 0.f;
      if (j < a.D_out) {
        if (k < a.K) v = weight_value<MODE>(a.w, j, (f0 + f) * a.K + k, Kdim);
        else v = weight_value<MODE>(a.wb, j, f0 + f, a.D_in);
        v = Act<MODE>::round(v);
      }
      Ws[n][c] = v;
    }
    __syncthreads();
#pragma unroll 4
    for (int c = 0; c < kc; ++c) {
      float av[RPT];
#pragma unroll
      for (int r = 0; r < RPT; ++r) av[r] = As[ty + TY * r][c];
#pragma unroll
      for (int j = 0; j < CPT; ++j) {
        const float w = Ws[tx + TX * j][c];
#pragma unroll
        for (int r = 0; r < RPT; ++r) acc[r][j] = fmaf(av[r], w, acc[r][j]);
      }
    }
    __syncthreads();
  }

  T* Y = (T*)a.Y;
  const T* bias = (const T*)a.bias;
#pragma unroll
  for (int r = 0; r < RPT; ++r) {
    const int row = row0 + ty + TY * r;
    if (row >= a.B) continue;
#pragma unroll
    for (int j = 0; j < CPT; ++j) {
      const int col = col0 + tx + TX * j;
      if (col >= a.D_out) continue;
      float v = acc[r][j];
      if (a.has_bias) v += Act<MODE>::to_f(bias[col]);
      Y[(size_t)row * a.D_out + col] = Act<MODE>::from_f(v);
    }
  }
}

template <int MODE, int BM>
static void launch_simt_tile(const LayerArgs& a, cudaStream_t s) {
  dim3 grid((a.D_out + SIMT_BN - 1) / SIMT_BN, (a.B + BM - 1) / BM);
  switch (BasisOf(a)) {
    case KAN_CHEBY: kan_simt_kernel<KAN_CHEBY, MODE, BM><<<grid, SIMT_THREADS, 0, s>>>(a); break;
    case KAN_RBF: kan_simt_kernel<KAN_RBF, MODE, BM><<<grid, SIMT_THREADS, 0, s>>>(a); break;
    case KAN_BSPLINE: kan_simt_kernel<KAN_BSPLINE, MODE, BM><<<grid, SIMT_THREADS, 0, s>>>(a); break;
    default: kan_simt_kernel<KAN_WAVELET, MODE, BM><<<grid, SIMT_THREADS, 0, s>>>(a); break;
  }
}

template <int MODE>
static cudaError_t launch_simt_mode(const LayerArgs& a, cudaStream_t s) {
  // the narrow tile when the wide one would leave most of the 148 SMs idle
  const long long wide = (long long)((a.D_out + SIMT_BN - 1) / SIMT_BN) *
                         ((a.B + SIMT_BM - 1) / SIMT_BM);
  if (wide < 148) launch_simt_tile<MODE, SIMT_BM_SMALL>(a, s);
  else launch_simt_tile<MODE, SIMT_BM>(a, s);
  return cudaGetLastError();
}

cudaError_t launch_simt(const LayerArgs& a, int act_dtype, cudaStream_t s) {
  note_launch();
  if (act_dtype == KAN_F32) return launch_simt_mode<MODE_F32>(a, s);
  if (act_dtype == KAN_F16) return launch_simt_mode<MODE_F16>(a, s);
  return launch_simt_mode<MODE_BF16>(a, s);
}

}  // namespace kan
