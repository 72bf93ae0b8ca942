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
    case KAN_WAVELET: kan_simt_kernel<KAN_WAVELET, MODE, BM><<<grid, SIMT_THREADS, 0, s>>>(a); break;
    case KAN_RELU: kan_simt_kernel<KAN_RELU, MODE, BM><<<grid, SIMT_THREADS, 0, s>>>(a); break;
    case KAN_FOURIER: kan_simt_kernel<KAN_FOURIER, MODE, BM><<<grid, SIMT_THREADS, 0, s>>>(a); break;
    default: kan_simt_kernel<KAN_JACOBI, MODE, BM><<<grid, SIMT_THREADS, 0, s>>>(a); break;
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

// ---------------------------------------------------------------------------------------------
// Dense fp32 weights: the CTA's weight panel streamed through a ring of cp.async stages.
//
// A CTA computes an 8-row x BN-column tile (BN = 64, or 32 when the grid of 64-wide tiles would
// not cover the SMs).  K runs in chunks of 64 columns -- the basis segment (W, basis values) then
// the base segment (W_base, silu values) -- and each chunk of the panel, [BN][64] fp32, is copied
// by 16-byte cp.async into stage t % S (S = 8 for BN = 32, 4 for BN = 64) S - 1 chunks ahead of
// its use, so the L2 round trips of several chunks overlap each other and the FMAs.  Layers of at
// most 16 chunks build their whole 8-row basis tile once, after the first S - 1 chunks' copies
// are issued (the input and weight latencies overlap); longer ones evaluate each chunk's 8 x 64
// basis values into a ring of A stages while its copies are in flight.  The eight warps split each
// chunk's columns (8 each: short dependent chains per warp, which bound this latency-limited
// kernel); a lane owns one or two output columns for all 8 rows, reads its
// weights as float4 (row pitch 68 floats: conflict-free) and the basis values as float4
// broadcasts, and the warps' partial tiles are summed in warp order at the end.
// ---------------------------------------------------------------------------------------------
constexpr int DN_BM = 8;
constexpr int DN_KC = 64;
constexpr int DN_PITCH = DN_KC + 4;
constexpr int DN_THREADS = 256;
constexpr int DN_COLS_PER_WARP = DN_KC / (DN_THREADS / 32);  // chunk columns per warp (8)
constexpr int DN_ACHUNKS = 16;  // basis-tile chunks kept: all of them when the layer has <= 16
// Weight-ring depth: 8 chunks for 32-wide tiles (the small-grid case, where the whole K loop of a
// short layer is then one memory latency), 4 for 64-wide tiles (shared memory).
template <int BN> struct DnStages { static constexpr int value = BN == 32 ? 8 : 4; };

template <int BN>
struct DnSmem {
  float W[DnStages<BN>::value][BN][DN_PITCH];
  // the whole basis tile (T <= 16 chunks: built once, before the K loop) or a ring of 4 chunks
  float A[DN_ACHUNKS][DN_BM][DN_PITCH];
  float red[DN_THREADS / 32][DN_BM][BN];
  float mean[DN_BM], rstd[DN_BM];
};

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, int src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src),
               "r"(src_bytes)
               : "memory");
}

template <int BASIS, int BN>
__global__ void __launch_bounds__(DN_THREADS) kan_simt_dense_kernel(LayerArgs a) {
  using Gen = typename GenFor<BASIS, MODE_F32>::type;
  constexpr int DN_STAGES = DnStages<BN>::value;
  extern __shared__ __align__(16) uint8_t dn_raw[];
  DnSmem<BN>& sm = *reinterpret_cast<DnSmem<BN>*>(dn_raw);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int col0 = blockIdx.x * BN, row0 = blockIdx.y * DN_BM;
  const int Kw = a.D_in * a.K;
  const int Tw = (Kw + DN_KC - 1) / DN_KC;
  const int T = Tw + (a.has_base ? (a.D_in + DN_KC - 1) / DN_KC : 0);
  const float* X = (const float*)a.X;
  const float* W = (const float*)a.w.data;
  const float* Wb = (const float*)a.wb.data;

  if (a.input_map == KAN_MAP_LAYERNORM) {
    row_stats<MODE_F32>(a, row0, DN_BM, sm.mean, sm.rstd);
    __syncthreads();
  }
  // whole basis tile at once when it fits: every input load of the CTA is in flight together
  // (one memory latency) instead of one dependent round trip per chunk
  const bool whole_a = T <= DN_ACHUNKS;

  // issue the copies of chunk t's weight panel and (ring mode) build its basis tile
  auto prepare = [&](int t) {
    const int st = t % DN_STAGES;
    const bool seg = t >= Tw;
    const int c0 = (seg ? t - Tw : t) * DN_KC;
    const int cols = seg ? a.D_in : Kw;
    const float* M = seg ? Wb : W;
    for (int q = tid; q < BN * (DN_KC / 4); q += DN_THREADS) {
      const int n = q / (DN_KC / 4), c = (q % (DN_KC / 4)) * 4;
      const int row = col0 + n, col = c0 + c;
      const bool ok = row < a.D_out && col < cols;
      cp_async16((uint32_t)__cvta_generic_to_shared(&sm.W[st][n][c]),
                 ok ? (const void*)(M + (size_t)row * cols + col) : (const void*)M, ok ? 16 : 0);
    }
    if (whole_a) return;
    if (!seg) {
      // (row, feature) items overlapping the chunk; features >= D_in and rows >= B give zeros
      const int i0 = c0 / a.K, i1 = (c0 + DN_KC - 1) / a.K;
      const int nf = i1 - i0 + 1;
      for (int it = tid; it < DN_BM * nf; it += DN_THREADS) {
        const int r = it / nf, i = i0 + it % nf;
        const int row = row0 + r;
        const bool ok = row < a.B && i < a.D_in;
        Gen g;
        if (ok) {
          const float xm = map_input<MODE_F32>(X[(size_t)row * a.D_in + i], a.input_map,
                                               sm.mean[r], sm.rstd[r]);
          g.init(xm, i, a);
        }
        for (int k = 0; k < a.K; ++k) {
          const float v = ok ? g.next() : 0.f;
          const int c = i * a.K + k - c0;
          if (c >= 0 && c < DN_KC) sm.A[st][r][c] = v;
        }
      }
    } else {
      for (int it = tid; it < DN_BM * DN_KC; it += DN_THREADS) {
        const int r = it / DN_KC, c = it % DN_KC;
        const int row = row0 + r, i = c0 + c;
        float v = 0.f;
        if (row < a.B && i < a.D_in)
          v = silu_value<MODE_F32>(map_input<MODE_F32>(X[(size_t)row * a.D_in + i], a.input_map,
                                                       sm.mean[r], sm.rstd[r]));
        sm.A[st][r][c] = v;
      }
    }
  };

  constexpr int NJ = BN / 32;
  float acc[DN_BM][NJ];
#pragma unroll
  for (int r = 0; r < DN_BM; ++r)
#pragma unroll
    for (int j = 0; j < NJ; ++j) acc[r][j] = 0.f;

  // the first chunks' weight copies go out before the basis tile is built, so that the two
  // memory latencies (weights from L2/HBM, inputs for the basis) overlap
#pragma unroll 1
  for (int t = 0; t < DN_STAGES - 1; ++t) {
    if (t < T) prepare(t);
    asm volatile("cp.async.commit_group;" ::: "memory");
  }
  if (whole_a) {
    // every row of the tile is written (zeros past B), and the columns past the last basis and
    // base column of their chunks are zeroed; the K loop's first barrier publishes the tile
    for (int it = tid; it < DN_BM * a.D_in; it += DN_THREADS) {
      const int r = it / a.D_in, i = it % a.D_in;
      const int row = row0 + r;
      const bool ok = row < a.B;
      Gen g;
      float xm = 0.f;
      if (ok) {
        xm = map_input<MODE_F32>(X[(size_t)row * a.D_in + i], a.input_map, sm.mean[r],
                                 sm.rstd[r]);
        g.init(xm, i, a);
      }
      for (int k = 0; k < a.K; ++k) {
        const int c = i * a.K + k;
        sm.A[c / DN_KC][r][c % DN_KC] = ok ? g.next() : 0.f;
      }
      if (a.has_base) sm.A[Tw + i / DN_KC][r][i % DN_KC] = ok ? silu_value<MODE_F32>(xm) : 0.f;
    }
    const int tail_w = Tw * DN_KC - Kw;  // unused columns of the last basis chunk
    for (int it = tid; it < DN_BM * tail_w; it += DN_THREADS)
      sm.A[Tw - 1][it / tail_w][DN_KC - tail_w + it % tail_w] = 0.f;
    if (a.has_base) {
      const int tail_b = (T - Tw) * DN_KC - a.D_in;
      for (int it = tid; it < DN_BM * tail_b; it += DN_THREADS)
        sm.A[T - 1][it / tail_b][DN_KC - tail_b + it % tail_b] = 0.f;
    }
  }
#pragma unroll 1
  for (int i = 0; i < T; ++i) {
    if (i + DN_STAGES - 1 < T) prepare(i + DN_STAGES - 1);
    asm volatile("cp.async.commit_group;" ::: "memory");
    // chunk i's copies (group i) have landed; its basis tile was written before the barrier
    asm volatile("cp.async.wait_group %0;" ::"n"(DN_STAGES - 1) : "memory");
    __syncthreads();
    const int st = i % DN_STAGES;
    const int sa = whole_a ? i : st;  // basis-tile chunk
#pragma unroll
    for (int s4 = 0; s4 < DN_COLS_PER_WARP / 4; ++s4) {
      const int c = warp * DN_COLS_PER_WARP + s4 * 4;
      float4 wv[NJ];
#pragma unroll
      for (int j = 0; j < NJ; ++j) wv[j] = *reinterpret_cast<const float4*>(&sm.W[st][lane + 32 * j][c]);
#pragma unroll
      for (int r = 0; r < DN_BM; ++r) {
        const float4 av = *reinterpret_cast<const float4*>(&sm.A[sa][r][c]);
#pragma unroll
        for (int j = 0; j < NJ; ++j) {
          acc[r][j] = fmaf(av.x, wv[j].x, acc[r][j]);
          acc[r][j] = fmaf(av.y, wv[j].y, acc[r][j]);
          acc[r][j] = fmaf(av.z, wv[j].z, acc[r][j]);
          acc[r][j] = fmaf(av.w, wv[j].w, acc[r][j]);
        }
      }
    }
    __syncthreads();  // stage st is refilled by the next iteration's prepare()
  }
  asm volatile("cp.async.wait_group 0;" ::: "memory");

#pragma unroll
  for (int r = 0; r < DN_BM; ++r)
#pragma unroll
    for (int j = 0; j < NJ; ++j) sm.red[warp][r][lane + 32 * j] = acc[r][j];
  __syncthreads();
  float* Y = (float*)a.Y;
  const float* bias = (const float*)a.bias;
  for (int o = tid; o < DN_BM * BN; o += DN_THREADS) {
    const int r = o / BN, n = o % BN;
    const int row = row0 + r, col = col0 + n;
    if (row >= a.B || col >= a.D_out) continue;
    float v = 0.f;
#pragma unroll
    for (int w = 0; w < DN_THREADS / 32; ++w) v += sm.red[w][r][n];
    if (a.has_bias) v += bias[col];
    Y[(size_t)row * a.D_out + col] = v;
  }
}

template <int BASIS, int BN>
static cudaError_t launch_dense_basis(const LayerArgs& a, cudaStream_t s) {
  const dim3 grid((a.D_out + BN - 1) / BN, (a.B + DN_BM - 1) / DN_BM);
  const int smem = (int)sizeof(DnSmem<BN>);
  static std::atomic<unsigned long long> configured{0};  // per device: smem limit raised
  cudaError_t e = ensure_smem_attr(kan_simt_dense_kernel<BASIS, BN>, smem, configured);
  if (e != cudaSuccess) return e;
  kan_simt_dense_kernel<BASIS, BN><<<grid, DN_THREADS, smem, s>>>(a);
  return cudaGetLastError();
}

template <int BN>
static cudaError_t launch_dense_bn(const LayerArgs& a, cudaStream_t s) {
  switch (BasisOf(a)) {
    case KAN_CHEBY: return launch_dense_basis<KAN_CHEBY, BN>(a, s);
    case KAN_RBF: return launch_dense_basis<KAN_RBF, BN>(a, s);
    case KAN_BSPLINE: return launch_dense_basis<KAN_BSPLINE, BN>(a, s);
    case KAN_WAVELET: return launch_dense_basis<KAN_WAVELET, BN>(a, s);
    case KAN_RELU: return launch_dense_basis<KAN_RELU, BN>(a, s);
    case KAN_FOURIER: return launch_dense_basis<KAN_FOURIER, BN>(a, s);
    default: return launch_dense_basis<KAN_JACOBI, BN>(a, s);
  }
}

// The streamed-panel kernel takes dense fp32 layers whose weight rows start on 16-byte
// boundaries (D_in * K and D_in multiples of 4, aligned base pointers).
static bool dense_f32_ok(const LayerArgs& a) {
  auto al = [](const void* p) { return ((uintptr_t)p & 15) == 0; };
  if (a.w.format != KAN_W_DENSE || (a.D_in * a.K) % 4 || !al(a.w.data)) return false;
  if (a.has_base && (a.wb.format != KAN_W_DENSE || a.D_in % 4 || !al(a.wb.data))) return false;
  return true;
}

cudaError_t launch_simt(const LayerArgs& a, int act_dtype, cudaStream_t s) {
  note_launch();
  if (act_dtype == KAN_F32 && dense_f32_ok(a)) {
    const long long wide = (long long)((a.D_out + 63) / 64) * ((a.B + DN_BM - 1) / DN_BM);
    return wide < 148 ? launch_dense_bn<32>(a, s) : launch_dense_bn<64>(a, s);
  }
  if (act_dtype == KAN_F32) return launch_simt_mode<MODE_F32>(a, s);
  if (act_dtype == KAN_F16) return launch_simt_mode<MODE_F16>(a, s);
  return launch_simt_mode<MODE_BF16>(a, s);
}

}  // namespace kan
