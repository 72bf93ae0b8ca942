// kan_extra.cu -- the three composite layer kinds of the reference that are not one basis
// expansion followed by one projection: MultKAN (an RBF layer whose extra outputs are multiplied
// in pairs), LowRankKAN (an RBF layer into a rank-r bottleneck, then an up projection plus the
// base branch) and RationalKAN (per input-output pair the rational function P(x) / (1 + |Q(x)|)
// of two Chebyshev expansions, fp32 only).  All three run on the CUDA cores: the multiplication
// is elementwise, the bottleneck projections have a contraction of r (<= a few dozen) and D_in
// terms, and the rational function divides per (row, output, input) triple -- none of them is a
// dense contraction the tensor cores could take.  The RBF stages run on the engine's layer
// kernels (kan_tc_kernel / kan_simt_kernel) before these.
#include <cuda_fp16.h>

#include "kan_device.cuh"
#include "kan_launch.h"

namespace kan {
namespace extra {

// -------------------------------------------------------------------------------------------
// MultKAN: out[b, j] = in[b, j] (j < num_add), in[b, num_add + m] * in[b, num_add + num_mult + m]
// (j = num_add + m), the product rounded once to the layer dtype (combine_mult_nodes,
// fused_kan.metal:368-389 and its fp16 twin :1615-1640).
// -------------------------------------------------------------------------------------------
template <int MODE>
__global__ void mult_combine_kernel(const void* in_, void* out_, int B, int num_add,
                                    int num_mult) {
  using T = typename Act<MODE>::T;
  const T* in = (const T*)in_;
  T* out = (T*)out_;
  const int total_out = num_add + num_mult, total_in = num_add + 2 * num_mult;
  const long long n = (long long)B * total_out;
  for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < n;
       e += (long long)gridDim.x * blockDim.x) {
    const int b = (int)(e / total_out), j = (int)(e % total_out);
    const T* row = in + (size_t)b * total_in;
    if (j < num_add) {
      out[e] = row[j];
    } else {
      const int m = j - num_add;
      const float u = Act<MODE>::to_f(row[num_add + m]);
      const float v = Act<MODE>::to_f(row[num_add + num_mult + m]);
      out[e] = Act<MODE>::from_f(u * v);  // exact product of two halves, rounded once
    }
  }
}

// -------------------------------------------------------------------------------------------
// Tiled CUDA-core contraction Y[b, j] = bias[j] + sum_k A(b, k) Bm(j, k) over a K dimension that
// is the concatenation of segments, each with its own A producer and weight matrix.  A CTA
// computes a 32-row x 32-column tile with 256 threads (4 outputs each: rows ty, ty+8, ...);
// 32-wide K chunks of A (evaluated once per row and chunk) and of the weights are staged in
// shared memory (pitch 33: conflict-free); fp32 accumulation, one rounding at the store.
// -------------------------------------------------------------------------------------------
constexpr int TM = 32, TN = 32, TK = 32, TH = 256;

// LowRankKAN second stage (metal_kan_bridge.mm:1535-1698): K = [rank | D_in],
// A = [Z | silu(x)] (Z: the bottleneck activations of the RBF stage, in the layer dtype),
// weights [W_up | W_base].
template <int MODE>
__global__ void __launch_bounds__(TH) lowrank_up_kernel(const void* Z_, const void* X_,
                                                        const void* Wup_, const void* Wb_,
                                                        const void* bias_, void* Y_, int B,
                                                        int D_in, int D_out, int rank,
                                                        int has_base, int has_bias) {
  using T = typename Act<MODE>::T;
  const T* Z = (const T*)Z_;
  const T* X = (const T*)X_;
  const T* Wup = (const T*)Wup_;
  const T* Wb = (const T*)Wb_;
  __shared__ float sA[TM][TK + 1];
  __shared__ float sW[TN][TK + 1];
  const int tid = threadIdx.x, tx = tid & 31, ty = tid >> 5;
  const int row0 = blockIdx.y * TM, col0 = blockIdx.x * TN;
  const int Ktot = rank + (has_base ? D_in : 0);
  float acc[TM / 8];
#pragma unroll
  for (int i = 0; i < TM / 8; ++i) acc[i] = 0.f;
  for (int k0 = 0; k0 < Ktot; k0 += TK) {
    for (int e = tid; e < TM * TK; e += TH) {
      const int r = e / TK, c = e % TK, k = k0 + c, row = row0 + r;
      float v = 0.f;
      if (row < B && k < Ktot)
        v = k < rank ? Act<MODE>::to_f(Z[(size_t)row * rank + k])
                     : silu_value<MODE>(Act<MODE>::to_f(X[(size_t)row * D_in + (k - rank)]));
      sA[r][c] = v;
    }
    for (int e = tid; e < TN * TK; e += TH) {
      const int n = e / TK, c = e % TK, k = k0 + c, col = col0 + n;
      float v = 0.f;
      if (col < D_out && k < Ktot)
        v = k < rank ? Act<MODE>::to_f(Wup[(size_t)col * rank + k])
                     : Act<MODE>::to_f(Wb[(size_t)col * D_in + (k - rank)]);
      sW[n][c] = v;
    }
    __syncthreads();
#pragma unroll 8
    for (int c = 0; c < TK; ++c) {
      const float w = sW[tx][c];
#pragma unroll
      for (int i = 0; i < TM / 8; ++i) acc[i] = fmaf(sA[ty + 8 * i][c], w, acc[i]);
    }
    __syncthreads();
  }
  const int col = col0 + tx;
  if (col >= D_out) return;
  const float b = has_bias ? Act<MODE>::to_f(((const T*)bias_)[col]) : 0.f;
#pragma unroll
  for (int i = 0; i < TM / 8; ++i) {
    const int row = row0 + ty + 8 * i;
    if (row < B) ((T*)Y_)[(size_t)row * D_out + col] = Act<MODE>::from_f(acc[i] + b);
  }
}

// -------------------------------------------------------------------------------------------
// RationalKAN (kan_rational_tiled, fused_kan.metal:996-1125), fp32:
//   y[b, j] = bias[j] + sum_i ( silu(xc) Wb[j, i] + P_ji / (1 + |Q_ji|) ),  xc = clamp(x, -1, 1)
//   P_ji = sum_{d < p} T_d(xc) Wp[j, i p + d],  Q_ji = sum_{d < q} T_d(xc) Wq[j, i q + d]
// with T_d the Chebyshev polynomials.  A CTA takes 8 rows x 32 outputs (warp = row, lane =
// output); per 16-feature chunk the rows' T_d(xc) and silu(xc) and the 32 outputs' Wp / Wq / Wb
// slices are staged in shared memory, and every thread runs its (row, output) pair through the
// chunk's features: p + q FMAs, one division and the base FMA per feature.
// -------------------------------------------------------------------------------------------
constexpr int RF = 16;       // features per chunk
constexpr int RMAXD = 16;    // max(p, q) supported
constexpr int RROWS = 8, RCOLS = 32, RTH = RROWS * RCOLS;

__global__ void __launch_bounds__(RTH) rational_kernel(const float* X, const float* Wp,
                                                       const float* Wq, const float* Wb,
                                                       const float* bias, float* Y, int B,
                                                       int D_in, int D_out, int p, int q,
                                                       int has_base, int has_bias) {
  __shared__ float sT[RROWS][RF][RMAXD + 1];
  __shared__ float sS[RROWS][RF];
  extern __shared__ float sw[];  // [RCOLS][RF * (p + q) + RF + 1]
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int row0 = blockIdx.y * RROWS, col0 = blockIdx.x * RCOLS;
  const int maxd = p > q ? p : q;
  const int wpitch = RF * (p + q) + RF + 1;
  const int row = row0 + warp, col = col0 + lane;
  float acc = (has_bias && col < D_out) ? bias[col] : 0.f;
  for (int i0 = 0; i0 < D_in; i0 += RF) {
    const int nf = min(RF, D_in - i0);
    // the rows' Chebyshev terms and silu of the clamped inputs
    for (int e = tid; e < RROWS * RF; e += RTH) {
      const int r = e / RF, f = e % RF, rr = row0 + r;
      float xc = 0.f;
      if (rr < B && f < nf) xc = fminf(fmaxf(X[(size_t)rr * D_in + i0 + f], -1.f), 1.f);
      float t0 = 1.f, t1 = xc;
      for (int d = 0; d < maxd; ++d) {
        float t;
        if (d == 0) {
          t = 1.f;
        } else if (d == 1) {
          t = xc;
        } else {
          t = 2.f * xc * t1 - t0;
          t0 = t1;
          t1 = t;
        }
        sT[r][f][d] = t;
      }
      sS[r][f] = has_base ? silu_value<MODE_F32>(xc) : 0.f;
    }
    // the outputs' weight slices: [Wp (nf * p) | Wq (nf * q) | Wb (nf)]
    for (int e = tid; e < RCOLS * RF * (p + q + 1); e += RTH) {
      const int n = e / (RF * (p + q + 1)), o = e % (RF * (p + q + 1)), cc = col0 + n;
      float v = 0.f;
      if (cc < D_out) {
        if (o < RF * p) {
          if (o < nf * p) v = Wp[(size_t)cc * D_in * p + (size_t)i0 * p + o];
        } else if (o < RF * (p + q)) {
          const int oq = o - RF * p;
          if (oq < nf * q) v = Wq[(size_t)cc * D_in * q + (size_t)i0 * q + oq];
        } else if (has_base) {
          const int ob = o - RF * (p + q);
          if (ob < nf) v = Wb[(size_t)cc * D_in + i0 + ob];
        }
      }
      sw[n * wpitch + o] = v;
    }
    __syncthreads();
    const float* w = sw + lane * wpitch;
    for (int f = 0; f < nf; ++f) {
      if (has_base) acc = fmaf(sS[warp][f], w[RF * (p + q) + f], acc);
      float P = 0.f, Q = 0.f;
      for (int d = 0; d < p; ++d) P = fmaf(sT[warp][f][d], w[f * p + d], P);
      for (int d = 0; d < q; ++d) Q = fmaf(sT[warp][f][d], w[RF * p + f * q + d], Q);
      acc += P / (1.f + fabsf(Q));
    }
    __syncthreads();
  }
  if (row < B && col < D_out) Y[(size_t)row * D_out + col] = acc;
}

}  // namespace extra

static unsigned grid_1d(long long n, int threads) {
  long long b = (n + threads - 1) / threads;
  const long long cap = 148LL * 16;  // a few waves of the SMs; the kernel strides
  return (unsigned)(b < 1 ? 1 : (b > cap ? cap : b));
}

cudaError_t launch_mult_combine(const void* in, void* out, int B, int num_add, int num_mult,
                                int act_dtype, cudaStream_t s) {
  if (B <= 0) return cudaSuccess;
  const unsigned g = grid_1d((long long)B * (num_add + num_mult), 256);
  note_launch();
  if (act_dtype == KAN_F32) extra::mult_combine_kernel<MODE_F32><<<g, 256, 0, s>>>(in, out, B, num_add, num_mult);
  else if (act_dtype == KAN_F16) extra::mult_combine_kernel<MODE_F16><<<g, 256, 0, s>>>(in, out, B, num_add, num_mult);
  else extra::mult_combine_kernel<MODE_BF16><<<g, 256, 0, s>>>(in, out, B, num_add, num_mult);
  return cudaGetLastError();
}

cudaError_t launch_lowrank_up(const void* Z, const void* X, const void* Wup, const void* Wb,
                              const void* bias, void* Y, int B, int D_in, int D_out, int rank,
                              int has_base, int has_bias, int act_dtype, cudaStream_t s) {
  if (B <= 0) return cudaSuccess;
  const dim3 grid((unsigned)((D_out + extra::TN - 1) / extra::TN),
                  (unsigned)((B + extra::TM - 1) / extra::TM));
  note_launch();
  if (act_dtype == KAN_F32)
    extra::lowrank_up_kernel<MODE_F32><<<grid, extra::TH, 0, s>>>(Z, X, Wup, Wb, bias, Y, B, D_in, D_out, rank, has_base, has_bias);
  else if (act_dtype == KAN_F16)
    extra::lowrank_up_kernel<MODE_F16><<<grid, extra::TH, 0, s>>>(Z, X, Wup, Wb, bias, Y, B, D_in, D_out, rank, has_base, has_bias);
  else
    extra::lowrank_up_kernel<MODE_BF16><<<grid, extra::TH, 0, s>>>(Z, X, Wup, Wb, bias, Y, B, D_in, D_out, rank, has_base, has_bias);
  return cudaGetLastError();
}

bool rational_supported(int p, int q) {
  return p >= 0 && q >= 0 && p <= extra::RMAXD && q <= extra::RMAXD && p + q > 0 &&
         p + q <= 16;  // the weight slices stay within the default 48 KB of shared memory
}

cudaError_t launch_rational(const float* X, const float* Wp, const float* Wq, const float* Wb,
                            const float* bias, float* Y, int B, int D_in, int D_out, int p, int q,
                            int has_base, int has_bias, cudaStream_t s) {
  if (B <= 0) return cudaSuccess;
  if (!rational_supported(p, q)) return cudaErrorInvalidValue;
  const dim3 grid((unsigned)((D_out + extra::RCOLS - 1) / extra::RCOLS),
                  (unsigned)((B + extra::RROWS - 1) / extra::RROWS));
  const size_t smem = sizeof(float) * extra::RCOLS * (extra::RF * (p + q) + extra::RF + 1);
  note_launch();
  extra::rational_kernel<<<grid, extra::RTH, smem, s>>>(X, Wp, Wq, Wb, bias, Y, B, D_in, D_out,
                                                        p, q, has_base, has_bias);
  return cudaGetLastError();
}

}  // namespace kan
