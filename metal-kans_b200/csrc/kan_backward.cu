// kan_backward.cu -- fused backward of a KAN layer (fp32, CUDA cores): dW, dW_base, dbias, dX.
//
// For y = bias + silu(x) Wb^T + Phi(x) W^T (Phi[b, i*K + k] = phi_k(x[b, i])):
//   dW[j, i*K + k] = sum_b dY[b, j] phi_k(x[b, i])        dWb[j, i] = sum_b dY[b, j] silu(x[b, i])
//   dbias[j]       = sum_b dY[b, j]
//   dX[b, i]       = sum_k phi_k'(x[b, i]) sum_j dY[b, j] W[j, i*K + k]
//                    + silu'(x[b, i]) sum_j dY[b, j] Wb[j, i]
// The reference evaluates Phi into a scratch buffer, runs three GEMMs (dY^T Phi, dY W and the
// base-branch pair) and a basis-derivative kernel over the materialised dPhi
// (metal_kan_bridge.mm:2715-2846; the fused Chebyshev variant :4532 streams the batch per
// weight, fused_kan.metal:2053-2163).  Here neither Phi nor dPhi reaches memory:
//
//   * dW: a CTA owns 64 outputs x F whole input features (F = 64 / (K + has_base): the K basis
//     columns of each feature, then its base column -- the tensor-core weight layout's blocking).
//     It walks the batch 16 rows at a time: the dY^T chunk and the basis values (and silu) of its
//     features for those rows are built in shared memory, and each thread accumulates a 4 x 4
//     register tile.  The epilogue scatters the tile to dW and dWb.
//   * dX: a CTA owns 64 batch rows x F features and walks D_out 16 outputs at a time with the dY
//     chunk and its features' weights (gathered from W and W_base) in shared memory; the 64 x
//     F*(K+1) sums then meet the basis derivatives and silu'(x) in the epilogue, giving dX in one
//     pass.
//   * dbias: column sums of dY.
//
// Derivatives follow the reference kernels (fused_kan.metal:1679-1882): Chebyshev on the clamped
// input, with the basis part zero outside [-1, 1]; Gaussian -2 (x - c) inv_den phi; tents
// -sign(x - g) inv_h where positive; the cubic
// B-spline pieces differentiated in u times inv_h on the clamped span; silu'(x) =
// sigma (1 + x (1 - sigma)) of the raw input.
#include "kan_device.cuh"
#include "kan_launch.h"

namespace kan {
namespace bwd {

constexpr int TILE = 64;     // outputs (dW) or batch rows (dX) per CTA, and padded columns
constexpr int CH = 16;       // reduction chunk (batch rows for dW, outputs for dX)
constexpr int PITCH = TILE + 4;
constexpr int THREADS = 256;

__device__ __forceinline__ float sigmoidf(float x) { return 1.0f / (1.0f + __expf(-x)); }

// Basis values phi_k(x) (k < K) of the forward's fp32 mode and their derivatives.
template <int BASIS>
__device__ __forceinline__ void basis_and_grad(const BackwardArgs& a, float x, float* phi,
                                               float* dphi) {
  if (BASIS == KAN_CHEBY) {
    const float xc = fminf(fmaxf(x, -1.0f), 1.0f);
    const bool inside = x >= -1.0f && x <= 1.0f;
    float t0 = 1.0f, t1 = xc, d0 = 0.0f, d1 = 1.0f;
    for (int k = 0; k < a.K; ++k) {
      float t, d;
      if (k == 0) {
        t = 1.0f;
        d = 0.0f;
      } else if (k == 1) {
        t = xc;
        d = 1.0f;
      } else {
        t = fmaf(2.0f * xc, t1, -t0);
        d = fmaf(2.0f * xc, d1, fmaf(2.0f, t1, -d0));
        t0 = t1;
        t1 = t;
        d0 = d1;
        d1 = d;
      }
      if (phi) phi[k] = t;
      if (dphi) dphi[k] = inside ? d : 0.0f;
    }
  } else if (BASIS == KAN_RBF) {
    for (int k = 0; k < a.K; ++k) {
      const float d = x - __ldg(a.grid + k);
      const float p = __expf(-(d * d) * a.inv_den);
      if (phi) phi[k] = p;
      if (dphi) dphi[k] = -2.0f * d * a.inv_den * p;
    }
  } else if (BASIS == KAN_RELU) {
    // tent: derivative -sign(x - g) inv_h where the tent is positive (fused_kan.metal:1787-1826)
    for (int k = 0; k < a.K; ++k) {
      const float d = x - __ldg(a.grid + k);
      const float v = 1.0f - fabsf(d) * a.inv_h;
      if (phi) phi[k] = fmaxf(0.0f, v);
      if (dphi) dphi[k] = v > 0.0f ? (d > 0.0f ? -a.inv_h : (d < 0.0f ? a.inv_h : 0.0f)) : 0.0f;
    }
  } else {  // cubic B-spline, G + 3 bases
    const float pos = (x - a.grid_min) * a.inv_h;
    const int span = (int)fminf(fmaxf(floorf(pos), 0.0f), (float)(a.grid_size - 1));
    const float u = fminf(fmaxf(pos - (float)span, 0.0f), 1.0f);
    const float om = 1.0f - u, u2 = u * u, u3 = u2 * u;
    const float inv6 = 1.0f / 6.0f;
    const float b[4] = {om * om * om * inv6, (3.0f * u3 - 6.0f * u2 + 4.0f) * inv6,
                        (-3.0f * u3 + 3.0f * u2 + 3.0f * u + 1.0f) * inv6, u3 * inv6};
    const float db[4] = {-0.5f * om * om * a.inv_h, (1.5f * u2 - 2.0f * u) * a.inv_h,
                         (-1.5f * u2 + u + 0.5f) * a.inv_h, 0.5f * u2 * a.inv_h};
    for (int k = 0; k < a.K; ++k) {
      const int d = k - span;
      const bool on = d >= 0 && d < 4;
      if (phi) phi[k] = on ? b[d] : 0.0f;
      if (dphi) dphi[k] = on ? db[d] : 0.0f;
    }
  }
}

// dW / dWb tile: 64 outputs x F features, batch in chunks of 16 rows.
template <int BASIS>
__global__ void __launch_bounds__(THREADS) bwd_dw_kernel(BackwardArgs a) {
  __shared__ __align__(16) float dYs[CH][PITCH];  // [batch row][output]
  __shared__ __align__(16) float Ps[CH][PITCH];   // [batch row][feature-blocked column]
  const int KT = a.K + (a.has_base ? 1 : 0);
  const int F = max(1, TILE / KT);
  const int j0 = blockIdx.x * TILE, i0 = blockIdx.y * F;
  const int tid = threadIdx.x, tj = tid / 16, tc = tid % 16;
  float acc[4][4];
#pragma unroll
  for (int p = 0; p < 4; ++p)
#pragma unroll
    for (int q = 0; q < 4; ++q) acc[p][q] = 0.f;
  float phi[64];

  for (int b0 = 0; b0 < a.B; b0 += CH) {
    for (int e = tid; e < CH * TILE; e += THREADS) {
      const int bb = e / TILE, jj = e % TILE;
      const int b = b0 + bb, j = j0 + jj;
      dYs[bb][jj] = (b < a.B && j < a.D_out) ? a.dY[(size_t)b * a.D_out + j] : 0.f;
    }
    for (int e = tid; e < CH * TILE; e += THREADS) {
      // columns past F * KT stay zero; the items below overwrite the real ones
      const int bb = e / TILE, c = e % TILE;
      if (c >= F * KT) Ps[bb][c] = 0.f;
    }
    for (int it = tid; it < CH * F; it += THREADS) {
      const int bb = it / F, f = it % F;
      const int b = b0 + bb, i = i0 + f;
      float* dst = &Ps[bb][f * KT];
      if (b < a.B && i < a.D_in) {
        const float x = a.X[(size_t)b * a.D_in + i];
        basis_and_grad<BASIS>(a, x, phi, nullptr);
        for (int k = 0; k < a.K; ++k) dst[k] = phi[k];
        if (a.has_base) dst[a.K] = x * sigmoidf(x);
      } else {
        for (int k = 0; k < KT; ++k) dst[k] = 0.f;
      }
    }
    __syncthreads();
#pragma unroll 4
    for (int bb = 0; bb < CH; ++bb) {
      const float4 y4 = *reinterpret_cast<const float4*>(&dYs[bb][tj * 4]);
      const float4 p4 = *reinterpret_cast<const float4*>(&Ps[bb][tc * 4]);
      const float yv[4] = {y4.x, y4.y, y4.z, y4.w}, pv[4] = {p4.x, p4.y, p4.z, p4.w};
#pragma unroll
      for (int p = 0; p < 4; ++p)
#pragma unroll
        for (int q = 0; q < 4; ++q) acc[p][q] = fmaf(yv[p], pv[q], acc[p][q]);
    }
    __syncthreads();
  }
  const int Kw = a.D_in * a.K;
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const int c = tc * 4 + q;
    const int f = c / KT, t = c - f * KT, i = i0 + f;
    if (f >= F || i >= a.D_in) continue;
#pragma unroll
    for (int p = 0; p < 4; ++p) {
      const int j = j0 + tj * 4 + p;
      if (j >= a.D_out) continue;
      if (t < a.K) {
        if (a.dW) a.dW[(size_t)j * Kw + i * a.K + t] = acc[p][q];
      } else if (a.dWb) {
        a.dWb[(size_t)j * a.D_in + i] = acc[p][q];
      }
    }
  }
}

// dX tile: 64 batch rows x F features, outputs in chunks of 16.
template <int BASIS>
__global__ void __launch_bounds__(THREADS) bwd_dx_kernel(BackwardArgs a) {
  __shared__ __align__(16) float dYs[CH][PITCH];  // [output][batch row]
  __shared__ __align__(16) float Ws[CH][PITCH];   // [output][feature-blocked column]
  __shared__ __align__(16) float G[TILE][PITCH];  // [batch row][column]: the contracted sums
  const int KT = a.K + (a.has_base ? 1 : 0);
  const int F = max(1, TILE / KT);
  const int i0 = blockIdx.x * F, b0 = blockIdx.y * TILE;
  const int tid = threadIdx.x, tb = tid / 16, tc = tid % 16;
  const int Kw = a.D_in * a.K;
  float acc[4][4];
#pragma unroll
  for (int p = 0; p < 4; ++p)
#pragma unroll
    for (int q = 0; q < 4; ++q) acc[p][q] = 0.f;

  for (int j0 = 0; j0 < a.D_out; j0 += CH) {
    for (int e = tid; e < CH * TILE; e += THREADS) {
      const int bb = e / CH, jj = e % CH;  // consecutive threads walk an output row of dY
      const int b = b0 + bb, j = j0 + jj;
      dYs[jj][bb] = (b < a.B && j < a.D_out) ? a.dY[(size_t)b * a.D_out + j] : 0.f;
    }
    for (int e = tid; e < CH * TILE; e += THREADS) {
      const int jj = e / TILE, c = e % TILE;
      const int j = j0 + jj;
      const int f = c / KT, t = c - f * KT, i = i0 + f;
      float w = 0.f;
      if (j < a.D_out && f < F && i < a.D_in)
        w = t < a.K ? a.W[(size_t)j * Kw + i * a.K + t] : a.Wb[(size_t)j * a.D_in + i];
      Ws[jj][c] = w;
    }
    __syncthreads();
#pragma unroll 4
    for (int jj = 0; jj < CH; ++jj) {
      const float4 y4 = *reinterpret_cast<const float4*>(&dYs[jj][tb * 4]);
      const float4 w4 = *reinterpret_cast<const float4*>(&Ws[jj][tc * 4]);
      const float yv[4] = {y4.x, y4.y, y4.z, y4.w}, wv[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
      for (int p = 0; p < 4; ++p)
#pragma unroll
        for (int q = 0; q < 4; ++q) acc[p][q] = fmaf(yv[p], wv[q], acc[p][q]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int p = 0; p < 4; ++p)
#pragma unroll
    for (int q = 0; q < 4; ++q) G[tb * 4 + p][tc * 4 + q] = acc[p][q];
  __syncthreads();
  float dphi[64];
  for (int it = tid; it < TILE * F; it += THREADS) {
    const int bb = it / F, f = it % F;
    const int b = b0 + bb, i = i0 + f;
    if (b >= a.B || i >= a.D_in) continue;
    const float x = a.X[(size_t)b * a.D_in + i];
    basis_and_grad<BASIS>(a, x, nullptr, dphi);
    const float* g = &G[bb][f * KT];
    float dx = 0.f;
    for (int k = 0; k < a.K; ++k) dx = fmaf(g[k], dphi[k], dx);
    if (a.has_base) {
      const float s = sigmoidf(x);
      dx = fmaf(g[a.K], s * (1.0f + x * (1.0f - s)), dx);
    }
    a.dX[(size_t)b * a.D_in + i] = dx;
  }
}

__global__ void bwd_dbias_kernel(BackwardArgs a) {
  const int j = blockIdx.x * blockDim.x + threadIdx.x;
  if (j >= a.D_out) return;
  float s = 0.f;
  for (int b = 0; b < a.B; ++b) s += a.dY[(size_t)b * a.D_out + j];
  a.dbias[j] = s;
}

// d_gate, d_up of hidden = silu(gate) * up, the SiLU argument clamped to +-20 in sigma
// (fused_kan.metal:2298-2316).
__global__ void swiglu_backward_kernel(const float* dh, const float* g, const float* u, float* dg,
                                       float* du, long long n) {
  for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < n;
       e += (long long)gridDim.x * blockDim.x) {
    const float gv = g[e], uv = u[e], d = dh[e];
    const float s = 1.0f / (1.0f + expf(-fminf(fmaxf(gv, -20.0f), 20.0f)));
    du[e] = d * (gv * s);
    dg[e] = d * uv * (s * (1.0f + gv * (1.0f - s)));
  }
}

}  // namespace bwd

bool backward_supported(const BackwardArgs& a) {
  if (a.basis != KAN_CHEBY && a.basis != KAN_RBF && a.basis != KAN_BSPLINE && a.basis != KAN_RELU)
    return false;
  if (a.K < 1 || a.K + (a.has_base ? 1 : 0) > 64 || a.B < 0 || a.D_in < 1 || a.D_out < 1)
    return false;
  if ((a.basis == KAN_RBF || a.basis == KAN_RELU) && !a.grid) return false;
  if (a.basis == KAN_BSPLINE && (a.grid_size < 1 || a.K != a.grid_size + 3)) return false;
  return true;
}

cudaError_t launch_backward(const BackwardArgs& a, cudaStream_t s) {
  using namespace bwd;
  if (a.B == 0) return cudaSuccess;
  const int KT = a.K + (a.has_base ? 1 : 0);
  const int F = TILE / KT > 0 ? TILE / KT : 1;
  const unsigned fblocks = (unsigned)((a.D_in + F - 1) / F);
  if (a.dW || a.dWb) {
    const dim3 grid((unsigned)((a.D_out + TILE - 1) / TILE), fblocks);
    note_launch();
    if (a.basis == KAN_CHEBY) bwd_dw_kernel<KAN_CHEBY><<<grid, THREADS, 0, s>>>(a);
    else if (a.basis == KAN_RBF) bwd_dw_kernel<KAN_RBF><<<grid, THREADS, 0, s>>>(a);
    else if (a.basis == KAN_RELU) bwd_dw_kernel<KAN_RELU><<<grid, THREADS, 0, s>>>(a);
    else bwd_dw_kernel<KAN_BSPLINE><<<grid, THREADS, 0, s>>>(a);
  }
  if (a.dX) {
    const dim3 grid(fblocks, (unsigned)((a.B + TILE - 1) / TILE));
    note_launch();
    if (a.basis == KAN_CHEBY) bwd_dx_kernel<KAN_CHEBY><<<grid, THREADS, 0, s>>>(a);
    else if (a.basis == KAN_RBF) bwd_dx_kernel<KAN_RBF><<<grid, THREADS, 0, s>>>(a);
    else if (a.basis == KAN_RELU) bwd_dx_kernel<KAN_RELU><<<grid, THREADS, 0, s>>>(a);
    else bwd_dx_kernel<KAN_BSPLINE><<<grid, THREADS, 0, s>>>(a);
  }
  if (a.dbias) {
    note_launch();
    bwd_dbias_kernel<<<(a.D_out + 255) / 256, 256, 0, s>>>(a);
  }
  return cudaGetLastError();
}

cudaError_t launch_swiglu_backward(const float* dh, const float* g, const float* u, float* dg,
                                   float* du, long long n, cudaStream_t s) {
  if (n <= 0) return cudaSuccess;
  long long blocks = (n + 255) / 256;
  if (blocks > 148LL * 16) blocks = 148LL * 16;
  note_launch();
  bwd::swiglu_backward_kernel<<<(unsigned)blocks, 256, 0, s>>>(dh, g, u, dg, du, n);
  return cudaGetLastError();
}

}  // namespace kan
