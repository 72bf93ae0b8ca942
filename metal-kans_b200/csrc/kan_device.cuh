// kan_device.cuh -- device-side building blocks shared by every KAN kernel.
//
// * activation-dtype traits (f32 / f16 / bf16),
// * the per-feature basis generators with the rounding points of the reference kernels
//   (Shuril/metal-kans metal_kans/kernels/fused_kan.metal, cited per generator),
// * weight decode (dense and the four packed formats of metal_kans/quantization.py),
// * the input maps (reference clamp, tanh, LayerNorm) and the device error word.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "../../include/kan_cuda.h"
#include "kan_args.h"

namespace kan {

// Generation modes: the arithmetic a basis value is produced with.
//   MODE_F32  - fp32 math (the reference's fp32 kernels)
//   MODE_F16  - the reference's *_fp16 kernels: half arithmetic where they use half, fp32 math
//               with a half store where they store half
//   MODE_BF16 - fp32 math, value rounded to bf16 (new; the reference has no bf16)
enum { MODE_F32 = 0, MODE_F16 = 1, MODE_BF16 = 2 };

template <int MODE> struct Act;
template <> struct Act<MODE_F32> {
  using T = float;
  static __device__ __forceinline__ float to_f(T v) { return v; }
  static __device__ __forceinline__ T from_f(float v) { return v; }
  static __device__ __forceinline__ float round(float v) { return v; }
};
template <> struct Act<MODE_F16> {
  using T = __half;
  static __device__ __forceinline__ float to_f(T v) { return __half2float(v); }
  static __device__ __forceinline__ T from_f(float v) { return __float2half_rn(v); }
  static __device__ __forceinline__ float round(float v) { return __half2float(__float2half_rn(v)); }
};
template <> struct Act<MODE_BF16> {
  using T = __nv_bfloat16;
  static __device__ __forceinline__ float to_f(T v) { return __bfloat162float(v); }
  static __device__ __forceinline__ T from_f(float v) { return __float2bfloat16_rn(v); }
  static __device__ __forceinline__ float round(float v) {
    return __bfloat162float(__float2bfloat16_rn(v));
  }
};


// ------------------------------------------------------------------------------------------
// device error word (bounded waits)
// ------------------------------------------------------------------------------------------
enum { DEVERR_TIMEOUT_FULL_A = 1, DEVERR_TIMEOUT_FULL_B = 2, DEVERR_TIMEOUT_EMPTY = 3,
       DEVERR_TIMEOUT_ACCUM = 4 };

__device__ __forceinline__ void raise_device_error(int* err, int code) {
  if (err) atomicCAS(err, 0, code);
}

// ------------------------------------------------------------------------------------------
// input maps
// ------------------------------------------------------------------------------------------
// The mapped value is handed to the basis in the activation dtype (rounded once).
template <int MODE>
__device__ __forceinline__ float map_input(float x, int input_map, float mean, float rstd) {
  if (input_map == KAN_MAP_TANH) return Act<MODE>::round(tanhf(x));
  if (input_map == KAN_MAP_LAYERNORM) return Act<MODE>::round((x - mean) * rstd);
  return x;
}

// ------------------------------------------------------------------------------------------
// SiLU of the base branch (applied to the mapped input)
// ------------------------------------------------------------------------------------------
// fp32: x / (1 + exp(-x))                         fused_kan.metal:116-138
// fp16: x / (1.0h + exp(-x)), three half roundings fused_kan.metal:1373-1397
// The quotient uses the fast reciprocal (within 2 ulp of fp32); for the f16/bf16 modes the
// result is then rounded to the operand dtype, for fp32 it stays far inside the 1e-5 budget.
template <int MODE>
__device__ __forceinline__ float silu_value(float x) {
  if (MODE == MODE_F16) {
    __half e = __float2half_rn(__expf(-x));
    __half d = __hadd(__float2half_rn(1.0f), e);
    return __half2float(__float2half_rn(__fdividef(x, __half2float(d))));
  }
  return Act<MODE>::round(__fdividef(x, 1.0f + __expf(-x)));
}

// ------------------------------------------------------------------------------------------
// basis generators: one object per (row, feature); term(k) is called for k = 0, 1, 2, ... in
// order (the Chebyshev recurrence relies on it).
// ------------------------------------------------------------------------------------------

// Chebyshev T_k(clamp(x, -1, 1)), K terms.  fp32: recurrence 2x T1 - T0 (fused_kan.metal:
// 205-238); fp16: fp32 recurrence fma(2x, T1, -T0) stored as half (:1399-1426).
template <int MODE>
struct ChebyGen {
  float x2, t0, t1;
  int k;
  __device__ __forceinline__ void init(float xm, int /*feature*/, const LayerArgs& /*a*/) {
    float xc = fminf(fmaxf(xm, -1.0f), 1.0f);
    x2 = 2.0f * xc;
    t0 = 1.0f;
    t1 = xc;
    k = 0;
  }
  __device__ __forceinline__ float next() {
    float v;
    if (k == 0) v = t0;
    else if (k == 1) v = t1;
    else {
      float t2 = fmaf(x2, t1, -t0);
      t0 = t1;
      t1 = t2;
      v = t2;
    }
    ++k;
    return Act<MODE>::round(v);
  }
};

// Gaussian RBF exp(-(x - c_k)^2 * inv_den).  fp32: fused_kan.metal:140-166; fp16 (:1428-1450):
// diff, -diff*diff and *inv_den in half arithmetic, exp of the half argument stored as half.
template <int MODE>
struct RbfGen {
  float x;
  const float* grid;
  float inv_den;
  int k;
  __device__ __forceinline__ void init(float xm, int, const LayerArgs& a) {
    x = xm;
    grid = a.grid;
    inv_den = a.inv_den;
    k = 0;
  }
  __device__ __forceinline__ float next() {
    float c = __ldg(grid + k);
    ++k;
    if (MODE == MODE_F16) {
      __half diff = __hsub(__float2half_rn(x), __float2half_rn(c));
      __half sq = __hmul(__hneg(diff), diff);
      __half t = __hmul(sq, __float2half_rn(inv_den));
      return __half2float(__float2half_rn(__expf(__half2float(t))));
    }
    float d = x - c;
    return Act<MODE>::round(__expf(-(d * d) * inv_den));
  }
};

// Closed-form uniform cubic B-spline, G+3 bases (fused_kan.metal:240-276; fp16 :1476-1512 uses the
// same fp32 math and stores half).  span = clamp(floor(pos), 0, G-1), u = clamp(pos-span, 0, 1).
template <int MODE>
struct BsplineGen {
  float b0, b1, b2, b3;
  int span, k;
  // The four nonzero terms (before rounding to the operand dtype) and the span of a mapped input.
  __device__ __forceinline__ static void terms(float xm, const LayerArgs& a, float& t0, float& t1,
                                               float& t2, float& t3, int& s) {
    float pos = (xm - a.grid_min) * a.inv_h;
    float fl = floorf(pos);
    s = (int)fminf(fmaxf(fl, 0.0f), (float)(a.grid_size - 1));
    float u = fminf(fmaxf(pos - (float)s, 0.0f), 1.0f);
    float om = 1.0f - u;
    const float inv6 = 1.0f / 6.0f;
    float u2 = u * u, u3 = u2 * u;
    t0 = om * om * om * inv6;
    t1 = (3.0f * u3 - 6.0f * u2 + 4.0f) * inv6;
    t2 = (-3.0f * u3 + 3.0f * u2 + 3.0f * u + 1.0f) * inv6;
    t3 = u3 * inv6;
  }
  __device__ __forceinline__ void init(float xm, int, const LayerArgs& a) {
    terms(xm, a, b0, b1, b2, b3, span);
    b0 = Act<MODE>::round(b0);
    b1 = Act<MODE>::round(b1);
    b2 = Act<MODE>::round(b2);
    b3 = Act<MODE>::round(b3);
    k = 0;
  }
  __device__ __forceinline__ float next() {
    int d = k - span;
    ++k;
    float v = 0.0f;
    v = (d == 0) ? b0 : v;
    v = (d == 1) ? b1 : v;
    v = (d == 2) ? b2 : v;
    v = (d == 3) ? b3 : v;
    return v;
  }
};

// Wavelets psi((x - t) * inv_s).  fp32 (fused_kan.metal:168-203): mexican hat (1-z^2) e^{-z^2/2},
// morlet cos(5z) e^{-z^2/2}, dog -z e^{-z^2/2}.  fp16 (:1514-1548): every step in half, and the
// Morlet frequency is 1.75 (the reference's half kernel differs from its fp32 one; mirrored).
template <int MODE>
struct WaveletGen {
  float x;
  const float* tr;
  const float* sc;
  int wtype, k;
  __device__ __forceinline__ void init(float xm, int feature, const LayerArgs& a) {
    x = xm;
    tr = a.translation + (size_t)feature * a.K;
    sc = a.inv_scale + (size_t)feature * a.K;
    wtype = a.wavelet_type;
    k = 0;
  }
  __device__ __forceinline__ float next() {
    float t = __ldg(tr + k), s = __ldg(sc + k);
    ++k;
    if (MODE == MODE_F16) {
      __half z = __hmul(__hsub(__float2half_rn(x), __float2half_rn(t)), __float2half_rn(s));
      __half ar = __hmul(__hmul(__float2half_rn(-0.5f), z), z);
      __half e = __float2half_rn(__expf(__half2float(ar)));
      __half psi;
      if (wtype == 0) psi = __hmul(__hsub(__float2half_rn(1.0f), __hmul(z, z)), e);
      else if (wtype == 1)
        psi = __hmul(__float2half_rn(cosf(__half2float(__hmul(__float2half_rn(1.75f), z)))), e);
      else psi = __hmul(__hneg(z), e);
      return __half2float(psi);
    }
    float z = (x - t) * s;
    float e = __expf(-0.5f * z * z);
    float psi;
    if (wtype == 0) psi = (1.0f - z * z) * e;
    else if (wtype == 1) psi = cosf(5.0f * z) * e;
    else psi = -z * e;
    return Act<MODE>::round(psi);
  }
};

// Tent (ReLUKAN) max(0, 1 - |x - g_k| inv_h) on the raw input (fused_kan.metal:278-303); fp16
// (:1452-1474): the difference, its magnitude, the product by half(inv_h) and 1 - that in half.
template <int MODE>
struct ReluGen {
  float x, inv_h;
  const float* grid;
  int k;
  __device__ __forceinline__ void init(float xm, int, const LayerArgs& a) {
    x = xm;
    grid = a.grid;
    inv_h = a.inv_h;
    k = 0;
  }
  __device__ __forceinline__ float next() {
    const float g = __ldg(grid + k);
    ++k;
    if (MODE == MODE_F16) {
      const __half d = __habs(__hsub(__float2half_rn(x), __float2half_rn(g)));
      const __half t = __hmul(d, __float2half_rn(inv_h));
      return __half2float(__hmax(__float2half_rn(0.0f), __hsub(__float2half_rn(1.0f), t)));
    }
    return Act<MODE>::round(fmaxf(0.0f, 1.0f - fabsf(x - g) * inv_h));
  }
};

// Fourier (FourierKAN) 1, cos(pi x), sin(pi x), ..., cos(F pi x), sin(F pi x) on the raw input
// (fused_kan.metal:306-329: angle (f pi) x in fp32); fp16 (:1550-1576): pi x and f (pi x) in
// half, the cosine and sine of that half angle stored as half.
template <int MODE>
struct FourierGen {
  float x, s;
  int k;
  __device__ __forceinline__ void init(float xm, int, const LayerArgs&) {
    x = xm;
    k = 0;
    s = 0.0f;
  }
  __device__ __forceinline__ float next() {
    const int kk = k++;
    if (kk == 0) return 1.0f;
    if ((kk & 1) == 0) return s;  // sin of the angle whose cos came just before
    const int f = (kk + 1) >> 1;
    float angle;
    if (MODE == MODE_F16) {
      const __half pix = __hmul(__float2half_rn(3.14159265358979f), __float2half_rn(x));
      angle = __half2float(__hmul(__float2half_rn((float)f), pix));
    } else {
      angle = ((float)f * 3.14159265358979f) * x;
    }
    float c;
    sincosf(angle, &s, &c);
    s = Act<MODE>::round(s);
    return Act<MODE>::round(c);
  }
};

// Jacobi P_k^(alpha, beta)(clamp(x, -1, 1)) by the three-term recurrence (fused_kan.metal:331-366;
// fp16 :1578-1613: the same fp32 recurrence, fma form, half store).
template <int MODE>
struct JacobiGen {
  float x, alpha, beta, p0, p1;
  int k;
  __device__ __forceinline__ void init(float xm, int, const LayerArgs& a) {
    x = fminf(fmaxf(xm, -1.0f), 1.0f);
    alpha = a.alpha;
    beta = a.beta;
    p0 = 1.0f;
    p1 = 0.0f;
    k = 0;
  }
  __device__ __forceinline__ float next() {
    const int n = k++;
    const float ab = alpha + beta;
    if (n == 0) return Act<MODE>::round(1.0f);
    if (n == 1) {
      p1 = 0.5f * (alpha - beta + (ab + 2.0f) * x);
      return Act<MODE>::round(p1);
    }
    const float fn = (float)n;
    const float an = 2.0f * fn * (fn + ab) * (2.0f * fn + ab - 2.0f);
    const float bn1 = (2.0f * fn + ab - 1.0f) * (2.0f * fn + ab) * (2.0f * fn + ab - 2.0f);
    const float bn2 = (2.0f * fn + ab - 1.0f) * (alpha * alpha - beta * beta);
    const float cn = 2.0f * (fn + alpha - 1.0f) * (fn + beta - 1.0f) * (2.0f * fn + ab);
    const float p = fmaf(fmaf(bn1, x, bn2), p1, -cn * p0) / an;
    p0 = p1;
    p1 = p;
    return Act<MODE>::round(p);
  }
};

template <int BASIS, int MODE> struct GenFor;
template <int MODE> struct GenFor<KAN_CHEBY, MODE> { using type = ChebyGen<MODE>; };
template <int MODE> struct GenFor<KAN_RBF, MODE> { using type = RbfGen<MODE>; };
template <int MODE> struct GenFor<KAN_BSPLINE, MODE> { using type = BsplineGen<MODE>; };
template <int MODE> struct GenFor<KAN_WAVELET, MODE> { using type = WaveletGen<MODE>; };
template <int MODE> struct GenFor<KAN_RELU, MODE> { using type = ReluGen<MODE>; };
template <int MODE> struct GenFor<KAN_FOURIER, MODE> { using type = FourierGen<MODE>; };
template <int MODE> struct GenFor<KAN_JACOBI, MODE> { using type = JacobiGen<MODE>; };

// Number of basis kinds (kan_basis), for dispatch tables.
constexpr int NUM_BASES = 7;

// ------------------------------------------------------------------------------------------
// weight decode: element (row, col) of a kan_weight as the exact fp32 value the reference's
// dequantiser produces (separate fp32 multiply and add; metal_kan_bridge.mm:4213-4232,
// :4278-4302, fused_kan.metal:2392-2441).  Dense weights are converted from the act dtype.
// ------------------------------------------------------------------------------------------
template <int MODE>
__device__ __forceinline__ float weight_value(const kan_weight& w, int row, int col, int cols) {
  switch (w.format) {
    case KAN_W_DENSE: {
      const typename Act<MODE>::T* p = (const typename Act<MODE>::T*)w.data;
      return Act<MODE>::to_f(p[(size_t)row * cols + col]);
    }
    case KAN_W_INT8:
    case KAN_W_INT4: {
      size_t e = (size_t)row * w.padded_cols + col;
      size_t g = e / (unsigned)w.group_size;
      int q;
      if (w.format == KAN_W_INT8) q = ((const uint8_t*)w.data)[e];
      else {
        uint8_t byte = ((const uint8_t*)w.data)[e >> 1];
        q = (e & 1) ? (byte >> 4) : (byte & 0xF);
      }
      return __fadd_rn(__fmul_rn((float)q, __ldg(w.scales + g)), __ldg(w.biases + g));
    }
    default: {  // 2-bit formats
      int words = (cols + 15) >> 4;
      int groups = (cols + w.group_size - 1) / w.group_size;
      uint32_t word = ((const uint32_t*)w.data)[(size_t)row * words + (col >> 4)];
      uint32_t code = (word >> ((col & 15) * 2)) & 3u;
      float s = __ldg(w.scales + (size_t)row * groups + col / w.group_size);
      float v;
      if (w.format == KAN_W_TERNARY) v = (code == 3u) ? 0.0f : (float)code - 1.0f;
      else v = __ldg(w.codebook + code);
      return __fmul_rn(v, s);
    }
  }
}

}  // namespace kan
