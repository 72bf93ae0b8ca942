// kan_misc.cu -- elementwise kernels: weight dequantisation (all packed formats), SwiGLU gating
// and dtype conversion; plus the device error word shared by the bounded waits.
#include "kan_device.cuh"
#include "kan_launch.h"

namespace kan {

// Written by kernels whose bounded waits expire; read (and cleared) by kan_device_error().
__device__ int g_kan_device_error = 0;

// Grid-stride launch size: enough blocks to fill 148 SMs x 16, never more than the work.
static int grid_blocks(long long n) {
  long long b = (n + 255) / 256;
  if (b > 148LL * 16) b = 148LL * 16;
  return b < 1 ? 1 : (int)b;
}

int* device_error_ptr() {
  void* p = nullptr;
  if (cudaGetSymbolAddress(&p, g_kan_device_error) != cudaSuccess) return nullptr;
  return (int*)p;
}

template <typename TO>
__device__ __forceinline__ TO cvt_out(float v);
template <> __device__ __forceinline__ float cvt_out<float>(float v) { return v; }
template <> __device__ __forceinline__ __half cvt_out<__half>(float v) { return __float2half_rn(v); }
template <> __device__ __forceinline__ __nv_bfloat16 cvt_out<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}

// Dequantise a [rows, cols] weight (fused_kan.metal:2392-2441 for the 2-bit formats,
// metal_kan_bridge.mm:4213 / :4278 for INT8/INT4): exact fp32 value, then rounded to TO.
template <typename TO>
__global__ void dequant_kernel(kan_weight w, int rows, int cols, TO* out) {
  long long total = (long long)rows * cols;
  for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < total;
       e += (long long)gridDim.x * blockDim.x) {
    int r = (int)(e / cols), c = (int)(e - (long long)r * cols);
    out[e] = cvt_out<TO>(weight_value<MODE_F32>(w, r, c, cols));
  }
}

cudaError_t launch_dequantize(const kan_weight& w, int rows, int cols, void* out, int out_dtype,
                              cudaStream_t s) {
  note_launch();
  long long total = (long long)rows * cols;
  int blocks = grid_blocks(total);
  if (blocks < 1) blocks = 1;
  kan_weight wd = w;
  if (wd.format == KAN_W_DENSE) return cudaErrorInvalidValue;
  if (out_dtype == KAN_F32) dequant_kernel<float><<<blocks, 256, 0, s>>>(wd, rows, cols, (float*)out);
  else if (out_dtype == KAN_F16)
    dequant_kernel<__half><<<blocks, 256, 0, s>>>(wd, rows, cols, (__half*)out);
  else dequant_kernel<__nv_bfloat16><<<blocks, 256, 0, s>>>(wd, rows, cols, (__nv_bfloat16*)out);
  return cudaGetLastError();
}

// hidden = g * sigmoid(clamp(g, -20, 20)) * u  (fused_kan.metal:2284-2296), fp32 math.
template <int MODE>
__global__ void swiglu_kernel(const typename Act<MODE>::T* g, const typename Act<MODE>::T* u,
                              typename Act<MODE>::T* out, long long n) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x) {
    float gv = Act<MODE>::to_f(g[i]), uv = Act<MODE>::to_f(u[i]);
    float sig = 1.0f / (1.0f + expf(-fminf(fmaxf(gv, -20.0f), 20.0f)));
    out[i] = Act<MODE>::from_f((gv * sig) * uv);
  }
}

cudaError_t launch_swiglu(const void* g, const void* u, void* out, long long n, int dtype,
                          cudaStream_t s) {
  note_launch();
  int blocks = grid_blocks(n);
  if (blocks < 1) blocks = 1;
  if (dtype == KAN_F32)
    swiglu_kernel<MODE_F32><<<blocks, 256, 0, s>>>((const float*)g, (const float*)u, (float*)out, n);
  else if (dtype == KAN_F16)
    swiglu_kernel<MODE_F16><<<blocks, 256, 0, s>>>((const __half*)g, (const __half*)u,
                                                   (__half*)out, n);
  else
    swiglu_kernel<MODE_BF16><<<blocks, 256, 0, s>>>((const __nv_bfloat16*)g,
                                                    (const __nv_bfloat16*)u,
                                                    (__nv_bfloat16*)out, n);
  return cudaGetLastError();
}

template <typename TI, typename TO>
__global__ void convert_kernel(const TI* src, TO* dst, long long n) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x) {
    float v;
    if constexpr (sizeof(TI) == 4) v = (float)src[i];
    else if constexpr (std::is_same<TI, __half>::value) v = __half2float(src[i]);
    else v = __bfloat162float(src[i]);
    dst[i] = cvt_out<TO>(v);
  }
}

template <typename TI>
static cudaError_t convert_from(const TI* src, void* dst, int ddt, long long n, int blocks,
                                cudaStream_t s) {
  if (ddt == KAN_F32) convert_kernel<TI, float><<<blocks, 256, 0, s>>>(src, (float*)dst, n);
  else if (ddt == KAN_F16) convert_kernel<TI, __half><<<blocks, 256, 0, s>>>(src, (__half*)dst, n);
  else convert_kernel<TI, __nv_bfloat16><<<blocks, 256, 0, s>>>(src, (__nv_bfloat16*)dst, n);
  return cudaGetLastError();
}

cudaError_t launch_convert(const void* src, int sdt, void* dst, int ddt, long long n,
                           cudaStream_t s) {
  note_launch();
  int blocks = grid_blocks(n);
  if (blocks < 1) blocks = 1;
  if (sdt == KAN_F32) return convert_from((const float*)src, dst, ddt, n, blocks, s);
  if (sdt == KAN_F16) return convert_from((const __half*)src, dst, ddt, n, blocks, s);
  return convert_from((const __nv_bfloat16*)src, dst, ddt, n, blocks, s);
}

}  // namespace kan
