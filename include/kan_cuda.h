/*
 * kan_cuda.h -- C ABI of libkan_cuda.so, the B200 (sm_100a) KAN inference engine.
 *
 * Two tiers:
 *
 *  1. Reference-compatible entry points.  Same names, argument order and meaning as the
 *     `extern "C"` functions of the reference bridge (Shuril/metal-kans,
 *     metal_kans/kernels/metal_kan_bridge.mm), which its ctypes loader binds in
 *     metal_kans/device.py:64-474.  All pointers are HOST pointers (C-contiguous, owned by the
 *     caller); fp16 arrays are passed as uint16_t.  Every operand is staged to the device, the
 *     result is copied back, and the call returns 0 on success or a negative status.  Unlike the
 *     reference, failures are never silent: a non-zero status comes with kan_last_error().
 *
 *  2. Device-resident entry points (new, prefix kan_).  Pointers are DEVICE pointers; work is
 *     enqueued on the given cudaStream_t (passed as void*, NULL = the library's stream of the
 *     current device) and the call returns without synchronising.
 *
 * Status codes are the KAN_ERR_* values below.  Nothing here falls back to a CPU path: without a
 * CUDA device every compute entry point returns KAN_ERR_NO_DEVICE.
 */
#ifndef KAN_CUDA_H_
#define KAN_CUDA_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------------------------------------ */
/* status                                                                                      */
/* ------------------------------------------------------------------------------------------ */
#define KAN_OK 0
#define KAN_ERR_ARG (-1)           /* bad pointer / size / enum                                 */
#define KAN_ERR_CUDA (-2)          /* a CUDA runtime/driver call failed                         */
#define KAN_ERR_UNSUPPORTED (-3)   /* valid request with no kernel for it                       */
#define KAN_ERR_NO_DEVICE (-4)     /* no CUDA device visible                                    */
#define KAN_ERR_DEVICE_TIMEOUT (-5)/* a kernel's bounded wait expired (kan_device_error())      */

/* Message of the last failing call on this thread ("" if none). */
const char* kan_last_error(void);
/* ABI version (major*100 + minor). */
int kan_abi_version(void);

/* ------------------------------------------------------------------------------------------ */
/* tier 1: reference-compatible, host pointers                                                */
/* ------------------------------------------------------------------------------------------ */

/* metal_kan_bridge.mm:289 metal_kan_init(const char* shader_path): the path is ignored (there is
 * no runtime shader compilation); initialises the current CUDA device. */
int metal_kan_init(const char* shader_path);
/* metal_kan_bridge.mm:275 / :280 -- async mode: forwards enqueue and return; metal_kan_sync()
 * waits and completes the pending host copies. */
int metal_kan_set_async(int enabled);
int metal_kan_sync(void);

/* metal_kan_bridge.mm:443 */
int metal_kan_cheby_forward(const float* X, const float* W_cheby, const float* W_base,
                            const float* bias, float* Y, int B, int D_in, int D_out, int K,
                            int has_base, int has_bias);
/* metal_kan_bridge.mm:1890 */
int metal_kan_cheby_forward_fp16(const uint16_t* X, const uint16_t* W_cheby,
                                 const uint16_t* W_base, const uint16_t* bias, uint16_t* Y, int B,
                                 int D_in, int D_out, int K, int has_base, int has_bias);
/* metal_kan_bridge.mm:532 */
int metal_kan_fastkan_forward(const float* X, const float* W_rbf, const float* W_base,
                              const float* grid, const float* bias, float* Y, int B, int D_in,
                              int D_out, int num_centers, float inv_denominator, int has_base,
                              int has_bias);
/* metal_kan_bridge.mm:1973 (grid is fp16 here, like the reference) */
int metal_kan_fastkan_forward_fp16(const uint16_t* X, const uint16_t* W_rbf,
                                   const uint16_t* W_base, const uint16_t* grid,
                                   const uint16_t* bias, uint16_t* Y, int B, int D_in, int D_out,
                                   int num_centers, float inv_denominator, int has_base,
                                   int has_bias);
/* metal_kan_bridge.mm:1069 (grid = {grid_min, inv_h}, float32; spline_order is ignored: the
 * reference evaluates closed-form uniform cubics whatever the order) */
int metal_kan_bspline_forward(const float* X, const float* W_spline, const float* W_base,
                              const float* grid, const float* bias, float* Y, int B, int D_in,
                              int D_out, int grid_size, int spline_order, int has_base,
                              int has_bias);
/* metal_kan_bridge.mm:2062 (grid stays float32, like the reference) */
int metal_kan_bspline_forward_fp16(const uint16_t* X, const uint16_t* W_spline,
                                   const uint16_t* W_base, const float* grid,
                                   const uint16_t* bias, uint16_t* Y, int B, int D_in, int D_out,
                                   int grid_size, int spline_order, int has_base, int has_bias);
/* metal_kan_bridge.mm:722 (wavelet_type 0 mexican hat, 1 morlet, 2 dog) */
int metal_kan_wavkan_forward(const float* X, const float* W_wav, const float* W_base,
                             const float* translation, const float* inv_scale, const float* bias,
                             float* Y, int B, int D_in, int D_out, int num_wavelets,
                             int wavelet_type, int has_base, int has_bias);
/* metal_kan_bridge.mm:2448 */
int metal_kan_wavkan_forward_fp16(const uint16_t* X, const uint16_t* W_wav,
                                  const uint16_t* W_base, const uint16_t* translation,
                                  const uint16_t* inv_scale, const uint16_t* bias, uint16_t* Y,
                                  int B, int D_in, int D_out, int num_wavelets, int wavelet_type,
                                  int has_base, int has_bias);
/* metal_kan_bridge.mm:1168 -- unlike the reference (which hard-codes 4 terms), degrees[] is
 * honoured per layer.  W_bases[l] / biases[l] may be NULL (no base / no bias for that layer). */
int metal_kan_chain_pipeline_cheby(const float* X, float* Y, int B, int num_layers,
                                   const int* layer_dims, const int* degrees,
                                   const float** W_chebys, const float** W_bases,
                                   const float** biases);
/* metal_kan_bridge.mm:4846 -- out = g * sigmoid(clamp(g, -20, 20)) * u */
int metal_kan_swiglu_forward(const float* gate, const float* up, float* out, int n_elems);

/* Host quantisers (metal_kan_bridge.mm:4177, :4234, :4634, :4735) and dequantisers (:4213,
 * :4278, :5073, :5109).  Bit-exact with the source text evaluated with one IEEE fp32 rounding per
 * operation.  Layouts: INT8 q[groups][gs]; INT4 q[groups][gs/2] (lo nibble = even element);
 * 2-bit P[D_out][ceil(K_dim/16)] (element k at bits 2*(k%16) of word k/16), scales
 * [D_out][ceil(K_dim/gs)]. */
int metal_kan_quantize_int8(const float* weights, uint8_t* qweight, float* scales, float* biases,
                            int num_groups, int group_size);
int metal_kan_quantize_int4(const float* weights, uint8_t* qweight, float* scales, float* biases,
                            int num_groups, int group_size);
int metal_kan_dequantize_int8(const uint8_t* qweight, const float* scales, const float* biases,
                              float* weights, int num_groups, int group_size);
int metal_kan_dequantize_int4(const uint8_t* qweight, const float* scales, const float* biases,
                              float* weights, int num_groups, int group_size);
int metal_kan_quantize_ternary(const float* W, uint32_t* W_packed, float* scales, int D_out,
                               int K_dim, int group_size);
int metal_kan_quantize_int2(const float* W, uint32_t* W_packed, float* scales,
                            const float* codebook, int D_out, int K_dim, int group_size);
/* These two run on the GPU, like the reference's dequantize_*_fast kernels. */
int metal_kan_dequantize_ternary(const uint32_t* packed, const float* scales, float* out,
                                 int D_out, int K_dim, int group_size);
int metal_kan_dequantize_int2(const uint32_t* packed, const float* scales, const float* codebook,
                              float* out, int D_out, int K_dim, int group_size);

/* metal_kan_bridge.mm:4684 / :4790 -- packed-weight ChebyKAN forward (no base branch), fp32.
 * degree = number of terms. */
int metal_kan_forward_ternary_cheby(const float* X, const uint32_t* W_packed, const float* scales,
                                    const float* bias, float* Y, int B, int D_in, int D_out,
                                    int degree, int group_size, int has_bias);
int metal_kan_forward_int2_cheby(const float* X, const uint32_t* W_packed, const float* scales,
                                 const float* codebook, const float* bias, float* Y, int B,
                                 int D_in, int D_out, int degree, int group_size, int has_bias);

/* metal_kan_bridge.mm:627 -- ReLUKAN (tent basis), grid [num_grids] */
int metal_kan_relu_forward(const float* X, const float* W_relu, const float* W_base,
                           const float* grid, const float* bias, float* Y, int B, int D_in,
                           int D_out, int num_grids, float inv_h, int has_base, int has_bias);
/* metal_kan_bridge.mm:2359 (grid is fp16 here, like the reference) */
int metal_kan_relu_forward_fp16(const uint16_t* X, const uint16_t* W_relu, const uint16_t* W_base,
                                const uint16_t* grid, const uint16_t* bias, uint16_t* Y, int B,
                                int D_in, int D_out, int num_grids, float inv_h, int has_base,
                                int has_bias);
/* metal_kan_bridge.mm:820 -- FourierKAN, 2 * num_frequencies + 1 bases per feature */
int metal_kan_fourier_forward(const float* X, const float* W_fourier, const float* W_base,
                              const float* bias, float* Y, int B, int D_in, int D_out,
                              int num_frequencies, int has_base, int has_bias);
/* metal_kan_bridge.mm:2539 */
int metal_kan_fourier_forward_fp16(const uint16_t* X, const uint16_t* W_fourier,
                                   const uint16_t* W_base, const uint16_t* bias, uint16_t* Y,
                                   int B, int D_in, int D_out, int num_frequencies, int has_base,
                                   int has_bias);
/* metal_kan_bridge.mm:910 -- JacobiKAN P_k^(alpha, beta), `degree` terms */
int metal_kan_jacobi_forward(const float* X, const float* W_jacobi, const float* W_base,
                             const float* bias, float* Y, int B, int D_in, int D_out, int degree,
                             float alpha, float beta, int has_base, int has_bias);
/* metal_kan_bridge.mm:2624 */
int metal_kan_jacobi_forward_fp16(const uint16_t* X, const uint16_t* W_jacobi,
                                  const uint16_t* W_base, const uint16_t* bias, uint16_t* Y, int B,
                                  int D_in, int D_out, int degree, float alpha, float beta,
                                  int has_base, int has_bias);
/* metal_kan_bridge.mm:1700 -- MultKAN: an RBF layer to num_add + 2 num_mult internal outputs,
 * then out[:, num_add + m] = internal[:, num_add + m] * internal[:, num_add + num_mult + m];
 * D_out = num_add + num_mult, W_rbf / W_base / bias sized for the internal outputs */
int metal_kan_mult_forward(const float* X, const float* W_rbf, const float* W_base,
                           const float* grid, const float* bias, float* Y, int B, int D_in,
                           int D_out, int num_add, int num_mult, int num_centers,
                           float inv_denominator, int has_base, int has_bias);
/* metal_kan_bridge.mm:2250 (grid is fp16 here, like the reference) */
int metal_kan_mult_forward_fp16(const uint16_t* X, const uint16_t* W_rbf, const uint16_t* W_base,
                                const uint16_t* grid, const uint16_t* bias, uint16_t* Y, int B,
                                int D_in, int D_out, int num_add, int num_mult, int num_centers,
                                float inv_denominator, int has_base, int has_bias);
/* metal_kan_bridge.mm:1535 -- LowRankKAN: Z = RBF layer to `rank` outputs (W_down, no base or
 * bias), Y = bias + Z W_up^T + silu(X) W_base^T */
int metal_kan_lowrank_forward(const float* X, const float* W_down, const float* W_up,
                              const float* W_base, const float* grid, const float* bias, float* Y,
                              int B, int D_in, int D_out, int rank, int num_centers,
                              float inv_denominator, int has_base, int has_bias);
/* metal_kan_bridge.mm:2153 */
int metal_kan_lowrank_forward_fp16(const uint16_t* X, const uint16_t* W_down,
                                   const uint16_t* W_up, const uint16_t* W_base,
                                   const uint16_t* grid, const uint16_t* bias, uint16_t* Y, int B,
                                   int D_in, int D_out, int rank, int num_centers,
                                   float inv_denominator, int has_base, int has_bias);
/* metal_kan_bridge.mm:1004 -- RationalKAN (fp32 only, like the reference): per input feature
 * P(xc) / (1 + |Q(xc)|) with Chebyshev expansions of xc = clamp(x, -1, 1) (W_p [D_out][D_in*p],
 * W_q [D_out][D_in*q]) plus silu(xc) W_base; p, q in 0..16, 1 <= p + q <= 16 */
int metal_kan_rational_forward(const float* X, const float* W_p, const float* W_q,
                               const float* W_base, const float* bias, float* Y, int B, int D_in,
                               int D_out, int p_degree, int q_degree, int has_base, int has_bias);

/* Backward of one fp32 layer, host pointers, synchronous (the reference's training path).
 * dY [B][D_out], X [B][D_in] (the forward's input), W / Wb the layer's weights; outputs dW
 * [D_out][D_in*K], dW_base [D_out][D_in] (if has_base), dbias [D_out] (if has_bias), dX
 * [B][D_in].  Same math as the reference: dW = dY^T Phi, dX = the basis derivatives contracted
 * with dY W (Chebyshev derivative zero outside [-1, 1]), silu' for the base branch. */
/* metal_kan_bridge.mm:2715 */
int metal_kan_cheby_backward(const float* dY, const float* X, const float* W_cheby,
                             const float* W_base, float* dW_cheby, float* dW_base, float* dbias,
                             float* dX, int B, int D_in, int D_out, int degree, int has_base,
                             int has_bias);
/* metal_kan_bridge.mm:4532 (same results as metal_kan_cheby_backward here: neither materialises
 * the basis matrix) */
int metal_kan_cheby_backward_fused(const float* dY, const float* X, const float* W_cheby,
                                   const float* W_base, float* dW_cheby, float* dW_base,
                                   float* dbias, float* dX, int B, int D_in, int D_out, int degree,
                                   int has_base, int has_bias);
/* metal_kan_bridge.mm:2847 */
int metal_kan_fastkan_backward(const float* dY, const float* X, const float* W_rbf,
                               const float* W_base, const float* grid, float* dW_rbf,
                               float* dW_base, float* dbias, float* dX, int B, int D_in, int D_out,
                               int num_centers, float inv_denominator, int has_base, int has_bias);
/* metal_kan_bridge.mm (ReLUKAN backward, bound at device.py:296) -- tent derivative
 * -sign(x - g) inv_h where the tent is positive (fused_kan.metal:1787-1826) */
int metal_kan_relu_backward(const float* dY, const float* X, const float* W_relu,
                            const float* W_base, const float* grid, float* dW_relu,
                            float* dW_base, float* dbias, float* dX, int B, int D_in, int D_out,
                            int num_grids, float inv_h, int has_base, int has_bias);
/* metal_kan_bridge.mm:3121 */
int metal_kan_bspline_backward(const float* dY, const float* X, const float* W_spline,
                               const float* W_base, float* dW_spline, float* dW_base, float* dbias,
                               float* dX, int B, int D_in, int D_out, int grid_size,
                               float grid_min, float inv_h, int has_base, int has_bias);
/* metal_kan_bridge.mm:4877 -- d_gate, d_up of hidden = silu(gate) * up (SiLU argument clamped to
 * +-20 in the sigmoid, fused_kan.metal:2298-2316) */
int metal_kan_swiglu_backward(const float* d_hidden, const float* gate, const float* up,
                              float* d_gate, float* d_up, int n_elems);

/* metal_kan_bridge.mm:1250-1371 -- mean milliseconds per full host-pointer forward (stage +
 * kernel + copy back), after `warmup` untimed calls; negative on error. */
double benchmark_metal_cheby(const float* X, const float* W_cheby, const float* W_base,
                             const float* bias, float* Y, int B, int D_in, int D_out, int K,
                             int has_base, int has_bias, int warmup, int iters);
double benchmark_metal_fastkan(const float* X, const float* W_rbf, const float* W_base,
                               const float* grid, const float* bias, float* Y, int B, int D_in,
                               int D_out, int num_centers, float inv_denominator, int has_base,
                               int has_bias, int warmup, int iters);
double benchmark_metal_bspline(const float* X, const float* W_spline, const float* W_base,
                               const float* grid, const float* bias, float* Y, int B, int D_in,
                               int D_out, int grid_size, int spline_order, int has_base,
                               int has_bias, int warmup, int iters);
double benchmark_metal_wavkan(const float* X, const float* W_wav, const float* W_base,
                              const float* translation, const float* inv_scale, const float* bias,
                              float* Y, int B, int D_in, int D_out, int num_wavelets,
                              int wavelet_type, int has_base, int has_bias, int warmup, int iters);
double benchmark_metal_relu(const float* X, const float* W_relu, const float* W_base,
                            const float* grid, const float* bias, float* Y, int B, int D_in,
                            int D_out, int num_grids, float inv_h, int has_base, int has_bias,
                            int warmup, int iters);
double benchmark_metal_fourier(const float* X, const float* W_fourier, const float* W_base,
                               const float* bias, float* Y, int B, int D_in, int D_out,
                               int num_frequencies, int has_base, int has_bias, int warmup,
                               int iters);
double benchmark_metal_jacobi(const float* X, const float* W_jacobi, const float* W_base,
                              const float* bias, float* Y, int B, int D_in, int D_out, int degree,
                              float alpha, float beta, int has_base, int has_bias, int warmup,
                              int iters);
double benchmark_metal_mult(const float* X, const float* W_rbf, const float* W_base,
                            const float* grid, const float* bias, float* Y, int B, int D_in,
                            int D_out, int num_add, int num_mult, int num_centers,
                            float inv_denominator, int has_base, int has_bias, int warmup,
                            int iters);
double benchmark_metal_lowrank(const float* X, const float* W_down, const float* W_up,
                               const float* W_base, const float* grid, const float* bias, float* Y,
                               int B, int D_in, int D_out, int rank, int num_centers,
                               float inv_denominator, int has_base, int has_bias, int warmup,
                               int iters);
double benchmark_metal_rational(const float* X, const float* W_p, const float* W_q,
                                const float* W_base, const float* bias, float* Y, int B, int D_in,
                                int D_out, int p_degree, int q_degree, int has_base, int has_bias,
                                int warmup, int iters);

/* ------------------------------------------------------------------------------------------ */
/* tier 2: device-resident engine (new)                                                       */
/* ------------------------------------------------------------------------------------------ */

enum kan_dtype { KAN_F32 = 0, KAN_F16 = 1, KAN_BF16 = 2 };
enum kan_basis {
  KAN_CHEBY = 0,   /* T_k(clamp(x, -1, 1))                                                       */
  KAN_RBF = 1,     /* exp(-(x - c_k)^2 inv_den), centres in grid[K]                             */
  KAN_BSPLINE = 2, /* uniform cubic B-spline, G + 3 bases                                       */
  KAN_WAVELET = 3, /* mexican hat / morlet / DoG of (x - t) inv_s                               */
  KAN_RELU = 4,    /* tent max(0, 1 - |x - g_k| inv_h), grid points in grid[K]                  */
  KAN_FOURIER = 5, /* 1, cos(pi x), sin(pi x), cos(2 pi x), ... (K = 2 F + 1)                   */
  KAN_JACOBI = 6   /* Jacobi P_k^(alpha, beta)(clamp(x, -1, 1))                                 */
};
enum kan_input_map { KAN_MAP_NONE = 0, KAN_MAP_TANH = 1, KAN_MAP_LAYERNORM = 2 };
enum kan_wformat {
  KAN_W_DENSE = 0,   /* act-dtype matrix [rows][cols]                                          */
  KAN_W_INT8 = 1,    /* u8 [rows*padded_cols/gs][gs], fp32 scales/biases per group             */
  KAN_W_INT4 = 2,    /* u8 [rows*padded_cols/gs][gs/2]                                          */
  KAN_W_TERNARY = 3, /* u32 [rows][ceil(cols/16)], fp32 scales [rows][ceil(cols/gs)]           */
  KAN_W_INT2 = 4     /* as ternary + fp32 codebook[4]                                          */
};
/* kan_weight.flags.  KAN_WFLAG_TERNARY_NO3: a ternary matrix holds no code 3 (the quantiser
   writes only 0, 1, 2; the dequantiser maps 3 to 0 like 1).  The CUDA-core small-batch kernel
   then decodes codes in place as c - 1 (fewer instructions per code); without the flag it uses
   the exact table decode.  A caller setting the flag on data that holds code 3 gets +1 instead
   of 0 for those weights. */
enum kan_wflags { KAN_WFLAG_TERNARY_NO3 = 1 };
/* Kernel selection for kan_forward_path.  KAN_PATH_AUTO: the CUDA-core small-batch kernel
   (GEMV_CC) when it applies (f16/bf16 layer of any basis and input map, ternary/INT8/INT4 weights,
   B <= 4), else the tensor-core small-batch kernel (GEMV: f16/bf16 Chebyshev layer, ternary/INT2
   weights, B <= 64, D_in >= 512, D_out >= 128), else the tensor-core kernel (TC) for f16/bf16,
   else the CUDA-core kernel (SIMT).  An explicit path a layer does not fit returns
   KAN_ERR_UNSUPPORTED. */
enum kan_path {
  KAN_PATH_AUTO = 0,
  KAN_PATH_SIMT = 1,
  KAN_PATH_TC = 2,
  KAN_PATH_GEMV = 3,
  KAN_PATH_GEMV_CC = 4
};

/* One weight matrix with `rows` = D_out and `cols` = D_in*K (basis) or D_in (base branch). */
typedef struct kan_weight {
  int32_t format;       /* enum kan_wformat */
  int32_t group_size;   /* quantised formats */
  int32_t padded_cols;  /* INT8/INT4: cols rounded up to a multiple of group_size */
  int32_t flags;        /* enum kan_wflags */
  const void* data;     /* device pointer */
  const float* scales;  /* device pointer or NULL */
  const float* biases;  /* device pointer or NULL (INT8/INT4 group minimum) */
  const float* codebook;/* device pointer or NULL (INT2) */
} kan_weight;

/* One KAN layer: y[b, j] = bias[j] + sum_i silu(m(x))[b,i] Wb[j,i]
 *                              + sum_i sum_k phi_k(m(x)[b,i]) W[j, i*K + k]
 * with m the input map.  All pointers are device pointers.  Basis parameters (grid,
 * translation, inv_scale) are float32 whatever the activation dtype; the fp16 mode rounds them
 * to half exactly where the reference's half kernels use half values. */
typedef struct kan_layer {
  int32_t basis;        /* enum kan_basis */
  int32_t act_dtype;    /* enum kan_dtype: X, Y, bias and dense weights */
  int32_t D_in, D_out;
  int32_t K;            /* basis terms per input feature (BSpline: grid_size + 3) */
  int32_t has_base, has_bias;
  int32_t input_map;    /* enum kan_input_map */
  int32_t wavelet_type; /* 0 mexican hat, 1 morlet, 2 dog */
  int32_t grid_size;    /* BSpline G */
  float inv_den;        /* RBF: exp(-(x-c)^2 * inv_den) */
  float grid_min, inv_h;/* BSpline */
  float ln_eps;         /* LayerNorm epsilon */
  const float* grid;    /* RBF centres [K] */
  const float* translation; /* wavelet [D_in][K] */
  const float* inv_scale;   /* wavelet [D_in][K] */
  const void* bias;     /* [D_out], act dtype */
  kan_weight w;         /* basis weights [D_out][D_in*K] */
  kan_weight wb;        /* base weights [D_out][D_in] */
  /* Optional: w and wb already packed by kan_tc_pack() into the tensor-core layout (device
   * pointer, act dtype).  When NULL the tensor-core path packs into library scratch on every
   * call; callers that keep weights resident should pack once and pass the buffer here. */
  const void* tc_weights;
  float alpha, beta;    /* Jacobi parameters (ReLU uses grid + inv_h) */
} kan_layer;

/* Tensor-core weight layout: 64-column blocks of whole input features -- F = 64 / KT features
 * per block, KT = K + has_base terms per feature (the basis terms, then the base weight), zero
 * padded -- rows = D_out, in the act dtype.  Packed weights are decoded (exact fp32 values) and
 * rounded to the act dtype.  kan_tc_packed_bytes() gives the buffer size. */
int kan_tc_packed_bytes(const kan_layer* layer, size_t* bytes);
int kan_tc_pack(const kan_layer* layer, void* out, void* stream);

/* Enqueue one layer forward: X [B][D_in] -> Y [B][D_out] (act dtype). */
int kan_forward(const kan_layer* layer, const void* X, void* Y, int B, void* stream);
/* Same with an explicit kernel path (tests, benchmarks). */
int kan_forward_path(const kan_layer* layer, const void* X, void* Y, int B, int path,
                     void* stream);
/* No counterpart in the reference.  The kernel plan kan_forward_path(layer, X, Y, B, path) would
 * run, without running it: info[0] = the path taken (KAN_PATH_SIMT / TC / GEMV; `path` may be
 * KAN_PATH_AUTO), and for the tensor-core path info[1] = tile width BN, info[2] = split-K factor
 * (cluster size), info[3] = M tiles, info[4] = N tiles, info[5] = 64-column K blocks; for the
 * tensor-core small-batch path info[3] = 128-row blocks; for the CUDA-core small-batch path
 * info[2] = K splits, info[3] = 32-row blocks.  Tests and benchmarks use it to name the plan they
 * check.  info must hold 6 ints. */
int kan_forward_plan(const kan_layer* layer, int B, int path, int* info);
/* No counterpart in the reference.  Limit of the tensor-core kernel's pipeline waits (a stage
 * filled or freed by another warp role), in SM clock cycles, for the launches that follow on any
 * device; 0 restores the default of about one second.  A short limit makes those waits expire,
 * so that the abort path (error word set, remaining work skipped, every copy and MMA in flight
 * still waited for with the full limit, TMEM released) can be driven by a test; the next call
 * then reports KAN_ERR_DEVICE_TIMEOUT.  Not for production use. */
int kan_set_wait_limit(long long cycles);
/* No counterpart in the reference's device API; replaces the host-pointer convention of the
 * bridge's forwards (metal_kan_bridge.mm:1890-1971: copy in, compute, copy out, synchronous) for
 * any kan_layer.  X [B][D_in] and Y [B][D_out] are HOST memory (page-locked for overlap);
 * returns when Y is written.  Large batches run as two chunks on separate copy and compute
 * streams, so that transfers overlap the kernels. */
int kan_forward_host(const kan_layer* layer, const void* X, void* Y, int B);

/* GatedKAN block: H = silu(gate(X)) * up(X) (act dtype, [B][D_ffn]); Y = down(H).  H is caller
 * memory ([B][gate.D_out] elements of the act dtype). */
int kan_gated_forward(const kan_layer* gate, const kan_layer* up, const kan_layer* down,
                      const void* X, void* H, void* Y, int B, void* stream);

/* No counterpart in the reference (gated_kan.py:112-131 runs gate and up as two layers).  Gate and
 * up of a GatedKAN read the same input through the same basis; kan_tc_pack_pair() packs both into
 * one tensor-core matrix (rows interleaved in blocks of 256; kan_tc_pair_bytes() gives its size)
 * and kan_gated_forward_pair() evaluates the basis once for both, applies SwiGLU in the epilogue
 * and runs down.  H equals kan_gated_forward's bit for bit where that one's gate and up launches
 * do not split K (otherwise the fp32 sums are ordered differently).  Needs two f16/bf16 Chebyshev layers
 * of one shape, K, base branch and input map; otherwise, for grids under 120 tiles, or with a
 * NULL pair, it runs kan_gated_forward(). */
int kan_tc_pair_bytes(const kan_layer* gate, const kan_layer* up, size_t* bytes);
int kan_tc_pack_pair(const kan_layer* gate, const kan_layer* up, void* out, void* stream);
int kan_gated_forward_pair(const kan_layer* gate, const kan_layer* up, const kan_layer* down,
                           const void* pair, const void* X, void* H, void* Y, int B,
                           void* stream);

/* No counterpart in the reference.  kan_gated_forward() for callers that cannot allocate device
 * memory (allocation forbidden after start-up by a memory arena or a serving runtime, or a
 * cudaMalloc that would synchronise or fail at that point): the gate and up activations live in
 * a fixed 32 MiB device array that every GPU loading the library holds until exit, so
 * 2 * B * gate->D_out * sizeof(act dtype) must be <= 32 MiB (else KAN_ERR_UNSUPPORTED).  H and
 * Y are the caller's, as in kan_gated_forward().  The first call on a device looks up the array's
 * device address (and sets up the library's per-device state); make it before any stream
 * capture.  All calls on a device share the array and keep the previous call's contents (nothing
 * in it needs zeroing), so calls that overlap on the GPU race.  f16/bf16 layers use the tensor
 * cores only if their tc_weights are packed in advance; without them they run on the CUDA-core
 * path, which needs no scratch. */
int kan_gated_forward_noalloc(const kan_layer* gate, const kan_layer* up, const kan_layer* down,
                              const void* X, void* H, void* Y, int B, void* stream);

/* No counterpart in the reference's device API (its backward is the host-pointer functions
 * above, which call this).  Backward of a dense fp32 layer with raw inputs (Chebyshev, RBF or
 * B-spline basis) on device pointers: X is the forward's input, dY [B][D_out]; writes dX
 * [B][D_in], dW [D_out][D_in*K], dWb [D_out][D_in] and dbias [D_out] -- any of them may be NULL
 * to skip it (dWb / dbias are ignored without a base branch / bias).  Enqueued on `stream`. */
int kan_backward(const kan_layer* layer, const void* X, const void* dY, void* dX, void* dW,
                 void* dWb, void* dbias, int B, void* stream);
/* Elementwise SwiGLU backward on device pointers (fp32, n elements). */
int kan_swiglu_backward(const void* d_hidden, const void* gate, const void* up, void* d_gate,
                        void* d_up, long long n, void* stream);

/* Dequantise any weight format to a dense matrix of `out_dtype` ([rows][cols]); the fp32 value
 * is bit-identical to the reference dequantiser, then rounded (RNE) for f16/bf16 outputs. */
int kan_dequantize(const kan_weight* w, int rows, int cols, void* out, int out_dtype,
                   void* stream);
/* Elementwise: out = g * sigmoid(clamp(g,-20,20)) * u, dtype act_dtype, n elements. */
int kan_swiglu(const void* gate, const void* up, void* out, long long n, int act_dtype,
               void* stream);
/* MultKAN pair products on device buffers: in [B][num_add + 2 num_mult] -> out
 * [B][num_add + num_mult] in `act_dtype` (metal_kan_bridge.mm:1788-1799). */
int kan_mult_combine(const void* in, void* out, int B, int num_add, int num_mult, int act_dtype,
                     void* stream);
/* LowRankKAN second stage on device buffers: Y = bias + Z W_up^T + silu(X) W_base^T, Z [B][rank]
 * the RBF stage's output (metal_kan_bridge.mm:1614-1636). */
int kan_lowrank_up(const void* Z, const void* X, const void* W_up, const void* W_base,
                   const void* bias, void* Y, int B, int D_in, int D_out, int rank, int has_base,
                   int has_bias, int act_dtype, void* stream);
/* RationalKAN on device buffers (fp32), as metal_kan_rational_forward. */
int kan_rational_forward(const float* X, const float* W_p, const float* W_q, const float* W_base,
                         const float* bias, float* Y, int B, int D_in, int D_out, int p_degree,
                         int q_degree, int has_base, int has_bias, void* stream);
/* Dtype conversion of n elements (any of KAN_F32/F16/BF16 to any). */
int kan_convert(const void* src, int src_dtype, void* dst, int dst_dtype, long long n,
                void* stream);

/* Device memory / stream helpers so that callers without a CUDA runtime binding (ctypes users)
 * can manage buffers.  kind: 1 = host->device, 2 = device->host, 3 = device->device. */
int kan_device_count(int* count);
int kan_set_device(int device);
int kan_get_device(int* device);
int kan_malloc(void** ptr, size_t bytes);
int kan_free(void* ptr);
int kan_host_alloc(void** ptr, size_t bytes); /* pinned host memory */
int kan_host_free(void* ptr);
int kan_memcpy(void* dst, const void* src, size_t bytes, int kind, void* stream);
int kan_memset(void* dst, int value, size_t bytes, void* stream);
int kan_stream_synchronize(void* stream);
void* kan_default_stream(void);

/* Device-side error word: non-zero when a kernel's bounded wait expired (the kernel then skipped
 * its remaining work and released its resources).  Reading clears it. */
int kan_device_error(int* code);

/* Number of kernels this library launched since load (evidence counter for benchmarks). */
long long kan_launch_count(void);

/* ------------------------------------------------------------------------------------------ */
/* training (fp32)                                                                             */
/* ------------------------------------------------------------------------------------------ */
/* Optimisers of kan_train_step / kan_optim_step; hyper = {lr, beta1, beta2, eps, weight_decay,
 * lr_t} (SGD: beta1 = momentum; lr_t = lr * sqrt(1 - beta2^t) / (1 - beta1^t) for the Adams). */
enum kan_optimizer { KAN_OPT_ADAMW = 0, KAN_OPT_ADAM = 1, KAN_OPT_SGD = 2, KAN_OPT_LION = 3 };
/* One training step of a dense fp32 layer on device buffers (metal_kan_bridge.mm:3432-3640):
 * forward, dY = (Y - target) * 2 / B (MSE), the weight / base / bias gradients, one optimiser
 * update of the layer's tensors in place (their pointers in `layer` must be writable).  State:
 * m (and v for the Adams) per tensor, NULL for absent base / bias. */
int kan_train_step(const kan_layer* layer, const float* X, const float* target, int B,
                   float* m_w, float* v_w, float* m_wb, float* v_wb, float* m_b, float* v_b,
                   int optimizer, const float* hyper, int nesterov, void* stream);
/* One optimiser update of n fp32 parameters on device buffers. */
int kan_optim_step(int optimizer, float* param, const float* grad, float* m, float* v,
                   long long n, const float* hyper, int nesterov, void* stream);
/* metal_kan_bridge.mm (adamw_step, fused_kan.metal:1896) -- host pointers, updated in place */
int metal_kan_adamw_step(float* param, const float* grad, float* m, float* v, float lr,
                         float beta1, float beta2, float eps, float weight_decay, float lr_t,
                         int n_elems);
/* adam_coupled_step: weight decay added to the gradient */
int metal_kan_adam_step(float* param, const float* grad, float* m, float* v, float lr,
                        float beta1, float beta2, float eps, float weight_decay, float lr_t,
                        int n_elems);
/* sgd_step (fused_kan.metal:1923) */
int metal_kan_sgd_step(float* param, const float* grad, float* velocity, float lr,
                       float momentum, float weight_decay, int nesterov, int n_elems);
/* lion_step (fused_kan.metal:1946) */
int metal_kan_lion_step(float* param, const float* grad, float* m, float lr, float beta1,
                        float beta2, float weight_decay, int n_elems);
/* metal_kan_bridge.mm:3432 -- fused AdamW training step of a ChebyKAN layer, host pointers;
 * weights and AdamW state updated in place */
int metal_kan_cheby_train_step(const float* X, const float* target, float* W_cheby,
                               float* W_base, float* bias, float* m_W, float* v_W, float* m_Wb,
                               float* v_Wb, float* m_b, float* v_b, int B, int D_in, int D_out,
                               int degree, int has_base, int has_bias, float lr, float beta1,
                               float beta2, float eps, float weight_decay, float lr_t);
/* FastKAN twin */
int metal_kan_fastkan_train_step(const float* X, const float* target, float* W_rbf,
                                 float* W_base, const float* grid, float* bias, float* m_W,
                                 float* v_W, float* m_Wb, float* v_Wb, float* m_b, float* v_b,
                                 int B, int D_in, int D_out, int num_centers,
                                 float inv_denominator, int has_base, int has_bias, float lr,
                                 float beta1, float beta2, float eps, float weight_decay,
                                 float lr_t);
/* metal_kan_bridge.mm:5148 -- the MSE loss gradient dY = (pred - target) * scale */
int metal_kan_calc_mse_loss_backward(const float* pred, const float* target, float* dY,
                                     int n_elems, float scale);
/* BSplineKAN twin (uniform grid [grid_min, grid_max] of grid_size intervals) */
int metal_kan_bspline_train_step(const float* X, const float* target, float* W_spline,
                                 float* W_base, float* bias, float* m_W, float* v_W, float* m_Wb,
                                 float* v_Wb, float* m_b, float* v_b, int B, int D_in, int D_out,
                                 int grid_size, float grid_min, float grid_max, int has_base,
                                 int has_bias, float lr, float beta1, float beta2, float eps,
                                 float weight_decay, float lr_t);

#ifdef __cplusplus
}
#endif
#endif /* KAN_CUDA_H_ */
