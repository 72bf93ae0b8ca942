// kan_launch.h -- host-side launchers of the device kernels (implemented in the .cu files) and
// the launch counter reported by kan_launch_count().
#pragma once

#include <cuda_runtime.h>

#include <atomic>

#include "kan_args.h"

namespace kan {

inline int BasisOf(const LayerArgs& a) { return a.basis; }

// Dynamic shared-memory limit of `kern` on the current device, set once per device: callers pass
// the largest size any launch of `kern` uses (a later, larger request would not be applied).
// cudaFuncSetAttribute acts on the current device only, so the "done" state is one bit per
// device in `done` (a static of the caller, one per kernel); the bit is set atomically, and two
// host threads that race on a device's first launch both set the same attribute, which is
// harmless.  Devices past the mask's width set it on every launch.
template <class Kern>
inline cudaError_t ensure_smem_attr(Kern kern, int smem_bytes,
                                    std::atomic<unsigned long long>& done) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const unsigned long long bit = dev < 64 ? (1ull << dev) : 0ull;
  if (bit && (done.load(std::memory_order_acquire) & bit)) return cudaSuccess;
  e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes);
  if (e == cudaSuccess && bit) done.fetch_or(bit, std::memory_order_acq_rel);
  return e;
}

// Limit of the tensor-core kernel's pipeline waits in SM clock cycles (0: the default of about
// one second).  A short limit makes those waits expire so that tests can drive the abort path;
// waits for copies and MMAs already in flight always keep the default (kan_abi.cpp).
long long pipeline_wait_limit();

void note_launch();
long long launch_count();
// Record `msg` as this thread's kan_last_error() and return `code` (kan_abi.cpp).
int set_error(int code, const char* msg);
// Address of the device error word on the current device (kan_misc.cu).
int* device_error_ptr();

// kan_simt.cu
cudaError_t launch_simt(const LayerArgs& a, int act_dtype, cudaStream_t s);
// kan_tc.cu: the tensor-core path.  tc_plan() picks the tile width and the split-K factor (the
// split CTAs of a tile form a cluster and reduce through distributed shared memory);
// launch_tc() needs a.tc_weights (the packed layout).
struct TcPlan {
  int BN, nb, mtiles, ntiles, splits;
};
bool tc_supported(const LayerArgs& a, int act_dtype);
TcPlan tc_plan(const LayerArgs& a);
cudaError_t launch_tc(const LayerArgs& a, int act_dtype, const TcPlan& plan, cudaStream_t s);
cudaError_t launch_tc_pack(const LayerArgs& a, int act_dtype, void* out, cudaStream_t s);
// GatedKAN gate/up pair: both layers packed into one [pair_rows(D_out)][NB*64] matrix, rows
// interleaved in blocks of PAIR_BLOCK (the layout a.fuse_swiglu launches read).
cudaError_t launch_tc_pack_pair(const LayerArgs& gate, const LayerArgs& up, int act_dtype,
                                void* out, cudaStream_t s);
// cuTensorMapEncodeTiled of the driver, looked up once (thread-safe); nullptr if unavailable
// (kan_tc.cu).
void* tensor_map_encoder();
// kan_gemv_cc.cu: small-batch path on the CUDA cores (B <= 4; ternary / INT8 / INT4 weights decoded
// on chip, integer dot products against a fixed-point basis matrix).  launch_gemv_cc also runs the
// basis pre-pass; `scratch` holds gemv_cc_scratch_bytes() of device memory, zeroed when allocated.
bool gemv_cc_supported(const LayerArgs& a, int act_dtype);
size_t gemv_cc_scratch_bytes(const LayerArgs& a);
int gemv_cc_splits(const LayerArgs& a);
cudaError_t launch_gemv_cc(const LayerArgs& a, int act_dtype, void* scratch, cudaStream_t s);
// kan_gemv.cu: small-batch path for 2-bit packed weights (weights as the MMA M operand, decoded
// from the packed codes into TMEM; no dense copy)
// launch_gemv also runs the basis pre-pass into `phi` (gemv_phi_bytes() of device scratch).
bool gemv_supported(const LayerArgs& a, int act_dtype);
size_t gemv_phi_bytes(const LayerArgs& a);
cudaError_t launch_gemv(const LayerArgs& a, int act_dtype, void* phi, cudaStream_t s);
// kan_backward.cu: fp32 layer backward (Chebyshev, RBF, B-spline bases; raw input)
bool backward_supported(const BackwardArgs& a);
cudaError_t launch_backward(const BackwardArgs& a, cudaStream_t s);
cudaError_t launch_swiglu_backward(const float* dh, const float* g, const float* u, float* dg,
                                   float* du, long long n, cudaStream_t s);
// kan_extra.cu: MultKAN pair products, LowRankKAN up projection (+ base branch), RationalKAN
cudaError_t launch_mult_combine(const void* in, void* out, int B, int num_add, int num_mult,
                                int act_dtype, cudaStream_t s);
cudaError_t launch_lowrank_up(const void* Z, const void* X, const void* Wup, const void* Wb,
                              const void* bias, void* Y, int B, int D_in, int D_out, int rank,
                              int has_base, int has_bias, int act_dtype, cudaStream_t s);
bool rational_supported(int p, int q);
cudaError_t launch_rational(const float* X, const float* Wp, const float* Wq, const float* Wb,
                            const float* bias, float* Y, int B, int D_in, int D_out, int p, int q,
                            int has_base, int has_bias, cudaStream_t s);
// kan_train.cu: MSE loss gradient and the optimiser updates of the fp32 training step
enum { OPTIM_ADAMW = 0, OPTIM_ADAM = 1, OPTIM_SGD = 2, OPTIM_LION = 3 };
struct OptimHyper {
  float lr, beta1, beta2, eps, weight_decay, lr_t;  // SGD: beta1 = momentum
  int nesterov;
};
cudaError_t launch_mse_grad(const float* pred, const float* target, float* dY, long long n,
                            float scale, cudaStream_t s);
// `count` (1..3) tensors in one launch; v may be null for SGD and Lion
cudaError_t launch_optim(int op, int count, float* const* param, const float* const* grad,
                         float* const* m, float* const* v, const long long* n,
                         const OptimHyper& h, cudaStream_t s);
// kan_misc.cu
cudaError_t launch_dequantize(const kan_weight& w, int rows, int cols, void* out, int out_dtype,
                              cudaStream_t s);
cudaError_t launch_swiglu(const void* g, const void* u, void* out, long long n, int dtype,
                          cudaStream_t s);
cudaError_t launch_convert(const void* src, int sdt, void* dst, int ddt, long long n,
                           cudaStream_t s);

}  // namespace kan
