// kan_launch.h -- host-side launchers of the device kernels (implemented in the .cu files) and
// the launch counter reported by kan_launch_count().
#pragma once

#include <cuda_runtime.h>

#include "kan_args.h"

namespace kan {

inline int BasisOf(const LayerArgs& a) { return a.basis; }

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
// kan_gemv.cu: small-batch path for 2-bit packed weights (weights as the MMA M operand, decoded
// from the packed codes into TMEM; no dense copy)
// launch_gemv also runs the basis pre-pass into `phi` (gemv_phi_bytes() of device scratch).
bool gemv_supported(const LayerArgs& a, int act_dtype);
size_t gemv_phi_bytes(const LayerArgs& a);
cudaError_t launch_gemv(const LayerArgs& a, int act_dtype, void* phi, cudaStream_t s);
// kan_misc.cu
cudaError_t launch_dequantize(const kan_weight& w, int rows, int cols, void* out, int out_dtype,
                              cudaStream_t s);
cudaError_t launch_swiglu(const void* g, const void* u, void* out, long long n, int dtype,
                          cudaStream_t s);
cudaError_t launch_convert(const void* src, int sdt, void* dst, int ddt, long long n,
                           cudaStream_t s);

}  // namespace kan
