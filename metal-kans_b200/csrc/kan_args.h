// kan_args.h -- the flattened per-call layer arguments every kernel receives (host + device).
#pragma once

#include "../../include/kan_cuda.h"

#ifdef __CUDACC__
#define KAN_HD __host__ __device__
#else
#define KAN_HD
#endif

namespace kan {

// Everything a kernel needs about one layer call (a flattened kan_layer + the call operands).
struct LayerArgs {
  int basis, act_dtype;
  int B, D_in, D_out, K, has_base, has_bias, input_map, wavelet_type, grid_size;
  float inv_den, grid_min, inv_h, ln_eps;
  const float* grid;
  const float* translation;
  const float* inv_scale;
  const void* X;
  void* Y;
  const void* bias;
  kan_weight w, wb;
  int* err;  // device error word (set when a bounded wait expires)
  const void* tc_weights;  // tensor-core layout weights (kan_tc_pack), act dtype
  // GatedKAN gate + up in one launch (tensor-core path only): tc_weights holds the two layers'
  // rows interleaved in blocks of 128 (kan_tc_pack_pair), D_out counts those rows, and the
  // epilogue writes Y = silu(gate) * up, [B][h_cols]; bias / has_bias belong to gate, bias2 /
  // has_bias2 to up
  int fuse_swiglu, h_cols, has_bias2;
  const void* bias2;
  // limit of the tensor-core kernel's pipeline waits, in SM clock cycles (waits on copies and
  // MMAs already in flight always use the default of about one second)
  long long wait_cycles;
  float alpha, beta;  // Jacobi parameters
};

// One fp32 layer backward (kan_backward.cu): device pointers; dW / dWb / dbias / dX may be null
// (not computed).
struct BackwardArgs {
  int basis, B, D_in, D_out, K, has_base, grid_size;
  float inv_den, grid_min, inv_h;
  const float* grid;  // RBF centres
  const float* X;     // [B][D_in]
  const float* dY;    // [B][D_out]
  const float* W;     // [D_out][D_in * K]
  const float* Wb;    // [D_out][D_in]
  float* dW;
  float* dWb;
  float* dbias;
  float* dX;
};

// Rows of a gate/up pair in the interleaved tensor-core layout: per 256 output columns, 256
// gate rows then 256 up rows (one wide tile of the tensor-core kernel).
constexpr int PAIR_BLOCK = 256;
KAN_HD inline int pair_rows(int d_ffn) {
  return (d_ffn + PAIR_BLOCK - 1) / PAIR_BLOCK * 2 * PAIR_BLOCK;
}

// Feature blocking of the tensor-core weight layout: F whole features of KT terms per 64-column
// block (KT = K + has_base: the K basis terms, then the base-branch weight).
struct TcBlocking {
  int KT, F, NB;
};
KAN_HD inline TcBlocking tc_blocking(int D_in, int K, int has_base) {
  TcBlocking b;
  b.KT = K + (has_base ? 1 : 0);
  b.F = b.KT > 0 ? 64 / b.KT : 0;
  b.NB = b.F > 0 ? (D_in + b.F - 1) / b.F : 0;
  return b;
}

}  // namespace kan
