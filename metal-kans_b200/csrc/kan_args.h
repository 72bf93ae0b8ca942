// kan_args.h -- the flattened per-call layer arguments every kernel receives (host + device).
#pragma once

#include "../../include/kan_cuda.h"

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
};

}  // namespace kan
