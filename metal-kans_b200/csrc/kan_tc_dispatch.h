// kan_tc_dispatch.h -- the tensor-core kernel instances, one per (activation dtype, basis), each
// compiled from kan_tc_inst.cu in its own translation unit.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include "kan_args.h"

namespace kan {
namespace tc {

// tw: the packed weights; tx: the input [B][D_in] in 64-feature x 128-row tiles, used when x_tma
using DispatchFn = cudaError_t (*)(const CUtensorMap& tw, const CUtensorMap& tx, int x_tma,
                                   const LayerArgs& a, int BN, int nb, int splits, dim3 grid,
                                   cudaStream_t s);

#define KAN_TC_DECL(MODE, BASIS)                                                              \
  cudaError_t dispatch_##MODE##_##BASIS(const CUtensorMap& tw, const CUtensorMap& tx,          \
                                        int x_tma, const LayerArgs& a, int BN, int nb,         \
                                        int splits, dim3 grid, cudaStream_t s);
KAN_TC_DECL(1, 0) KAN_TC_DECL(1, 1) KAN_TC_DECL(1, 2) KAN_TC_DECL(1, 3)
KAN_TC_DECL(1, 4) KAN_TC_DECL(1, 5) KAN_TC_DECL(1, 6)
KAN_TC_DECL(2, 0) KAN_TC_DECL(2, 1) KAN_TC_DECL(2, 2) KAN_TC_DECL(2, 3)
KAN_TC_DECL(2, 4) KAN_TC_DECL(2, 5) KAN_TC_DECL(2, 6)
#undef KAN_TC_DECL

}  // namespace tc
}  // namespace kan
