// kan_tc_inst.cu -- compiled once per (KAN_TC_MODE, KAN_TC_BASIS) pair by build.py; instantiates
// the tensor-core kernels of that activation dtype and basis (see kan_tc_kernel.cuh).
#include "kan_tc_dispatch.h"
#include "kan_tc_kernel.cuh"

#if !defined(KAN_TC_MODE) || !defined(KAN_TC_BASIS)
#error "build with -DKAN_TC_MODE=<1|2> -DKAN_TC_BASIS=<0..6>"
#endif

#define KAN_CAT2(a, b, c) a##b##_##c
#define KAN_CAT(a, b, c) KAN_CAT2(a, b, c)

namespace kan {
namespace tc {

cudaError_t KAN_CAT(dispatch_, KAN_TC_MODE, KAN_TC_BASIS)(const CUtensorMap& tw,
                                                          const CUtensorMap& tx, int x_tma,
                                                          const LayerArgs& a, int BN, int nb,
                                                          int splits, dim3 grid, cudaStream_t s) {
  return dispatch_k<KAN_TC_BASIS, KAN_TC_MODE>(tw, tx, x_tma, a, BN, nb, splits, grid, s);
}

}  // namespace tc
}  // namespace kan
