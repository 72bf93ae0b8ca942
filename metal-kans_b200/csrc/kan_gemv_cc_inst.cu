// kan_gemv_cc_inst.cu -- main-kernel instances of the CUDA-core small-batch path for one
// (activation dtype, batch size) pair, given as KAN_CC_MODE and KAN_CC_NB: every weight format,
// ternary decoder and flush width.  One translation unit per pair so that they compile in
// parallel.
#include "kan_gemv_cc.cuh"

#ifndef KAN_CC_MODE
#error "define KAN_CC_MODE and KAN_CC_NB"
#endif

namespace kan {
namespace cc {

template <>
MainFn select_main<KAN_CC_MODE, KAN_CC_NB>(int fmt, bool fast, int fu) {
  constexpr int M = KAN_CC_MODE, N = KAN_CC_NB;
  if (fmt == KAN_W_TERNARY) {
    if (fast) {
      if (fu == 1) return kan_gemv_cc_kernel<M, KAN_W_TERNARY, true, 1, N>;
      if (fu == 2) return kan_gemv_cc_kernel<M, KAN_W_TERNARY, true, 2, N>;
      return kan_gemv_cc_kernel<M, KAN_W_TERNARY, true, 4, N>;
    }
    if (fu == 1) return kan_gemv_cc_kernel<M, KAN_W_TERNARY, false, 1, N>;
    if (fu == 2) return kan_gemv_cc_kernel<M, KAN_W_TERNARY, false, 2, N>;
    return kan_gemv_cc_kernel<M, KAN_W_TERNARY, false, 4, N>;
  }
  if (fmt == KAN_W_INT4) {
    if (fu == 1) return kan_gemv_cc_kernel<M, KAN_W_INT4, false, 1, N>;
    return kan_gemv_cc_kernel<M, KAN_W_INT4, false, 2, N>;
  }
  return kan_gemv_cc_kernel<M, KAN_W_INT8, false, 1, N>;
}

}  // namespace cc
}  // namespace kan
