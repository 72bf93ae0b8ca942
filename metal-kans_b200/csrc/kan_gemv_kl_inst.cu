// kan_gemv_kl_inst.cu -- instances of the lanes-along-K small-batch kernel for one (activation
// dtype, batch size) pair, given as KAN_KL_MODE and KAN_KL_NB: both ternary decoders.  One
// translation unit per pair so that they compile in parallel.
#include <type_traits>

#include "kan_gemv_kl.cuh"

#ifndef KAN_KL_MODE
#error "define KAN_KL_MODE and KAN_KL_NB"
#endif

namespace kan {
namespace kl {

template <>
KlFn select_kl<KAN_KL_MODE, KAN_KL_NB>(bool fast) {
  if (fast) return kan_gemv_kl_kernel<KAN_KL_MODE, true, KAN_KL_NB>;
  return kan_gemv_kl_kernel<KAN_KL_MODE, false, KAN_KL_NB>;
}

}  // namespace kl
}  // namespace kan
