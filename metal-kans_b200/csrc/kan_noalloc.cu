// kan_noalloc.cu -- GatedKAN block forward that allocates no memory.
//
// Some callers cannot call cudaMalloc at all: code that runs inside a framework's memory arena or
// a serving runtime that forbids allocation after start-up, code on a path where a cudaMalloc
// would synchronise the device or fail for lack of free memory at the wrong moment, and callers
// that only hold pointers handed to them.  kan_gated_forward() keeps the gate and up activations
// in scratch it allocates on first use (and grows later); this variant keeps them in a fixed
// device array that exists from the moment the library is loaded, so a call never allocates.
//
// The array is shared by every call on a device and keeps the previous call's contents.  Nothing
// in it needs to start at zero: the gate and up kernels overwrite every element they later read.
// Calls that overlap on the GPU (different streams, or host threads racing on one device) use
// the same array and therefore race; callers must order them.
#include <cuda_runtime.h>

#include <mutex>

#include "../../include/kan_cuda.h"
#include "kan_launch.h"

namespace {

// Gate and up activations of one call: 2 * B * D_ffn elements of the act dtype.
constexpr size_t kNoallocScratchBytes = 32u << 20;  // 32 MiB per device that loads the library
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoallocScratchBytes];

constexpr int kMaxDevices = 16;
std::mutex g_mu;
void* g_scratch_addr[kMaxDevices] = {};

// Device address of the array on the current device, looked up once per device with that device
// current (in host code the array's name only stands for it and must never reach a kernel).
int scratch_address(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return KAN_ERR_NO_DEVICE;
  if (dev < 0 || dev >= kMaxDevices) return KAN_ERR_ARG;
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_scratch_addr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p) return KAN_ERR_CUDA;
    g_scratch_addr[dev] = p;
  }
  *out = g_scratch_addr[dev];
  return KAN_OK;
}

}  // namespace

extern "C" {

// GatedKAN forward without any allocation: Y = down(silu(gate(X)) * up(X)), H the caller's
// [B][gate->D_out] buffer for the gated activations.  The gate/up activations live in a fixed
// 32 MiB device array, so 2 * B * gate->D_out * sizeof(act dtype) must not exceed 32 MiB.  f16/bf16
// layers run on the tensor cores only when their tc_weights are packed in advance
// (kan_tc_pack); otherwise they run on the CUDA-core path, which needs no scratch either.
int kan_gated_forward_noalloc(const kan_layer* gate, const kan_layer* up, const kan_layer* down,
                              const void* X, void* H, void* Y, int B, void* stream) {
  if (!gate || !up || !down || !H || B < 0)
    return kan::set_error(KAN_ERR_ARG, "kan_gated_forward_noalloc: NULL argument or B < 0");
  if (gate->D_out != up->D_out || down->D_in != gate->D_out || gate->D_in != up->D_in ||
      gate->act_dtype != up->act_dtype || down->act_dtype != gate->act_dtype)
    return kan::set_error(KAN_ERR_ARG,
                          "kan_gated_forward_noalloc: inconsistent gate/up/down shapes or dtypes");
  const size_t esz = gate->act_dtype == KAN_F32 ? 4 : 2;
  const size_t one = (size_t)B * (size_t)gate->D_out * esz;  // gate (or up) activations
  const size_t up_off = (one + 255) & ~size_t(255);
  if (up_off + one > kNoallocScratchBytes)
    return kan::set_error(KAN_ERR_UNSUPPORTED,
                          "kan_gated_forward_noalloc: 2 * B * D_ffn * sizeof(dtype) exceeds the "
                          "fixed 32 MiB scratch; split the batch or use kan_gated_forward");
  if (B == 0) return KAN_OK;
  void* base = nullptr;
  int rc = scratch_address(&base);
  if (rc) return kan::set_error(rc, "kan_gated_forward_noalloc: no device scratch address");
  void* g = base;
  void* u = static_cast<unsigned char*>(base) + up_off;
  const kan_layer* layers[3] = {gate, up, down};
  int path[3];
  for (int i = 0; i < 3; ++i) {
    const bool lowp = layers[i]->act_dtype != KAN_F32;
    path[i] = (lowp && layers[i]->tc_weights) ? KAN_PATH_TC : KAN_PATH_SIMT;
  }
  // a layer the tensor cores cannot take (e.g. no tensor-map encoder in this driver) runs on the
  // CUDA cores, as kan_gated_forward() would run it; neither path allocates
  auto run = [&](const kan_layer* L, const void* in, void* out, int p) {
    int r = kan_forward_path(L, in, out, B, p, stream);
    if (r == KAN_ERR_UNSUPPORTED && p == KAN_PATH_TC)
      r = kan_forward_path(L, in, out, B, KAN_PATH_SIMT, stream);
    return r;
  };
  if ((rc = run(gate, X, g, path[0]))) return rc;
  if ((rc = run(up, X, u, path[1]))) return rc;
  if ((rc = kan_swiglu(g, u, H, (long long)B * gate->D_out, gate->act_dtype, stream))) return rc;
  return run(down, H, Y, path[2]);
}

}  // extern "C"
