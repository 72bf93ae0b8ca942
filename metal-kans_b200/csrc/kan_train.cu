// kan_train.cu -- the elementwise pieces of the fp32 training step: the MSE loss gradient and the
// optimiser updates (AdamW, Adam with coupled weight decay, SGD with momentum / Nesterov, Lion),
// each one grid-stride pass over fp32 parameter, gradient and state arrays.  The update formulas
// and their order of operations follow the reference's kernels (fused_kan.metal:1884-1970 and
// the coupled Adam beside them), so a step moves the parameters by the same fp32 values.  They
// are HBM-bound: 16-24 bytes per parameter read and written once.
#include "kan_device.cuh"
#include "kan_launch.h"

namespace kan {
namespace train {

__global__ void mse_grad_kernel(const float* __restrict__ pred, const float* __restrict__ target,
                                float* __restrict__ dY, long long n, float scale) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x)
    dY[i] = (pred[i] - target[i]) * scale;
}

// One parameter tensor per blockIdx.y (up to three: weights, base weights, bias), so that a
// layer's whole update is one launch.
struct OptimTensors {
  float* param[3];
  const float* grad[3];
  float* m[3];
  float* v[3];
  long long n[3];
};

template <int OP>
__global__ void optim_kernel(OptimTensors t, OptimHyper h) {
  const int k = blockIdx.y;
  float* __restrict__ param = t.param[k];
  const float* __restrict__ grad = t.grad[k];
  float* __restrict__ m = t.m[k];
  float* __restrict__ v = t.v[k];
  const long long n = t.n[k];
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x) {
    float p = param[i];
    float g = grad[i];
    if (OP == OPTIM_ADAMW) {  // decoupled decay (adamw_step)
      if (h.weight_decay > 0.0f) p -= h.lr * h.weight_decay * p;
      const float mv = h.beta1 * m[i] + (1.0f - h.beta1) * g;
      const float vv = h.beta2 * v[i] + (1.0f - h.beta2) * (g * g);
      m[i] = mv;
      v[i] = vv;
      param[i] = p - h.lr_t * (mv / (sqrtf(vv) + h.eps));
    } else if (OP == OPTIM_ADAM) {  // decay added to the gradient (adam_coupled_step)
      if (h.weight_decay > 0.0f) g += h.weight_decay * p;
      const float mv = h.beta1 * m[i] + (1.0f - h.beta1) * g;
      const float vv = h.beta2 * v[i] + (1.0f - h.beta2) * (g * g);
      m[i] = mv;
      v[i] = vv;
      param[i] = p - h.lr_t * (mv / (sqrtf(vv) + h.eps));
    } else if (OP == OPTIM_SGD) {  // m = velocity (sgd_step)
      if (h.weight_decay > 0.0f) g += h.weight_decay * p;
      const float vel = h.beta1 * m[i] + g;  // beta1 = momentum
      m[i] = vel;
      const float upd = h.nesterov ? (g + h.beta1 * vel) : vel;
      param[i] = p - h.lr * upd;
    } else {  // OPTIM_LION (lion_step)
      if (h.weight_decay > 0.0f) p -= h.lr * h.weight_decay * p;
      const float mv = m[i];
      const float u = h.beta1 * mv + (1.0f - h.beta1) * g;
      const float s = u > 0.0f ? 1.0f : (u < 0.0f ? -1.0f : 0.0f);
      param[i] = p - h.lr * s;
      m[i] = h.beta2 * mv + (1.0f - h.beta2) * g;
    }
  }
}

static unsigned blocks_for(long long n) {
  long long b = (n + 255) / 256;
  const long long cap = 148LL * 8;  // the kernels stride; a few waves cover any size
  return (unsigned)(b < 1 ? 1 : (b > cap ? cap : b));
}

}  // namespace train

cudaError_t launch_mse_grad(const float* pred, const float* target, float* dY, long long n,
                            float scale, cudaStream_t s) {
  if (n <= 0) return cudaSuccess;
  note_launch();
  train::mse_grad_kernel<<<train::blocks_for(n), 256, 0, s>>>(pred, target, dY, n, scale);
  return cudaGetLastError();
}

cudaError_t launch_optim(int op, int count, float* const* param, const float* const* grad,
                         float* const* m, float* const* v, const long long* n,
                         const OptimHyper& h, cudaStream_t s) {
  if (count < 1 || count > 3) return cudaErrorInvalidValue;
  train::OptimTensors t = {};
  long long nmax = 0;
  for (int k = 0; k < count; ++k) {
    t.param[k] = param[k];
    t.grad[k] = grad[k];
    t.m[k] = m[k];
    t.v[k] = v ? v[k] : nullptr;
    t.n[k] = n[k];
    nmax = n[k] > nmax ? n[k] : nmax;
  }
  if (nmax <= 0) return cudaSuccess;
  const dim3 grid(train::blocks_for(nmax), (unsigned)count);
  note_launch();
  switch (op) {
    case OPTIM_ADAMW: train::optim_kernel<OPTIM_ADAMW><<<grid, 256, 0, s>>>(t, h); break;
    case OPTIM_ADAM: train::optim_kernel<OPTIM_ADAM><<<grid, 256, 0, s>>>(t, h); break;
    case OPTIM_SGD: train::optim_kernel<OPTIM_SGD><<<grid, 256, 0, s>>>(t, h); break;
    case OPTIM_LION: train::optim_kernel<OPTIM_LION><<<grid, 256, 0, s>>>(t, h); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

}  // namespace kan
