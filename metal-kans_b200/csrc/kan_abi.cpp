// kan_abi.cpp -- the C ABI of libkan_cuda.so (declared in include/kan_cuda.h).
//
// Host runtime of the engine: per-device state (stream, staging buffers, scratch), kernel
// dispatch for kan_forward, the reference-compatible host-pointer entry points (the symbols the
// reference's ctypes loader binds, metal_kans/device.py:64-474), the host quantisers and the
// memory helpers.  No CPU compute fallback exists: every forward runs a CUDA kernel or fails.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <chrono>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <functional>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/kan_cuda.h"
#include "kan_launch.h"

namespace kan {

// ------------------------------------------------------------------------------------------
// errors
// ------------------------------------------------------------------------------------------
static thread_local std::string t_err;

static int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  t_err = buf;
  return code;
}

#define KAN_CUDA_TRY(expr)                                                                 \
  do {                                                                                     \
    cudaError_t e_ = (expr);                                                               \
    if (e_ != cudaSuccess)                                                                 \
      return fail(KAN_ERR_CUDA, "%s failed: %s (%s:%d)", #expr, cudaGetErrorString(e_),   \
                  __FILE__, __LINE__);                                                     \
  } while (0)

int set_error(int code, const char* msg) { return fail(code, "%s", msg); }

static std::atomic<long long> g_launches{0};
void note_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }
long long launch_count() { return g_launches.load(); }

// kan_set_wait_limit(): 0 = the kernels' default (about one second of SM clocks)
static std::atomic<long long> g_wait_limit{0};
long long pipeline_wait_limit() { return g_wait_limit.load(std::memory_order_relaxed); }

// ------------------------------------------------------------------------------------------
// per-device state
// ------------------------------------------------------------------------------------------
constexpr int MAX_DEVICES = 16;
enum Slot { S_X, S_W, S_WB, S_BIAS, S_Y, S_GRID, S_TRANS, S_ISC, S_SC, S_BI, S_CB, S_T0, S_T1,
            S_DY, S_DW, S_DWB, S_DBIAS, S_DX, NUM_SLOTS };

struct PendingCopy {
  void* pinned;
  void* user;
  size_t bytes;
};

// Engine scratch of one stream: packed tensor-core weights (when the caller passes none) and the
// GatedKAN gate/up activations.  Kept per stream so that work queued on different streams never
// shares a buffer.
enum ScratchId { SC_TCW, SC_GATE, SC_UP, SC_PHI, SC_HX, SC_HY, SC_CC, SC_TY, SC_TDY, SC_TDW,
                 SC_TDWB, SC_TDB, NUM_SCRATCH };
struct Scratch {
  cudaStream_t stream = nullptr;
  void* ptr[NUM_SCRATCH] = {};
  size_t cap[NUM_SCRATCH] = {};
};

struct DeviceState {
  bool init = false;
  cudaStream_t stream = nullptr;
  int* err_word = nullptr;
  int* err_host = nullptr;  // pinned mirror of the error word (read back on the engine stream)
  void* slot_ptr[NUM_SLOTS] = {};
  size_t slot_cap[NUM_SLOTS] = {};
  std::vector<PendingCopy> pending;     // async-mode results waiting for metal_kan_sync()
  std::vector<std::pair<void*, size_t>> pinned_free;  // reusable pinned buffers
  std::vector<Scratch*> scratch;        // one per stream that ran the engine
  // kan_forward_host: copy streams (host->device, device->host) and per-chunk events
  cudaStream_t h2d = nullptr, d2h = nullptr;
  static constexpr int kMaxChunks = 4;  // kan_forward_host: copy/compute overlap chunks
  cudaEvent_t ev_in[kMaxChunks] = {}, ev_done[kMaxChunks] = {};
};

static DeviceState g_dev[MAX_DEVICES];
static std::mutex g_mu;
static thread_local int t_async = 0;

static int current_state(DeviceState** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0)
      return fail(KAN_ERR_NO_DEVICE, "no CUDA device: %s", cudaGetErrorString(e));
    return fail(KAN_ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
  }
  if (dev < 0 || dev >= MAX_DEVICES) return fail(KAN_ERR_ARG, "device index %d too large", dev);
  DeviceState& d = g_dev[dev];
  if (!d.init) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (!d.init) {
      KAN_CUDA_TRY(cudaStreamCreateWithFlags(&d.stream, cudaStreamNonBlocking));
      d.err_word = device_error_ptr();
      if (!d.err_word) return fail(KAN_ERR_CUDA, "device error word unavailable");
      KAN_CUDA_TRY(cudaHostAlloc((void**)&d.err_host, sizeof(int), cudaHostAllocDefault));
      d.init = true;
    }
  }
  *out = &d;
  return KAN_OK;
}

static int slot(DeviceState* d, int s, size_t bytes, void** out) {
  if (bytes == 0) bytes = 16;
  if (d->slot_cap[s] < bytes) {
    if (d->slot_ptr[s]) {
      cudaStreamSynchronize(d->stream);
      cudaFree(d->slot_ptr[s]);
      d->slot_ptr[s] = nullptr;
      d->slot_cap[s] = 0;
    }
    size_t cap = std::max<size_t>(bytes, 4096);
    KAN_CUDA_TRY(cudaMalloc(&d->slot_ptr[s], cap));
    d->slot_cap[s] = cap;
  }
  *out = d->slot_ptr[s];
  return KAN_OK;
}

static Scratch* scratch_for(DeviceState* d, cudaStream_t s) {
  std::lock_guard<std::mutex> lk(g_mu);
  for (Scratch* sc : d->scratch)
    if (sc->stream == s) return sc;
  Scratch* sc = new Scratch();
  sc->stream = s;
  d->scratch.push_back(sc);
  return sc;
}

// Grow-only scratch buffer `id` of stream s; new buffers are zeroed when `zero` is set.
static int scratch_buf(DeviceState* d, cudaStream_t s, int id, size_t bytes, bool zero,
                       void** out) {
  Scratch* sc = scratch_for(d, s);
  if (bytes == 0) bytes = 16;
  if (sc->cap[id] < bytes) {
    if (sc->ptr[id]) {
      KAN_CUDA_TRY(cudaStreamSynchronize(s));
      cudaFree(sc->ptr[id]);
      sc->ptr[id] = nullptr;
      sc->cap[id] = 0;
    }
    KAN_CUDA_TRY(cudaMalloc(&sc->ptr[id], bytes));
    sc->cap[id] = bytes;
    if (zero) KAN_CUDA_TRY(cudaMemsetAsync(sc->ptr[id], 0, bytes, s));
  }
  *out = sc->ptr[id];
  return KAN_OK;
}

static int stage_in(DeviceState* d, int s, const void* host, size_t bytes, void** dev) {
  int rc = slot(d, s, bytes, dev);
  if (rc) return rc;
  if (host && bytes) KAN_CUDA_TRY(cudaMemcpyAsync(*dev, host, bytes, cudaMemcpyHostToDevice, d->stream));
  return KAN_OK;
}

// Read (and clear) the device error word through the pinned mirror on the engine stream: a
// 4-byte copy ordered after the work already queued there, no device-wide synchronisation.
static int read_device_error(DeviceState* d, int* out) {
  KAN_CUDA_TRY(cudaMemcpyAsync(d->err_host, d->err_word, sizeof(int), cudaMemcpyDeviceToHost,
                               d->stream));
  KAN_CUDA_TRY(cudaStreamSynchronize(d->stream));
  const int v = *d->err_host;
  if (v) {
    KAN_CUDA_TRY(cudaMemsetAsync(d->err_word, 0, sizeof(int), d->stream));
    KAN_CUDA_TRY(cudaStreamSynchronize(d->stream));
  }
  *out = v;
  return KAN_OK;
}

static int check_device_error(DeviceState* d) {
  int v = 0;
  int rc = read_device_error(d, &v);
  if (rc) return rc;
  if (v) return fail(KAN_ERR_DEVICE_TIMEOUT, "a kernel's bounded wait expired (code %d)", v);
  return KAN_OK;
}

// Copy the result back: synchronously, or (async mode) into pinned memory completed by sync().
static int stage_out(DeviceState* d, void* host, const void* dev, size_t bytes) {
  if (!t_async) {
    KAN_CUDA_TRY(cudaMemcpyAsync(host, dev, bytes, cudaMemcpyDeviceToHost, d->stream));
    KAN_CUDA_TRY(cudaStreamSynchronize(d->stream));
    return check_device_error(d);
  }
  void* pin = nullptr;
  for (size_t i = 0; i < d->pinned_free.size(); ++i) {
    if (d->pinned_free[i].second >= bytes) {
      pin = d->pinned_free[i].first;
      d->pinned_free.erase(d->pinned_free.begin() + i);
      break;
    }
  }
  if (!pin) KAN_CUDA_TRY(cudaHostAlloc(&pin, std::max<size_t>(bytes, 4096), cudaHostAllocDefault));
  KAN_CUDA_TRY(cudaMemcpyAsync(pin, dev, bytes, cudaMemcpyDeviceToHost, d->stream));
  d->pending.push_back({pin, host, std::max<size_t>(bytes, 4096)});
  d->pending.back().bytes = bytes;
  return KAN_OK;
}

static int sync_pending(DeviceState* d) {
  KAN_CUDA_TRY(cudaStreamSynchronize(d->stream));
  for (auto& p : d->pending) {
    std::memcpy(p.user, p.pinned, p.bytes);
    d->pinned_free.push_back({p.pinned, std::max<size_t>(p.bytes, 4096)});
  }
  d->pending.clear();
  return check_device_error(d);
}

// ------------------------------------------------------------------------------------------
// validation + dispatch
// ------------------------------------------------------------------------------------------
static size_t dtype_size(int dt) { return dt == KAN_F32 ? 4 : 2; }

static int validate_weight(const kan_weight& w, const char* name, int act_dtype) {
  switch (w.format) {
    case KAN_W_DENSE:
      if (!w.data) return fail(KAN_ERR_ARG, "%s: dense weight pointer is NULL", name);
      return KAN_OK;
    case KAN_W_INT8:
    case KAN_W_INT4:
      if (!w.data || !w.scales || !w.biases || w.group_size <= 0 || w.padded_cols <= 0 ||
          (w.format == KAN_W_INT4 && (w.group_size & 1)))
        return fail(KAN_ERR_ARG, "%s: incomplete INT8/INT4 weight", name);
      return KAN_OK;
    case KAN_W_TERNARY:
    case KAN_W_INT2:
      if (!w.data || !w.scales || w.group_size <= 0 ||
          (w.format == KAN_W_INT2 && !w.codebook))
        return fail(KAN_ERR_ARG, "%s: incomplete 2-bit weight", name);
      return KAN_OK;
    default:
      return fail(KAN_ERR_ARG, "%s: unknown weight format %d", name, w.format);
  }
  (void)act_dtype;
}

static int make_args(const kan_layer* L, const void* X, void* Y, int B, DeviceState* d,
                     LayerArgs* a) {
  if (!L) return fail(KAN_ERR_ARG, "layer descriptor is NULL");
  if (B < 0) return fail(KAN_ERR_ARG, "B = %d", B);
  if (L->D_in <= 0 || L->D_out <= 0 || L->K <= 0)
    return fail(KAN_ERR_ARG, "bad layer dims D_in=%d D_out=%d K=%d", L->D_in, L->D_out, L->K);
  if (L->K > 64) return fail(KAN_ERR_UNSUPPORTED, "K=%d terms per feature (max 64)", L->K);
  if (L->act_dtype < KAN_F32 || L->act_dtype > KAN_BF16)
    return fail(KAN_ERR_ARG, "act_dtype %d", L->act_dtype);
  if (L->basis < KAN_CHEBY || L->basis > KAN_JACOBI) return fail(KAN_ERR_ARG, "basis %d", L->basis);
  if (B > 0 && (!X || !Y)) return fail(KAN_ERR_ARG, "X or Y is NULL");
  if ((L->basis == KAN_RBF || L->basis == KAN_RELU) && !L->grid)
    return fail(KAN_ERR_ARG, "RBF / ReLU layer without grid");
  if (L->basis == KAN_WAVELET && (!L->translation || !L->inv_scale))
    return fail(KAN_ERR_ARG, "wavelet layer without translation/inv_scale");
  if (L->basis == KAN_BSPLINE && (L->grid_size <= 0 || L->K != L->grid_size + 3))
    return fail(KAN_ERR_ARG, "BSpline layer needs K = grid_size + 3 (K=%d G=%d)", L->K,
                L->grid_size);
  if (L->has_bias && !L->bias) return fail(KAN_ERR_ARG, "has_bias without bias pointer");
  int rc = validate_weight(L->w, "w", L->act_dtype);
  if (rc) return rc;
  if (L->has_base) {
    rc = validate_weight(L->wb, "wb", L->act_dtype);
    if (rc) return rc;
  }
  std::memset(a, 0, sizeof(*a));
  a->basis = L->basis;
  a->act_dtype = L->act_dtype;
  a->B = B;
  a->D_in = L->D_in;
  a->D_out = L->D_out;
  a->K = L->K;
  a->has_base = L->has_base ? 1 : 0;
  a->has_bias = L->has_bias ? 1 : 0;
  a->input_map = L->input_map;
  a->wavelet_type = L->wavelet_type;
  a->grid_size = L->grid_size;
  a->inv_den = L->inv_den;
  a->grid_min = L->grid_min;
  a->inv_h = L->inv_h;
  a->ln_eps = L->ln_eps > 0.f ? L->ln_eps : 1e-5f;
  a->grid = L->grid;
  a->translation = L->translation;
  a->inv_scale = L->inv_scale;
  a->X = X;
  a->Y = Y;
  a->bias = L->bias;
  a->w = L->w;
  a->wb = L->wb;
  a->err = d->err_word;
  a->tc_weights = L->tc_weights;
  a->wait_cycles = pipeline_wait_limit();
  a->alpha = L->alpha;
  a->beta = L->beta;
  return KAN_OK;
}

// Tensor-core launch: packs the weights into scratch when the caller did not.
static int run_tc(LayerArgs& a, int act_dtype, cudaStream_t s, DeviceState* d) {
  const TcPlan p = tc_plan(a);
  int rc;
  if (!a.tc_weights) {
    const TcBlocking bl = tc_blocking(a.D_in, a.K, a.has_base);
    void* buf;
    if ((rc = scratch_buf(d, s, SC_TCW, (size_t)bl.NB * 64 * a.D_out * 2, false, &buf))) return rc;
    cudaError_t e = launch_tc_pack(a, act_dtype, buf, s);
    if (e != cudaSuccess) return fail(KAN_ERR_CUDA, "weight pack: %s", cudaGetErrorString(e));
    a.tc_weights = buf;
  }
  cudaError_t e = launch_tc(a, act_dtype, p, s);
  if (e != cudaSuccess) return fail(KAN_ERR_CUDA, "tensor-core launch: %s", cudaGetErrorString(e));
  return KAN_OK;
}

// KAN_PATH_AUTO: the small-batch kernel where it applies, else the tensor cores for f16/bf16,
// else the CUDA cores.
static int auto_path(const LayerArgs& a, int act_dtype) {
  if (gemv_cc_supported(a, act_dtype)) return KAN_PATH_GEMV_CC;
  if (gemv_supported(a, act_dtype)) return KAN_PATH_GEMV;
  if (act_dtype != KAN_F32 && tc_supported(a, act_dtype)) return KAN_PATH_TC;
  return KAN_PATH_SIMT;
}

static int run_forward(const kan_layer* L, const void* X, void* Y, int B, int path,
                       cudaStream_t s, DeviceState* d) {
  LayerArgs a;
  int rc = make_args(L, X, Y, B, d, &a);
  if (rc) return rc;
  if (B == 0) return KAN_OK;
  cudaError_t e;
  const bool gemv_ok = gemv_supported(a, L->act_dtype);
  if (path == KAN_PATH_AUTO) path = auto_path(a, L->act_dtype);
  if (path == KAN_PATH_TC) {
    if (!tc_supported(a, L->act_dtype))
      return fail(KAN_ERR_UNSUPPORTED,
                  "tensor-core path needs an f16/bf16 layer with K + has_base <= 64");
    return run_tc(a, L->act_dtype, s, d);
  } else if (path == KAN_PATH_GEMV) {
    if (!gemv_ok)
      return fail(KAN_ERR_UNSUPPORTED,
                  "small-batch path needs an f16/bf16 Chebyshev layer with ternary/INT2 weights "
                  "(group 32/64/128), B <= 64, D_in >= 512, D_out >= 256");
    void* phi;
    if ((rc = scratch_buf(d, s, SC_PHI, gemv_phi_bytes(a), false, &phi))) return rc;
    e = launch_gemv(a, L->act_dtype, phi, s);
  } else if (path == KAN_PATH_GEMV_CC) {
    if (!gemv_cc_supported(a, L->act_dtype))
      return fail(KAN_ERR_UNSUPPORTED,
                  "CUDA-core small-batch path needs an f16/bf16 layer with ternary/INT8/INT4 "
                  "weights (group a multiple of 16), B <= 4, and code rows of >= 128 bytes");
    void* scratch;
    // zeroed when first allocated: the split counters start at zero (the pre-pass resets them)
    if ((rc = scratch_buf(d, s, SC_CC, gemv_cc_scratch_bytes(a), true, &scratch))) return rc;
    e = launch_gemv_cc(a, L->act_dtype, scratch, s);
  } else if (path == KAN_PATH_SIMT) {
    e = launch_simt(a, L->act_dtype, s);
  } else {
    return fail(KAN_ERR_ARG, "unknown path %d", path);
  }
  if (e != cudaSuccess) return fail(KAN_ERR_CUDA, "kernel launch: %s", cudaGetErrorString(e));
  return KAN_OK;
}

static cudaStream_t pick_stream(void* s, DeviceState* d) {
  return s ? (cudaStream_t)s : d->stream;
}

}  // namespace kan

using namespace kan;

// ==========================================================================================
// tier 2: device-resident engine
// ==========================================================================================
extern "C" {

const char* kan_last_error(void) { return t_err.c_str(); }
int kan_abi_version(void) { return 100; }
long long kan_launch_count(void) { return launch_count(); }

int kan_forward_path(const kan_layer* layer, const void* X, void* Y, int B, int path,
                     void* stream) {
  DeviceState* d;
  int rc = current_state(&d);
  if (rc) return rc;
  return run_forward(layer, X, Y, B, path, pick_stream(stream, d), d);
}

int kan_forward(const kan_layer* layer, const void* X, void* Y, int B, void* stream) {
  return kan_forward_path(layer, X, Y, B, KAN_PATH_AUTO, stream);
}

int kan_forward_plan(const kan_layer* layer, int B, int path, int* info) {
  DeviceState* d;
  int rc = current_state(&d);
  if (rc) return rc;
  if (!info) return fail(KAN_ERR_ARG, "forward_plan: NULL info");
  // any non-null pointers: the plan depends on shapes, formats and alignment of the weights only
  static const uint8_t dummy[16] = {};
  LayerArgs a;
  if ((rc = make_args(layer, dummy, (void*)dummy, B, d, &a))) return rc;
  if (path == KAN_PATH_AUTO) path = auto_path(a, layer->act_dtype);
  for (int i = 0; i < 6; ++i) info[i] = 0;
  info[0] = path;
  if (path == KAN_PATH_TC) {
    if (!tc_supported(a, layer->act_dtype))
      return fail(KAN_ERR_UNSUPPORTED, "forward_plan: the layer does not fit the tensor cores");
    const TcPlan p = tc_plan(a);
    info[1] = p.BN;
    info[2] = p.splits;
    info[3] = p.mtiles;
    info[4] = p.ntiles;
    info[5] = p.nb;
  } else if (path == KAN_PATH_GEMV) {
    if (!gemv_supported(a, layer->act_dtype))
      return fail(KAN_ERR_UNSUPPORTED, "forward_plan: the layer does not fit the small-batch path");
    info[3] = (layer->D_out + 127) / 128;
  } else if (path == KAN_PATH_GEMV_CC) {
    if (!gemv_cc_supported(a, layer->act_dtype))
      return fail(KAN_ERR_UNSUPPORTED,
                  "forward_plan: the layer does not fit the CUDA-core small-batch path");
    info[2] = gemv_cc_splits(a);
    info[3] = (layer->D_out + 31) / 32;
  } else if (path != KAN_PATH_SIMT) {
    return fail(KAN_ERR_ARG, "forward_plan: unknown path %d", path);
  }
  return KAN_OK;
}

int kan_set_wait_limit(long long cycles) {
  if (cycles < 0) return fail(KAN_ERR_ARG, "wait limit %lld < 0", cycles);
  g_wait_limit.store(cycles, std::memory_order_relaxed);
  return KAN_OK;
}

int kan_forward_host(const kan_layer* layer, const void* X, void* Y, int B) {
  DeviceState* d;
  int rc = current_state(&d);
  if (rc) return rc;
  if (!layer) return fail(KAN_ERR_ARG, "forward_host: NULL layer");
  if (B < 0) return fail(KAN_ERR_ARG, "forward_host: B < 0");
  if (B == 0) return KAN_OK;
  if (!X || !Y) return fail(KAN_ERR_ARG, "forward_host: NULL X or Y");
  const size_t esz = dtype_size(layer->act_dtype);
  const size_t xrow = (size_t)layer->D_in * esz, yrow = (size_t)layer->D_out * esz;
  if (!d->h2d) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (!d->h2d) {
      KAN_CUDA_TRY(cudaStreamCreateWithFlags(&d->d2h, cudaStreamNonBlocking));
      for (int c = 0; c < DeviceState::kMaxChunks; ++c) {
        KAN_CUDA_TRY(cudaEventCreateWithFlags(&d->ev_in[c], cudaEventDisableTiming));
        KAN_CUDA_TRY(cudaEventCreateWithFlags(&d->ev_done[c], cudaEventDisableTiming));
      }
      cudaStream_t h;
      KAN_CUDA_TRY(cudaStreamCreateWithFlags(&h, cudaStreamNonBlocking));
      d->h2d = h;
    }
  }
  void *dX, *dY;
  if ((rc = scratch_buf(d, d->stream, SC_HX, (size_t)B * xrow, false, &dX))) return rc;
  if ((rc = scratch_buf(d, d->stream, SC_HY, (size_t)B * yrow, false, &dY))) return rc;
  // chunks (at 128-row boundaries) once the copies are worth overlapping: chunk c + 1's input
  // crosses the link while chunk c computes, and chunk c's result returns while chunk c + 1
  // computes, so only the first input and the last result copy stay exposed.  Four chunks from
  // 32768 rows (each still fills the GPU with row tiles), two from 2048 rows and 2 MB of copies.
  const bool big = (size_t)B * (xrow + yrow) >= ((size_t)2 << 20);
  const int nc = (big && B >= 32768) ? DeviceState::kMaxChunks : ((big && B >= 2048) ? 2 : 1);
  const int per = (B / nc + 127) / 128 * 128;
  for (int c = 0; c < nc; ++c) {
    const int r0 = std::min(B, c * per);
    const int rows = c == nc - 1 ? B - r0 : std::min(per, B - r0);
    if (rows <= 0) break;
    const char* xs = (const char*)X + (size_t)r0 * xrow;
    char* xd = (char*)dX + (size_t)r0 * xrow;
    char* yd = (char*)dY + (size_t)r0 * yrow;
    KAN_CUDA_TRY(cudaMemcpyAsync(xd, xs, (size_t)rows * xrow, cudaMemcpyHostToDevice, d->h2d));
    KAN_CUDA_TRY(cudaEventRecord(d->ev_in[c], d->h2d));
    KAN_CUDA_TRY(cudaStreamWaitEvent(d->stream, d->ev_in[c], 0));
    if ((rc = run_forward(layer, xd, yd, rows, KAN_PATH_AUTO, d->stream, d))) {
      cudaStreamSynchronize(d->h2d);
      cudaStreamSynchronize(d->stream);
      return rc;
    }
    KAN_CUDA_TRY(cudaEventRecord(d->ev_done[c], d->stream));
    KAN_CUDA_TRY(cudaStreamWaitEvent(d->d2h, d->ev_done[c], 0));
    KAN_CUDA_TRY(cudaMemcpyAsync((char*)Y + (size_t)r0 * yrow, yd, (size_t)rows * yrow,
                                 cudaMemcpyDeviceToHost, d->d2h));
  }
  // the device error word rides on the same copy stream (after the last kernel, which the last
  // result copy waited for): one synchronisation for the results and the error check
  KAN_CUDA_TRY(cudaMemcpyAsync(d->err_host, d->err_word, sizeof(int), cudaMemcpyDeviceToHost,
                               d->d2h));
  KAN_CUDA_TRY(cudaStreamSynchronize(d->d2h));
  if (*d->err_host) return check_device_error(d);  // reads it again on the engine stream, clears it
  return KAN_OK;
}

// Gate and up of a GatedKAN share their input and their basis (Chebyshev, same K, base branch and
// input map): one launch can evaluate the basis once for both.
static bool pair_compatible(const kan_layer* g, const kan_layer* u) {
  return g && u && g->basis == KAN_CHEBY && u->basis == KAN_CHEBY &&
         (g->act_dtype == KAN_F16 || g->act_dtype == KAN_BF16) && g->act_dtype == u->act_dtype &&
         g->K == u->K && g->D_in == u->D_in && g->D_out == u->D_out &&
         (g->has_base != 0) == (u->has_base != 0) && g->input_map == u->input_map;
}

int kan_tc_pair_bytes(const kan_layer* gate, const kan_layer* up, size_t* bytes) {
  if (!bytes) return fail(KAN_ERR_ARG, "pair_bytes: NULL output");
  if (!pair_compatible(gate, up))
    return fail(KAN_ERR_UNSUPPORTED, "gate/up pair: needs two f16/bf16 Chebyshev layers of one "
                                     "shape, K, base branch and input map");
  const TcBlocking bl = tc_blocking(gate->D_in, gate->K, gate->has_base);
  *bytes = (size_t)pair_rows(gate->D_out) * bl.NB * 64 * 2;
  return KAN_OK;
}

int kan_tc_pack_pair(const kan_layer* gate, const kan_layer* up, void* out, void* stream) {
  DeviceState* d;
  int rc = current_state(&d);
  if (rc) return rc;
  size_t bytes;
  if ((rc = kan_tc_pair_bytes(gate, up, &bytes))) return rc;
  if (!out) return fail(KAN_ERR_ARG, "pack_pair: NULL output");
  LayerArgs ag, au;
  if ((rc = make_args(gate, nullptr, nullptr, 0, d, &ag))) return rc;
  if ((rc = make_args(up, nullptr, nullptr, 0, d, &au))) return rc;
  cudaError_t e = launch_tc_pack_pair(ag, au, gate->act_dtype, out, pick_stream(stream, d));
  if (e != cudaSuccess) return fail(KAN_ERR_CUDA, "pair pack: %s", cudaGetErrorString(e));
  return KAN_OK;
}

int kan_gated_forward(const kan_layer* gate, const kan_layer* up, const kan_layer* down,
                      const void* X, void* H, void* Y, int B, void* stream) {
  DeviceState* d;
  int rc = current_state(&d);
  if (rc) return rc;
  if (!gate || !up || !down || !H) return fail(KAN_ERR_ARG, "gated: NULL argument");
  if (gate->D_out != up->D_out || down->D_in != gate->D_out || gate->D_in != up->D_in ||
      gate->act_dtype != up->act_dtype || down->act_dtype != gate->act_dtype)
    return fail(KAN_ERR_ARG, "gated: inconsistent gate/up/down shapes or dtypes");
  cudaStream_t s = pick_stream(stream, d);
  const size_t esz = dtype_size(gate->act_dtype);
  const size_t n = (size_t)B * gate->D_out;
  void *g, *u;
  if ((rc = scratch_buf(d, s, SC_GATE, n * esz, false, &g))) return rc;
  if ((rc = scratch_buf(d, s, SC_UP, n * esz, false, &u))) return rc;
  if ((rc = run_forward(gate, X, g, B, KAN_PATH_AUTO, s, d))) return rc;
  if ((rc = run_forward(up, X, u, B, KAN_PATH_AUTO, s, d))) return rc;
  cudaError_t e = launch_swiglu(g, u, H, (long long)n, gate->act_dtype, s);
  if (e != cudaSuccess) return fail(KAN_ERR_CUDA, "swiglu launch: %s", cudaGetErrorString(e));
  return run_forward(down, H, Y, B, KAN_PATH_AUTO, s, d);
}

int kan_gated_forward_pair(const kan_layer* gate, const kan_layer* up, const kan_layer* down,
                           const void* pair, const void* X, void* H, void* Y, int B,
                           void* stream) {
  DeviceState* d;
  int rc = current_state(&d);
  if (rc) return rc;
  if (!gate || !up || !down || !H) return fail(KAN_ERR_ARG, "gated: NULL argument");
  if (!pair || !pair_compatible(gate, up) || down->D_in != gate->D_out ||
      down->act_dtype != gate->act_dtype)
    return kan_gated_forward(gate, up, down, X, H, Y, B, stream);
  cudaStream_t s = pick_stream(stream, d);
  LayerArgs a, au;
  if ((rc = make_args(gate, X, H, B, d, &a))) return rc;
  if ((rc = make_args(up, X, H, B, d, &au))) return rc;
  if (B == 0) return KAN_OK;
  a.D_out = pair_rows(gate->D_out);
  a.tc_weights = pair;
  a.fuse_swiglu = 1;
  a.h_cols = gate->D_out;
  a.bias2 = au.bias;
  a.has_bias2 = au.has_bias;
  TcPlan p = tc_plan(a);
  // the fused epilogue needs wide, unsplit tiles; smaller grids take the separate launches
  if (!tc_supported(a, gate->act_dtype) || p.BN != 2 * PAIR_BLOCK || p.splits != 1)
    return kan_gated_forward(gate, up, down, X, H, Y, B, stream);
  cudaError_t e = launch_tc(a, gate->act_dtype, p, s);
  if (e != cudaSuccess) return fail(KAN_ERR_CUDA, "gate/up launch: %s", cudaGetErrorString(e));
  return run_forward(down, H, Y, B, KAN_PATH_AUTO, s, d);
}

int kan_tc_packed_bytes(const kan_layer* layer, size_t* bytes) {
  if (!layer || !bytes) return fail(KAN_ERR_ARG, "NULL argument");
  const int KT = layer->K + (layer->has_base ? 1 : 0);
  if (layer->D_in <= 0 || layer->D_out <= 0 || layer->K <= 0 || KT > 64)
    return fail(KAN_ERR_ARG, "tc layout needs D_in, D_out, K > 0 and K + has_base <= 64");
  const TcBlocking bl = tc_blocking(layer->D_in, layer->K, layer->has_base);
  *bytes = (size_t)bl.NB * 64 * layer->D_out * 2;
  return KAN_OK;
}

int kan_tc_pack(const kan_layer* layer, void* out, void* stream) {
  DeviceState* d;
  int rc = current_state(&d);
  if (rc) return rc;
  size_t bytes;
  if ((rc = kan_tc_packed_bytes(layer, &bytes))) return rc;
  if (!out) return fail(KAN_ERR_ARG, "tc pack: NULL output");
  if (layer->act_dtype != KAN_F16 && layer->act_dtype != KAN_BF16)
    return fail(KAN_ERR_ARG, "tc pack: the tensor-core layout is f16/bf16");
  LayerArgs a;
  // X/Y are not used by the pack kernel; B = 0 skips their checks
  if ((rc = make_args(layer, nullptr, nullptr, 0, d, &a))) return rc;
  cudaError_t e = launch_tc_pack(a, layer->act_dtype, out, pick_stream(stream, d));
  if (e != cudaSuccess) return fail(KAN_ERR_CUDA, "tc pack: %s", cudaGetErrorString(e));
  return KAN_OK;
}

int kan_dequantize(const kan_weight* w, int rows, int cols, void* out, int out_dtype,
                   void* stream) {
  DeviceState* d;
  int rc = current_state(&d);
  if (rc) return rc;
  if (!w || !out || rows <= 0 || cols <= 0) return fail(KAN_ERR_ARG, "dequantize: bad args");
  if ((rc = validate_weight(*w, "w", out_dtype))) return rc;
  if (w->format == KAN_W_DENSE) return fail(KAN_ERR_ARG, "dequantize: weight is already dense");
  cudaError_t e = launch_dequantize(*w, rows, cols, out, out_dtype, pick_stream(stream, d));
  if (e != cudaSuccess) return fail(KAN_ERR_CUDA, "dequantize launch: %s", cudaGetErrorString(e));
  return KAN_OK;
}

int kan_swiglu(const void* gate, const void* up, void* out, long long n, int act_dtype,
               void* stream) {
  DeviceState* d;
  int rc = current_state(&d);
  if (rc) return rc;
  if (n < 0 || (n > 0 && (!gate || !up || !out))) return fail(KAN_ERR_ARG, "swiglu: bad args");
  if (n == 0) return KAN_OK;
  cudaError_t e = launch_swiglu(gate, up, out, n, act_dtype, pick_stream(stream, d));
  if (e != cudaSuccess) return fail(KAN_ERR_CUDA, "swiglu launch: %s", cudaGetErrorString(e));
  return KAN_OK;
}

int kan_mult_combine(const void* in, void* out, int B, int num_add, int num_mult,
                     int act_dtype, void* stream) {
  DeviceState* d;
  int rc = current_state(&d);
  if (rc) return rc;
  if (B < 0 || num_add < 0 || num_mult < 0 || (B > 0 && (!in || !out)))
    return fail(KAN_ERR_ARG, "mult_combine: bad args");
  cudaError_t e = launch_mult_combine(in, out, B, num_add, num_mult, act_dtype,
                                      pick_stream(stream, d));
  if (e != cudaSuccess) return fail(KAN_ERR_CUDA, "mult_combine: %s", cudaGetErrorString(e));
  return KAN_OK;
}

int kan_lowrank_up(const void* Z, const void* X, const void* Wup, const void* Wb,
                   const void* bias, void* Y, int B, int D_in, int D_out, int rank, int has_base,
                   int has_bias, int act_dtype, void* stream) {
  DeviceState* d;
  int rc = current_state(&d);
  if (rc) return rc;
  if (B < 0 || D_in <= 0 || D_out <= 0 || rank <= 0 ||
      (B > 0 && (!Z || !Y || !Wup || (has_base && (!X || !Wb)) || (has_bias && !bias))))
    return fail(KAN_ERR_ARG, "lowrank_up: bad args");
  cudaError_t e = launch_lowrank_up(Z, X, Wup, Wb, bias, Y, B, D_in, D_out, rank, has_base,
                                    has_bias, act_dtype, pick_stream(stream, d));
  if (e != cudaSuccess) return fail(KAN_ERR_CUDA, "lowrank_up: %s", cudaGetErrorString(e));
  return KAN_OK;
}

int kan_rational_forward(const float* X, const float* Wp, const float* Wq, const float* Wb,
                         const float* bias, float* Y, int B, int D_in, int D_out, int p, int q,
                         int has_base, int has_bias, void* stream) {
  DeviceState* d;
  int rc = current_state(&d);
  if (rc) return rc;
  if (!rational_supported(p, q)) return fail(KAN_ERR_UNSUPPORTED, "rational: degrees");
  if (B < 0 || D_in <= 0 || D_out <= 0 ||
      (B > 0 && (!X || !Y || (p && !Wp) || (q && !Wq) || (has_base && !Wb) ||
                 (has_bias && !bias))))
    return fail(KAN_ERR_ARG, "rational: bad args");
  cudaError_t e = launch_rational(X, Wp, Wq, Wb, bias, Y, B, D_in, D_out, p, q, has_base,
                                  has_bias, pick_stream(stream, d));
  if (e != cudaSuccess) return fail(KAN_ERR_CUDA, "rational: %s", cudaGetErrorString(e));
  return KAN_OK;
}

int kan_convert(const void* src, int src_dtype, void* dst, int dst_dtype, long long n,
                void* stream) {
  DeviceState* d;
  int rc = current_state(&d);
  if (rc) return rc;
  if (n < 0 || (n > 0 && (!src || !dst))) return fail(KAN_ERR_ARG, "convert: bad args");
  if (n == 0) return KAN_OK;
  cudaError_t e = launch_convert(src, src_dtype, dst, dst_dtype, n, pick_stream(stream, d));
  if (e != cudaSuccess) return fail(KAN_ERR_CUDA, "convert launch: %s", cudaGetErrorString(e));
  return KAN_OK;
}

int kan_device_count(int* count) {
  if (!count) return fail(KAN_ERR_ARG, "NULL");
  cudaError_t e = cudaGetDeviceCount(count);
  if (e != cudaSuccess) {
    *count = 0;
    return fail(KAN_ERR_NO_DEVICE, "cudaGetDeviceCount: %s", cudaGetErrorString(e));
  }
  return KAN_OK;
}
int kan_set_device(int device) {
  KAN_CUDA_TRY(cudaSetDevice(device));
  return KAN_OK;
}
int kan_get_device(int* device) {
  if (!device) return fail(KAN_ERR_ARG, "NULL");
  KAN_CUDA_TRY(cudaGetDevice(device));
  return KAN_OK;
}
int kan_malloc(void** ptr, size_t bytes) {
  if (!ptr) return fail(KAN_ERR_ARG, "NULL");
  KAN_CUDA_TRY(cudaMalloc(ptr, bytes ? bytes : 16));
  return KAN_OK;
}
int kan_free(void* ptr) {
  if (ptr) KAN_CUDA_TRY(cudaFree(ptr));
  return KAN_OK;
}
int kan_host_alloc(void** ptr, size_t bytes) {
  if (!ptr) return fail(KAN_ERR_ARG, "NULL");
  KAN_CUDA_TRY(cudaHostAlloc(ptr, bytes ? bytes : 16, cudaHostAllocDefault));
  return KAN_OK;
}
int kan_host_free(void* ptr) {
  if (ptr) KAN_CUDA_TRY(cudaFreeHost(ptr));
  return KAN_OK;
}
int kan_memcpy(void* dst, const void* src, size_t bytes, int kind, void* stream) {
  DeviceState* d;
  int rc = current_state(&d);
  if (rc) return rc;
  if (bytes == 0) return KAN_OK;
  if (!dst || !src) return fail(KAN_ERR_ARG, "memcpy: NULL pointer");
  cudaMemcpyKind k = kind == 1 ? cudaMemcpyHostToDevice
                     : kind == 2 ? cudaMemcpyDeviceToHost
                                 : cudaMemcpyDeviceToDevice;
  KAN_CUDA_TRY(cudaMemcpyAsync(dst, src, bytes, k, pick_stream(stream, d)));
  return KAN_OK;
}
int kan_memset(void* dst, int value, size_t bytes, void* stream) {
  DeviceState* d;
  int rc = current_state(&d);
  if (rc) return rc;
  if (bytes == 0) return KAN_OK;
  KAN_CUDA_TRY(cudaMemsetAsync(dst, value, bytes, pick_stream(stream, d)));
  return KAN_OK;
}
int kan_stream_synchronize(void* stream) {
  DeviceState* d;
  int rc = current_state(&d);
  if (rc) return rc;
  KAN_CUDA_TRY(cudaStreamSynchronize(pick_stream(stream, d)));
  return KAN_OK;
}
void* kan_default_stream(void) {
  DeviceState* d;
  if (current_state(&d)) return nullptr;
  return (void*)d->stream;
}
int kan_device_error(int* code) {
  DeviceState* d;
  int rc = current_state(&d);
  if (rc) return rc;
  int v = 0;
  if ((rc = read_device_error(d, &v))) return rc;
  if (code) *code = v;
  return KAN_OK;
}

// ==========================================================================================
// tier 1: reference-compatible host-pointer entry points
// ==========================================================================================

int metal_kan_init(const char* shader_path) {
  (void)shader_path;
  DeviceState* d;
  return current_state(&d);
}

int metal_kan_set_async(int enabled) {
  if (!enabled && t_async) {
    t_async = 0;
    return metal_kan_sync();
  }
  t_async = enabled ? 1 : 0;
  return KAN_OK;
}

int metal_kan_sync(void) {
  DeviceState* d;
  int rc = current_state(&d);
  if (rc) return rc;
  return sync_pending(d);
}

}  // extern "C"

namespace kan {

// Stage a host-pointer layer call, run it, copy Y back.
struct HostLayer {
  kan_layer L;
  const void* X;
  void* Y;
  int B;
  // host sources for the dense operands
  const void* hW = nullptr;
  const void* hWb = nullptr;
  const void* hBias = nullptr;
  std::vector<float> grid, trans, isc;  // basis parameters, already fp32
  // optional second stage on the device output: (state, device X, device Y of the layer) ->
  // the buffer and size to copy back (MultKAN's pair products, LowRankKAN's up projection)
  std::function<int(DeviceState*, void*, void*, void**, size_t*)> post;
};

static int run_host_layer(HostLayer& h) {
  DeviceState* d;
  int rc = current_state(&d);
  if (rc) return rc;
  kan_layer& L = h.L;
  if (h.B < 0 || L.D_in <= 0 || L.D_out <= 0) return fail(KAN_ERR_ARG, "bad sizes");
  if (h.B > 0 && (!h.X || !h.Y || !h.hW)) return fail(KAN_ERR_ARG, "NULL X/Y/W");
  if (L.has_base && !h.hWb) return fail(KAN_ERR_ARG, "has_base with NULL W_base");
  if (L.has_bias && !h.hBias) return fail(KAN_ERR_ARG, "has_bias with NULL bias");
  if (h.B == 0) return KAN_OK;
  const size_t es = dtype_size(L.act_dtype);
  void *dX, *dY, *dW, *dWb = nullptr, *dB = nullptr, *dG = nullptr, *dT = nullptr, *dS = nullptr;
  if ((rc = stage_in(d, S_X, h.X, (size_t)h.B * L.D_in * es, &dX))) return rc;
  if ((rc = stage_in(d, S_W, h.hW, (size_t)L.D_out * L.D_in * L.K * es, &dW))) return rc;
  if (L.has_base && (rc = stage_in(d, S_WB, h.hWb, (size_t)L.D_out * L.D_in * es, &dWb))) return rc;
  if (L.has_bias && (rc = stage_in(d, S_BIAS, h.hBias, (size_t)L.D_out * es, &dB))) return rc;
  if (!h.grid.empty() && (rc = stage_in(d, S_GRID, h.grid.data(), h.grid.size() * 4, &dG))) return rc;
  if (!h.trans.empty() && (rc = stage_in(d, S_TRANS, h.trans.data(), h.trans.size() * 4, &dT))) return rc;
  if (!h.isc.empty() && (rc = stage_in(d, S_ISC, h.isc.data(), h.isc.size() * 4, &dS))) return rc;
  if ((rc = slot(d, S_Y, (size_t)h.B * L.D_out * es, &dY))) return rc;
  L.w.format = KAN_W_DENSE;
  L.w.data = dW;
  L.wb.format = KAN_W_DENSE;
  L.wb.data = dWb;
  L.bias = dB;
  L.grid = (const float*)dG;
  L.translation = (const float*)dT;
  L.inv_scale = (const float*)dS;
  if ((rc = run_forward(&L, dX, dY, h.B, KAN_PATH_AUTO, d->stream, d))) return rc;
  void* dOut = dY;
  size_t out_bytes = (size_t)h.B * L.D_out * es;
  if (h.post && (rc = h.post(d, dX, dY, &dOut, &out_bytes))) return rc;
  return stage_out(d, h.Y, dOut, out_bytes);
}

static kan_layer base_layer(int basis, int dt, int D_in, int D_out, int K, int hb, int hbi) {
  kan_layer L;
  std::memset(&L, 0, sizeof(L));
  L.basis = basis;
  L.act_dtype = dt;
  L.D_in = D_in;
  L.D_out = D_out;
  L.K = K;
  L.has_base = hb ? 1 : 0;
  L.has_bias = hbi ? 1 : 0;
  L.ln_eps = 1e-5f;
  return L;
}

static std::vector<float> half_to_float(const uint16_t* p, size_t n) {
  std::vector<float> v(n);
  for (size_t i = 0; i < n; ++i) {
    __half_raw r;
    r.x = p[i];
    v[i] = __half2float(__half(r));
  }
  return v;
}

}  // namespace kan

namespace kan {
// host-timed loop behind benchmark_metal_* (metal_kan_bridge.mm:1250-1371)
template <class F>
static double bench_loop(F&& fwd, int warmup, int iters) {
  if (iters <= 0) {
    fail(KAN_ERR_ARG, "iters must be > 0");
    return -1.0;
  }
  for (int i = 0; i < warmup; ++i)
    if (fwd()) return -1.0;
  auto t0 = std::chrono::steady_clock::now();
  for (int i = 0; i < iters; ++i)
    if (fwd()) return -1.0;
  auto t1 = std::chrono::steady_clock::now();
  return std::chrono::duration<double, std::milli>(t1 - t0).count() / iters;
}

}  // namespace kan

extern "C" {

int metal_kan_cheby_forward(const float* X, const float* W, const float* Wb, const float* bias,
                            float* Y, int B, int D_in, int D_out, int K, int hb, int hbi) {
  HostLayer h{base_layer(KAN_CHEBY, KAN_F32, D_in, D_out, K, hb, hbi), X, Y, B, W, Wb, bias};
  return run_host_layer(h);
}

int metal_kan_cheby_forward_fp16(const uint16_t* X, const uint16_t* W, const uint16_t* Wb,
                                 const uint16_t* bias, uint16_t* Y, int B, int D_in, int D_out,
                                 int K, int hb, int hbi) {
  HostLayer h{base_layer(KAN_CHEBY, KAN_F16, D_in, D_out, K, hb, hbi), X, Y, B, W, Wb, bias};
  return run_host_layer(h);
}

int metal_kan_fastkan_forward(const float* X, const float* W, const float* Wb, const float* grid,
                              const float* bias, float* Y, int B, int D_in, int D_out, int K,
                              float inv_den, int hb, int hbi) {
  if (!grid || K <= 0) return fail(KAN_ERR_ARG, "fastkan: NULL grid");
  HostLayer h{base_layer(KAN_RBF, KAN_F32, D_in, D_out, K, hb, hbi), X, Y, B, W, Wb, bias};
  h.L.inv_den = inv_den;
  h.grid.assign(grid, grid + K);
  return run_host_layer(h);
}

int metal_kan_fastkan_forward_fp16(const uint16_t* X, const uint16_t* W, const uint16_t* Wb,
                                   const uint16_t* grid, const uint16_t* bias, uint16_t* Y, int B,
                                   int D_in, int D_out, int K, float inv_den, int hb, int hbi) {
  if (!grid || K <= 0) return fail(KAN_ERR_ARG, "fastkan: NULL grid");
  HostLayer h{base_layer(KAN_RBF, KAN_F16, D_in, D_out, K, hb, hbi), X, Y, B, W, Wb, bias};
  h.L.inv_den = inv_den;
  h.grid = half_to_float(grid, K);
  return run_host_layer(h);
}

static int bspline_common(int dt, const void* X, const void* W, const void* Wb,
                          const float* grid, const void* bias, void* Y, int B, int D_in,
                          int D_out, int G, int hb, int hbi) {
  if (!grid || G <= 0) return fail(KAN_ERR_ARG, "bspline: NULL grid or grid_size <= 0");
  HostLayer h{base_layer(KAN_BSPLINE, dt, D_in, D_out, G + 3, hb, hbi), X, Y, B, W, Wb, bias};
  h.L.grid_size = G;
  h.L.grid_min = grid[0];
  h.L.inv_h = grid[1];
  return run_host_layer(h);
}

int metal_kan_bspline_forward(const float* X, const float* W, const float* Wb, const float* grid,
                              const float* bias, float* Y, int B, int D_in, int D_out, int G,
                              int spline_order, int hb, int hbi) {
  (void)spline_order;
  return bspline_common(KAN_F32, X, W, Wb, grid, bias, Y, B, D_in, D_out, G, hb, hbi);
}

int metal_kan_bspline_forward_fp16(const uint16_t* X, const uint16_t* W, const uint16_t* Wb,
                                   const float* grid, const uint16_t* bias, uint16_t* Y, int B,
                                   int D_in, int D_out, int G, int spline_order, int hb,
                                   int hbi) {
  (void)spline_order;
  return bspline_common(KAN_F16, X, W, Wb, grid, bias, Y, B, D_in, D_out, G, hb, hbi);
}

int metal_kan_wavkan_forward(const float* X, const float* W, const float* Wb, const float* trans,
                             const float* isc, const float* bias, float* Y, int B, int D_in,
                             int D_out, int nw, int wtype, int hb, int hbi) {
  if (!trans || !isc || nw <= 0) return fail(KAN_ERR_ARG, "wavkan: NULL translation/scale");
  HostLayer h{base_layer(KAN_WAVELET, KAN_F32, D_in, D_out, nw, hb, hbi), X, Y, B, W, Wb, bias};
  h.L.wavelet_type = wtype;
  h.trans.assign(trans, trans + (size_t)D_in * nw);
  h.isc.assign(isc, isc + (size_t)D_in * nw);
  return run_host_layer(h);
}

int metal_kan_wavkan_forward_fp16(const uint16_t* X, const uint16_t* W, const uint16_t* Wb,
                                  const uint16_t* trans, const uint16_t* isc,
                                  const uint16_t* bias, uint16_t* Y, int B, int D_in, int D_out,
                                  int nw, int wtype, int hb, int hbi) {
  if (!trans || !isc || nw <= 0) return fail(KAN_ERR_ARG, "wavkan: NULL translation/scale");
  HostLayer h{base_layer(KAN_WAVELET, KAN_F16, D_in, D_out, nw, hb, hbi), X, Y, B, W, Wb, bias};
  h.L.wavelet_type = wtype;
  h.trans = half_to_float(trans, (size_t)D_in * nw);
  h.isc = half_to_float(isc, (size_t)D_in * nw);
  return run_host_layer(h);
}

int metal_kan_relu_forward(const float* X, const float* W, const float* Wb, const float* grid,
                           const float* bias, float* Y, int B, int D_in, int D_out, int G,
                           float inv_h, int hb, int hbi) {
  if (!grid || G <= 0) return fail(KAN_ERR_ARG, "relu: NULL grid");
  HostLayer h{base_layer(KAN_RELU, KAN_F32, D_in, D_out, G, hb, hbi), X, Y, B, W, Wb, bias};
  h.L.inv_h = inv_h;
  h.grid.assign(grid, grid + G);
  return run_host_layer(h);
}

int metal_kan_relu_forward_fp16(const uint16_t* X, const uint16_t* W, const uint16_t* Wb,
                                const uint16_t* grid, const uint16_t* bias, uint16_t* Y, int B,
                                int D_in, int D_out, int G, float inv_h, int hb, int hbi) {
  if (!grid || G <= 0) return fail(KAN_ERR_ARG, "relu_fp16: NULL grid");
  HostLayer h{base_layer(KAN_RELU, KAN_F16, D_in, D_out, G, hb, hbi), X, Y, B, W, Wb, bias};
  h.L.inv_h = inv_h;
  h.grid = half_to_float(grid, (size_t)G);
  return run_host_layer(h);
}

int metal_kan_fourier_forward(const float* X, const float* W, const float* Wb, const float* bias,
                              float* Y, int B, int D_in, int D_out, int num_freqs, int hb,
                              int hbi) {
  if (num_freqs < 0) return fail(KAN_ERR_ARG, "fourier: num_frequencies < 0");
  HostLayer h{base_layer(KAN_FOURIER, KAN_F32, D_in, D_out, 2 * num_freqs + 1, hb, hbi), X, Y, B,
              W, Wb, bias};
  return run_host_layer(h);
}

int metal_kan_fourier_forward_fp16(const uint16_t* X, const uint16_t* W, const uint16_t* Wb,
                                   const uint16_t* bias, uint16_t* Y, int B, int D_in, int D_out,
                                   int num_freqs, int hb, int hbi) {
  if (num_freqs < 0) return fail(KAN_ERR_ARG, "fourier_fp16: num_frequencies < 0");
  HostLayer h{base_layer(KAN_FOURIER, KAN_F16, D_in, D_out, 2 * num_freqs + 1, hb, hbi), X, Y, B,
              W, Wb, bias};
  return run_host_layer(h);
}

int metal_kan_jacobi_forward(const float* X, const float* W, const float* Wb, const float* bias,
                             float* Y, int B, int D_in, int D_out, int degree, float alpha,
                             float beta, int hb, int hbi) {
  HostLayer h{base_layer(KAN_JACOBI, KAN_F32, D_in, D_out, degree, hb, hbi), X, Y, B, W, Wb, bias};
  h.L.alpha = alpha;
  h.L.beta = beta;
  return run_host_layer(h);
}

int metal_kan_jacobi_forward_fp16(const uint16_t* X, const uint16_t* W, const uint16_t* Wb,
                                  const uint16_t* bias, uint16_t* Y, int B, int D_in, int D_out,
                                  int degree, float alpha, float beta, int hb, int hbi) {
  HostLayer h{base_layer(KAN_JACOBI, KAN_F16, D_in, D_out, degree, hb, hbi), X, Y, B, W, Wb, bias};
  h.L.alpha = alpha;
  h.L.beta = beta;
  return run_host_layer(h);
}

// MultKAN (metal_kan_bridge.mm:1700-1802, fp16 :2250-2350): the RBF layer to num_add +
// 2 num_mult internal outputs, then the pair products.  `grid` is in the layer dtype.
static int mult_common(int dt, const void* X, const void* W, const void* Wb, const void* grid,
                       const void* bias, void* Y, int B, int D_in, int D_out, int num_add,
                       int num_mult, int K, float inv_den, int hb, int hbi) {
  if (!grid || K <= 0) return fail(KAN_ERR_ARG, "mult: NULL grid");
  if (num_add < 0 || num_mult < 0 || num_add + num_mult != D_out)
    return fail(KAN_ERR_ARG, "mult: num_add + num_mult must equal D_out");
  const int internal = num_add + 2 * num_mult;
  HostLayer h{base_layer(KAN_RBF, dt, D_in, internal, K, hb, hbi), X, Y, B, W, Wb, bias};
  h.L.inv_den = inv_den;
  h.grid = dt == KAN_F16 ? half_to_float((const uint16_t*)grid, (size_t)K)
                         : std::vector<float>((const float*)grid, (const float*)grid + K);
  if (num_mult > 0) {
    h.post = [=](DeviceState* d, void*, void* dIn, void** dOut, size_t* bytes) {
      const size_t es = dtype_size(dt);
      int rc = slot(d, S_T1, (size_t)B * D_out * es, dOut);
      if (rc) return rc;
      cudaError_t e = launch_mult_combine(dIn, *dOut, B, num_add, num_mult, dt, d->stream);
      if (e != cudaSuccess) return fail(KAN_ERR_CUDA, "mult combine: %s", cudaGetErrorString(e));
      *bytes = (size_t)B * D_out * es;
      return KAN_OK;
    };
  }
  return run_host_layer(h);
}

int metal_kan_mult_forward(const float* X, const float* W, const float* Wb, const float* grid,
                           const float* bias, float* Y, int B, int D_in, int D_out, int num_add,
                           int num_mult, int K, float inv_den, int hb, int hbi) {
  return mult_common(KAN_F32, X, W, Wb, grid, bias, Y, B, D_in, D_out, num_add, num_mult, K,
                     inv_den, hb, hbi);
}

int metal_kan_mult_forward_fp16(const uint16_t* X, const uint16_t* W, const uint16_t* Wb,
                                const uint16_t* grid, const uint16_t* bias, uint16_t* Y, int B,
                                int D_in, int D_out, int num_add, int num_mult, int K,
                                float inv_den, int hb, int hbi) {
  return mult_common(KAN_F16, X, W, Wb, grid, bias, Y, B, D_in, D_out, num_add, num_mult, K,
                     inv_den, hb, hbi);
}

// LowRankKAN (metal_kan_bridge.mm:1535-1698, fp16 :2153-2248): Z = RBF layer to `rank` outputs
// (no base, no bias; Z in the layer dtype), then Y = bias + Z W_up^T + silu(x) W_base^T.
static int lowrank_common(int dt, const void* X, const void* Wdown, const void* Wup,
                          const void* Wb, const void* grid, const void* bias, void* Y, int B,
                          int D_in, int D_out, int rank, int K, float inv_den, int hb, int hbi) {
  if (!grid || K <= 0 || rank <= 0 || !Wup) return fail(KAN_ERR_ARG, "lowrank: bad arguments");
  if (hb && !Wb) return fail(KAN_ERR_ARG, "lowrank: has_base with NULL W_base");
  if (hbi && !bias) return fail(KAN_ERR_ARG, "lowrank: has_bias with NULL bias");
  HostLayer h{base_layer(KAN_RBF, dt, D_in, rank, K, 0, 0), X, Y, B, Wdown, nullptr, nullptr};
  h.L.inv_den = inv_den;
  h.grid = dt == KAN_F16 ? half_to_float((const uint16_t*)grid, (size_t)K)
                         : std::vector<float>((const float*)grid, (const float*)grid + K);
  h.post = [=](DeviceState* d, void* dX, void* dZ, void** dOut, size_t* bytes) {
    const size_t es = dtype_size(dt);
    void *dWup, *dWb = nullptr, *dB = nullptr;
    int rc;
    if ((rc = stage_in(d, S_T0, Wup, (size_t)D_out * rank * es, &dWup))) return rc;
    if (hb && (rc = stage_in(d, S_WB, Wb, (size_t)D_out * D_in * es, &dWb))) return rc;
    if (hbi && (rc = stage_in(d, S_BIAS, bias, (size_t)D_out * es, &dB))) return rc;
    if ((rc = slot(d, S_T1, (size_t)B * D_out * es, dOut))) return rc;
    cudaError_t e = launch_lowrank_up(dZ, dX, dWup, dWb, dB, *dOut, B, D_in, D_out, rank, hb,
                                      hbi, dt, d->stream);
    if (e != cudaSuccess) return fail(KAN_ERR_CUDA, "lowrank up: %s", cudaGetErrorString(e));
    *bytes = (size_t)B * D_out * es;
    return KAN_OK;
  };
  return run_host_layer(h);
}

int metal_kan_lowrank_forward(const float* X, const float* Wdown, const float* Wup,
                              const float* Wb, const float* grid, const float* bias, float* Y,
                              int B, int D_in, int D_out, int rank, int K, float inv_den, int hb,
                              int hbi) {
  return lowrank_common(KAN_F32, X, Wdown, Wup, Wb, grid, bias, Y, B, D_in, D_out, rank, K,
                        inv_den, hb, hbi);
}

int metal_kan_lowrank_forward_fp16(const uint16_t* X, const uint16_t* Wdown,
                                   const uint16_t* Wup, const uint16_t* Wb, const uint16_t* grid,
                                   const uint16_t* bias, uint16_t* Y, int B, int D_in, int D_out,
                                   int rank, int K, float inv_den, int hb, int hbi) {
  return lowrank_common(KAN_F16, X, Wdown, Wup, Wb, grid, bias, Y, B, D_in, D_out, rank, K,
                        inv_den, hb, hbi);
}

// RationalKAN (metal_kan_bridge.mm:1004-1067), fp32 only like the reference.
int metal_kan_rational_forward(const float* X, const float* Wp, const float* Wq, const float* Wb,
                               const float* bias, float* Y, int B, int D_in, int D_out, int p,
                               int q, int hb, int hbi) {
  DeviceState* d;
  int rc = current_state(&d);
  if (rc) return rc;
  if (B < 0 || D_in <= 0 || D_out <= 0) return fail(KAN_ERR_ARG, "rational: bad sizes");
  if (!rational_supported(p, q)) return fail(KAN_ERR_UNSUPPORTED, "rational: degrees p, q in 0..16 with p + q in 1..16");
  if (B == 0) return KAN_OK;
  if (!X || !Y || (p && !Wp) || (q && !Wq) || (hb && !Wb) || (hbi && !bias))
    return fail(KAN_ERR_ARG, "rational: NULL pointer");
  void *dX, *dWp = nullptr, *dWq = nullptr, *dWb = nullptr, *dB = nullptr, *dY;
  if ((rc = stage_in(d, S_X, X, (size_t)B * D_in * 4, &dX))) return rc;
  if (p && (rc = stage_in(d, S_W, Wp, (size_t)D_out * D_in * p * 4, &dWp))) return rc;
  if (q && (rc = stage_in(d, S_T0, Wq, (size_t)D_out * D_in * q * 4, &dWq))) return rc;
  if (hb && (rc = stage_in(d, S_WB, Wb, (size_t)D_out * D_in * 4, &dWb))) return rc;
  if (hbi && (rc = stage_in(d, S_BIAS, bias, (size_t)D_out * 4, &dB))) return rc;
  if ((rc = slot(d, S_Y, (size_t)B * D_out * 4, &dY))) return rc;
  cudaError_t e = launch_rational((const float*)dX, (const float*)dWp, (const float*)dWq,
                                  (const float*)dWb, (const float*)dB, (float*)dY, B, D_in, D_out,
                                  p, q, hb, hbi, d->stream);
  if (e != cudaSuccess) return fail(KAN_ERR_CUDA, "rational launch: %s", cudaGetErrorString(e));
  return stage_out(d, Y, dY, (size_t)B * D_out * 4);
}

int metal_kan_chain_pipeline_cheby(const float* X, float* Y, int B, int num_layers,
                                   const int* dims, const int* degrees, const float** W,
                                   const float** Wb, const float** bias) {
  DeviceState* d;
  int rc = current_state(&d);
  if (rc) return rc;
  if (!X || !Y || !dims || !degrees || !W || num_layers <= 0 || B < 0)
    return fail(KAN_ERR_ARG, "chain: bad arguments");
  if (B == 0) return KAN_OK;
  int max_dim = 0;
  for (int l = 0; l <= num_layers; ++l) {
    if (dims[l] <= 0) return fail(KAN_ERR_ARG, "chain: dims[%d] = %d", l, dims[l]);
    max_dim = std::max(max_dim, dims[l]);
  }
  // ping-pong activations stay on the device between layers
  void *act[2], *dW, *dWb, *dB;
  if ((rc = slot(d, S_T0, (size_t)B * max_dim * 4, &act[0]))) return rc;
  if ((rc = slot(d, S_T1, (size_t)B * max_dim * 4, &act[1]))) return rc;
  KAN_CUDA_TRY(cudaMemcpyAsync(act[0], X, (size_t)B * dims[0] * 4, cudaMemcpyHostToDevice, d->stream));
  int cur = 0;
  for (int l = 0; l < num_layers; ++l) {
    const int din = dims[l], dout = dims[l + 1], K = degrees[l];
    if (K <= 0 || !W[l]) return fail(KAN_ERR_ARG, "chain: layer %d weights/degree", l);
    const int hb = (Wb && Wb[l]) ? 1 : 0, hbi = (bias && bias[l]) ? 1 : 0;
    // weights of every layer are staged into distinct slots only one layer at a time, so the
    // copy for layer l must wait until layer l-1 has consumed the slot: same stream, in order.
    if ((rc = stage_in(d, S_W, W[l], (size_t)dout * din * K * 4, &dW))) return rc;
    dWb = nullptr;
    dB = nullptr;
    if (hb && (rc = stage_in(d, S_WB, Wb[l], (size_t)dout * din * 4, &dWb))) return rc;
    if (hbi && (rc = stage_in(d, S_BIAS, bias[l], (size_t)dout * 4, &dB))) return rc;
    kan_layer L = base_layer(KAN_CHEBY, KAN_F32, din, dout, K, hb, hbi);
    L.w.format = KAN_W_DENSE;
    L.w.data = dW;
    L.wb.format = KAN_W_DENSE;
    L.wb.data = dWb;
    L.bias = dB;
    if ((rc = run_forward(&L, act[cur], act[cur ^ 1], B, KAN_PATH_AUTO, d->stream, d))) return rc;
    cur ^= 1;
  }
  return stage_out(d, Y, act[cur], (size_t)B * dims[num_layers] * 4);
}

int metal_kan_swiglu_forward(const float* gate, const float* up, float* out, int n) {
  DeviceState* d;
  int rc = current_state(&d);
  if (rc) return rc;
  if (!gate || !up || !out || n <= 0) return fail(KAN_ERR_ARG, "swiglu: bad arguments");
  void *g, *u, *o;
  if ((rc = stage_in(d, S_X, gate, (size_t)n * 4, &g))) return rc;
  if ((rc = stage_in(d, S_W, up, (size_t)n * 4, &u))) return rc;
  if ((rc = slot(d, S_Y, (size_t)n * 4, &o))) return rc;
  cudaError_t e = launch_swiglu(g, u, o, n, KAN_F32, d->stream);
  if (e != cudaSuccess) return fail(KAN_ERR_CUDA, "swiglu: %s", cudaGetErrorString(e));
  return stage_out(d, out, o, (size_t)n * 4);
}

// ---------------------------------------------------------------- host quantisers
// Source-level IEEE fp32 semantics of metal_kan_bridge.mm:4177-4302 / :4634-4682 / :4735-4788:
// each operation rounds once (this file is compiled with -ffp-contract=off).

int metal_kan_quantize_int8(const float* w, uint8_t* q, float* s, float* b, int groups, int gs) {
  if (!w || !q || !s || !b || groups <= 0 || gs <= 0)
    return fail(KAN_ERR_ARG, "quantize_int8: bad arguments");
  for (int g = 0; g < groups; ++g) {
    const float* grp = w + (size_t)g * gs;
    float mn = grp[0], mx = grp[0];
    for (int i = 1; i < gs; ++i) {
      mn = grp[i] < mn ? grp[i] : mn;
      mx = grp[i] > mx ? grp[i] : mx;
    }
    float range = std::max(mx - mn, 1e-7f);
    float scale = range / 255.0f;
    s[g] = scale;
    b[g] = mn;
    float inv = 1.0f / scale;
    for (int i = 0; i < gs; ++i) {
      float v = (grp[i] - mn) * inv + 0.5f;
      int qi = (int)v;
      q[(size_t)g * gs + i] = (uint8_t)(qi < 0 ? 0 : qi > 255 ? 255 : qi);
    }
  }
  return KAN_OK;
}

int metal_kan_quantize_int4(const float* w, uint8_t* q, float* s, float* b, int groups, int gs) {
  if (!w || !q || !s || !b || groups <= 0 || gs <= 0 || (gs & 1))
    return fail(KAN_ERR_ARG, "quantize_int4: bad arguments");
  const int half = gs / 2;
  for (int g = 0; g < groups; ++g) {
    const float* grp = w + (size_t)g * gs;
    float mn = grp[0], mx = grp[0];
    for (int i = 1; i < gs; ++i) {
      mn = grp[i] < mn ? grp[i] : mn;
      mx = grp[i] > mx ? grp[i] : mx;
    }
    float range = std::max(mx - mn, 1e-7f);
    float scale = range / 15.0f;
    s[g] = scale;
    b[g] = mn;
    float inv = 1.0f / scale;
    for (int i = 0; i < half; ++i) {
      int q0 = (int)((grp[2 * i] - mn) * inv + 0.5f);
      int q1 = (int)((grp[2 * i + 1] - mn) * inv + 0.5f);
      q0 = q0 < 0 ? 0 : q0 > 15 ? 15 : q0;
      q1 = q1 < 0 ? 0 : q1 > 15 ? 15 : q1;
      q[(size_t)g * half + i] = (uint8_t)(q0 | (q1 << 4));
    }
  }
  return KAN_OK;
}

int metal_kan_dequantize_int8(const uint8_t* q, const float* s, const float* b, float* out,
                              int groups, int gs) {
  if (!q || !s || !b || !out || groups <= 0 || gs <= 0)
    return fail(KAN_ERR_ARG, "dequantize_int8: bad arguments");
  for (int g = 0; g < groups; ++g)
    for (int i = 0; i < gs; ++i) {
      float m = (float)q[(size_t)g * gs + i] * s[g];
      out[(size_t)g * gs + i] = m + b[g];
    }
  return KAN_OK;
}

int metal_kan_dequantize_int4(const uint8_t* q, const float* s, const float* b, float* out,
                              int groups, int gs) {
  if (!q || !s || !b || !out || groups <= 0 || gs <= 0 || (gs & 1))
    return fail(KAN_ERR_ARG, "dequantize_int4: bad arguments");
  const int half = gs / 2;
  for (int g = 0; g < groups; ++g)
    for (int i = 0; i < half; ++i) {
      uint8_t byte = q[(size_t)g * half + i];
      float m0 = (float)(byte & 0xF) * s[g];
      float m1 = (float)((byte >> 4) & 0xF) * s[g];
      out[(size_t)g * gs + 2 * i] = m0 + b[g];
      out[(size_t)g * gs + 2 * i + 1] = m1 + b[g];
    }
  return KAN_OK;
}

int metal_kan_quantize_ternary(const float* W, uint32_t* P, float* s, int D_out, int K_dim,
                               int gs) {
  if (!W || !P || !s || D_out <= 0 || K_dim <= 0 || gs <= 0)
    return fail(KAN_ERR_ARG, "quantize_ternary: bad arguments");
  const int words = (K_dim + 15) / 16, G = (K_dim + gs - 1) / gs;
  std::memset(P, 0, (size_t)D_out * words * sizeof(uint32_t));
  for (int j = 0; j < D_out; ++j) {
    const float* row = W + (size_t)j * K_dim;
    for (int g = 0; g < G; ++g) {
      const int st = g * gs, en = std::min(st + gs, K_dim), cnt = en - st;
      double sum = 0.0;
      for (int k = st; k < en; ++k) sum += std::fabs((double)row[k]);
      float sc = (cnt > 0 && sum > 0.0) ? (float)(sum / cnt) : 1e-4f;
      s[(size_t)j * G + g] = sc;
      float inv = 1.0f / sc;
      for (int k = st; k < en; ++k) {
        float v = row[k] * inv;
        uint32_t c = v < -0.5f ? 0u : (v > 0.5f ? 2u : 1u);
        P[(size_t)j * words + k / 16] |= c << ((k % 16) * 2);
      }
    }
  }
  return KAN_OK;
}

int metal_kan_quantize_int2(const float* W, uint32_t* P, float* s, const float* cb, int D_out,
                            int K_dim, int gs) {
  if (!W || !P || !s || !cb || D_out <= 0 || K_dim <= 0 || gs <= 0)
    return fail(KAN_ERR_ARG, "quantize_int2: bad arguments");
  const int words = (K_dim + 15) / 16, G = (K_dim + gs - 1) / gs;
  std::memset(P, 0, (size_t)D_out * words * sizeof(uint32_t));
  for (int j = 0; j < D_out; ++j) {
    const float* row = W + (size_t)j * K_dim;
    for (int g = 0; g < G; ++g) {
      const int st = g * gs, en = std::min(st + gs, K_dim);
      float mx = 0.0f;
      for (int k = st; k < en; ++k) mx = std::max(mx, std::fabs(row[k]));
      float sc = mx > 0.0f ? mx : 1e-4f;
      s[(size_t)j * G + g] = sc;
      float inv = 1.0f / sc;
      for (int k = st; k < en; ++k) {
        float v = row[k] * inv;
        int best = 0;
        float bd = std::fabs(v - cb[0]);
        for (int c = 1; c < 4; ++c) {
          float dd = std::fabs(v - cb[c]);
          if (dd < bd) {
            bd = dd;
            best = c;
          }
        }
        P[(size_t)j * words + k / 16] |= (uint32_t)best << ((k % 16) * 2);
      }
    }
  }
  return KAN_OK;
}

static int dequant_2bit_host(int fmt, const uint32_t* P, const float* s, const float* cb,
                             float* out, int D_out, int K_dim, int gs) {
  DeviceState* d;
  int rc = current_state(&d);
  if (rc) return rc;
  if (!P || !s || !out || D_out <= 0 || K_dim <= 0 || gs <= 0 || (fmt == KAN_W_INT2 && !cb))
    return fail(KAN_ERR_ARG, "dequantize (2-bit): bad arguments");
  const int words = (K_dim + 15) / 16, G = (K_dim + gs - 1) / gs;
  void *dP, *dS, *dC = nullptr, *dO;
  if ((rc = stage_in(d, S_W, P, (size_t)D_out * words * 4, &dP))) return rc;
  if ((rc = stage_in(d, S_SC, s, (size_t)D_out * G * 4, &dS))) return rc;
  if (cb && (rc = stage_in(d, S_CB, cb, 16, &dC))) return rc;
  if ((rc = slot(d, S_Y, (size_t)D_out * K_dim * 4, &dO))) return rc;
  kan_weight w;
  std::memset(&w, 0, sizeof(w));
  w.format = fmt;
  w.group_size = gs;
  w.data = dP;
  w.scales = (const float*)dS;
  w.codebook = (const float*)dC;
  cudaError_t e = launch_dequantize(w, D_out, K_dim, dO, KAN_F32, d->stream);
  if (e != cudaSuccess) return fail(KAN_ERR_CUDA, "dequantize: %s", cudaGetErrorString(e));
  return stage_out(d, out, dO, (size_t)D_out * K_dim * 4);
}

int metal_kan_dequantize_ternary(const uint32_t* P, const float* s, float* out, int D_out,
                                 int K_dim, int gs) {
  return dequant_2bit_host(KAN_W_TERNARY, P, s, nullptr, out, D_out, K_dim, gs);
}

int metal_kan_dequantize_int2(const uint32_t* P, const float* s, const float* cb, float* out,
                              int D_out, int K_dim, int gs) {
  return dequant_2bit_host(KAN_W_INT2, P, s, cb, out, D_out, K_dim, gs);
}

static int packed_cheby_host(int fmt, const float* X, const uint32_t* P, const float* s,
                             const float* cb, const float* bias, float* Y, int B, int D_in,
                             int D_out, int deg, int gs, int hbi) {
  DeviceState* d;
  int rc = current_state(&d);
  if (rc) return rc;
  if (!X || !P || !s || !Y || B <= 0 || D_in <= 0 || D_out <= 0 || deg <= 0 || gs <= 0 ||
      (fmt == KAN_W_INT2 && !cb) || (hbi && !bias))
    return fail(KAN_ERR_ARG, "packed cheby forward: bad arguments");
  const int K_dim = D_in * deg, words = (K_dim + 15) / 16, G = (K_dim + gs - 1) / gs;
  void *dX, *dP, *dS, *dC = nullptr, *dB = nullptr, *dY;
  if ((rc = stage_in(d, S_X, X, (size_t)B * D_in * 4, &dX))) return rc;
  if ((rc = stage_in(d, S_W, P, (size_t)D_out * words * 4, &dP))) return rc;
  if ((rc = stage_in(d, S_SC, s, (size_t)D_out * G * 4, &dS))) return rc;
  if (cb && (rc = stage_in(d, S_CB, cb, 16, &dC))) return rc;
  if (hbi && (rc = stage_in(d, S_BIAS, bias, (size_t)D_out * 4, &dB))) return rc;
  if ((rc = slot(d, S_Y, (size_t)B * D_out * 4, &dY))) return rc;
  kan_layer L = base_layer(KAN_CHEBY, KAN_F32, D_in, D_out, deg, 0, hbi);
  L.w.format = fmt;
  L.w.group_size = gs;
  L.w.data = dP;
  L.w.scales = (const float*)dS;
  L.w.codebook = (const float*)dC;
  L.bias = dB;
  if ((rc = run_forward(&L, dX, dY, B, KAN_PATH_AUTO, d->stream, d))) return rc;
  return stage_out(d, Y, dY, (size_t)B * D_out * 4);
}

int metal_kan_forward_ternary_cheby(const float* X, const uint32_t* P, const float* s,
                                    const float* bias, float* Y, int B, int D_in, int D_out,
                                    int degree, int gs, int hbi) {
  return packed_cheby_host(KAN_W_TERNARY, X, P, s, nullptr, bias, Y, B, D_in, D_out, degree, gs,
                           hbi);
}

int metal_kan_forward_int2_cheby(const float* X, const uint32_t* P, const float* s,
                                 const float* cb, const float* bias, float* Y, int B, int D_in,
                                 int D_out, int degree, int gs, int hbi) {
  return packed_cheby_host(KAN_W_INT2, X, P, s, cb, bias, Y, B, D_in, D_out, degree, gs, hbi);
}

double benchmark_metal_cheby(const float* X, const float* W, const float* Wb, const float* bias,
                             float* Y, int B, int D_in, int D_out, int K, int hb, int hbi,
                             int warmup, int iters) {
  return bench_loop([&] { return metal_kan_cheby_forward(X, W, Wb, bias, Y, B, D_in, D_out, K, hb, hbi); },
                    warmup, iters);
}
double benchmark_metal_fastkan(const float* X, const float* W, const float* Wb, const float* grid,
                               const float* bias, float* Y, int B, int D_in, int D_out, int K,
                               float inv_den, int hb, int hbi, int warmup, int iters) {
  return bench_loop([&] {
    return metal_kan_fastkan_forward(X, W, Wb, grid, bias, Y, B, D_in, D_out, K, inv_den, hb, hbi);
  }, warmup, iters);
}
double benchmark_metal_bspline(const float* X, const float* W, const float* Wb, const float* grid,
                               const float* bias, float* Y, int B, int D_in, int D_out, int G,
                               int order, int hb, int hbi, int warmup, int iters) {
  return bench_loop([&] {
    return metal_kan_bspline_forward(X, W, Wb, grid, bias, Y, B, D_in, D_out, G, order, hb, hbi);
  }, warmup, iters);
}
double benchmark_metal_wavkan(const float* X, const float* W, const float* Wb, const float* tr,
                              const float* isc, const float* bias, float* Y, int B, int D_in,
                              int D_out, int nw, int wt, int hb, int hbi, int warmup, int iters) {
  return bench_loop([&] {
    return metal_kan_wavkan_forward(X, W, Wb, tr, isc, bias, Y, B, D_in, D_out, nw, wt, hb, hbi);
  }, warmup, iters);
}

double benchmark_metal_relu(const float* X, const float* W, const float* Wb, const float* grid,
                            const float* bias, float* Y, int B, int D_in, int D_out, int G,
                            float inv_h, int hb, int hbi, int warmup, int iters) {
  return bench_loop([&] {
    return metal_kan_relu_forward(X, W, Wb, grid, bias, Y, B, D_in, D_out, G, inv_h, hb, hbi);
  }, warmup, iters);
}
double benchmark_metal_fourier(const float* X, const float* W, const float* Wb, const float* bias,
                               float* Y, int B, int D_in, int D_out, int num_freqs, int hb,
                               int hbi, int warmup, int iters) {
  return bench_loop([&] {
    return metal_kan_fourier_forward(X, W, Wb, bias, Y, B, D_in, D_out, num_freqs, hb, hbi);
  }, warmup, iters);
}
double benchmark_metal_jacobi(const float* X, const float* W, const float* Wb, const float* bias,
                              float* Y, int B, int D_in, int D_out, int degree, float alpha,
                              float beta, int hb, int hbi, int warmup, int iters) {
  return bench_loop([&] {
    return metal_kan_jacobi_forward(X, W, Wb, bias, Y, B, D_in, D_out, degree, alpha, beta, hb,
                                    hbi);
  }, warmup, iters);
}

double benchmark_metal_mult(const float* X, const float* W, const float* Wb, const float* grid,
                            const float* bias, float* Y, int B, int D_in, int D_out, int num_add,
                            int num_mult, int K, float inv_den, int hb, int hbi, int warmup,
                            int iters) {
  return bench_loop([&] {
    return metal_kan_mult_forward(X, W, Wb, grid, bias, Y, B, D_in, D_out, num_add, num_mult, K,
                                  inv_den, hb, hbi);
  }, warmup, iters);
}

double benchmark_metal_lowrank(const float* X, const float* Wdown, const float* Wup,
                               const float* Wb, const float* grid, const float* bias, float* Y,
                               int B, int D_in, int D_out, int rank, int K, float inv_den, int hb,
                               int hbi, int warmup, int iters) {
  return bench_loop([&] {
    return metal_kan_lowrank_forward(X, Wdown, Wup, Wb, grid, bias, Y, B, D_in, D_out, rank, K,
                                     inv_den, hb, hbi);
  }, warmup, iters);
}

double benchmark_metal_rational(const float* X, const float* Wp, const float* Wq,
                                const float* Wb, const float* bias, float* Y, int B, int D_in,
                                int D_out, int p, int q, int hb, int hbi, int warmup, int iters) {
  return bench_loop([&] {
    return metal_kan_rational_forward(X, Wp, Wq, Wb, bias, Y, B, D_in, D_out, p, q, hb, hbi);
  }, warmup, iters);
}

}  // extern "C"

// ==========================================================================================
// backward (fp32): device entry points and the reference's host-pointer functions
// ==========================================================================================
namespace kan {

static int make_backward_args(const kan_layer* L, const void* X, const void* dY, void* dX,
                              void* dW, void* dWb, void* dbias, int B, BackwardArgs* a) {
  if (!L) return fail(KAN_ERR_ARG, "backward: NULL layer");
  if (B < 0) return fail(KAN_ERR_ARG, "backward: B < 0");
  if (L->act_dtype != KAN_F32)
    return fail(KAN_ERR_UNSUPPORTED, "backward: fp32 layers only (the reference trains in fp32)");
  if (L->w.format != KAN_W_DENSE || !L->w.data || (L->has_base && (L->wb.format != KAN_W_DENSE ||
                                                                   !L->wb.data)))
    return fail(KAN_ERR_UNSUPPORTED, "backward: dense weights only");
  if (L->input_map != KAN_MAP_NONE)
    return fail(KAN_ERR_UNSUPPORTED, "backward: raw inputs only (no tanh / LayerNorm map)");
  if (B > 0 && (!X || !dY)) return fail(KAN_ERR_ARG, "backward: NULL X or dY");
  std::memset(a, 0, sizeof(*a));
  a->basis = L->basis;
  a->B = B;
  a->D_in = L->D_in;
  a->D_out = L->D_out;
  a->K = L->K;
  a->has_base = L->has_base ? 1 : 0;
  a->grid_size = L->grid_size;
  a->inv_den = L->inv_den;
  a->grid_min = L->grid_min;
  a->inv_h = L->inv_h;
  a->grid = L->grid;
  a->X = (const float*)X;
  a->dY = (const float*)dY;
  a->W = (const float*)L->w.data;
  a->Wb = (const float*)L->wb.data;
  a->dW = (float*)dW;
  a->dWb = L->has_base ? (float*)dWb : nullptr;
  a->dbias = (float*)dbias;
  a->dX = (float*)dX;
  if (!backward_supported(*a))
    return fail(KAN_ERR_UNSUPPORTED,
                "backward: Chebyshev, RBF, B-spline or ReLU layers with K + has_base <= 64");
  return KAN_OK;
}

// Host-pointer backward: stage dY, X and the weights, run, copy the requested gradients back.
static int run_host_backward(kan_layer L, const float* dY, const float* X, const float* W,
                             const float* Wb, const float* grid, float* dW, float* dWb,
                             float* dbias, float* dX, int B) {
  DeviceState* d;
  int rc = current_state(&d);
  if (rc) return rc;
  if (B <= 0 || L.D_in <= 0 || L.D_out <= 0 || L.K <= 0 || !dY || !X || !W || !dX)
    return fail(KAN_ERR_ARG, "backward: bad sizes or NULL dY / X / W / dX");
  if (L.has_base && !Wb) return fail(KAN_ERR_ARG, "backward: has_base with NULL W_base");
  const size_t kw = (size_t)L.D_in * L.K;
  void *ddY, *dXin, *dWt, *dWbt = nullptr, *dG = nullptr, *oW = nullptr, *oWb = nullptr,
             *oB = nullptr, *oX;
  if ((rc = stage_in(d, S_DY, dY, (size_t)B * L.D_out * 4, &ddY))) return rc;
  if ((rc = stage_in(d, S_X, X, (size_t)B * L.D_in * 4, &dXin))) return rc;
  if ((rc = stage_in(d, S_W, W, (size_t)L.D_out * kw * 4, &dWt))) return rc;
  if (L.has_base && (rc = stage_in(d, S_WB, Wb, (size_t)L.D_out * L.D_in * 4, &dWbt))) return rc;
  if (grid && (rc = stage_in(d, S_GRID, grid, (size_t)L.K * 4, &dG))) return rc;
  if (dW && (rc = slot(d, S_DW, (size_t)L.D_out * kw * 4, &oW))) return rc;
  if (L.has_base && dWb && (rc = slot(d, S_DWB, (size_t)L.D_out * L.D_in * 4, &oWb))) return rc;
  if (L.has_bias && dbias && (rc = slot(d, S_DBIAS, (size_t)L.D_out * 4, &oB))) return rc;
  if ((rc = slot(d, S_DX, (size_t)B * L.D_in * 4, &oX))) return rc;
  L.w.format = KAN_W_DENSE;
  L.w.data = dWt;
  L.wb.format = KAN_W_DENSE;
  L.wb.data = dWbt;
  L.grid = (const float*)dG;
  BackwardArgs a;
  if ((rc = make_backward_args(&L, dXin, ddY, oX, oW, oWb, oB, B, &a))) return rc;
  cudaError_t e = launch_backward(a, d->stream);
  if (e != cudaSuccess) return fail(KAN_ERR_CUDA, "backward launch: %s", cudaGetErrorString(e));
  if (oW) KAN_CUDA_TRY(cudaMemcpyAsync(dW, oW, (size_t)L.D_out * kw * 4, cudaMemcpyDeviceToHost,
                                       d->stream));
  if (oWb) KAN_CUDA_TRY(cudaMemcpyAsync(dWb, oWb, (size_t)L.D_out * L.D_in * 4,
                                        cudaMemcpyDeviceToHost, d->stream));
  if (oB) KAN_CUDA_TRY(cudaMemcpyAsync(dbias, oB, (size_t)L.D_out * 4, cudaMemcpyDeviceToHost,
                                       d->stream));
  KAN_CUDA_TRY(cudaMemcpyAsync(dX, oX, (size_t)B * L.D_in * 4, cudaMemcpyDeviceToHost, d->stream));
  KAN_CUDA_TRY(cudaStreamSynchronize(d->stream));
  return check_device_error(d);
}

// One fp32 training step on device buffers (metal_kan_bridge.mm:3432-3640 for the Chebyshev
// layer; the FastKAN and B-spline steps are alike): forward, dY = (Y - T) * 2 / B, the weight,
// base-weight and bias gradients (no input gradient), then one optimiser launch over the layer's
// tensors -- which the layer's own weight pointers are, updated in place.
static int run_train_step(DeviceState* d, cudaStream_t s, const kan_layer* L, const float* X,
                          const float* T, int B, float* const* m, float* const* v, int op,
                          const OptimHyper& h) {
  if (!L) return fail(KAN_ERR_ARG, "train_step: NULL layer");
  if (B <= 0 || !X || !T) return fail(KAN_ERR_ARG, "train_step: bad batch or NULL X / target");
  if (L->act_dtype != KAN_F32) return fail(KAN_ERR_UNSUPPORTED, "train_step: fp32 layers only");
  const int n_t = 1 + (L->has_base ? 1 : 0) + (L->has_bias ? 1 : 0);
  for (int k = 0; k < n_t; ++k)
    if (!m[k] || ((op == OPTIM_ADAMW || op == OPTIM_ADAM) && !v[k]))
      return fail(KAN_ERR_ARG, "train_step: NULL optimiser state");
  const size_t nw = (size_t)L->D_out * L->D_in * L->K, nb = (size_t)L->D_out * L->D_in;
  void *Y, *dY, *dW, *dWb = nullptr, *db = nullptr;
  int rc;
  if ((rc = scratch_buf(d, s, SC_TY, (size_t)B * L->D_out * 4, false, &Y))) return rc;
  if ((rc = scratch_buf(d, s, SC_TDY, (size_t)B * L->D_out * 4, false, &dY))) return rc;
  if ((rc = scratch_buf(d, s, SC_TDW, nw * 4, false, &dW))) return rc;
  if (L->has_base && (rc = scratch_buf(d, s, SC_TDWB, nb * 4, false, &dWb))) return rc;
  if (L->has_bias && (rc = scratch_buf(d, s, SC_TDB, (size_t)L->D_out * 4, false, &db))) return rc;
  BackwardArgs a;
  if ((rc = make_backward_args(L, X, dY, nullptr, dW, dWb, db, B, &a))) return rc;
  if ((rc = run_forward(L, X, Y, B, KAN_PATH_AUTO, s, d))) return rc;
  cudaError_t e = launch_mse_grad((const float*)Y, T, (float*)dY, (long long)B * L->D_out,
                                  2.0f / (float)B, s);
  if (e == cudaSuccess) e = launch_backward(a, s);
  float* params[3];
  const float* grads[3];
  long long n[3];
  int c = 0;
  params[c] = (float*)L->w.data, grads[c] = (const float*)dW, n[c++] = (long long)nw;
  if (L->has_base) params[c] = (float*)L->wb.data, grads[c] = (const float*)dWb, n[c++] = (long long)nb;
  if (L->has_bias) params[c] = (float*)L->bias, grads[c] = (const float*)db, n[c++] = L->D_out;
  if (e == cudaSuccess) e = launch_optim(op, c, params, grads, m, v, n, h, s);
  if (e != cudaSuccess) return fail(KAN_ERR_CUDA, "train_step: %s", cudaGetErrorString(e));
  return KAN_OK;
}

static OptimHyper hyper_of(const float* hp, int nesterov) {
  OptimHyper h = {hp[0], hp[1], hp[2], hp[3], hp[4], hp[5], nesterov};
  return h;
}

// Host-pointer training step: stage the batch, the layer and its AdamW state, run, copy the
// updated weights and state back (in place, as the reference's shared-memory buffers are).
static int run_host_train_step(kan_layer L, const float* X, const float* T, float* W, float* Wb,
                               float* bias, const float* grid, float* mW, float* vW, float* mWb,
                               float* vWb, float* mb, float* vb, int B, const OptimHyper& h) {
  DeviceState* d;
  int rc = current_state(&d);
  if (rc) return rc;
  if (B <= 0 || L.D_in <= 0 || L.D_out <= 0 || L.K <= 0 || !X || !T || !W || !mW || !vW)
    return fail(KAN_ERR_ARG, "train_step: bad sizes or NULL pointer");
  if ((L.has_base && (!Wb || !mWb || !vWb)) || (L.has_bias && (!bias || !mb || !vb)))
    return fail(KAN_ERR_ARG, "train_step: NULL base / bias tensor or state");
  const size_t nw = (size_t)L.D_out * L.D_in * L.K * 4, nb = (size_t)L.D_out * L.D_in * 4,
               nbias = (size_t)L.D_out * 4;
  void *dX, *dT, *dW, *dWb = nullptr, *dB = nullptr, *dG = nullptr;
  void *dmW, *dvW, *dmWb = nullptr, *dvWb = nullptr, *dmb = nullptr, *dvb = nullptr;
  if ((rc = stage_in(d, S_X, X, (size_t)B * L.D_in * 4, &dX))) return rc;
  if ((rc = stage_in(d, S_DY, T, (size_t)B * L.D_out * 4, &dT))) return rc;
  if ((rc = stage_in(d, S_W, W, nw, &dW))) return rc;
  if ((rc = stage_in(d, S_DW, mW, nw, &dmW))) return rc;
  if ((rc = stage_in(d, S_DWB, vW, nw, &dvW))) return rc;
  if (L.has_base) {
    if ((rc = stage_in(d, S_WB, Wb, nb, &dWb))) return rc;
    if ((rc = stage_in(d, S_DBIAS, mWb, nb, &dmWb))) return rc;
    if ((rc = stage_in(d, S_DX, vWb, nb, &dvWb))) return rc;
  }
  if (L.has_bias) {
    if ((rc = stage_in(d, S_BIAS, bias, nbias, &dB))) return rc;
    if ((rc = stage_in(d, S_SC, mb, nbias, &dmb))) return rc;
    if ((rc = stage_in(d, S_BI, vb, nbias, &dvb))) return rc;
  }
  if (grid && (rc = stage_in(d, S_GRID, grid, (size_t)L.K * 4, &dG))) return rc;
  L.w.format = KAN_W_DENSE;
  L.w.data = dW;
  L.wb.format = KAN_W_DENSE;
  L.wb.data = dWb;
  L.bias = dB;
  L.grid = (const float*)dG;
  float* m[3] = {(float*)dmW, nullptr, nullptr};
  float* v[3] = {(float*)dvW, nullptr, nullptr};
  int c = 1;
  if (L.has_base) m[c] = (float*)dmWb, v[c++] = (float*)dvWb;
  if (L.has_bias) m[c] = (float*)dmb, v[c++] = (float*)dvb;
  if ((rc = run_train_step(d, d->stream, &L, (const float*)dX, (const float*)dT, B, m, v,
                           OPTIM_ADAMW, h)))
    return rc;
  struct Back { void* host; const void* dev; size_t bytes; } back[9] = {
      {W, dW, nw}, {mW, dmW, nw}, {vW, dvW, nw}, {Wb, dWb, L.has_base ? nb : 0},
      {mWb, dmWb, L.has_base ? nb : 0}, {vWb, dvWb, L.has_base ? nb : 0},
      {bias, dB, L.has_bias ? nbias : 0}, {mb, dmb, L.has_bias ? nbias : 0},
      {vb, dvb, L.has_bias ? nbias : 0}};
  for (const Back& b : back)
    if (b.bytes) KAN_CUDA_TRY(cudaMemcpyAsync(b.host, b.dev, b.bytes, cudaMemcpyDeviceToHost, d->stream));
  KAN_CUDA_TRY(cudaStreamSynchronize(d->stream));
  return check_device_error(d);
}

// Host-pointer optimiser step on one tensor (the reference's metal_kan_*_step): param, m (and v)
// updated in place.
static int run_host_optim(int op, float* param, const float* grad, float* m, float* v, long long n,
                          const OptimHyper& h) {
  DeviceState* d;
  int rc = current_state(&d);
  if (rc) return rc;
  if (n < 0 || (n > 0 && (!param || !grad || !m || ((op == OPTIM_ADAMW || op == OPTIM_ADAM) && !v))))
    return fail(KAN_ERR_ARG, "optimiser step: bad arguments");
  if (n == 0) return KAN_OK;
  const size_t bytes = (size_t)n * 4;
  void *dp, *dg, *dm, *dv = nullptr;
  if ((rc = stage_in(d, S_T0, param, bytes, &dp))) return rc;
  if ((rc = stage_in(d, S_T1, grad, bytes, &dg))) return rc;
  if ((rc = stage_in(d, S_SC, m, bytes, &dm))) return rc;
  if (v && (rc = stage_in(d, S_BI, v, bytes, &dv))) return rc;
  float* P[1] = {(float*)dp};
  const float* G[1] = {(const float*)dg};
  float* M[1] = {(float*)dm};
  float* V[1] = {(float*)dv};
  cudaError_t e = launch_optim(op, 1, P, G, M, V, &n, h, d->stream);
  if (e != cudaSuccess) return fail(KAN_ERR_CUDA, "optimiser step: %s", cudaGetErrorString(e));
  KAN_CUDA_TRY(cudaMemcpyAsync(param, dp, bytes, cudaMemcpyDeviceToHost, d->stream));
  KAN_CUDA_TRY(cudaMemcpyAsync(m, dm, bytes, cudaMemcpyDeviceToHost, d->stream));
  if (v) KAN_CUDA_TRY(cudaMemcpyAsync(v, dv, bytes, cudaMemcpyDeviceToHost, d->stream));
  KAN_CUDA_TRY(cudaStreamSynchronize(d->stream));
  return check_device_error(d);
}

}  // namespace kan

extern "C" {

int kan_backward(const kan_layer* layer, const void* X, const void* dY, void* dX, void* dW,
                 void* dWb, void* dbias, int B, void* stream) {
  DeviceState* d;
  int rc = current_state(&d);
  if (rc) return rc;
  BackwardArgs a;
  if ((rc = make_backward_args(layer, X, dY, dX, dW, dWb, layer && layer->has_bias ? dbias : nullptr,
                               B, &a)))
    return rc;
  cudaError_t e = launch_backward(a, pick_stream(stream, d));
  if (e != cudaSuccess) return fail(KAN_ERR_CUDA, "backward launch: %s", cudaGetErrorString(e));
  return KAN_OK;
}

int kan_swiglu_backward(const void* d_hidden, const void* gate, const void* up, void* d_gate,
                        void* d_up, long long n, void* stream) {
  DeviceState* d;
  int rc = current_state(&d);
  if (rc) return rc;
  if (n < 0 || (n > 0 && (!d_hidden || !gate || !up || !d_gate || !d_up)))
    return fail(KAN_ERR_ARG, "swiglu_backward: bad arguments");
  cudaError_t e = launch_swiglu_backward((const float*)d_hidden, (const float*)gate,
                                         (const float*)up, (float*)d_gate, (float*)d_up, n,
                                         pick_stream(stream, d));
  if (e != cudaSuccess) return fail(KAN_ERR_CUDA, "swiglu_backward: %s", cudaGetErrorString(e));
  return KAN_OK;
}

int metal_kan_cheby_backward(const float* dY, const float* X, const float* W, const float* Wb,
                             float* dW, float* dWb, float* dbias, float* dX, int B, int D_in,
                             int D_out, int degree, int has_base, int has_bias) {
  return run_host_backward(base_layer(KAN_CHEBY, KAN_F32, D_in, D_out, degree, has_base, has_bias),
                           dY, X, W, Wb, nullptr, dW, dWb, dbias, dX, B);
}

int metal_kan_cheby_backward_fused(const float* dY, const float* X, const float* W,
                                   const float* Wb, float* dW, float* dWb, float* dbias, float* dX,
                                   int B, int D_in, int D_out, int degree, int has_base,
                                   int has_bias) {
  // one implementation: neither backward materialises the basis matrix here
  return metal_kan_cheby_backward(dY, X, W, Wb, dW, dWb, dbias, dX, B, D_in, D_out, degree,
                                  has_base, has_bias);
}

int metal_kan_fastkan_backward(const float* dY, const float* X, const float* W, const float* Wb,
                               const float* grid, float* dW, float* dWb, float* dbias, float* dX,
                               int B, int D_in, int D_out, int num_centers, float inv_den,
                               int has_base, int has_bias) {
  if (!grid) return fail(KAN_ERR_ARG, "fastkan_backward: NULL grid");
  kan_layer L = base_layer(KAN_RBF, KAN_F32, D_in, D_out, num_centers, has_base, has_bias);
  L.inv_den = inv_den;
  return run_host_backward(L, dY, X, W, Wb, grid, dW, dWb, dbias, dX, B);
}

int metal_kan_relu_backward(const float* dY, const float* X, const float* W, const float* Wb,
                            const float* grid, float* dW, float* dWb, float* dbias, float* dX,
                            int B, int D_in, int D_out, int num_grids, float inv_h, int has_base,
                            int has_bias) {
  if (!grid) return fail(KAN_ERR_ARG, "relu_backward: NULL grid");
  kan_layer L = base_layer(KAN_RELU, KAN_F32, D_in, D_out, num_grids, has_base, has_bias);
  L.inv_h = inv_h;
  return run_host_backward(L, dY, X, W, Wb, grid, dW, dWb, dbias, dX, B);
}

int metal_kan_bspline_backward(const float* dY, const float* X, const float* W, const float* Wb,
                               float* dW, float* dWb, float* dbias, float* dX, int B, int D_in,
                               int D_out, int grid_size, float grid_min, float inv_h,
                               int has_base, int has_bias) {
  kan_layer L = base_layer(KAN_BSPLINE, KAN_F32, D_in, D_out, grid_size + 3, has_base, has_bias);
  L.grid_size = grid_size;
  L.grid_min = grid_min;
  L.inv_h = inv_h;
  return run_host_backward(L, dY, X, W, Wb, nullptr, dW, dWb, dbias, dX, B);
}

int metal_kan_swiglu_backward(const float* d_hidden, const float* gate, const float* up,
                              float* d_gate, float* d_up, int n) {
  DeviceState* d;
  int rc = current_state(&d);
  if (rc) return rc;
  if (!d_hidden || !gate || !up || !d_gate || !d_up || n <= 0)
    return fail(KAN_ERR_ARG, "swiglu_backward: bad arguments");
  void *dh, *g, *u, *dg, *du;
  if ((rc = stage_in(d, S_DY, d_hidden, (size_t)n * 4, &dh))) return rc;
  if ((rc = stage_in(d, S_X, gate, (size_t)n * 4, &g))) return rc;
  if ((rc = stage_in(d, S_W, up, (size_t)n * 4, &u))) return rc;
  if ((rc = slot(d, S_DW, (size_t)n * 4, &dg))) return rc;
  if ((rc = slot(d, S_DX, (size_t)n * 4, &du))) return rc;
  cudaError_t e = launch_swiglu_backward((const float*)dh, (const float*)g, (const float*)u,
                                         (float*)dg, (float*)du, n, d->stream);
  if (e != cudaSuccess) return fail(KAN_ERR_CUDA, "swiglu_backward: %s", cudaGetErrorString(e));
  KAN_CUDA_TRY(cudaMemcpyAsync(d_gate, dg, (size_t)n * 4, cudaMemcpyDeviceToHost, d->stream));
  KAN_CUDA_TRY(cudaMemcpyAsync(d_up, du, (size_t)n * 4, cudaMemcpyDeviceToHost, d->stream));
  KAN_CUDA_TRY(cudaStreamSynchronize(d->stream));
  return check_device_error(d);
}

// ---- training step and optimisers (fp32) ---------------------------------------------------

int kan_train_step(const kan_layer* layer, const float* X, const float* target, int B,
                   float* m_w, float* v_w, float* m_wb, float* v_wb, float* m_b, float* v_b,
                   int optimizer, const float* hyper, int nesterov, void* stream) {
  DeviceState* d;
  int rc = current_state(&d);
  if (rc) return rc;
  if (!hyper || optimizer < OPTIM_ADAMW || optimizer > OPTIM_LION)
    return fail(KAN_ERR_ARG, "train_step: bad optimiser or NULL hyper-parameters");
  if (layer && (layer->w.format != KAN_W_DENSE || (layer->has_base && layer->wb.format != KAN_W_DENSE)))
    return fail(KAN_ERR_UNSUPPORTED, "train_step: dense weights only");
  float* m[3] = {m_w, nullptr, nullptr};
  float* v[3] = {v_w, nullptr, nullptr};
  int c = 1;
  if (layer && layer->has_base) m[c] = m_wb, v[c++] = v_wb;
  if (layer && layer->has_bias) m[c] = m_b, v[c++] = v_b;
  return run_train_step(d, pick_stream(stream, d), layer, X, target, B, m, v, optimizer,
                        hyper_of(hyper, nesterov));
}

int kan_optim_step(int optimizer, float* param, const float* grad, float* m, float* v,
                   long long n, const float* hyper, int nesterov, void* stream) {
  DeviceState* d;
  int rc = current_state(&d);
  if (rc) return rc;
  if (!hyper || optimizer < OPTIM_ADAMW || optimizer > OPTIM_LION || n < 0 ||
      (n > 0 && (!param || !grad || !m ||
                 ((optimizer == OPTIM_ADAMW || optimizer == OPTIM_ADAM) && !v))))
    return fail(KAN_ERR_ARG, "optim_step: bad arguments");
  if (n == 0) return KAN_OK;
  float* P[1] = {param};
  const float* G[1] = {grad};
  float* M[1] = {m};
  float* V[1] = {v};
  cudaError_t e = launch_optim(optimizer, 1, P, G, M, V, &n, hyper_of(hyper, nesterov),
                               pick_stream(stream, d));
  if (e != cudaSuccess) return fail(KAN_ERR_CUDA, "optim_step: %s", cudaGetErrorString(e));
  return KAN_OK;
}

int metal_kan_adamw_step(float* param, const float* grad, float* m, float* v, float lr,
                         float beta1, float beta2, float eps, float weight_decay, float lr_t,
                         int n) {
  const OptimHyper h = {lr, beta1, beta2, eps, weight_decay, lr_t, 0};
  return run_host_optim(OPTIM_ADAMW, param, grad, m, v, n, h);
}

int metal_kan_adam_step(float* param, const float* grad, float* m, float* v, float lr,
                        float beta1, float beta2, float eps, float weight_decay, float lr_t,
                        int n) {
  const OptimHyper h = {lr, beta1, beta2, eps, weight_decay, lr_t, 0};
  return run_host_optim(OPTIM_ADAM, param, grad, m, v, n, h);
}

int metal_kan_sgd_step(float* param, const float* grad, float* velocity, float lr,
                       float momentum, float weight_decay, int nesterov, int n) {
  const OptimHyper h = {lr, momentum, 0.f, 0.f, weight_decay, 0.f, nesterov ? 1 : 0};
  return run_host_optim(OPTIM_SGD, param, grad, velocity, nullptr, n, h);
}

int metal_kan_lion_step(float* param, const float* grad, float* m, float lr, float beta1,
                        float beta2, float weight_decay, int n) {
  const OptimHyper h = {lr, beta1, beta2, 0.f, weight_decay, 0.f, 0};
  return run_host_optim(OPTIM_LION, param, grad, m, nullptr, n, h);
}

int metal_kan_cheby_train_step(const float* X, const float* T, float* W, float* Wb, float* bias,
                               float* mW, float* vW, float* mWb, float* vWb, float* mb, float* vb,
                               int B, int D_in, int D_out, int degree, int hb, int hbi, float lr,
                               float beta1, float beta2, float eps, float weight_decay,
                               float lr_t) {
  const OptimHyper h = {lr, beta1, beta2, eps, weight_decay, lr_t, 0};
  return run_host_train_step(base_layer(KAN_CHEBY, KAN_F32, D_in, D_out, degree, hb, hbi), X, T,
                             W, Wb, bias, nullptr, mW, vW, mWb, vWb, mb, vb, B, h);
}

int metal_kan_fastkan_train_step(const float* X, const float* T, float* W, float* Wb,
                                 const float* grid, float* bias, float* mW, float* vW,
                                 float* mWb, float* vWb, float* mb, float* vb, int B, int D_in,
                                 int D_out, int num_centers, float inv_den, int hb, int hbi,
                                 float lr, float beta1, float beta2, float eps,
                                 float weight_decay, float lr_t) {
  if (!grid) return fail(KAN_ERR_ARG, "fastkan train_step: NULL grid");
  kan_layer L = base_layer(KAN_RBF, KAN_F32, D_in, D_out, num_centers, hb, hbi);
  L.inv_den = inv_den;
  const OptimHyper h = {lr, beta1, beta2, eps, weight_decay, lr_t, 0};
  return run_host_train_step(L, X, T, W, Wb, bias, grid, mW, vW, mWb, vWb, mb, vb, B, h);
}

int metal_kan_bspline_train_step(const float* X, const float* T, float* W, float* Wb,
                                 float* bias, float* mW, float* vW, float* mWb, float* vWb,
                                 float* mb, float* vb, int B, int D_in, int D_out, int grid_size,
                                 float grid_min, float grid_max, int hb, int hbi, float lr,
                                 float beta1, float beta2, float eps, float weight_decay,
                                 float lr_t) {
  if (grid_size <= 0 || !(grid_max > grid_min))
    return fail(KAN_ERR_ARG, "bspline train_step: bad grid");
  kan_layer L = base_layer(KAN_BSPLINE, KAN_F32, D_in, D_out, grid_size + 3, hb, hbi);
  L.grid_size = grid_size;
  L.grid_min = grid_min;
  L.inv_h = (float)grid_size / (grid_max - grid_min);  // metal_kan_bridge.mm bspline train step
  const OptimHyper h = {lr, beta1, beta2, eps, weight_decay, lr_t, 0};
  return run_host_train_step(L, X, T, W, Wb, bias, nullptr, mW, vW, mWb, vWb, mb, vb, B, h);
}

/* metal_kan_bridge.mm:5148 -- dY = (pred - target) * scale, host pointers */
int metal_kan_calc_mse_loss_backward(const float* pred, const float* target, float* dY, int n,
                                     float scale) {
  DeviceState* d;
  int rc = current_state(&d);
  if (rc) return rc;
  if (!pred || !target || !dY || n <= 0) return fail(KAN_ERR_ARG, "mse_loss_backward: bad arguments");
  const size_t bytes = (size_t)n * 4;
  void *dp, *dt, *dd;
  if ((rc = stage_in(d, S_T0, pred, bytes, &dp))) return rc;
  if ((rc = stage_in(d, S_T1, target, bytes, &dt))) return rc;
  if ((rc = slot(d, S_SC, bytes, &dd))) return rc;
  cudaError_t e = launch_mse_grad((const float*)dp, (const float*)dt, (float*)dd, n, scale, d->stream);
  if (e != cudaSuccess) return fail(KAN_ERR_CUDA, "mse_loss_backward: %s", cudaGetErrorString(e));
  KAN_CUDA_TRY(cudaMemcpyAsync(dY, dd, bytes, cudaMemcpyDeviceToHost, d->stream));
  KAN_CUDA_TRY(cudaStreamSynchronize(d->stream));
  return check_device_error(d);
}

}  // extern "C"
