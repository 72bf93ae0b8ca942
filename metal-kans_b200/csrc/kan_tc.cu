// kan_tc.cu -- host side of the tensor-core path: launch planning (tile width, split-K factor),
// the TMA descriptor of the packed weights, dispatch to the kernel instances (kan_tc_inst.cu),
// and the kernel that packs weights into the feature-blocked layout (kan_tc_pack).
#include <cuda.h>

#include <mutex>

#include "kan_device.cuh"
#include "kan_launch.h"
#include "kan_tc_dispatch.h"

namespace kan {
namespace tc {

constexpr int BM = 128;
constexpr int BK = 64;
constexpr int MAX_SPLITS = 4;  // split-K cluster size (reduction slots sized for it)

// Pack W (basis terms) and Wb (base weights) into Wp[D_out][NB*64]: block b, column j holds term
// t = j % KT of feature i = b*F + j/KT (t < K: W[o, i*K + t]; t == K: Wb[o, i]); zero elsewhere.
// Packed formats are decoded to their exact fp32 value, then rounded to the act dtype.
// part >= 0: the layer is half of a gate/up pair and its row o goes to row
// (o / PAIR_BLOCK) * 2 * PAIR_BLOCK + part * PAIR_BLOCK + o % PAIR_BLOCK of `out`.
template <int MODE>
__global__ void pack_kernel(LayerArgs a, typename Act<MODE>::T* out, int KT, int F, int NB,
                            int part) {
  const long long cols = (long long)NB * BK;
  const long long total = cols * a.D_out;
  const int Kdim = a.D_in * a.K;
  for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < total;
       e += (long long)gridDim.x * blockDim.x) {
    const int o = (int)(e / cols);
    const int c = (int)(e - (long long)o * cols);
    const int b = c / BK, jj = c - b * BK;
    const int f = jj / KT, t = jj - f * KT;
    const int i = b * F + f;
    float v = 0.f;
    if (f < F && i < a.D_in) {
      v = (t < a.K) ? weight_value<MODE>(a.w, o, i * a.K + t, Kdim)
                    : weight_value<MODE>(a.wb, o, i, a.D_in);
    }
    const long long orow = part < 0 ? o
                                    : (long long)(o / PAIR_BLOCK) * 2 * PAIR_BLOCK +
                                          part * PAIR_BLOCK + o % PAIR_BLOCK;
    out[orow * cols + c] = Act<MODE>::from_f(v);
  }
}

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn get_encode() { return (EncodeTiledFn)tensor_map_encoder(); }

// 2-D tensor map over the packed [rows][cols] 16-bit matrix, box = 64 columns x box_rows,
// 128-byte swizzle, zero fill out of range (rows beyond D_out).  cols is a multiple of 64, so the
// row pitch is a multiple of 128 bytes and every box starts on a 128-byte boundary.
static bool make_tmap(CUtensorMap* m, const void* base, int rows, long long cols, int box_rows,
                      int mode) {
  EncodeTiledFn enc = get_encode();
  if (!enc || ((uintptr_t)base & 15)) return false;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
  cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(m, mode == MODE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                        : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                   2, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// 2-D tensor map over the input X[B][D_in] (16-bit), box = 64 features x 128 rows, 128-byte
// swizzle; zero fill beyond B rows and D_in features.  Needs 16-byte aligned rows.
static bool make_tmap_x(CUtensorMap* m, const void* base, int B, int D_in, int mode) {
  EncodeTiledFn enc = get_encode();
  if (!enc || ((uintptr_t)base & 15) || (D_in % 8) != 0) return false;
  cuuint64_t dims[2] = {(cuuint64_t)D_in, (cuuint64_t)B};
  cuuint64_t strides[1] = {(cuuint64_t)D_in * 2};
  cuuint32_t box[2] = {64, (cuuint32_t)BM};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(m, mode == MODE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                        : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                   2, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

static const DispatchFn kDispatch[3][NUM_BASES] = {
    {nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr},
    {dispatch_1_0, dispatch_1_1, dispatch_1_2, dispatch_1_3, dispatch_1_4, dispatch_1_5,
     dispatch_1_6},
    {dispatch_2_0, dispatch_2_1, dispatch_2_2, dispatch_2_3, dispatch_2_4, dispatch_2_5,
     dispatch_2_6}};

}  // namespace tc

void* tensor_map_encoder() {
  static void* fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = p;
  });
  return fn;
}

bool tc_supported(const LayerArgs& a, int act_dtype) {
  if (act_dtype != KAN_F16 && act_dtype != KAN_BF16) return false;
  if (a.B <= 0 || a.D_in <= 0 || a.D_out <= 0 || a.K <= 0) return false;
  if (a.K + (a.has_base ? 1 : 0) > 64) return false;
  return tc::get_encode() != nullptr;
}

TcPlan tc_plan(const LayerArgs& a) {
  TcPlan p;
  p.BN = a.D_out > 128 ? 256 : (a.D_out > 64 ? 128 : 64);
  const TcBlocking bl = tc_blocking(a.D_in, a.K, a.has_base);
  p.nb = bl.NB;
  p.mtiles = (a.B + tc::BM - 1) / tc::BM;
  // wide tiles (two N = 256 accumulators per basis block) halve the basis work per output; taken
  // when the grid of wide tiles fills the GPU, or does with K split in two (the producers then
  // build half the blocks per CTA: 64 wide tiles x 2 splits run in one wave where 128 narrow
  // tiles each build every block), never for the staged LayerNorm input
  if (a.D_out >= 512 && a.input_map != KAN_MAP_LAYERNORM) {
    const long long wide_tiles = (long long)p.mtiles * ((a.D_out + 511) / 512);
    const int wide_splits = wide_tiles >= 120 ? 1 : (wide_tiles * 2 >= 120 && p.nb / 2 >= 32) ? 2 : 0;
    if (wide_splits) {
      p.BN = 512;
      p.ntiles = (a.D_out + 511) / 512;
      p.splits = wide_splits;
      return p;
    }
  }
  p.ntiles = (a.D_out + p.BN - 1) / p.BN;
  const long long tiles = (long long)p.mtiles * p.ntiles;
  int splits = 1;
  if (tiles < 120) {
    // split K over a cluster so that the grid covers the 148 SMs; the cluster reduction needs
    // BN % (32 * splits) == 0, and each split keeps at least 4 K blocks
    splits = (int)(148 / tiles);
    const int max_by_k = p.nb / 4;
    splits = splits > max_by_k ? max_by_k : splits;
    splits = splits > tc::MAX_SPLITS ? tc::MAX_SPLITS : splits;
    while (splits > 1 && (p.BN % (32 * splits)) != 0) --splits;
    splits = splits < 1 ? 1 : splits;
  } else {
    // several waves of one-CTA-per-SM tiles: the last wave of tiles * S CTAs on 148 SMs runs
    // partly empty.  Split K (S = 2 or 4, at least 32 K blocks per split, so the cluster
    // reduction stays small against the main loop) when that fills the waves better by more
    // than 2 %: e.g. 512 tiles = 3.46 waves (86 % filled), split in two = 6.92 waves (99 %).
    auto fill = [&](int S) {
      const long long ctas = tiles * S;
      const long long waves = (ctas + 147) / 148;
      return (double)ctas / (double)(waves * 148);
    };
    double best = fill(1);
    for (int S = 2; S <= tc::MAX_SPLITS; S *= 2) {
      if (p.BN % (32 * S) != 0 || p.nb / S < 32) continue;
      const double f = fill(S);
      if (f > best + 0.02) {
        best = f;
        splits = S;
      }
    }
  }
  p.splits = splits;
  return p;
}

cudaError_t launch_tc(const LayerArgs& a, int act_dtype, const TcPlan& p, cudaStream_t s) {
  if (!tc_supported(a, act_dtype) || !a.tc_weights) return cudaErrorNotSupported;
  const int mode = act_dtype == KAN_F16 ? MODE_F16 : MODE_BF16;
  CUtensorMap tw;
  if (!tc::make_tmap(&tw, a.tc_weights, a.D_out, (long long)p.nb * tc::BK, p.BN > 256 ? 256 : p.BN,
                     mode))
    return cudaErrorInvalidValue;
  // the input in 64-feature x 128-row tiles for the producers (rows of 16-byte multiples only)
  CUtensorMap tx = tw;
  const int x_tma = tc::make_tmap_x(&tx, a.X, a.B, a.D_in, mode) ? 1 : 0;
  note_launch();
  dim3 grid(p.mtiles, p.ntiles, p.splits);
  return tc::kDispatch[mode][a.basis](tw, tx, x_tma, a, p.BN, p.nb, p.splits, grid, s);
}

static cudaError_t pack_part(const LayerArgs& a, int act_dtype, void* out, int part,
                             cudaStream_t s) {
  const TcBlocking bl = tc_blocking(a.D_in, a.K, a.has_base);
  if (bl.F <= 0) return cudaErrorInvalidValue;
  note_launch();
  const long long total = (long long)bl.NB * tc::BK * a.D_out;
  long long blocks = (total + 255) / 256;
  if (blocks > 148LL * 16) blocks = 148LL * 16;
  if (blocks < 1) blocks = 1;
  if (act_dtype == KAN_F16)
    tc::pack_kernel<MODE_F16><<<(int)blocks, 256, 0, s>>>(a, (__half*)out, bl.KT, bl.F, bl.NB,
                                                         part);
  else
    tc::pack_kernel<MODE_BF16><<<(int)blocks, 256, 0, s>>>(a, (__nv_bfloat16*)out, bl.KT, bl.F,
                                                          bl.NB, part);
  return cudaGetLastError();
}

cudaError_t launch_tc_pack(const LayerArgs& a, int act_dtype, void* out, cudaStream_t s) {
  return pack_part(a, act_dtype, out, -1, s);
}

cudaError_t launch_tc_pack_pair(const LayerArgs& gate, const LayerArgs& up, int act_dtype,
                                void* out, cudaStream_t s) {
  const TcBlocking bl = tc_blocking(gate.D_in, gate.K, gate.has_base);
  // rows past D_out in either half stay zero
  cudaError_t e = cudaMemsetAsync(out, 0, (size_t)pair_rows(gate.D_out) * bl.NB * tc::BK * 2, s);
  if (e != cudaSuccess) return e;
  if ((e = pack_part(gate, act_dtype, out, 0, s)) != cudaSuccess) return e;
  return pack_part(up, act_dtype, out, 1, s);
}

}  // namespace kan
