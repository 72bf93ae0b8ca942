// kan_gemv_cc.cu -- host side of the small-batch path on the CUDA cores (kan_gemv_cc.cuh): the
// launch plan, tensor maps, the basis pre-pass instances and the launch.
#include <cuda.h>

#include <algorithm>
#include <atomic>
#include <map>
#include <mutex>
#include <tuple>

#include "kan_gemv_cc.cuh"

namespace kan {
namespace cc {

// ---------------------------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------------------------
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// [rows][cols] matrix of `esz`-byte elements, box = box_cols x ROWS, zero fill outside.
static bool make_map(CUtensorMap* m, const void* base, int rows, long long cols, int box_cols,
                     bool codes) {
  EncodeTiledFn enc = (EncodeTiledFn)tensor_map_encoder();
  const int esz = codes ? 1 : 4;
  if (!enc || ((uintptr_t)base & 15) || ((cols * esz) % 16)) return false;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(cols * esz)};
  cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)ROWS};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(m, codes ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2,
                   const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE,
                   codes ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// Code bytes and groups of one row of a packed weight with `cols` logical columns.
struct RowShape {
  long long bytes;
  int groups;
};
static RowShape row_shape(const kan_weight& w, int cols) {
  RowShape s = {0, 0};
  if (w.format == KAN_W_TERNARY || w.format == KAN_W_INT2) {
    s.bytes = (long long)((cols + 15) / 16) * 4;
    s.groups = (cols + w.group_size - 1) / w.group_size;
  } else if (w.format == KAN_W_INT8 || w.format == KAN_W_INT4) {
    s.bytes = w.format == KAN_W_INT8 ? w.padded_cols : w.padded_cols / 2;
    s.groups = w.group_size > 0 ? w.padded_cols / w.group_size : 0;
  }
  return s;
}

static int sm_count() {
  static int n[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (!n[dev]) {
    int v = 0;
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v <= 0)
      v = 148;
    n[dev] = v;
  }
  return n[dev];
}

// The main-kernel instance for a launch (ternary flags and flush width from the plan).
static MainFn main_kernel(int mode, int B, int fmt, bool fast, int fu) {
  if (mode == MODE_F16) {
    switch (B) {
      case 1: return select_main<MODE_F16, 1>(fmt, fast, fu);
      case 2: return select_main<MODE_F16, 2>(fmt, fast, fu);
      case 3: return select_main<MODE_F16, 3>(fmt, fast, fu);
      default: return select_main<MODE_F16, 4>(fmt, fast, fu);
    }
  }
  switch (B) {
    case 1: return select_main<MODE_BF16, 1>(fmt, fast, fu);
    case 2: return select_main<MODE_BF16, 2>(fmt, fast, fu);
    case 3: return select_main<MODE_BF16, 3>(fmt, fast, fu);
    default: return select_main<MODE_BF16, 4>(fmt, fast, fu);
  }
}

// The dynamic shared-memory limit every instance is given (once per device): the CTA maximum,
// so that a launch of any stage size stays within it.
constexpr int SMEM_MAX = 227 * 1024;

// Per instance and device: the shared-memory limit has been raised (bit per device).
static std::atomic<unsigned long long>& configured(MainFn k) {
  static std::mutex mu;
  static std::map<MainFn, std::atomic<unsigned long long>*> m;
  std::lock_guard<std::mutex> lk(mu);
  auto it = m.find(k);
  if (it == m.end()) it = m.emplace(k, new std::atomic<unsigned long long>(0)).first;
  return *it->second;
}

// Resident CTAs per SM of a main-kernel instance at `smem` bytes (cached per device, instance
// and size); raises the instance's dynamic shared-memory limit on this device first.
static int occupancy(MainFn k, int smem) {
  if (ensure_smem_attr(k, SMEM_MAX, configured(k)) != cudaSuccess) {
    (void)cudaGetLastError();
    return 1;
  }
  static std::mutex mu;
  static std::map<std::tuple<int, MainFn, int>, int> cache;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) dev = 0;
  std::lock_guard<std::mutex> lk(mu);
  const auto key = std::make_tuple(dev, k, smem);
  auto it = cache.find(key);
  if (it != cache.end()) return it->second;
  int v = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&v, k, THREADS, smem) != cudaSuccess ||
      v <= 0) {
    (void)cudaGetLastError();
    v = 1;
  }
  cache.emplace(key, v);
  return v;
}

static size_t align256(size_t v) { return (v + 255) & ~size_t(255); }

// Floats per row of the scale tile of a segment with `groups` groups per row: the groups one
// stage touches, 4-aligned at both ends, at most the whole row.
static int scale_box(int gps, int groups) { return std::min((gps + 3) / 4 * 4 + 4, groups); }

// The launch plan; `scratch` (may be null) fills the scratch pointers.  Returns the scratch
// bytes needed.
static size_t plan(const LayerArgs& a, int act_dtype, Params& p, void* scratch) {
  p = Params{};
  p.fmt = a.w.format;
  p.cpb = p.fmt == KAN_W_TERNARY ? 4 : (p.fmt == KAN_W_INT4 ? 2 : 1);
  p.fast = p.fmt == KAN_W_TERNARY && (a.w.flags & KAN_WFLAG_TERNARY_NO3) &&
           (!a.has_base || (a.wb.flags & KAN_WFLAG_TERNARY_NO3));
  p.gs = a.w.group_size;
  p.lg = 0;
  while ((16 << p.lg) < p.gs) ++p.lg;
  const int upc = p.cpb;                       // 16-code units per 16-byte chunk
  p.fu = std::min(upc, 1 << p.lg);             // a flush never crosses a group or a chunk
  const RowShape rw = row_shape(a.w, a.D_in * a.K);
  const RowShape rbs = a.has_base ? row_shape(a.wb, a.D_in) : RowShape{0, 0};
  p.stages_w = (int)((rw.bytes + ROW_BYTES - 1) / ROW_BYTES);
  p.stages_b = (int)((rbs.bytes + ROW_BYTES - 1) / ROW_BYTES);
  p.nst = p.stages_w + p.stages_b;
  const int ups = ROW_BYTES * p.cpb / 16;  // units per stage
  p.units_w = p.stages_w * ups;
  p.units_b = p.stages_b * ups;
  p.phi_pitch = (p.units_w + p.units_b) * 16;
  const int gps = std::max(1, ROW_BYTES * p.cpb / std::max(1, p.gs));  // groups per stage
  p.groups_w = rw.groups;
  p.groups_b = rbs.groups;
  p.sbox_w = scale_box(gps, rw.groups);
  p.sbox_b = a.has_base ? scale_box(gps, rbs.groups) : 4;
  p.sbox_max = std::max(p.sbox_w, p.sbox_b);
  const bool affine = p.fmt != KAN_W_TERNARY;
  p.ups = ups;
  const int Bs = std::min(MAXB, std::max(1, a.B));
  p.off_phi = CODE_TILE + ROWS * p.sbox_max * 4 * (affine ? 2 : 1);        // multiple of 512
  p.off_aux = p.off_phi + Bs * 2 * ups * 16;
  p.tile_bytes = p.off_aux + Bs * 2 * ups * 4;
  p.tile_bytes = (p.tile_bytes + 1023) / 1024 * 1024;  // 128-byte swizzle: 1 KB aligned stages
  p.off_red = STAGES * p.tile_bytes;
  p.off_bar = p.off_red + NWARPS * MAXB * ROWS * 4;
  p.smem = p.off_bar + 2 * STAGES * 8 + 16 + 1024;
  p.rowblocks = (a.D_out + ROWS - 1) / ROWS;
  const int mode = act_dtype == KAN_F16 ? MODE_F16 : MODE_BF16;
  const int occ = occupancy(main_kernel(mode, Bs, p.fmt, p.fast != 0, p.fu), p.smem);
  // as many K splits as keep the whole grid resident at once (one wave), at least 2 stages each
  int S = std::max(1, sm_count() * occ / std::max(1, p.rowblocks));
  S = std::min(S, std::max(1, p.nst / 2));
  p.S = S;
  const int Bn = std::max(1, a.B);
  size_t off = 0;
  const size_t o_hi = off;
  off = align256(off + (size_t)Bn * p.phi_pitch);
  const size_t o_lo = off;
  off = align256(off + (size_t)Bn * p.phi_pitch);
  const size_t o_sum = off;
  off = align256(off + (size_t)Bn * (p.units_w + p.units_b) * 4);
  const size_t o_p2b = off;
  off = align256(off + (size_t)Bn * std::max(1, p.units_b) * 4);
  const size_t o_part = off;
  off = align256(off + (size_t)S * Bn * a.D_out * 4);
  const size_t o_cnt = off;
  off = align256(off + (size_t)p.rowblocks * 4);
  if (scratch) {
    uint8_t* base = (uint8_t*)scratch;
    p.phi_hi = (int8_t*)(base + o_hi);
    p.phi_lo = (int8_t*)(base + o_lo);
    p.sumphi = (float*)(base + o_sum);
    p.p2b = (float*)(base + o_p2b);
    p.part = (float*)(base + o_part);
    p.counters = (int*)(base + o_cnt);
  }
  return off;
}

}  // namespace cc

bool gemv_cc_supported(const LayerArgs& a, int act_dtype) {
  using namespace cc;
  if (act_dtype != KAN_F16 && act_dtype != KAN_BF16) return false;
  if (a.B < 1 || a.B > MAXB || a.D_in < 1 || a.D_out < 1 || a.K < 1) return false;
  // the fixed-point basis matrix needs |phi| <= 1: every basis but Jacobi (whose polynomials
  // exceed 1 for alpha or beta > 0)
  if (a.basis == KAN_JACOBI) return false;
  if (pre_smem_bytes(a.K) > 48 * 1024) return false;  // the pre-pass stages 64 features' terms
  const int fmt = a.w.format;
  if (fmt != KAN_W_TERNARY && fmt != KAN_W_INT8 && fmt != KAN_W_INT4) return false;
  const int gs = a.w.group_size;
  if (gs < 16 || (gs & (gs - 1)) || gs > 4096) return false;  // group index by shift
  if (a.has_base && (a.wb.format != fmt || a.wb.group_size != gs)) return false;
  // TMA: rows of 16-byte multiples at least one box wide, whole 4-float groups of scales
  auto fits = [&](const RowShape& s) {
    return s.bytes % 16 == 0 && s.bytes >= BOX_BYTES && s.groups % 4 == 0 && s.groups >= 4;
  };
  if (!fits(row_shape(a.w, a.D_in * a.K))) return false;
  if (a.has_base && !fits(row_shape(a.wb, a.D_in))) return false;
  if (fmt != KAN_W_TERNARY) {
    // the padded row holds whole groups: codes of a row start at row * padded_cols
    if (a.w.padded_cols % gs || a.w.padded_cols < a.D_in * a.K) return false;
    if (a.has_base && (a.wb.padded_cols % gs || a.wb.padded_cols < a.D_in)) return false;
  }
  auto al = [](const void* ptr) { return ((uintptr_t)ptr & 15) == 0; };
  if (!al(a.w.data) || !al(a.w.scales) || (fmt != KAN_W_TERNARY && !al(a.w.biases))) return false;
  if (a.has_base &&
      (!al(a.wb.data) || !al(a.wb.scales) || (fmt != KAN_W_TERNARY && !al(a.wb.biases))))
    return false;
  return tensor_map_encoder() != nullptr;
}

size_t gemv_cc_scratch_bytes(const LayerArgs& a) {
  cc::Params p;
  return cc::plan(a, a.act_dtype, p, nullptr);
}

int gemv_cc_splits(const LayerArgs& a) {
  cc::Params p;
  cc::plan(a, a.act_dtype, p, nullptr);
  return p.S;
}

template <int MODE>
static void launch_phi(const LayerArgs& a, const cc::Params& p, cudaStream_t s) {
  const dim3 grid((unsigned)((a.D_in + cc::PRE_FEATURES - 1) / cc::PRE_FEATURES), (unsigned)a.B);
  const size_t sm = (size_t)cc::pre_smem_bytes(a.K);
  switch (a.basis) {
    case KAN_CHEBY: cc::cc_phi_kernel<MODE, KAN_CHEBY><<<grid, cc::PRE_THREADS, sm, s>>>(a, p); break;
    case KAN_RBF: cc::cc_phi_kernel<MODE, KAN_RBF><<<grid, cc::PRE_THREADS, sm, s>>>(a, p); break;
    case KAN_BSPLINE:
      cc::cc_phi_kernel<MODE, KAN_BSPLINE><<<grid, cc::PRE_THREADS, sm, s>>>(a, p);
      break;
    case KAN_WAVELET:
      cc::cc_phi_kernel<MODE, KAN_WAVELET><<<grid, cc::PRE_THREADS, sm, s>>>(a, p);
      break;
    case KAN_RELU: cc::cc_phi_kernel<MODE, KAN_RELU><<<grid, cc::PRE_THREADS, sm, s>>>(a, p); break;
    default: cc::cc_phi_kernel<MODE, KAN_FOURIER><<<grid, cc::PRE_THREADS, sm, s>>>(a, p); break;
  }
}

cudaError_t launch_gemv_cc(const LayerArgs& a, int act_dtype, void* scratch, cudaStream_t s) {
  using namespace cc;
  Params p;
  plan(a, act_dtype, p, scratch);
  const int mode = act_dtype == KAN_F16 ? MODE_F16 : MODE_BF16;
  const int fmt = p.fmt;
  CUtensorMap cw, sw, mw, cb, sb, mb;
  const RowShape rw = row_shape(a.w, a.D_in * a.K);
  if (!make_map(&cw, a.w.data, a.D_out, rw.bytes, BOX_BYTES, true) ||
      !make_map(&sw, a.w.scales, a.D_out, rw.groups, p.sbox_w, false))
    return cudaErrorInvalidValue;
  mw = sw;
  if (fmt != KAN_W_TERNARY && !make_map(&mw, a.w.biases, a.D_out, rw.groups, p.sbox_w, false))
    return cudaErrorInvalidValue;
  cb = cw;
  sb = sw;
  mb = mw;
  if (a.has_base) {
    const RowShape rbs = row_shape(a.wb, a.D_in);
    if (!make_map(&cb, a.wb.data, a.D_out, rbs.bytes, BOX_BYTES, true) ||
        !make_map(&sb, a.wb.scales, a.D_out, rbs.groups, p.sbox_b, false))
      return cudaErrorInvalidValue;
    if (fmt != KAN_W_TERNARY && !make_map(&mb, a.wb.biases, a.D_out, rbs.groups, p.sbox_b, false))
      return cudaErrorInvalidValue;
  }
  if (mode == MODE_F16) launch_phi<MODE_F16>(a, p, s);
  else launch_phi<MODE_BF16>(a, p, s);
  note_launch();
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;

  const MainFn kern = main_kernel(mode, a.B, fmt, p.fast != 0, p.fu);
  if ((e = ensure_smem_attr(kern, SMEM_MAX, configured(kern))) != cudaSuccess) return e;
  if (p.smem > SMEM_MAX) return cudaErrorInvalidValue;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)p.rowblocks, (unsigned)p.S, 1);
  cfg.blockDim = dim3(THREADS, 1, 1);
  cfg.dynamicSmemBytes = (size_t)p.smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  // programmatic dependent launch: the weight stream starts while the pre-pass runs
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  note_launch();
  return cudaLaunchKernelEx(&cfg, kern, cw, sw, mw, cb, sb, mb, a, p);
}

}  // namespace kan
