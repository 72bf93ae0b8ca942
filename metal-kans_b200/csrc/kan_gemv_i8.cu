// kan_gemv_i8.cu -- host side and instances of the 8-bit tensor-core small-batch kernel
// (kan_gemv_i8.cuh): the launch plan, tensor maps, the basis pre-pass and the launch.
#include <cuda.h>

#include <algorithm>
#include <atomic>
#include <map>
#include <mutex>

#include "kan_gemv_i8.cuh"

namespace kan {
namespace i8 {

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

constexpr int SMEM_MAX = 227 * 1024;

// [rows][cols] matrix of 1-byte (codes, basis bytes) or 4-byte (scales) elements, box =
// box_cols x box_rows, zero fill outside.
static bool make_map(CUtensorMap* m, const void* base, int rows, long long cols, int box_cols,
                     int box_rows, bool bytes, bool swizzle) {
  EncodeTiledFn enc = (EncodeTiledFn)tensor_map_encoder();
  const int esz = bytes ? 1 : 4;
  if (!enc || ((uintptr_t)base & 15) || ((cols * esz) % 16)) return false;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(cols * esz)};
  cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(m, bytes ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2,
                   const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE,
                   swizzle ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
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

static size_t align256(size_t v) { return (v + 255) & ~size_t(255); }

struct Scratch {
  size_t counters, part, hi, lo, sums, p2b, bytes;
};

// The launch plan and the scratch layout.
static Scratch plan(const LayerArgs& a, Params& p) {
  p = Params{};
  const int NP = a.B <= 8 ? 8 : 16;
  const long long kdim = (long long)a.D_in * a.K;
  p.Ww = (int)((kdim + WIN_CODES - 1) / WIN_CODES);
  const int Wb = a.has_base ? (a.D_in + WIN_CODES - 1) / WIN_CODES : 0;
  p.W = p.Ww + Wb;
  p.gpu = a.w.group_size / UNIT;
  p.sfl = WIN_CODES / a.w.group_size;
  p.units_w = p.Ww * (WIN_CODES / 16);
  p.units_b = Wb * (WIN_CODES / 16);
  p.off_phi = CODE_TILE;
  p.off_scale = p.off_phi + 4 * (2 * NP * 128);
  p.off_p2b = p.off_scale + ROWS * p.sfl * 4;
  p.stage_bytes = (p.off_p2b + NP * 128 + 1023) / 1024 * 1024;
  p.off_bar = STAGES * p.stage_bytes;
  const int nbars = 2 * STAGES + 2 * ASLOTS + 2 * ACC_SLOTS + NISS;
  p.smem = p.off_bar + nbars * 8 + 16 + 1024;
  p.rowblocks = (a.D_out + ROWS - 1) / ROWS;
  p.tasks = (long long)p.rowblocks * p.W;
  p.G = (int)std::min<long long>(p.tasks, sm_count());
  p.maxc = 1;
  for (int rb = 0; rb < p.rowblocks; ++rb)
    p.maxc = std::max(p.maxc, kl::owner((long long)rb * p.W + p.W - 1, p.tasks, p.G) -
                                  kl::owner((long long)rb * p.W, p.tasks, p.G) + 1);
  Scratch sc;
  const int Bn = std::max(1, a.B);
  const size_t pitch = (size_t)(p.units_w + p.units_b) * 16;
  size_t off = 0;
  sc.counters = off;
  off = align256(off + (size_t)p.rowblocks * 8);
  sc.part = off;
  off = align256(off + (size_t)p.rowblocks * p.maxc * NP * ROWS * 4);
  sc.hi = off;
  off = align256(off + (size_t)Bn * pitch);
  sc.lo = off;
  off = align256(off + (size_t)Bn * pitch);
  sc.sums = off;
  off = align256(off + (size_t)Bn * (p.units_w + p.units_b) * 4);
  sc.p2b = off;
  off = align256(off + (size_t)Bn * std::max(1, p.units_b) * 4);
  sc.bytes = off;
  return sc;
}

using I8Fn = void (*)(const CUtensorMap, const CUtensorMap, const CUtensorMap, const CUtensorMap,
                      const CUtensorMap, const CUtensorMap, LayerArgs, Params);

static I8Fn kernel_for(int act_dtype, int NP) {
  if (act_dtype == KAN_F16) return NP == 8 ? kan_gemv_i8_kernel<MODE_F16, 8> : kan_gemv_i8_kernel<MODE_F16, 16>;
  return NP == 8 ? kan_gemv_i8_kernel<MODE_BF16, 8> : kan_gemv_i8_kernel<MODE_BF16, 16>;
}

static std::atomic<unsigned long long>& configured(I8Fn k) {
  static std::mutex mu;
  static std::map<I8Fn, std::atomic<unsigned long long>*> m;
  std::lock_guard<std::mutex> lk(mu);
  auto it = m.find(k);
  if (it == m.end()) it = m.emplace(k, new std::atomic<unsigned long long>(0)).first;
  return *it->second;
}

}  // namespace i8

// Ternary layers (basis and base branch alike) in groups of 64 or 128 codes at 5 <= B <= 16, any
// basis with |phi| <= 1 (not Jacobi), code rows of 16-byte multiples and whole 4-float groups of
// scales per row.
bool gemv_i8_supported(const LayerArgs& a, int act_dtype) {
  using namespace i8;
  if (act_dtype != KAN_F16 && act_dtype != KAN_BF16) return false;
  if (a.B < 5 || a.B > 16 || a.D_in < 1 || a.D_out < 1 || a.K < 1) return false;
  if (a.basis == KAN_JACOBI) return false;
  if (cc::pre_smem_bytes(a.K) > 48 * 1024) return false;
  if (a.w.format != KAN_W_TERNARY) return false;
  const int gs = a.w.group_size;
  if (gs != 64 && gs != 128) return false;
  if (a.has_base && (a.wb.format != KAN_W_TERNARY || a.wb.group_size != gs)) return false;
  const long long bytes_w = ((long long)a.D_in * a.K + 15) / 16 * 4;
  const long long groups_w = ((long long)a.D_in * a.K + gs - 1) / gs;
  if (bytes_w % 16 || groups_w % 4) return false;
  if (a.has_base) {
    const long long bytes_b = ((long long)a.D_in + 15) / 16 * 4, groups_b = (a.D_in + gs - 1) / gs;
    if (bytes_b % 16 || groups_b % 4) return false;
  }
  auto al = [](const void* ptr) { return ((uintptr_t)ptr & 15) == 0; };
  if (!al(a.w.data) || !al(a.w.scales)) return false;
  if (a.has_base && (!al(a.wb.data) || !al(a.wb.scales))) return false;
  Params p;
  plan(a, p);
  if (p.smem > SMEM_MAX) return false;
  return tensor_map_encoder() != nullptr;
}

size_t gemv_i8_scratch_bytes(const LayerArgs& a) {
  i8::Params p;
  return i8::plan(a, p).bytes;
}

int gemv_i8_splits(const LayerArgs& a) {
  i8::Params p;
  i8::plan(a, p);
  return p.maxc;
}

cudaError_t launch_gemv_i8(const LayerArgs& a, int act_dtype, void* scratch, cudaStream_t s) {
  using namespace i8;
  Params p;
  const Scratch sc = plan(a, p);
  uint8_t* base = (uint8_t*)scratch;
  p.counters = (unsigned long long*)(base + sc.counters);
  p.part = (float*)(base + sc.part);
  p.p2b = (const float*)(base + sc.p2b);
  p.epoch = kl::next_epoch();
  const int NP = a.B <= 8 ? 8 : 16;
  const int gs = a.w.group_size;
  const long long bytes_w = ((long long)a.D_in * a.K + 15) / 16 * 4;
  const long long groups_w = ((long long)a.D_in * a.K + gs - 1) / gs;
  const long long pitch = (long long)(p.units_w + p.units_b) * 16;
  CUtensorMap cw, sw, cb, sb, thi, tlo;
  if (!make_map(&cw, a.w.data, a.D_out, bytes_w, 128, ROWS, true, true) ||
      !make_map(&sw, a.w.scales, a.D_out, groups_w, p.sfl, ROWS, false, false) ||
      !make_map(&thi, base + sc.hi, a.B, pitch, 128, NP, true, true) ||
      !make_map(&tlo, base + sc.lo, a.B, pitch, 128, NP, true, true))
    return cudaErrorInvalidValue;
  cb = cw;
  sb = sw;
  if (a.has_base) {
    const long long bytes_b = ((long long)a.D_in + 15) / 16 * 4, groups_b = (a.D_in + gs - 1) / gs;
    if (!make_map(&cb, a.wb.data, a.D_out, bytes_b, 128, ROWS, true, true) ||
        !make_map(&sb, a.wb.scales, a.D_out, groups_b, p.sfl, ROWS, false, false))
      return cudaErrorInvalidValue;
  }
  // the basis matrix in the table decoder's byte order (no unit sums: the decoded codes are
  // signed), its padding columns zeroed by the pre-pass
  cc::Params pp = {};
  pp.fmt = KAN_W_TERNARY;
  pp.fast = 0;
  pp.fu = 1;
  pp.units_w = p.units_w;
  pp.units_b = p.units_b;
  pp.phi_pitch = (int)pitch;
  pp.rowblocks = 0;
  pp.phi_hi = (int8_t*)(base + sc.hi);
  pp.phi_lo = (int8_t*)(base + sc.lo);
  pp.sumphi = (float*)(base + sc.sums);
  pp.p2b = (float*)(base + sc.p2b);
  cudaError_t e = launch_cc_prepass(a, act_dtype, pp, s);
  if (e != cudaSuccess) return e;

  const I8Fn kern = kernel_for(act_dtype, NP);
  if ((e = ensure_smem_attr(kern, SMEM_MAX, configured(kern))) != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)p.G, 1, 1);
  cfg.blockDim = dim3(THREADS, 1, 1);
  cfg.dynamicSmemBytes = (size_t)p.smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  // programmatic dependent launch: the code stream starts while the basis pre-pass runs
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  note_launch();
  return cudaLaunchKernelEx(&cfg, kern, cw, sw, cb, sb, thi, tlo, a, p);
}

}  // namespace kan
