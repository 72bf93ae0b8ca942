// tcgen05_mma_rate.cu -- issue rate of tcgen05.mma.cta_group::1.kind::f16 per instruction shape.
//
// One CTA; thread 0 issues 512 MMAs back to back (fully unrolled, descriptors precomputed, the
// accumulator in TMEM, A from shared memory (SS) or from TMEM (TS)); optionally warps 4-7 store
// into TMEM (tcgen05.st.32x32b.x32 + wait::st) at the same time.  Prints cycles per MMA for the
// issue loop and until the commit's mbarrier completes.  This measurement sets the small-batch
// kernel's design floor: below N = 128 an MMA costs the same ~50 cycles whatever its N.
//
//   nvcc -gencode arch=compute_100a,code=sm_100a -O3 -std=c++17 -I include \
//        -o tcgen05_mma_rate metal-kans_b200/microbench/tcgen05_mma_rate.cu && ./tcgen05_mma_rate
#include <cstdio>
#include <cuda.h>
#include "../csrc/kan_tc_kernel.cuh"
using namespace kan::tc;

__device__ __forceinline__ void mma_ts2(uint32_t d, uint32_t a, uint64_t bdesc, uint32_t idesc, uint32_t acc) {
  asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
               "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}\n"
               ::"r"(d), "r"(a), "l"(bdesc), "r"(idesc), "r"(acc) : "memory");
}

__device__ __forceinline__ void st32(uint32_t taddr, uint32_t v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1};" ::"r"(taddr), "r"(v) : "memory");
}
template <int MODE, int ND>
__global__ void bench(long long* out, int M, int N, int niter, int nst) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  const uint32_t sb = smem_u32(smem);
  for (int i = threadIdx.x; i < (48 * 1024) / 16; i += blockDim.x)
    reinterpret_cast<uint4*>(smem)[i] = make_uint4(0, 0, 0, 0);
  const uint32_t bar = sb + 48 * 1024, slot = bar + 8;
  if (threadIdx.x == 0) { mbar_init(bar, 1); asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
  if (threadIdx.x < 32) tmem_alloc(slot, 512);
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(smem + 48 * 1024 + 8);
  if (threadIdx.x >= 128) {
    const int q = (threadIdx.x >> 5) & 3;
    long long t0 = clock64();
    for (int i = 0; i < nst; ++i) {
      st32(tmem + ((uint32_t)(q * 32) << 16) + 64 + (uint32_t)((i & 3) * 32), (uint32_t)i);
      asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
    }
    if ((threadIdx.x & 31) == 0) out[8 + q] = clock64() - t0;
  }
  if (threadIdx.x == 0) {
    const uint32_t idesc = instr_desc(1, N, M);
    uint64_t ad[4], bd[4];
    uint32_t ta[4], dd[ND];
#pragma unroll
    for (int k = 0; k < 4; ++k) { ad[k] = smem_desc_sw128(sb) + 2 * k; bd[k] = smem_desc_sw128(sb + 16 * 1024) + 2 * k; ta[k] = tmem + k * 8; }
#pragma unroll
    for (int j = 0; j < ND; ++j) dd[j] = tmem + 256 + j * N;
    long long t0 = clock64();
#pragma unroll 1
    for (int i = 0; i < niter; i += 4 * ND) {
#pragma unroll
      for (int j = 0; j < ND; ++j)
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          if (MODE == 0) mma_f16(dd[j], ad[k], bd[k], idesc, (i > 0 || k > 0) ? 1u : 0u);
          else mma_ts2(dd[j], ta[k], bd[k], idesc, (i > 0 || k > 0) ? 1u : 0u);
        }
    }
    long long t1 = clock64();
    mma_commit(bar);
    bool ok = mbar_wait(bar, 0);
    long long t2 = clock64();
    out[0] = t1 - t0; out[1] = t2 - t0; out[2] = ok;
  }
  tc_fence_before();
  __syncthreads();
  if (threadIdx.x < 32) { tc_fence_after(); tmem_dealloc(tmem, 512); }
}

template <int MODE, int ND>
static void run(long long* d, int M, int N, const char* name, int nst = 0) {
  cudaFuncSetAttribute(bench<MODE, ND>, cudaFuncAttributeMaxDynamicSharedMemorySize, 50 * 1024 + 1024);
  for (int rep = 0; rep < 2; ++rep) {
    bench<MODE, ND><<<1, nst ? 256 : 128, 50 * 1024 + 1024>>>(d, M, N, 512, nst);
    cudaError_t e = cudaDeviceSynchronize();
    if (e != cudaSuccess) { printf("%s: error %s\n", name, cudaGetErrorString(e)); exit(1); }
    long long hh[12];
    cudaMemcpy(hh, d, 96, cudaMemcpyDeviceToHost);
    if (rep) printf("%-18s issue %6.1f  complete %6.1f cycles/MMA  ok=%lld  (ideal full-rate %5.1f)  st: %lld st.x32 per warp, %.1f cycles each\n", name,
                    hh[0] / 512.0, hh[1] / 512.0, hh[2], (double)M * N * 16 * 2 / 8192.0, (long long)nst, nst ? hh[8] / (double)nst : 0.0);
  }
}
int main() {
  long long* d;
  cudaMalloc(&d, 128);
  run<0, 1>(d, 128, 16, "SS M128 N16");
  run<1, 1>(d, 128, 16, "TS M128 N16");
  run<1, 4>(d, 128, 16, "TS M128 N16 d4");
  run<0, 1>(d, 128, 64, "SS M128 N64");
  run<0, 1>(d, 128, 128, "SS M128 N128");
  run<0, 1>(d, 128, 256, "SS M128 N256");
  run<0, 1>(d, 64, 256, "SS M64 N256");
  run<1, 1>(d, 128, 16, "TS M128 N16 +st", 400);
  run<1, 4>(d, 128, 16, "TS M128 N16 d4 +st", 400);
  return 0;
}
