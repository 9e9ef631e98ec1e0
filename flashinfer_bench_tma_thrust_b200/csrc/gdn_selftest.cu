// gdn_selftest.cu — known-answer check of the tcgen05 building blocks.
//
// One 128x64x128 bf16 GEMM D = A * B through shared-memory descriptors in the
// K-major or MN-major 128B-swizzled layouts, the MMA, commit-to-mbarrier and
// the TMEM load path that the chunked prefill kernel is built from. The GPU
// tests compare D with a torch matmul, for all four major-ness combinations.
#include "gdn_b200.h"
#include "gdn_common.cuh"
#include "sm100_umma.cuh"

namespace gdn {
namespace {

using namespace sm100;

// A: [128 (m)][128 (k)] row-major bf16; B: [128 (k)][64 (n)] row-major bf16; D [128][64] fp32.
__global__ void __launch_bounds__(128) umma_selftest_kernel(const __nv_bfloat16* A,
                                                            const __nv_bfloat16* B, float* D,
                                                            int a_mn, int b_mn, int* status) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = align_smem<1024>(smem_raw);
  uint8_t* sA = smem;            // 32 KB
  uint8_t* sB = smem + 32768;    // 16 KB
  __shared__ uint64_t bar;
  __shared__ uint32_t tmem_base;
  const int t = threadIdx.x;
  const int warp = t >> 5;

  // Fill A. K-major: 2 tiles (k halves) of 128 rows (m) x 64 cols (k).
  //         MN-major: 2 tiles (m blocks) of 128 rows (k) x 64 cols (m).
  for (int idx = t; idx < 128 * 128; idx += 128) {
    const int m = idx / 128, k = idx % 128;
    const __nv_bfloat16 val = A[idx];
    uint32_t off;
    if (!a_mn) off = (k / 64) * 16384 + sw128_offset(m, k % 64);
    else off = (m / 64) * 16384 + sw128_offset(k, m % 64);
    *reinterpret_cast<__nv_bfloat16*>(sA + off) = val;
  }
  // Fill B. K-major: 2 tiles (k halves) of 64 rows (n) x 64 cols (k).
  //         MN-major: 1 tile of 128 rows (k) x 64 cols (n).
  for (int idx = t; idx < 128 * 64; idx += 128) {
    const int k = idx / 64, n = idx % 64;
    const __nv_bfloat16 val = B[idx];
    uint32_t off;
    if (!b_mn) off = (k / 64) * 8192 + sw128_offset(n, k % 64);
    else off = sw128_offset(k, n);
    *reinterpret_cast<__nv_bfloat16*>(sB + off) = val;
  }
  if (t == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
  }
  if (warp == 0) tmem_alloc(&tmem_base, 64);
  fence_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = tmem_base;
  if (t == 0) {
    const uint32_t idesc = idesc_bf16(128, 64, a_mn != 0, b_mn != 0);
    const uint32_t a0 = smem_u32(sA), b0 = smem_u32(sB);
    for (int s = 0; s < 8; ++s) {
      const uint64_t ad = a_mn ? desc_mnmajor(a0 + s * 2048, 16384)
                               : desc_kmajor(a0 + (s / 4) * 16384 + (s % 4) * 32);
      const uint64_t bd = b_mn ? desc_mnmajor(b0 + s * 2048, 8192)
                               : desc_kmajor(b0 + (s / 4) * 8192 + (s % 4) * 32);
      mma_bf16(tbase, ad, bd, idesc, s > 0);
    }
    mma_commit(&bar);
  }
  const bool ok = mbar_wait(&bar, 0);
  tc_fence_after();
  if (!ok) {
    if (t == 0) atomicExch(status, 1);
  } else {
    for (int c = 0; c < 64; c += 32) {
      float r[32];
      tmem_ld32(tbase + ((warp * 32u) << 16) + c, r);
      tmem_ld_wait();
#pragma unroll
      for (int j = 0; j < 32; ++j) D[t * 64 + c + j] = r[j];
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tbase, 64);
}

// A from TMEM (written by tcgen05.st, row m in lane m, bf16 pairs per column), B
// K-major from shared memory: D[128 x N] = A[128 x 128] B[128 x N], N = 128.
__global__ void __launch_bounds__(128) umma_ts_selftest_kernel(const __nv_bfloat16* A,
                                                               const __nv_bfloat16* B, float* D,
                                                               int* status) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = align_smem<1024>(smem_raw);
  uint8_t* sB = smem;  // 2 k-halves x 128 rows (n) x 128 B = 32 KB
  __shared__ uint64_t bar;
  __shared__ uint32_t tmem_base;
  const int t = threadIdx.x;
  const int warp = t >> 5;
  for (int idx = t; idx < 128 * 128; idx += 128) {
    const int k = idx / 128, n = idx % 128;  // B given as [k][n] row-major
    *reinterpret_cast<__nv_bfloat16*>(sB + (k / 64) * 16384 + sw128_offset(n, k % 64)) = B[idx];
  }
  if (t == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
  }
  if (warp == 0) tmem_alloc(&tmem_base, 256);
  fence_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = tmem_base;
  const uint32_t lane_addr = tbase + ((warp * 32u) << 16);
  // A row t -> columns [128, 192) of lane t: 64 words of two bf16
  for (int c0 = 0; c0 < 64; c0 += 32) {
    float w[32];
    for (int j = 0; j < 32; ++j) {
      const int c = c0 + j;
      const uint32_t lo = __bfloat16_as_ushort(A[t * 128 + 2 * c]);
      const uint32_t hi = __bfloat16_as_ushort(A[t * 128 + 2 * c + 1]);
      w[j] = __uint_as_float(lo | (hi << 16));
    }
    tmem_st32(lane_addr + 128 + c0, w);
  }
  tmem_st_wait();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (t == 0) {
    const uint32_t idesc = idesc_bf16(128, 128, false, false);
    for (int s = 0; s < 8; ++s)
      mma_bf16_ts(tbase, tbase + 128 + s * 8,
                  desc_kmajor(smem_u32(sB) + (s / 4) * 16384 + (s % 4) * 32), idesc, s > 0);
    mma_commit(&bar);
  }
  const bool ok = mbar_wait(&bar, 0);
  tc_fence_after();
  if (!ok) {
    if (t == 0) atomicExch(status, 1);
  } else {
    for (int c = 0; c < 128; c += 32) {
      float r[32];
      tmem_ld32(lane_addr + c, r);
      tmem_ld_wait();
      for (int j = 0; j < 32; ++j) D[t * 128 + c + j] = r[j];
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tbase, 256);
}

}  // namespace
}  // namespace gdn

extern "C" int gdn_selftest_umma_ts(const void* A, const void* B, float* D, int* status,
                                    void* stream) {
  if (!A || !B || !D || !status) return GDN_ERR_INVALID_ARG;
  const int smem = 32768 + 1024;
  if (cudaFuncSetAttribute(gdn::umma_ts_selftest_kernel,
                           cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
    return GDN_ERR_CUDA;
  gdn::umma_ts_selftest_kernel<<<1, 128, smem, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(A), static_cast<const __nv_bfloat16*>(B), D, status);
  return cudaGetLastError() == cudaSuccess ? GDN_OK : GDN_ERR_CUDA;
}

extern "C" int gdn_selftest_umma(const void* A, const void* B, float* D, int a_mn_major,
                                 int b_mn_major, int* status, void* stream) {
  if (!A || !B || !D || !status) return GDN_ERR_INVALID_ARG;
  const int smem = 32768 + 16384 + 1024;
  if (cudaFuncSetAttribute(gdn::umma_selftest_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           smem) != cudaSuccess)
    return GDN_ERR_CUDA;
  gdn::umma_selftest_kernel<<<1, 128, smem, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(A), static_cast<const __nv_bfloat16*>(B), D, a_mn_major,
      b_mn_major, status);
  return cudaGetLastError() == cudaSuccess ? GDN_OK : GDN_ERR_CUDA;
}

namespace gdn {
namespace {

// Waits on an mbarrier phase that nothing completes: the bounded wait must give up
// (after about a second) and the kernel must report it instead of hanging.
__global__ void wait_timeout_kernel(int* status, long long* waited_ns) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) {
    sm100::mbar_init(&bar, 1);
    sm100::fence_mbar_init();
  }
  __syncthreads();
  const uint64_t t0 = sm100::globaltimer_ns();
  const bool ok = sm100::mbar_wait(&bar, 0);
  const uint64_t t1 = sm100::globaltimer_ns();
  if (threadIdx.x == 0) {
    *status = ok ? 0 : 1;
    *waited_ns = static_cast<long long>(t1 - t0);
  }
}

}  // namespace
}  // namespace gdn

extern "C" int gdn_selftest_wait_timeout(int* status, long long* waited_ns, void* stream) {
  if (!status || !waited_ns) return GDN_ERR_INVALID_ARG;
  gdn::wait_timeout_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(status, waited_ns);
  return cudaGetLastError() == cudaSuccess ? GDN_OK : GDN_ERR_CUDA;
}
