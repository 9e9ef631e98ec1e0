// gdn_chunk_common.cuh — pieces shared by the chunk-64 prefill kernels
// (the fused single-kernel path in gdn_prefill_chunked.cu and the two-phase
// prep/scan path in gdn_prefill_twophase.cu): operand helpers, the gate scan,
// the construction of A and [I; M], the blocked triangular solve and the
// TMA tensor maps of q/k. The algebra is described in gdn_prefill_chunked.cu.
#pragma once

#include <cuda.h>

#include "gdn_common.cuh"
#include "sm100_umma.cuh"

namespace gdn {
namespace chunk {

using namespace sm100;

constexpr int kC = 64;        // chunk length
constexpr int kVT = 64;       // V columns per state tile
constexpr int kTiles = kHeadDim / kVT;
constexpr float kLog2e = 1.4426950408889634f;

// fp32 64 x 64 matrices with the 16-byte column groups XOR-swizzled by row, so
// that row-per-thread float4 writes and column reads are free of bank conflicts.
__device__ __forceinline__ int fidx(int r, int c) {
  return r * 64 + ((((c >> 2) ^ r) & 15) << 2) + (c & 3);
}

constexpr uint32_t ID_KK = idesc_bf16(128, 64, false, false);  // A K-major, B K-major
constexpr uint32_t ID_KM = idesc_bf16(128, 64, false, true);   // A K-major, B MN-major
constexpr uint32_t ID_MM = idesc_bf16(128, 64, true, true);    // A MN-major, B MN-major

// Split 64 fp32 values into bf16 hi/lo and write them as row `row` of two
// 128B-swizzled tiles (8 chunks of 16 bytes each).
__device__ __forceinline__ void store_row_split(uint8_t* hi, uint8_t* lo, uint32_t row,
                                                const float* v) {
#pragma unroll
  for (int c = 0; c < 8; ++c) {
    uint32_t h[4], l[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      __nv_bfloat16 h0, l0, h1, l1;
      split_bf16(v[c * 8 + 2 * e], h0, l0);
      split_bf16(v[c * 8 + 2 * e + 1], h1, l1);
      h[e] = pack_bf16(h0, h1);
      l[e] = pack_bf16(l0, l1);
    }
    const uint32_t off = sw128_chunk(row, c);
    *reinterpret_cast<uint4*>(hi + off) = make_uint4(h[0], h[1], h[2], h[3]);
    *reinterpret_cast<uint4*>(lo + off) = make_uint4(l[0], l[1], l[2], l[3]);
  }
}

__device__ __forceinline__ void tmem_ld64(uint32_t taddr, float* out) {
  float a[32], b[32];
  tmem_ld32(taddr, a);
  tmem_ld32(taddr + 32, b);
  tmem_ld_wait();
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    out[i] = a[i];
    out[32 + i] = b[i];
  }
}

__device__ __forceinline__ void tmem_st64(uint32_t taddr, const float* in) {
  float a[32], b[32];
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    a[i] = in[i];
    b[i] = in[32 + i];
  }
  tmem_st32(taddr, a);
  tmem_st32(taddr + 32, b);
  tmem_st_wait();
}

// Make this thread's shared-memory operand writes and TMEM accesses visible to
// the MMA issued after the block-wide barrier.
__device__ __forceinline__ void sync_before_mma() {
  fence_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
}

// Issue `ksteps` MMAs of the three-term split product (hi*hi + hi*lo + lo*hi)
// or of a plain product when a_lo == 0 and b_lo == 0 (exact bf16 operands).
struct Operand {
  uint32_t hi, lo;   // shared addresses of the two halves (lo == 0: exact, no second half)
  bool mn;           // MN-major
  uint32_t lbo;      // MN-major: byte distance of 64-wide MN blocks
  uint32_t kstep;    // byte advance per 16-element K step
  uint32_t khalf;    // K-major operands spanning 2 swizzle atoms: byte distance of the atoms
};

__device__ __forceinline__ uint64_t op_desc(const Operand& o, uint32_t base, int s) {
  if (o.mn) return desc_mnmajor(base + s * o.kstep, o.lbo);
  return desc_kmajor(base + (s >> 2) * o.khalf + (s & 3) * 32);
}

__device__ __forceinline__ void issue_gemm(uint32_t d, const Operand& a, const Operand& b,
                                           uint32_t idesc, int ksteps) {
  int n = 0;
  for (int s = 0; s < ksteps; ++s) mma_bf16(d, op_desc(a, a.hi, s), op_desc(b, b.hi, s), idesc, n++ > 0);
  if (b.lo)
    for (int s = 0; s < ksteps; ++s) mma_bf16(d, op_desc(a, a.hi, s), op_desc(b, b.lo, s), idesc, 1);
  if (a.lo)
    for (int s = 0; s < ksteps; ++s) mma_bf16(d, op_desc(a, a.lo, s), op_desc(b, b.hi, s), idesc, 1);
}

// Gates of the chunk's tokens (threads 0..63 hold the raw a, b of token t) and the
// inclusive in-chunk cumulative log decay, in log2 units: sG[t] = Gamma_t * log2(e),
// sBeta[t] = beta_t; padded tokens (t >= L) get log g = 0 and beta = 0. Block-wide.
__device__ __forceinline__ void chunk_gates(float ra, float rb, int L, float A_log, float dtb,
                                            float* sG, float* sBeta) {
  const int t = threadIdx.x, lane = t & 31;
  // ---- gates and in-chunk cumulative log decay (log2 units) ----------------------
  if (t < kC) {
    const bool valid = t < L;
    const float lg = valid ? gate_log_decay(A_log, ra, dtb) * kLog2e : 0.0f;
    const float beta = valid ? gate_beta(rb) : 0.0f;
    float x = lg;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
    sG[t] = x;  // warp 1 adds warp 0's total below
    sBeta[t] = beta;
  }
  __syncthreads();
  if (t >= 32 && t < kC) sG[t] += sG[31];
  __syncthreads();

}

// From S = [K;Q] K^T in TMEM (this thread's lane): thread t < 64 writes row t of
// A = strict_lower(beta_i e^{Gamma_i-Gamma_j} S_kk) (fp32, for the solve) and the
// identity row t of [I; M]; thread t >= 64 writes row t of [I; M] with
// M = lower(e^{Gamma_i-Gamma_j} S_qk), as bf16 hi/lo K-major rows.
__device__ __forceinline__ void build_a_m(uint32_t ts_row, float* sAf, const float* sG,
                                          const float* sBeta, uint8_t* a2_hi, uint8_t* a2_lo) {
  const int t = threadIdx.x;
  {
    float srow[64];
    tmem_ld64(ts_row, srow);
    if (t < kC) {
      // A row i = t (fp32, for the solve); identity row of [I; M]
      const float gi = sG[t], bi = sBeta[t];
#pragma unroll
      for (int j = 0; j < kC; j += 4) {
        float4 w;
        w.x = (j + 0 < t) ? bi * ex2(gi - sG[j + 0]) * srow[j + 0] : 0.f;
        w.y = (j + 1 < t) ? bi * ex2(gi - sG[j + 1]) * srow[j + 1] : 0.f;
        w.z = (j + 2 < t) ? bi * ex2(gi - sG[j + 2]) * srow[j + 2] : 0.f;
        w.w = (j + 3 < t) ? bi * ex2(gi - sG[j + 3]) * srow[j + 3] : 0.f;
        *reinterpret_cast<float4*>(sAf + fidx(t, j)) = w;
      }
#pragma unroll
      for (int j = 0; j < kC; ++j) srow[j] = (j == t) ? 1.0f : 0.0f;
      store_row_split(a2_hi, a2_lo, t, srow);
    } else {
      // M row i = t - 64
      const int i = t - kC;
      const float gi = sG[i];
#pragma unroll
      for (int j = 0; j < kC; ++j) srow[j] = (j <= i) ? ex2(gi - sG[j]) * srow[j] : 0.f;
      store_row_split(a2_hi, a2_lo, t, srow);
    }
  }
}

// T_b = (I + A)^-1 diag(beta), written as the MN-major bf16 hi/lo B operand (rows j,
// cols n). A: strictly lower 64 x 64 fp32 in sAf (fidx layout); sTf receives T, its
// upper blocks serve as scratch. Block-wide: every thread of the 128 calls it.
__device__ __forceinline__ void solve_tb(float* sAf, float* sTf, const float* sBeta,
                                         uint8_t* tb_hi, uint8_t* tb_lo) {
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  // ---- T = (I + A)^-1, blocked 16 x 16 ---------------------------------------------
  if (lane < 16) {
    const int b0 = warp * 16;
    float tc[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      float s = 0.f;
#pragma unroll
      for (int j = 0; j < i; ++j) s = fmaf(sAf[fidx(b0 + i, b0 + j)], tc[j], s);
      tc[i] = (i < lane) ? 0.f : ((i == lane) ? 1.f : -s);
    }
#pragma unroll
    for (int i = 0; i < 16; ++i) sTf[fidx(b0 + i, b0 + lane)] = tc[i];
  }
  __syncthreads();
  // Off-diagonal blocks by distance d = I - J: one warp per block, each lane
  // owns row r = lane/2 and 8 columns c0 = 8*(lane&1) of the 16 x 16 block.
  {
    const int r = lane >> 1, c0 = (lane & 1) * 8;
    for (int d = 1; d < 4; ++d) {
      const int I = d + warp, J = warp;
      float w[8];
      if (warp < 4 - d) {  // W_IJ = sum_{K=J}^{I-1} A_IK T_KJ  -> scratch block (J, I)
#pragma unroll
        for (int e = 0; e < 8; ++e) w[e] = 0.f;
        for (int K = J; K < I; ++K) {
#pragma unroll
          for (int k = 0; k < 16; ++k) {
            const float a = sAf[fidx(16 * I + r, 16 * K + k)];
            const float4 t0 = *reinterpret_cast<const float4*>(sTf + fidx(16 * K + k, 16 * J + c0));
            const float4 t1 = *reinterpret_cast<const float4*>(sTf + fidx(16 * K + k, 16 * J + c0 + 4));
            w[0] = fmaf(a, t0.x, w[0]); w[1] = fmaf(a, t0.y, w[1]);
            w[2] = fmaf(a, t0.z, w[2]); w[3] = fmaf(a, t0.w, w[3]);
            w[4] = fmaf(a, t1.x, w[4]); w[5] = fmaf(a, t1.y, w[5]);
            w[6] = fmaf(a, t1.z, w[6]); w[7] = fmaf(a, t1.w, w[7]);
          }
        }
        *reinterpret_cast<float4*>(sTf + fidx(16 * J + r, 16 * I + c0)) =
            make_float4(w[0], w[1], w[2], w[3]);
        *reinterpret_cast<float4*>(sTf + fidx(16 * J + r, 16 * I + c0 + 4)) =
            make_float4(w[4], w[5], w[6], w[7]);
      }
      __syncwarp();
      if (warp < 4 - d) {  // T_IJ = -T_II W_IJ (W read back from the scratch block)
#pragma unroll
        for (int e = 0; e < 8; ++e) w[e] = 0.f;
#pragma unroll
        for (int k = 0; k < 16; ++k) {
          const float a = sTf[fidx(16 * I + r, 16 * I + k)];
          const float4 t0 = *reinterpret_cast<const float4*>(sTf + fidx(16 * J + k, 16 * I + c0));
          const float4 t1 = *reinterpret_cast<const float4*>(sTf + fidx(16 * J + k, 16 * I + c0 + 4));
          w[0] = fmaf(a, t0.x, w[0]); w[1] = fmaf(a, t0.y, w[1]);
          w[2] = fmaf(a, t0.z, w[2]); w[3] = fmaf(a, t0.w, w[3]);
          w[4] = fmaf(a, t1.x, w[4]); w[5] = fmaf(a, t1.y, w[5]);
          w[6] = fmaf(a, t1.z, w[6]); w[7] = fmaf(a, t1.w, w[7]);
        }
        *reinterpret_cast<float4*>(sTf + fidx(16 * I + r, 16 * J + c0)) =
            make_float4(-w[0], -w[1], -w[2], -w[3]);
        *reinterpret_cast<float4*>(sTf + fidx(16 * I + r, 16 * J + c0 + 4)) =
            make_float4(-w[4], -w[5], -w[6], -w[7]);
      }
      __syncthreads();
    }
  }
  {
    // T_b = T diag(beta) as the MN-major B operand: row j, cols n (half of the row per
    // thread); written over A, which the solve no longer needs
    const int j = t & (kC - 1), half = t >> 6;
    float vals[32];
#pragma unroll
    for (int c = 0; c < 32; ++c) {
      const int nn = half * 32 + c;
      const bool lower = (nn >> 4) < (j >> 4) || ((nn >> 4) == (j >> 4) && nn <= j);
      vals[c] = lower ? sTf[fidx(j, nn)] * sBeta[nn] : 0.f;
    }
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      uint32_t hw[4], lw[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        __nv_bfloat16 h0, l0, h1, l1;
        split_bf16(vals[c * 8 + 2 * e], h0, l0);
        split_bf16(vals[c * 8 + 2 * e + 1], h1, l1);
        hw[e] = pack_bf16(h0, h1);
        lw[e] = pack_bf16(l0, l1);
      }
      const uint32_t off = sw128_chunk(j, half * 4 + c);
      *reinterpret_cast<uint4*>(tb_hi + off) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
      *reinterpret_cast<uint4*>(tb_lo + off) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
    }
  }

}

struct ChunkTmaps {
  CUtensorMap k;  // [T, HQ, 128] bf16: dims {128, HQ, T}, box {64, 1, 64}, 128B swizzle
  CUtensorMap q;
};

// ------------------------------------------------------------------ host side
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiledFn get_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  }
  return fn;
}

inline bool encode_qk_map(CUtensorMap* map, const void* base, int64_t T, int HQ) {
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) return false;
  const cuuint64_t dims[3] = {static_cast<cuuint64_t>(kHeadDim), static_cast<cuuint64_t>(HQ),
                              static_cast<cuuint64_t>(T)};
  const cuuint64_t strides[2] = {static_cast<cuuint64_t>(kHeadDim) * 2,
                                 static_cast<cuuint64_t>(HQ) * kHeadDim * 2};
  const cuuint32_t box[3] = {64, 1, kC};
  const cuuint32_t estr[3] = {1, 1, 1};
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides,
             box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) ==
         CUDA_SUCCESS;
}


}  // namespace chunk
}  // namespace gdn
