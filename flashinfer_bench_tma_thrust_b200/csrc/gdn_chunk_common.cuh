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

// Layouts of the fp32 64 x 64 solve matrices. SwzLayout: stride 64 with the 16-byte
// column groups XOR-swizzled by row (16 KB, for kernels short of shared memory).
// PadLayout: stride 68 (17 KB): addresses are affine in the column, so unrolled loops
// fold them into immediates, and row-per-thread float4 writes stay conflict-free.
struct SwzLayout {
  static __device__ __forceinline__ int idx(int r, int c) { return fidx(r, c); }
};
struct PadLayout {
  static __device__ __forceinline__ int idx(int r, int c) { return r * 68 + c; }
};


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
      split2(v[c * 8 + 2 * e], v[c * 8 + 2 * e + 1], h[e], l[e]);
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
// Called by all lanes of one warp (warp-level MMA issue; see mma_bf16_w).
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

// Byte offset of K step s from step 0 (added to the start-address field, which
// holds address >> 4 in its low 14 bits; shared addresses stay below 256 KB).
__device__ __forceinline__ uint64_t op_step(const Operand& o, int s) {
  const uint32_t off = o.mn ? s * o.kstep : (s >> 2) * o.khalf + (s & 3) * 32;
  return static_cast<uint64_t>(off >> 4);
}

__device__ __forceinline__ void issue_gemm(uint32_t d, const Operand& a, const Operand& b,
                                           uint32_t idesc, int ksteps) {
  const uint64_t ah = op_desc(a, a.hi, 0), bh = op_desc(b, b.hi, 0);
  const uint64_t al = a.lo ? op_desc(a, a.lo, 0) : 0, bl = b.lo ? op_desc(b, b.lo, 0) : 0;
#pragma unroll
  for (int s = 0; s < ksteps; ++s) mma_bf16_w(d, ah + op_step(a, s), bh + op_step(b, s), idesc, s > 0);
  if (b.lo) {
#pragma unroll
    for (int s = 0; s < ksteps; ++s) mma_bf16_w(d, ah + op_step(a, s), bl + op_step(b, s), idesc, 1);
  }
  if (a.lo) {
#pragma unroll
    for (int s = 0; s < ksteps; ++s) mma_bf16_w(d, al + op_step(a, s), bh + op_step(b, s), idesc, 1);
  }
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

__device__ __forceinline__ void named_bar_sync(uint32_t id, uint32_t nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}


// From S = [K;Q] K^T in TMEM (this thread's lane): thread t < 64 writes row t of
// A = strict_lower(beta_i e^{Gamma_i-Gamma_j} S_kk) (fp32, for the solve) and the
// identity row t of [I; M]; thread t >= 64 writes row t of [I; M] with
// M = lower(e^{Gamma_i-Gamma_j} S_qk), as bf16 hi/lo K-major rows.
template <class Lay>
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
        *reinterpret_cast<float4*>(sAf + Lay::idx(t, j)) = w;
      }
      // identity row: one nonzero bf16 (1.0 = 0x3f80) in chunk t/8; lo half is zero
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        uint32_t w[4] = {0u, 0u, 0u, 0u};
        if (c == (t >> 3)) w[(t & 7) >> 1] = (t & 1) ? 0x3f800000u : 0x00003f80u;
        const uint32_t off = sw128_chunk(t, c);
        *reinterpret_cast<uint4*>(a2_hi + off) = make_uint4(w[0], w[1], w[2], w[3]);
        *reinterpret_cast<uint4*>(a2_lo + off) = make_uint4(0u, 0u, 0u, 0u);
      }
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

// One warp: W = A_{I,K} T_{K,J} (16 x 16 x 16) stored into the scratch block at
// block coordinates (sr, sc). Lane owns row lane/2 and 8 columns.
template <class Lay>
__device__ __forceinline__ void solve_partial(const float* sAf, float* sTf, int I, int K, int J,
                                              int sr, int sc, int lane) {
  const int r = lane >> 1, c0 = (lane & 1) * 8;
  float w[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) w[e] = 0.f;
#pragma unroll
  for (int k = 0; k < 16; ++k) {
    const float a = sAf[Lay::idx(16 * I + r, 16 * K + k)];
    const float4 t0 = *reinterpret_cast<const float4*>(sTf + Lay::idx(16 * K + k, 16 * J + c0));
    const float4 t1 =
        *reinterpret_cast<const float4*>(sTf + Lay::idx(16 * K + k, 16 * J + c0 + 4));
    w[0] = fmaf(a, t0.x, w[0]); w[1] = fmaf(a, t0.y, w[1]);
    w[2] = fmaf(a, t0.z, w[2]); w[3] = fmaf(a, t0.w, w[3]);
    w[4] = fmaf(a, t1.x, w[4]); w[5] = fmaf(a, t1.y, w[5]);
    w[6] = fmaf(a, t1.z, w[6]); w[7] = fmaf(a, t1.w, w[7]);
  }
  *reinterpret_cast<float4*>(sTf + Lay::idx(16 * sr + r, 16 * sc + c0)) =
      make_float4(w[0], w[1], w[2], w[3]);
  *reinterpret_cast<float4*>(sTf + Lay::idx(16 * sr + r, 16 * sc + c0 + 4)) =
      make_float4(w[4], w[5], w[6], w[7]);
}

// T_IJ = -T_II (sum of NP scratch blocks), computed by a group of G threads (g = rank
// in the group): each owns 256/G outputs of one row.
template <class Lay, int NP, int G>
__device__ __forceinline__ void solve_finish(float* sTf, int I, int J, int sr0, int sc0, int sr1,
                                             int sc1, int sr2, int sc2, int g) {
  constexpr int kCols = 256 / G;  // 8, 4 or 2 columns per thread
  constexpr int kPerRow = 16 / kCols;
  const int r = g / kPerRow, c0 = (g % kPerRow) * kCols;
  float w[kCols];
#pragma unroll
  for (int e = 0; e < kCols; ++e) w[e] = 0.f;
#pragma unroll
  for (int k = 0; k < 16; ++k) {
    const float a = sTf[Lay::idx(16 * I + r, 16 * I + k)];
#pragma unroll
    for (int e = 0; e < kCols; ++e) {
      w[e] = fmaf(a, sTf[Lay::idx(16 * sr0 + k, 16 * sc0 + c0 + e)], w[e]);
      if (NP > 1) w[e] = fmaf(a, sTf[Lay::idx(16 * sr1 + k, 16 * sc1 + c0 + e)], w[e]);
      if (NP > 2) w[e] = fmaf(a, sTf[Lay::idx(16 * sr2 + k, 16 * sc2 + c0 + e)], w[e]);
    }
  }
#pragma unroll
  for (int e = 0; e < kCols; ++e) sTf[Lay::idx(16 * I + r, 16 * J + c0 + e)] = -w[e];
}

// T_b = (I + A)^-1 diag(beta), written as the MN-major bf16 hi/lo B operand (rows j,
// cols n). A: strictly lower 64 x 64 fp32 in sAf; sTf receives T, its upper blocks
// serve as scratch for the partial products. Blocked by 16: the four diagonal blocks
// by forward substitution (one warp each), then the off-diagonal blocks by distance,
// T_IJ = -T_II sum_{K=J}^{I-1} A_IK T_KJ, with the partial products of one block
// spread over warps. Block-wide: all 128 threads call it.
template <class Lay>
__device__ __forceinline__ void solve_tb(float* sAf, float* sTf, const float* sBeta,
                                         uint8_t* tb_hi, uint8_t* tb_lo) {
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  if (lane < 16) {
    const int b0 = warp * 16;
    float tc[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      float s = 0.f;
#pragma unroll
      for (int j = 0; j < i; ++j) s = fmaf(sAf[Lay::idx(b0 + i, b0 + j)], tc[j], s);
      tc[i] = (i < lane) ? 0.f : ((i == lane) ? 1.f : -s);
    }
#pragma unroll
    for (int i = 0; i < 16; ++i) sTf[Lay::idx(b0 + i, b0 + lane)] = tc[i];
  }
  __syncthreads();
  // distance 1: blocks (1,0), (2,1), (3,2), one warp each; scratch (J, I)
  if (warp < 3) {
    const int I = warp + 1, J = warp;
    solve_partial<Lay>(sAf, sTf, I, J, J, J, I, lane);
    __syncwarp();
    solve_finish<Lay, 1, 32>(sTf, I, J, J, I, 0, 0, 0, 0, lane);
  }
  __syncthreads();
  // distance 2: blocks (2,0) [warps 0,1] and (3,1) [warps 2,3]; one partial per warp
  {
    const int b = warp >> 1, I = 2 + b, J = b, K = J + (warp & 1);
    // scratch: (J, I) for K = J, (J, J+1) for K = J+1 (free since distance 1 finished)
    solve_partial<Lay>(sAf, sTf, I, K, J, J, (warp & 1) ? J + 1 : I, lane);
  }
  __syncthreads();
  {
    const int b = warp >> 1, I = 2 + b, J = b;
    solve_finish<Lay, 2, 64>(sTf, I, J, J, I, J, J + 1, 0, 0, t & 63);
  }
  __syncthreads();
  // distance 3: block (3,0); partials K = 0, 1, 2 on warps 0..2 into (0,3), (0,1), (0,2)
  if (warp < 3) solve_partial<Lay>(sAf, sTf, 3, warp, 0, 0, warp == 0 ? 3 : warp, lane);
  __syncthreads();
  {
    solve_finish<Lay, 3, 128>(sTf, 3, 0, 0, 3, 0, 1, 0, 2, t);
  }
  __syncthreads();
  {
    // T_b = T diag(beta) as the MN-major B operand: row j, cols n (half of the row per
    // thread)
    const int j = t & (kC - 1), half = t >> 6;
    float vals[32];
#pragma unroll
    for (int c = 0; c < 32; ++c) {
      const int nn = half * 32 + c;
      const bool lower = (nn >> 4) < (j >> 4) || ((nn >> 4) == (j >> 4) && nn <= j);
      vals[c] = lower ? sTf[Lay::idx(j, nn)] * sBeta[nn] : 0.f;
    }
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      uint32_t hw[4], lw[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        split2(vals[c * 8 + 2 * e], vals[c * 8 + 2 * e + 1], hw[e], lw[e]);
      }
      const uint32_t off = sw128_chunk(j, half * 4 + c);
      *reinterpret_cast<uint4*>(tb_hi + off) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
      *reinterpret_cast<uint4*>(tb_lo + off) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
    }
  }
}


// ------------------------------------------------------------ 256-thread variants
// Thread t owns row r = t % 128 (its TMEM lane) and the 32 columns [32c, 32c+32)
// of it, c = t / 128.

// From S = [K;Q] K^T in TMEM (ts_row already points at this thread's lane and column
// half): rows r < 64 write A row r (fp32) into sAf; rows r >= 64 write row r - 64 of M
// as bf16 hi/lo K-major rows of the m_hi / m_lo tiles.
template <class Lay>
__device__ __forceinline__ void build_a_m_256(uint32_t ts_row, float* sAf, const float* sG,
                                              const float* sBeta, uint8_t* m_hi, uint8_t* m_lo) {
  const int t = threadIdx.x, r = t & 127, c0 = (t >> 7) * 32;
  // where this warp's 32 x 32 quarter lies against the diagonal (warp-uniform): its
  // row block rb and column block cb within A or M
  const int rb = (r & 63) >> 5, cb = t >> 7;
  if (r < kC) {
    if (cb > rb) return;  // above the diagonal: the solve reads only A's strict lower part
    float srow[32];
    tmem_ld32(ts_row, srow);
    tmem_ld_wait();
    const float gi = sG[r], bi = sBeta[r];
#pragma unroll
    for (int j = 0; j < 32; j += 4) {
      float4 w;
      const int jj = c0 + j;
      const float4 g = *reinterpret_cast<const float4*>(sG + jj);
      // unmasked: the solve reads only the strict lower triangle of A
      w.x = bi * ex2(gi - g.x) * srow[j + 0];
      w.y = bi * ex2(gi - g.y) * srow[j + 1];
      w.z = bi * ex2(gi - g.z) * srow[j + 2];
      w.w = bi * ex2(gi - g.w) * srow[j + 3];
      *reinterpret_cast<float4*>(sAf + Lay::idx(r, jj)) = w;
    }
  } else {
    const int i = r - kC;
    if (cb > rb) {  // above the diagonal: M is zero there
      const uint4 z = make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const uint32_t off = sw128_chunk(i, (c0 >> 3) + c);
        *reinterpret_cast<uint4*>(m_hi + off) = z;
        *reinterpret_cast<uint4*>(m_lo + off) = z;
      }
      return;
    }
    float srow[32];
    tmem_ld32(ts_row, srow);
    tmem_ld_wait();
    const float gi = sG[i];
    if (cb < rb) {  // below the diagonal: no mask
#pragma unroll
      for (int j = 0; j < 32; j += 4) {
        const float4 g = *reinterpret_cast<const float4*>(sG + c0 + j);
        srow[j] = ex2(gi - g.x) * srow[j];
        srow[j + 1] = ex2(gi - g.y) * srow[j + 1];
        srow[j + 2] = ex2(gi - g.z) * srow[j + 2];
        srow[j + 3] = ex2(gi - g.w) * srow[j + 3];
      }
    } else {
#pragma unroll
      for (int j = 0; j < 32; j += 4) {
        const float4 g = *reinterpret_cast<const float4*>(sG + c0 + j);
        srow[j] = (c0 + j <= i) ? ex2(gi - g.x) * srow[j] : 0.f;
        srow[j + 1] = (c0 + j + 1 <= i) ? ex2(gi - g.y) * srow[j + 1] : 0.f;
        srow[j + 2] = (c0 + j + 2 <= i) ? ex2(gi - g.z) * srow[j + 2] : 0.f;
        srow[j + 3] = (c0 + j + 3 <= i) ? ex2(gi - g.w) * srow[j + 3] : 0.f;
      }
    }
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      uint32_t hw[4], lw[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) split2(srow[c * 8 + 2 * e], srow[c * 8 + 2 * e + 1], hw[e], lw[e]);
      const uint32_t off = sw128_chunk(i, (c0 >> 3) + c);
      *reinterpret_cast<uint4*>(m_hi + off) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
      *reinterpret_cast<uint4*>(m_lo + off) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
    }
  }
}

// solve_tb for 256 threads (8 warps): the 16 x 16 diagonal blocks by right-looking
// substitution (each step's updates are independent), then the off-diagonal blocks
// in two levels of the block-diagonal inverse formula (16 -> 32, 32 -> 64), each
// spread over all 8 warps so that the dependent chain is short.
template <class Lay>
__device__ __forceinline__ void solve_tb_256(float* sAf, float* sTf, const float* sBeta,
                                             uint8_t* tb_hi, uint8_t* tb_lo) {
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  if (warp < 2) {
    // column `lane % 16` of the inverse of the unit lower block b0 (each half-warp one
    // block): x_i = d_i - sum_{j<i} A_ij x_j, right-looking two columns per step so
    // that A_{i,j}, A_{i,j+1} come as one broadcast 64-bit load (same order of updates
    // per x_i as one column per step)
    const int b0 = (2 * warp + (lane >> 4)) * 16, l = lane & 15;
    float x[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) x[i] = (i == l) ? 1.f : 0.f;
#pragma unroll
    for (int j = 0; j < 16; j += 2) {
      x[j + 1] = fmaf(-sAf[Lay::idx(b0 + j + 1, b0 + j)], x[j], x[j + 1]);
#pragma unroll
      for (int i = j + 2; i < 16; ++i) {
        const float2 a = *reinterpret_cast<const float2*>(sAf + Lay::idx(b0 + i, b0 + j));
        x[i] = fmaf(-a.x, x[j], x[i]);
        x[i] = fmaf(-a.y, x[j + 1], x[i]);
      }
    }
#pragma unroll
    for (int i = 0; i < 16; ++i) sTf[Lay::idx(b0 + i, b0 + l)] = x[i];
  } else if (warp >= 4 && warp < 6) {
    // block (0, 1) of T must read as zero in the level-2 product below
    const int q = t - 128, row = q >> 2, col = 16 + (q & 3) * 4;
    *reinterpret_cast<float4*>(sTf + Lay::idx(row, col)) = make_float4(0.f, 0.f, 0.f, 0.f);
  }
  __syncthreads();
  // Two levels, every warp busy at each (T_IJ = -T_II A_IJ T_JJ for the lower blocks
  // of a block-diagonal inverse). Lanes own columns: the left operand of a k-quad comes
  // as one broadcast float4 per row, the right operand as one conflict-free 32-bit load
  // per lane (a float4 per lane over eight addresses would cost four shared-memory
  // wavefronts for four products).
  // level 1, 16 -> 32: blocks (1,0) [warps 0-3] and (3,2) [warps 4-7]; rows r0, r0 + 1
  // and column c per thread; scratch W in block (0, 2 + g).
  {
    const int g = warp >> 2, r0 = 4 * (warp & 3) + 2 * (lane >> 4), c = lane & 15;
    const int I = 2 * g + 1, J = 2 * g;
    {
      // W = A_IJ T_JJ with warps over column quads (row = lane % 16, two columns per
      // lane): T_JJ is lower triangular, so the warp's k loop starts at its first column
      const int cq = 4 * (warp & 3), cw = cq + 2 * (lane >> 4), rw = lane & 15;
      float w0 = 0.f, w1 = 0.f;
#pragma unroll 1
      for (int k = cq; k < 16; k += 4) {
        const float4 a = *reinterpret_cast<const float4*>(sAf + Lay::idx(16 * I + rw, 16 * J + k));
        float2 tv[4];
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          tv[kk] = *reinterpret_cast<const float2*>(sTf + Lay::idx(16 * J + k + kk, 16 * J + cw));
        w0 = fmaf(a.x, tv[0].x, w0); w0 = fmaf(a.y, tv[1].x, w0);
        w0 = fmaf(a.z, tv[2].x, w0); w0 = fmaf(a.w, tv[3].x, w0);
        w1 = fmaf(a.x, tv[0].y, w1); w1 = fmaf(a.y, tv[1].y, w1);
        w1 = fmaf(a.z, tv[2].y, w1); w1 = fmaf(a.w, tv[3].y, w1);
      }
      *reinterpret_cast<float2*>(sTf + Lay::idx(rw, 32 + 16 * g + cw)) = make_float2(w0, w1);
    }
    named_bar_sync(2 + g, 128);
    // T_II is lower triangular: rows of this warp need k < 4 (warp % 4) + 4 only
    const int kmax = 4 * (warp & 3) + 4;
    float v0 = 0.f, v1 = 0.f;
#pragma unroll 1
    for (int k = 0; k < kmax; k += 4) {
      const float4 a0 = *reinterpret_cast<const float4*>(sTf + Lay::idx(16 * I + r0, 16 * I + k));
      const float4 a1 =
          *reinterpret_cast<const float4*>(sTf + Lay::idx(16 * I + r0 + 1, 16 * I + k));
      const float t0 = sTf[Lay::idx(k, 32 + 16 * g + c)];
      const float t1 = sTf[Lay::idx(k + 1, 32 + 16 * g + c)];
      const float t2 = sTf[Lay::idx(k + 2, 32 + 16 * g + c)];
      const float t3 = sTf[Lay::idx(k + 3, 32 + 16 * g + c)];
      v0 = fmaf(a0.x, t0, v0); v0 = fmaf(a0.y, t1, v0);
      v0 = fmaf(a0.z, t2, v0); v0 = fmaf(a0.w, t3, v0);
      v1 = fmaf(a1.x, t0, v1); v1 = fmaf(a1.y, t1, v1);
      v1 = fmaf(a1.z, t2, v1); v1 = fmaf(a1.w, t3, v1);
    }
    sTf[Lay::idx(16 * I + r0, 16 * J + c)] = -v0;
    sTf[Lay::idx(16 * I + r0 + 1, 16 * J + c)] = -v1;
  }
  __syncthreads();
  // level 2, 32 -> 64: block rows 32..63 x cols 0..31; warp w owns rows 4w..4w+3 and
  // lane = column; scratch W in rows 0..31 x cols 32..63 (the level-1 scratch is consumed)
  {
    const int r0 = 4 * warp, c = lane;
    {
      // W = A_21 T_11 with warp w over columns 4w..4w+3 and lane = row: T_11 is lower
      // triangular, so the warp's k loop starts at 4w
      const int cq = 4 * warp;
      float w[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 1
      for (int k = cq; k < 32; k += 4) {
        const float4 a = *reinterpret_cast<const float4*>(sAf + Lay::idx(32 + lane, k));
        float4 tv[4];
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          tv[kk] = *reinterpret_cast<const float4*>(sTf + Lay::idx(k + kk, cq));
        w[0] = fmaf(a.x, tv[0].x, w[0]); w[0] = fmaf(a.y, tv[1].x, w[0]);
        w[0] = fmaf(a.z, tv[2].x, w[0]); w[0] = fmaf(a.w, tv[3].x, w[0]);
        w[1] = fmaf(a.x, tv[0].y, w[1]); w[1] = fmaf(a.y, tv[1].y, w[1]);
        w[1] = fmaf(a.z, tv[2].y, w[1]); w[1] = fmaf(a.w, tv[3].y, w[1]);
        w[2] = fmaf(a.x, tv[0].z, w[2]); w[2] = fmaf(a.y, tv[1].z, w[2]);
        w[2] = fmaf(a.z, tv[2].z, w[2]); w[2] = fmaf(a.w, tv[3].z, w[2]);
        w[3] = fmaf(a.x, tv[0].w, w[3]); w[3] = fmaf(a.y, tv[1].w, w[3]);
        w[3] = fmaf(a.z, tv[2].w, w[3]); w[3] = fmaf(a.w, tv[3].w, w[3]);
      }
      *reinterpret_cast<float4*>(sTf + Lay::idx(lane, 32 + cq)) =
          make_float4(w[0], w[1], w[2], w[3]);
    }
    __syncthreads();
    // T_{[32,64)} is lower triangular: rows of warp w need k < 4w + 4
    const int kmax = r0 + 4;
    float v[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 1
    for (int k = 0; k < kmax; k += 4) {
      float wv[4];
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) wv[kk] = sTf[Lay::idx(k + kk, 32 + c)];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float4 a = *reinterpret_cast<const float4*>(sTf + Lay::idx(32 + r0 + i, 32 + k));
        v[i] = fmaf(a.x, wv[0], v[i]); v[i] = fmaf(a.y, wv[1], v[i]);
        v[i] = fmaf(a.z, wv[2], v[i]); v[i] = fmaf(a.w, wv[3], v[i]);
      }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) sTf[Lay::idx(32 + r0 + i, c)] = -v[i];
  }
  __syncthreads();
  {
    // T_b = T diag(beta), MN-major rows j x cols n: a quarter row (2 chunks) per thread.
    // Warp-uniform cases: the warp's 16 columns lie right of all its 32 rows (zero),
    // left of all of them (no mask), or across the diagonal (masked: T's upper triangle
    // holds scratch).
    const int j = t & (kC - 1), qq = t >> 6, jb = (t >> 5) & 1;
    if (16 * qq > 32 * jb + 31) {
      const uint4 z = make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        const uint32_t off = sw128_chunk(j, qq * 2 + c);
        *reinterpret_cast<uint4*>(tb_hi + off) = z;
        *reinterpret_cast<uint4*>(tb_lo + off) = z;
      }
    } else {
      const bool full = 16 * qq + 15 <= 32 * jb;
      float vals[16];
#pragma unroll
      for (int c = 0; c < 16; c += 4) {
        const int nn = qq * 16 + c;
        const float4 tv = *reinterpret_cast<const float4*>(sTf + Lay::idx(j, nn));
        const float4 bv = *reinterpret_cast<const float4*>(sBeta + nn);
        vals[c] = tv.x * bv.x;
        vals[c + 1] = tv.y * bv.y;
        vals[c + 2] = tv.z * bv.z;
        vals[c + 3] = tv.w * bv.w;
      }
      if (!full) {
#pragma unroll
        for (int c = 0; c < 16; ++c)
          if (qq * 16 + c > j) vals[c] = 0.f;
      }
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        uint32_t hw[4], lw[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) split2(vals[c * 8 + 2 * e], vals[c * 8 + 2 * e + 1], hw[e], lw[e]);
        const uint32_t off = sw128_chunk(j, qq * 2 + c);
        *reinterpret_cast<uint4*>(tb_hi + off) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
        *reinterpret_cast<uint4*>(tb_lo + off) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
      }
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
