// gdn_prefill_chunked.cu — chunk-64 varlen GDN prefill on the sm_100a tensor cores.
//
// Semantics: gdn/prefill/baseline/triton/kernel.py:18-100 (per-token recurrence,
// empty sequences pass their state through). Algorithm: the chunkwise
// (WY / UT-transform) form of the gated delta rule. Per (sequence, v-head) and
// chunk of 64 tokens, with H the k-first state [K=128, V] entering the chunk and
// Gamma the in-chunk cumulative log decay:
//
//   S     = [K; Q] K^T                                   (tensor cores, bf16 exact)
//   A     = strict_lower(beta_i e^{Gamma_i-Gamma_j} S_kk)  M = lower(e^{Gamma_i-Gamma_j} S_qk)
//   T_b   = (I + A)^-1 diag(beta)                        (blocked 16x16 solve, CUDA cores)
//   [T_b; P] = [I; M] T_b                                 (tensor cores)
//   [KH; QH] = [K; Q] H                                   (tensor cores)
//   X     = V - diag(gamma) KH
//   [U; O'] = [T_b; P] X                                  (tensor cores)
//   O     = scale (diag(gamma) QH + O')                   -> bf16 output
//   H    <- gamma_last H + K^T diag(f) U,  f_j = e^{Gamma_last-Gamma_j}     (tensor cores)
//
// One thread block (128 threads, one warpgroup) per (sequence, v-head, 64-wide
// V tile) walks the sequence chunk by chunk. The state tile H [128 x 64] stays
// in TMEM in fp32 for the whole sequence (TMEM lane = k). Operands that are not
// exact bf16 (H, T_b, P, X, U) enter the bf16 tensor core as hi + lo bf16
// pairs (hi*hi + hi*lo + lo*hi), which keeps about 16 significant bits; q, k and
// v are bf16 inputs and enter exactly. K and Q chunk tiles arrive by TMA
// (128B-swizzled, 3-D tensor maps over [token, head, dim]); the next chunk's
// tile is requested as soon as the state-update GEMM has consumed the current
// one. Shared memory is kept under 100 KB so that two blocks run per SM and
// each hides the other's MMA, TMA and barrier latency.
// Padded rows of a partial chunk carry beta = 0 and log g = 0, which makes
// their contribution to U, O and H exactly zero; their outputs are not stored.
#include <cuda.h>

#include "gdn_common.cuh"
#include "gdn_launch.h"
#include "sm100_umma.cuh"

namespace gdn {
namespace {

using namespace sm100;

constexpr int kC = 64;        // chunk length
constexpr int kVT = 64;       // V columns per thread block
constexpr int kTiles = kHeadDim / kVT;
constexpr float kLog2e = 1.4426950408889634f;

// Shared memory map (bytes from a 1024-aligned base), 97 KB so that two blocks
// share an SM. Regions are reused across the phases of a chunk:
//   KQ   [k half][K rows 0..63 | Q rows 64..127], K-major, filled by TMA. The Q
//        halves are dead once [KH; QH] is computed and then hold X (later U).
//   H    H hi/lo (MN-major B operand of [K;Q] H). Dead between that MMA and the
//        state update, so the fp32 solve matrices A and T live there, and T_b
//        (hi/lo) replaces A once the solve is done.
//   A2   [I; M] and then [T_b; P] hi/lo, K-major rows m (128) x cols j.
constexpr uint32_t OFF_KQ = 0;           // 32 KB
constexpr uint32_t OFF_X_HI = 8192;      // 8 KB (Q half 0): X then diag(f) U, MN-major rows j x cols v
constexpr uint32_t OFF_X_LO = 24576;     // 8 KB (Q half 1)
constexpr uint32_t OFF_H_HI = 32768;     // 16 KB: H, MN-major: rows k (128) x cols v (64)
constexpr uint32_t OFF_H_LO = 49152;
constexpr uint32_t OFF_AF = 32768;       // 64 x 64 fp32 A (swizzled columns), aliases H hi
constexpr uint32_t OFF_TF = 49152;       // 64 x 64 fp32 T (upper blocks: scratch), aliases H lo
constexpr uint32_t OFF_TB_HI = 32768;    // 8 KB: T_b, MN-major rows j x cols n (after the solve)
constexpr uint32_t OFF_TB_LO = 40960;
constexpr uint32_t OFF_A2_HI = 65536;    // 16 KB
constexpr uint32_t OFF_A2_LO = 81920;
constexpr uint32_t OFF_G = 98304;        // 64 fp32: Gamma * log2(e)
constexpr uint32_t OFF_BETA = 98560;     // 64 fp32: beta
constexpr uint32_t OFF_BAR = 98816;      // 2 mbarriers + TMEM base
constexpr uint32_t kSmemUsed = 98880;
constexpr uint32_t kSmemBytes = kSmemUsed + 1024;  // + alignment slack

// fp32 64 x 64 matrices with the 16-byte column groups XOR-swizzled by row, so
// that row-per-thread float4 writes and column reads are free of bank conflicts.
__device__ __forceinline__ int fidx(int r, int c) {
  return r * 64 + ((((c >> 2) ^ r) & 15) << 2) + (c & 3);
}

// TMEM columns (fp32, lane = row of M = 128)
constexpr uint32_t kTmemCols = 256;
constexpr uint32_t TM_H = 0;     // persistent state H (lane k, col v)
constexpr uint32_t TM_S = 64;    // S = [K;Q] K^T, then [T_b; P]
constexpr uint32_t TM_1 = 128;   // [KH; QH]
constexpr uint32_t TM_2 = 192;   // [U; O'], then Kt^T U

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

#ifdef GDN_PHASE_PROFILE
// Debug-only phase timer (block 0, thread 0): accumulates clock64 deltas per phase.
__device__ long long g_phase_cycles[16];
#define PHASE(i)                                                   \
  do {                                                             \
    if (blockIdx.x == 0 && threadIdx.x == 0) {                     \
      const long long now_ = clock64();                            \
      g_phase_cycles[i] += now_ - phase_last_;                     \
      phase_last_ = now_;                                          \
    }                                                              \
  } while (0)
#else
#define PHASE(i) \
  do {           \
  } while (0)
#endif

struct ChunkTmaps {
  CUtensorMap k;  // [T, HQ, 128] bf16: dims {128, HQ, T}, box {64, 1, 64}, 128B swizzle
  CUtensorMap q;
};

__global__ void __launch_bounds__(128, 2)
    prefill_chunked_kernel(const PrefillParams p, const __grid_constant__ ChunkTmaps maps) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                           ~uintptr_t(1023));
  float* sAf = reinterpret_cast<float*>(sm + OFF_AF);  // (aliases H hi, see the map)
  float* sTf = reinterpret_cast<float*>(sm + OFF_TF);
  float* sG = reinterpret_cast<float*>(sm + OFF_G);
  float* sBeta = reinterpret_cast<float*>(sm + OFF_BETA);
  uint64_t* bar_tma = reinterpret_cast<uint64_t*>(sm + OFF_BAR);
  uint64_t* bar_mma = bar_tma + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + OFF_BAR + 16);

  const int t = threadIdx.x;
  const int warp = t >> 5;
  const int lane = t & 31;
  const int64_t unit = blockIdx.x;
  const int vt = static_cast<int>(unit % kTiles);
  const int h = static_cast<int>((unit / kTiles) % p.HV);
  const int64_t n = unit / (kTiles * p.HV);
  const int qh = h / (p.HV / p.HQ);

  int64_t start = load_index(p.cu_seqlens, p.cu_dtype, n);
  int64_t end = load_index(p.cu_seqlens, p.cu_dtype, n + 1);
  start = start < 0 ? 0 : (start > p.T ? p.T : start);
  end = end < 0 ? 0 : (end > p.T ? p.T : end);

  // state rows of this tile: S[n, h, vt*64 + v, k]; thread t owns k = t
  const int64_t sbase = ((n * p.HV + h) * kHeadDim + vt * kVT) * kHeadDim + t;
  float hrow[kVT];
#pragma unroll
  for (int v = 0; v < kVT; ++v) hrow[v] = p.state ? p.state[sbase + v * kHeadDim] : 0.0f;

  if (end <= start) {  // empty sequence: pass the state through
#pragma unroll
    for (int v = 0; v < kVT; ++v) p.new_state[sbase + v * kHeadDim] = hrow[v];
    return;
  }

  if (t == 0) {
    mbar_init(bar_tma, 1);
    mbar_init(bar_mma, 1);
    fence_mbar_init();
    tma_prefetch_desc(&maps.k);
    tma_prefetch_desc(&maps.q);
  }
  if (warp == 0) tmem_alloc(tmem_slot, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t lane_base = static_cast<uint32_t>(warp * 32) << 16;
  const uint32_t trow = tmem + lane_base;  // this thread's TMEM lane

  // initial state -> TMEM (fp32) and the hi/lo MN-major operand tile
  tmem_st64(trow + TM_H, hrow);
  store_row_split(sm + OFF_H_HI, sm + OFF_H_LO, t, hrow);

  const float A_log = load_scalar(p.A_log, p.A_log_dtype, h);
  const float dtb = load_scalar(p.dt_bias, p.dt_bias_dtype, h);
  const int64_t HV = p.HV;

  // K/Q tiles by TMA (thread 0); raw gates of the chunk's tokens (threads 0..63)
  auto issue_tma = [&](int64_t cs) {
    if (t == 0) {
      fence_async_smem();  // order earlier generic accesses of the tile before the TMA writes
      mbar_arrive_expect_tx(bar_tma, 4 * 8192);
      const int tok = static_cast<int>(cs);
      tma_load_3d(sm + OFF_KQ, &maps.k, bar_tma, 0, qh, tok);
      tma_load_3d(sm + OFF_KQ + 8192, &maps.q, bar_tma, 0, qh, tok);
      tma_load_3d(sm + OFF_KQ + 16384, &maps.k, bar_tma, 64, qh, tok);
      tma_load_3d(sm + OFF_KQ + 16384 + 8192, &maps.q, bar_tma, 64, qh, tok);
    }
  };
  auto load_gates = [&](int64_t cs, int64_t ce, float& ra, float& rb) {
    if (t < kC) {
      const int64_t tok = cs + t;
      const bool valid = tok < ce;
      ra = valid ? load_scalar(p.a, p.a_dtype, tok * HV + h) : 0.0f;
      rb = valid ? load_scalar(p.b, p.b_dtype, tok * HV + h) : 0.0f;
    }
  };

  uint32_t tma_phase = 0, mma_phase = 0;
  bool ok = true;
#ifdef GDN_PHASE_PROFILE
  long long phase_last_ = clock64();
#endif
  float ra = 0.f, rb = 0.f;
  issue_tma(start);
  load_gates(start, end, ra, rb);

  for (int64_t cs = start; cs < end; cs += kC) {
    const int L = static_cast<int>((end - cs) < kC ? (end - cs) : kC);
    const int64_t next = cs + kC;

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

    PHASE(0);  // gates + scan
    // ---- wait for K/Q, then S = [K;Q] K^T and [KH;QH] = [K;Q] H ----------------------
    ok = mbar_wait(bar_tma, tma_phase);
    tma_phase ^= 1;
    sync_before_mma();
    if (!__syncthreads_and(ok)) break;
    PHASE(1);  // TMA wait
    if (t == 0) {
      const Operand kq{smem_u32(sm + OFF_KQ), 0, false, 0, 0, 16384};
      const Operand hB{smem_u32(sm + OFF_H_HI), smem_u32(sm + OFF_H_LO), true, 8192, 2048, 0};
      issue_gemm(tmem + TM_S, kq, kq, ID_KK, 8);
      issue_gemm(tmem + TM_1, kq, hB, ID_KM, 8);
      mma_commit(bar_mma);
    }
    // V row of this thread's token (independent of the MMAs; latency overlaps them)
    uint4 vraw[8];
    if (t < kC) {
      if (t < L) {
        const uint4* src = reinterpret_cast<const uint4*>(
            p.v + ((cs + t) * HV + h) * kHeadDim + vt * kVT);
#pragma unroll
        for (int c = 0; c < 8; ++c) vraw[c] = src[c];
      } else {
#pragma unroll
        for (int c = 0; c < 8; ++c) vraw[c] = make_uint4(0u, 0u, 0u, 0u);
      }
    }
    ok = mbar_wait(bar_mma, mma_phase);
    mma_phase ^= 1;
    tc_fence_after();
    if (!__syncthreads_and(ok)) break;

    PHASE(2);  // S, G1 MMA
    const float g_last = sG[kC - 1];
    {
      float srow[64];
      tmem_ld64(trow + TM_S, srow);
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
        store_row_split(sm + OFF_A2_HI, sm + OFF_A2_LO, t, srow);
      } else {
        // M row i = t - 64
        const int i = t - kC;
        const float gi = sG[i];
#pragma unroll
        for (int j = 0; j < kC; ++j) srow[j] = (j <= i) ? ex2(gi - sG[j]) * srow[j] : 0.f;
        store_row_split(sm + OFF_A2_HI, sm + OFF_A2_LO, t, srow);
      }
    }
    if (t < kC) {
      // X row j = t:  V_j - gamma_j (K H)_j, into the dead Q half of the tile
      float xr[64];
      tmem_ld64(trow + TM_1, xr);
      const float gam = ex2(sG[t]);
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        const uint32_t w[4] = {vraw[c].x, vraw[c].y, vraw[c].z, vraw[c].w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          xr[c * 8 + 2 * e] = __uint_as_float(w[e] << 16) - gam * xr[c * 8 + 2 * e];
          xr[c * 8 + 2 * e + 1] = __uint_as_float(w[e] & 0xffff0000u) - gam * xr[c * 8 + 2 * e + 1];
        }
      }
      store_row_split(sm + OFF_X_HI, sm + OFF_X_LO, t, xr);
    }
    __syncthreads();

    PHASE(3);  // A/M/X build
    float nra = 0.f, nrb = 0.f;
    if (next < end) load_gates(next, end, nra, nrb);

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
    PHASE(4);  // diag solve
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
    PHASE(5);  // off-diag solve
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
        *reinterpret_cast<uint4*>(sm + OFF_TB_HI + off) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
        *reinterpret_cast<uint4*>(sm + OFF_TB_LO + off) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
      }
    }

    PHASE(6);  // T_b write
    // ---- [T_b; P] = [I; M] T_b -----------------------------------------------------
    sync_before_mma();
    if (t == 0) {
      const Operand a2{smem_u32(sm + OFF_A2_HI), smem_u32(sm + OFF_A2_LO), false, 0, 0, 0};
      const Operand tb{smem_u32(sm + OFF_TB_HI), smem_u32(sm + OFF_TB_LO), true, 8192, 2048, 0};
      issue_gemm(tmem + TM_S, a2, tb, ID_KM, 4);
      mma_commit(bar_mma);
    }
    ok = mbar_wait(bar_mma, mma_phase);
    mma_phase ^= 1;
    tc_fence_after();
    if (!__syncthreads_and(ok)) break;
    PHASE(7);  // P MMA
    {
      float r[64];
      tmem_ld64(trow + TM_S, r);
      store_row_split(sm + OFF_A2_HI, sm + OFF_A2_LO, t, r);
    }

    PHASE(8);  // A2 write
    // ---- [U; O'] = [T_b; P] X ----------------------------------------------------------
    sync_before_mma();
    if (t == 0) {
      const Operand a2{smem_u32(sm + OFF_A2_HI), smem_u32(sm + OFF_A2_LO), false, 0, 0, 0};
      const Operand xb{smem_u32(sm + OFF_X_HI), smem_u32(sm + OFF_X_LO), true, 8192, 2048, 0};
      issue_gemm(tmem + TM_2, a2, xb, ID_KM, 4);
      mma_commit(bar_mma);
    }
    ok = mbar_wait(bar_mma, mma_phase);
    mma_phase ^= 1;
    tc_fence_after();
    if (!__syncthreads_and(ok)) break;
    PHASE(9);  // G2 MMA
    if (t < kC) {
      // f_j U_j with f_j = e^{Gamma_last - Gamma_j} (0 for padded rows): the state
      // update then reads the raw K tile, dH = K^T diag(f) U
      float u[64];
      tmem_ld64(trow + TM_2, u);
      const float f = (t < L) ? ex2(g_last - sG[t]) : 0.0f;
#pragma unroll
      for (int v = 0; v < kVT; ++v) u[v] *= f;
      store_row_split(sm + OFF_X_HI, sm + OFF_X_LO, t, u);  // overwrites X (G2 is done)
    } else {
      const int i = t - kC;
      float o[64], qhv[64];
      tmem_ld64(trow + TM_2, o);
      tmem_ld64(trow + TM_1, qhv);
      if (i < L) {
        const float gam = ex2(sG[i]);
        __nv_bfloat16* dst = p.out + ((cs + i) * HV + h) * kHeadDim + vt * kVT;
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          uint32_t w[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int v0 = c * 8 + 2 * e;
            const float o0 = p.scale * fmaf(gam, qhv[v0], o[v0]);
            const float o1 = p.scale * fmaf(gam, qhv[v0 + 1], o[v0 + 1]);
            w[e] = pack_bf16(__float2bfloat16_rn(o0), __float2bfloat16_rn(o1));
          }
          *reinterpret_cast<uint4*>(dst + c * 8) = make_uint4(w[0], w[1], w[2], w[3]);
        }
      }
    }

    PHASE(10);  // U / O
    // ---- dH = K^T diag(f) U;  H <- gamma_last H + dH ----------------------------------------
    sync_before_mma();
    if (t == 0) {
      const Operand kt{smem_u32(sm + OFF_KQ), 0, true, 16384, 2048, 0};
      const Operand ub{smem_u32(sm + OFF_X_HI), smem_u32(sm + OFF_X_LO), true, 8192, 2048, 0};
      issue_gemm(tmem + TM_2, kt, ub, ID_MM, 4);
      mma_commit(bar_mma);
    }
    ok = mbar_wait(bar_mma, mma_phase);
    mma_phase ^= 1;
    tc_fence_after();
    if (!__syncthreads_and(ok)) break;
    // the K/Q tile is free: fetch the next chunk while the state is updated
    if (next < end) issue_tma(next);
    PHASE(11);  // G3 MMA
    {
      float dh[64];
      tmem_ld64(trow + TM_2, dh);
      tmem_ld64(trow + TM_H, hrow);
      const float gl = ex2(g_last);
#pragma unroll
      for (int v = 0; v < kVT; ++v) hrow[v] = fmaf(gl, hrow[v], dh[v]);
      tmem_st64(trow + TM_H, hrow);
      store_row_split(sm + OFF_H_HI, sm + OFF_H_LO, t, hrow);
    }
    PHASE(12);  // H update
    ra = nra;
    rb = nrb;
  }

  if (ok) {
    tmem_ld64(trow + TM_H, hrow);
#pragma unroll
    for (int v = 0; v < kVT; ++v) p.new_state[sbase + v * kHeadDim] = hrow[v];
  } else if (t == 0 && p.status) {
    atomicExch(p.status, 1);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, kTmemCols);
}

// ------------------------------------------------------------------ host side
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn get_encode_fn() {
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

bool encode_qk_map(CUtensorMap* map, const void* base, int64_t T, int HQ) {
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

}  // namespace

int launch_prefill_chunked(const PrefillParams& p, cudaStream_t stream) {
  const int64_t units = p.N * p.HV * kTiles;
  if (units == 0) return 0;
  ChunkTmaps maps;
  // a zero-token batch still launches (every sequence passes its state through);
  // the maps then describe a 1-token extent that no block reads
  const int64_t Tm = p.T > 0 ? p.T : 1;
  const void* kb = p.T > 0 ? static_cast<const void*>(p.k) : static_cast<const void*>(p.new_state);
  const void* qb = p.T > 0 ? static_cast<const void*>(p.q) : static_cast<const void*>(p.new_state);
  if (!encode_qk_map(&maps.k, kb, Tm, p.HQ) || !encode_qk_map(&maps.q, qb, Tm, p.HQ)) return -2;
  static bool attr_set = false;
  if (!attr_set) {
    if (cudaFuncSetAttribute(prefill_chunked_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             kSmemBytes) != cudaSuccess)
      return -1;
    attr_set = true;
  }
  prefill_chunked_kernel<<<static_cast<unsigned>(units), 128, kSmemBytes, stream>>>(p, maps);
  return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

}  // namespace gdn

#ifdef GDN_PHASE_PROFILE
// Debug builds only: copy (and optionally reset) the per-phase cycle counters.
extern "C" __attribute__((visibility("default"))) int gdn_debug_phase_cycles(long long* host,
                                                                               int reset) {
  if (cudaMemcpyFromSymbol(host, gdn::g_phase_cycles, sizeof(long long) * 16) != cudaSuccess)
    return -1;
  if (reset) {
    long long z[16] = {0};
    if (cudaMemcpyToSymbol(gdn::g_phase_cycles, z, sizeof(z)) != cudaSuccess) return -1;
  }
  return 0;
}
#endif
