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
#include "gdn_chunk_common.cuh"

namespace gdn {
namespace {

using namespace sm100;
using namespace chunk;


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

// TMEM columns (fp32, lane = row of M = 128)
constexpr uint32_t kTmemCols = 256;
constexpr uint32_t TM_H = 0;     // persistent state H (lane k, col v)
constexpr uint32_t TM_S = 64;    // S = [K;Q] K^T, then [T_b; P]
constexpr uint32_t TM_1 = 128;   // [KH; QH]
constexpr uint32_t TM_2 = 192;   // [U; O'], then Kt^T U


__global__ void __launch_bounds__(128, 2)
    prefill_chunked_kernel(const PrefillParams p, const __grid_constant__ ChunkTmaps maps) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = align_smem<1024>(smem_raw);
  float* sAf = reinterpret_cast<float*>(sm + OFF_AF);  // (aliases H hi, see the map)
  float* sTf = reinterpret_cast<float*>(sm + OFF_TF);
  float* sG = reinterpret_cast<float*>(sm + OFF_G);
  float* sBeta = reinterpret_cast<float*>(sm + OFF_BETA);
  uint64_t* bar_tma = reinterpret_cast<uint64_t*>(sm + OFF_BAR);
  uint64_t* bar_mma = bar_tma + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + OFF_BAR + 16);

  const int t = threadIdx.x;
  const int warp = t >> 5;
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
  float ra = 0.f, rb = 0.f;
  issue_tma(start);
  load_gates(start, end, ra, rb);

  for (int64_t cs = start; cs < end; cs += kC) {
    const int L = static_cast<int>((end - cs) < kC ? (end - cs) : kC);
    const int64_t next = cs + kC;

    chunk_gates(ra, rb, L, A_log, dtb, sG, sBeta);
    // ---- wait for K/Q, then S = [K;Q] K^T and [KH;QH] = [K;Q] H ----------------------
    ok = mbar_wait(bar_tma, tma_phase);
    tma_phase ^= 1;
    sync_before_mma();
    if (!__syncthreads_and(ok)) break;
    if (t < 32) {  // warp 0 issues
      const Operand kq{smem_u32(sm + OFF_KQ), 0, false, 0, 0, 16384};
      const Operand hB{smem_u32(sm + OFF_H_HI), smem_u32(sm + OFF_H_LO), true, 8192, 2048, 0};
      issue_gemm(tmem + TM_S, kq, kq, ID_KK, 8);
      issue_gemm(tmem + TM_1, kq, hB, ID_KM, 8);
      mma_commit_w(bar_mma);
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

    const float g_last = sG[kC - 1];
    build_a_m<SwzLayout>(trow + TM_S, sAf, sG, sBeta, sm + OFF_A2_HI, sm + OFF_A2_LO);
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

    float nra = 0.f, nrb = 0.f;
    if (next < end) load_gates(next, end, nra, nrb);

    solve_tb<SwzLayout>(sAf, sTf, sBeta, sm + OFF_TB_HI, sm + OFF_TB_LO);
    // ---- [T_b; P] = [I; M] T_b -----------------------------------------------------
    sync_before_mma();
    if (t < 32) {  // warp 0 issues
      const Operand a2{smem_u32(sm + OFF_A2_HI), smem_u32(sm + OFF_A2_LO), false, 0, 0, 0};
      const Operand tb{smem_u32(sm + OFF_TB_HI), smem_u32(sm + OFF_TB_LO), true, 8192, 2048, 0};
      issue_gemm(tmem + TM_S, a2, tb, ID_KM, 4);
      mma_commit_w(bar_mma);
    }
    ok = mbar_wait(bar_mma, mma_phase);
    mma_phase ^= 1;
    tc_fence_after();
    if (!__syncthreads_and(ok)) break;
    {
      float r[64];
      tmem_ld64(trow + TM_S, r);
      store_row_split(sm + OFF_A2_HI, sm + OFF_A2_LO, t, r);
    }

    // ---- [U; O'] = [T_b; P] X ----------------------------------------------------------
    sync_before_mma();
    if (t < 32) {  // warp 0 issues
      const Operand a2{smem_u32(sm + OFF_A2_HI), smem_u32(sm + OFF_A2_LO), false, 0, 0, 0};
      const Operand xb{smem_u32(sm + OFF_X_HI), smem_u32(sm + OFF_X_LO), true, 8192, 2048, 0};
      issue_gemm(tmem + TM_2, a2, xb, ID_KM, 4);
      mma_commit_w(bar_mma);
    }
    ok = mbar_wait(bar_mma, mma_phase);
    mma_phase ^= 1;
    tc_fence_after();
    if (!__syncthreads_and(ok)) break;
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
            w[e] = pack2_rn(o0, o1);
          }
          *reinterpret_cast<uint4*>(dst + c * 8) = make_uint4(w[0], w[1], w[2], w[3]);
        }
      }
    }

    // ---- dH = K^T diag(f) U;  H <- gamma_last H + dH ----------------------------------------
    sync_before_mma();
    if (t < 32) {  // warp 0 issues
      const Operand kt{smem_u32(sm + OFF_KQ), 0, true, 16384, 2048, 0};
      const Operand ub{smem_u32(sm + OFF_X_HI), smem_u32(sm + OFF_X_LO), true, 8192, 2048, 0};
      issue_gemm(tmem + TM_2, kt, ub, ID_MM, 4);
      mma_commit_w(bar_mma);
    }
    ok = mbar_wait(bar_mma, mma_phase);
    mma_phase ^= 1;
    tc_fence_after();
    if (!__syncthreads_and(ok)) break;
    // the K/Q tile is free: fetch the next chunk while the state is updated
    if (next < end) issue_tma(next);
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
    ra = nra;
    rb = nrb;
  }

  if (ok) {
    tmem_ld64(trow + TM_H, hrow);
#pragma unroll
    for (int v = 0; v < kVT; ++v) p.new_state[sbase + v * kHeadDim] = hrow[v];
  } else if (t == 0 && p.status) {
    atomicOr(p.status, 1);  // bit 0: a bounded wait gave up
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, kTmemCols);
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
  // a per-device attribute: set it on every launch (a cheap host call)
  if (cudaFuncSetAttribute(prefill_chunked_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           kSmemBytes) != cudaSuccess)
    return -1;
  prefill_chunked_kernel<<<static_cast<unsigned>(units), 128, kSmemBytes, stream>>>(p, maps);
  return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

}  // namespace gdn

