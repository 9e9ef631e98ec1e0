// gdn_prefill_twophase.cu — chunk-64 varlen GDN prefill split into a parallel
// prep phase and a sequential scan phase (the default prefill path).
//
// Same algebra as gdn_prefill_chunked.cu (chunkwise / UT-transform gated delta
// rule; semantics of gdn/prefill/baseline/triton/kernel.py:18-100). The work of
// a chunk splits into a part that does not depend on the state and a part that
// does:
//
//   prep (one block per (chunk, v-head), all chunks of all sequences at once):
//     S = [K;Q] K^T, A, M, T_b = (I + A)^-1 diag(beta), [T_b; P] = [I; M] T_b
//     -> the bf16 image of [T_b; P] (hi 128 rows, lo rows 0..63: 24 KB) written to
//        the workspace in the 128B-swizzled layout the scan kernel's MMA reads.
//   scan (one 256-thread block per (sequence, v-head), chunk by chunk; the products
//   are taken transposed so that the chain's own operands live in TMEM):
//     [KH; QH] = [K;Q] H,  X = V - gamma KH,  [U; O'] = [T_b; P] X,
//     O = scale (gamma QH + O'),  H <- gamma_last H + K^T diag(f) U.
//
// The prep phase has (T/64 + N) x HV independent blocks, so the triangular solve
// and the operand construction run at full occupancy instead of on the critical
// path of each sequence; the scan keeps only the state chain and receives
// [T_b; P] with one bulk copy per chunk, double-buffered with the K/Q and V tiles.
// P enters the tensor core as hi only (its rounding only touches the output, which
// is bf16), T_b as hi + lo.
// A tiny first kernel turns cu_seqlens into per-sequence chunk offsets so that
// no host synchronisation is needed.
#include "gdn_chunk_common.cuh"
#include "gdn_launch.h"

namespace gdn {
namespace {

using namespace sm100;
using namespace chunk;

constexpr uint32_t kA2Bytes = 24576;

#ifdef GDN_PHASE_PROFILE
// Debug-only phase timer of the scan (block 0, thread 0): clock64 deltas per phase.
__device__ long long g_scan_cycles[16];
#define SPHASE(i)                                     \
  do {                                                \
    if (blockIdx.x == 0 && threadIdx.x == 0) {        \
      const long long now_ = clock64();               \
      g_scan_cycles[i] += now_ - sphase_last_;        \
      sphase_last_ = now_;                            \
    }                                                 \
  } while (0)
__device__ long long g_prep_cycles[16];
#define PPHASE(i)                                     \
  do {                                                \
    if (blockIdx.x == 0 && threadIdx.x == 0) {        \
      const long long now_ = clock64();               \
      g_prep_cycles[i] += now_ - pphase_last_;        \
      pphase_last_ = now_;                            \
    }                                                 \
  } while (0)
#define PPHASE_INIT long long pphase_last_ = clock64()
#else
#define SPHASE(i) \
  do {            \
  } while (0)
#define PPHASE(i) \
  do {            \
  } while (0)
#define PPHASE_INIT
#endif  // per (chunk, v-head): hi 16 KB + lo rows 0..63 8 KB

__device__ __forceinline__ void seq_bounds(const PrefillParams& p, int64_t n, int64_t& start,
                                           int64_t& end) {
  start = load_index(p.cu_seqlens, p.cu_dtype, n);
  end = load_index(p.cu_seqlens, p.cu_dtype, n + 1);
  start = start < 0 ? 0 : (start > p.T ? p.T : start);
  end = end < 0 ? 0 : (end > p.T ? p.T : end);
}

// ------------------------------------------------------------------ chunk offsets
// offs[n] = number of 64-token chunks in sequences 0..n-1 (offs[0] = 0). One block.
__global__ void __launch_bounds__(1024) chunk_offsets_kernel(const PrefillParams p,
                                                             int64_t* offs) {
  __shared__ int64_t warp_sums[32];
  __shared__ int64_t carry;
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  if (t == 0) {
    carry = 0;
    offs[0] = 0;
  }
  __syncthreads();
  for (int64_t base = 0; base < p.N; base += 1024) {
    const int64_t n = base + t;
    int64_t cnt = 0;
    if (n < p.N) {
      int64_t s, e;
      seq_bounds(p, n, s, e);
      cnt = e > s ? (e - s + kC - 1) / kC : 0;
    }
    int64_t x = cnt;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int64_t y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
    if (lane == 31) warp_sums[warp] = x;
    __syncthreads();
    if (warp == 0) {
      int64_t w = warp_sums[lane];
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int64_t y = __shfl_up_sync(0xffffffffu, w, o);
        if (lane >= o) w += y;
      }
      warp_sums[lane] = w;  // inclusive over warps
    }
    __syncthreads();
    const int64_t incl = x + (warp > 0 ? warp_sums[warp - 1] : 0) + carry;
    if (n < p.N) offs[n + 1] = incl;
    __syncthreads();
    if (t == 1023) carry = incl;
    __syncthreads();
  }
}

// ------------------------------------------------------------------ scan order
// order[i] = the sequence the i-th group of scan blocks processes: longest first
// (most chunks), ties by index, so that the longest chains start in the first wave
// and short ones fill the tail. Rank sort, one thread per sequence (N <= kMaxSortN;
// beyond that the identity order).
constexpr int64_t kMaxSortN = 4096;
__global__ void __launch_bounds__(256) scan_order_kernel(int64_t N, const int64_t* offs,
                                                         int32_t* order) {
  const int64_t n = blockIdx.x * 256 + threadIdx.x;
  if (n >= N) return;
  if (N > kMaxSortN) {
    order[n] = static_cast<int32_t>(n);
    return;
  }
  const int64_t cn = offs[n + 1] - offs[n];
  int64_t rank = 0;
  for (int64_t m = 0; m < N; ++m) {
    const int64_t cm = offs[m + 1] - offs[m];
    rank += (cm > cn || (cm == cn && m < n)) ? 1 : 0;
  }
  order[rank] = static_cast<int32_t>(n);
}

// ------------------------------------------------------------------ prep
// 256 threads; thread t owns TMEM lane / row t % 128 and a 32-column half of it.
// Shared memory: the K/Q tile (32 KB, TMA) is dead after S and then holds the fp32 A
// and T of the solve (padded rows, 17 KB each), then T_b hi/lo over A. M hi/lo (rows
// 0..63 of the A operand of P = M T_b; the operand's rows 64..127 read whatever
// follows — those result rows are not used).
constexpr uint32_t P_OFF_KQ = 0;
constexpr uint32_t P_OFF_AF = 0;
constexpr uint32_t P_OFF_TF = 17408;
constexpr uint32_t P_OFF_TB_HI = 0;
constexpr uint32_t P_OFF_TB_LO = 8192;
constexpr uint32_t P_OFF_M_HI = 35840;   // 1024-aligned, after T
constexpr uint32_t P_OFF_M_LO = 44032;   // rows 64..127 of the hi operand = these rows
constexpr uint32_t P_OFF_G = 60416;      // (52224..60416: rows 64..127 of the lo operand)
constexpr uint32_t P_OFF_BETA = 60672;
constexpr uint32_t P_OFF_BAR = 60928;
constexpr uint32_t kPrepSmem = 60992 + 1024;
constexpr uint32_t kPrepTmemCols = 128;
constexpr uint32_t PT_S = 0, PT_P = 64;
constexpr int kPrepThreads = 256;

__global__ void __launch_bounds__(kPrepThreads, 3)
    prep_kernel(const PrefillParams p, const __grid_constant__ ChunkTmaps maps,
                const int64_t* __restrict__ offs, uint8_t* __restrict__ a2_out) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                           ~uintptr_t(1023));
  float* sAf = reinterpret_cast<float*>(sm + P_OFF_AF);
  float* sTf = reinterpret_cast<float*>(sm + P_OFF_TF);
  float* sG = reinterpret_cast<float*>(sm + P_OFF_G);
  float* sBeta = reinterpret_cast<float*>(sm + P_OFF_BETA);
  uint64_t* bar_tma = reinterpret_cast<uint64_t*>(sm + P_OFF_BAR);
  uint64_t* bar_mma = bar_tma + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + P_OFF_BAR + 16);

  const int t = threadIdx.x, warp = t >> 5, r = t & 127, c0 = (t >> 7) * 32;
  const int h = static_cast<int>(blockIdx.x % p.HV);
  const int64_t gchunk = blockIdx.x / p.HV;
  const int64_t total = offs[p.N];
  if (gchunk >= total) return;
  // sequence containing this chunk: the last n with offs[n] <= gchunk
  int64_t lo = 0, hi = p.N;
  while (lo < hi) {
    const int64_t mid = (lo + hi + 1) >> 1;
    if (offs[mid] <= gchunk) lo = mid;
    else hi = mid - 1;
  }
  const int64_t n = lo;
  int64_t start, end;
  seq_bounds(p, n, start, end);
  const int64_t cs = start + (gchunk - offs[n]) * kC;
  const int L = static_cast<int>((end - cs) < kC ? (end - cs) : kC);
  const int qh = h / (p.HV / p.HQ);

  if (t == 0) {
    mbar_init(bar_tma, 1);
    mbar_init(bar_mma, 1);
    fence_mbar_init();
    mbar_arrive_expect_tx(bar_tma, 4 * 8192);
    const int tok = static_cast<int>(cs);
    tma_load_3d(sm + P_OFF_KQ, &maps.k, bar_tma, 0, qh, tok);
    tma_load_3d(sm + P_OFF_KQ + 8192, &maps.q, bar_tma, 0, qh, tok);
    tma_load_3d(sm + P_OFF_KQ + 16384, &maps.k, bar_tma, 64, qh, tok);
    tma_load_3d(sm + P_OFF_KQ + 16384 + 8192, &maps.q, bar_tma, 64, qh, tok);
  }
  if (warp == 0) tmem_alloc(tmem_slot, kPrepTmemCols);
  float ra = 0.f, rb = 0.f;
  if (t < kC && t < L) {
    ra = load_scalar(p.a, p.a_dtype, (cs + t) * p.HV + h);
    rb = load_scalar(p.b, p.b_dtype, (cs + t) * p.HV + h);
  }
  const float A_log = load_scalar(p.A_log, p.A_log_dtype, h);
  const float dtb = load_scalar(p.dt_bias, p.dt_bias_dtype, h);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t trow = tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16) + c0;

  PPHASE_INIT;
  chunk_gates(ra, rb, L, A_log, dtb, sG, sBeta);
  PPHASE(0);  // gates
  bool ok = mbar_wait(bar_tma, 0);
  PPHASE(1);  // TMA wait
  sync_before_mma();
  if (__syncthreads_and(ok)) {
    if (t < 32) {  // warp 0 issues
      const Operand kq{smem_u32(sm + P_OFF_KQ), 0, false, 0, 0, 16384};
      issue_gemm(tmem + PT_S, kq, kq, ID_KK, 8);
      mma_commit_w(bar_mma);
    }
    ok = mbar_wait(bar_mma, 0);
    tc_fence_after();
    PPHASE(2);  // S MMA
    if (__syncthreads_and(ok)) {
      // the K/Q tile is dead: A, T and T_b reuse its space
      build_a_m_256<PadLayout>(trow + PT_S, sAf, sG, sBeta, sm + P_OFF_M_HI, sm + P_OFF_M_LO);
      __syncthreads();
      PPHASE(3);  // build A, M
      solve_tb_256<PadLayout>(sAf, sTf, sBeta, sm + P_OFF_TB_HI, sm + P_OFF_TB_LO);
      PPHASE(4);  // solve + T_b
      sync_before_mma();
      if (t < 32) {  // warp 0 issues  // P = M T_b (result rows 0..63)
        const Operand mA{smem_u32(sm + P_OFF_M_HI), smem_u32(sm + P_OFF_M_LO), false, 0, 0, 0};
        const Operand tb{smem_u32(sm + P_OFF_TB_HI), smem_u32(sm + P_OFF_TB_LO), true, 8192,
                         2048, 0};
        issue_gemm(tmem + PT_P, mA, tb, ID_KM, 4);
        mma_commit_w(bar_mma);
      }
      // meanwhile: the T_b rows of [T_b; P] are the T_b tiles themselves (same swizzled
      // row image): copy hi to rows 0..63 of the hi part, lo to the lo part
      uint8_t* dst = a2_out + (static_cast<uint64_t>(gchunk) * p.HV + h) * kA2Bytes;
      {
        const uint4* src_hi = reinterpret_cast<const uint4*>(sm + P_OFF_TB_HI);
        const uint4* src_lo = reinterpret_cast<const uint4*>(sm + P_OFF_TB_LO);
#pragma unroll
        for (int q = 0; q < 2; ++q) {
          const int idx = t + q * kPrepThreads;  // 512 x 16 B = 8 KB per tile
          reinterpret_cast<uint4*>(dst)[idx] = src_hi[idx];
          reinterpret_cast<uint4*>(dst + 16384)[idx] = src_lo[idx];
        }
      }
      PPHASE(5);  // P issue + T_b copy
      ok = mbar_wait(bar_mma, 1);
      tc_fence_after();
      PPHASE(6);  // P wait
      if (__syncthreads_and(ok) && r < kC) {
        // row r of P -> hi only (P only reaches the bf16 output), rows 64..127 of the hi part
        float pr[32];
        tmem_ld32(trow + PT_P, pr);
        tmem_ld_wait();
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t w[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) w[e] = pack2_rn(pr[c * 8 + 2 * e], pr[c * 8 + 2 * e + 1]);
          *reinterpret_cast<uint4*>(dst + 8192 + sw128_chunk(r, (c0 >> 3) + c)) =
              make_uint4(w[0], w[1], w[2], w[3]);
        }
      }
      PPHASE(7);  // P rows write
    }
  }
  if (!ok && t == 0 && p.status) atomicExch(p.status, 1);
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, kPrepTmemCols);
}

// ------------------------------------------------------------------ scan, transposed
// One 256-thread block per (sequence, v-head): the whole 128 x 128 state. The
// products are taken transposed so that everything the chain produces is an A
// operand read from TMEM (lane = state row v) and every B operand is a tile that
// arrived by TMA / bulk copy:
//   D1 = S [K;Q]^T        -> [ (KH)^T | (QH)^T ]          (A = S hi/lo from TMEM)
//   X^T = V^T - (KH)^T diag(gamma)                         (written to TMEM as bf16 hi/lo)
//   D2 = X^T [T_b; P]^T   -> [ U^T | (P X)^T ]
//   U'^T = U^T diag(f);  O^T = scale ((QH)^T diag(gamma) + (P X)^T)
//   dS = U'^T K;  S <- gamma_last S + dS                   (S = H^T, k-last, in registers)
// Thread t owns state row v = t % 128 and quarter c = t / 128 of every row-sliced
// quantity (k in [32c, 32c+32) of S; j in [16c, 16c+16) of X, U; i likewise of O).
// K/Q, V and [T_b; P] are double-buffered: chunk c+1's tiles are requested when
// chunk c starts.
constexpr uint32_t T_OFF_KQ = 0;          // 2 x 32 KB
constexpr uint32_t T_OFF_A2 = 65536;      // 2 x 32 KB: hi 16 KB | lo 16 KB (rows 64..127 zero)
constexpr uint32_t T_OFF_V = 131072;      // 2 x 16 KB: V tile, rows j x 128 v (256 B rows)
constexpr uint32_t T_OFF_G = 163840;      // 2 x 64 fp32
constexpr uint32_t T_OFF_BETA = 164352;   // 2 x 64 fp32 (written by the gate scan, unused)
constexpr uint32_t T_OFF_GAM = 164864;    // 2 x 64 fp32: gamma_j = e^{Gamma_j}
constexpr uint32_t T_OFF_F = 165376;      // 2 x 64 fp32: f_j = e^{Gamma_last - Gamma_j} (0 if padded)
constexpr uint32_t T_OFF_BAR = 165888;    // ld[2], a2[2], mma; TMEM slot
constexpr uint32_t T_OFF_O = 166912;      // 2 x 16 KB: output tile, rows i x 128 v (TMA store)
constexpr uint32_t kScanTSmem = 166912 + 32768 + 1024;
constexpr uint32_t kScanTTmemCols = 512;
constexpr uint32_t TT_S = 0;    // S operand: hi [0, 64) | lo [64, 128); later dS (fp32, 128)
constexpr uint32_t TT_D1 = 128; // 128 fp32 columns
constexpr uint32_t TT_X = 256;  // X^T then U'^T operand: hi [256, 288) | lo [288, 320)
constexpr uint32_t TT_D2 = 320; // 128 fp32 columns
constexpr uint32_t ID_T_K = idesc_bf16(128, 128, false, false);   // B K-major
constexpr uint32_t ID_T_MN = idesc_bf16(128, 128, false, true);   // B MN-major
// N = 64: the lo (correction) terms are taken only for the columns that feed the state
// (KH and U); the QH and PX columns reach the bf16 output alone and take hi x hi
constexpr uint32_t ID_T_K64 = idesc_bf16(128, 64, false, false);
constexpr int kScanTThreads = 512;
constexpr int kScanTGateBase = 128;  // warps 4-5 compute the next chunk's gates

struct ScanMaps {
  CUtensorMap k, q, v, o;
};

// 2n fp32 -> n bf16x2 words, hi and lo parts
template <int NW>
__device__ __forceinline__ void split_words(const float* x, uint32_t (&hi)[NW], uint32_t (&lo)[NW]) {
#pragma unroll
  for (int w = 0; w < NW; ++w) split2(x[2 * w], x[2 * w + 1], hi[w], lo[w]);
}

__global__ void __launch_bounds__(kScanTThreads, 1)
    scan_t_kernel(const PrefillParams p, const __grid_constant__ ScanMaps maps,
                  const int64_t* __restrict__ offs, const int32_t* __restrict__ order,
                  const uint8_t* __restrict__ a2_in) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                           ~uintptr_t(1023));
  float* sG0 = reinterpret_cast<float*>(sm + T_OFF_G);
  float* sBeta0 = reinterpret_cast<float*>(sm + T_OFF_BETA);
  float* sGam0 = reinterpret_cast<float*>(sm + T_OFF_GAM);
  float* sF0 = reinterpret_cast<float*>(sm + T_OFF_F);
  uint64_t* bar_ld = reinterpret_cast<uint64_t*>(sm + T_OFF_BAR);  // [2]
  uint64_t* bar_a2 = bar_ld + 2;                                   // [2]
  uint64_t* bar_mma = bar_ld + 4;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + T_OFF_BAR + 48);

  const int t = threadIdx.x, warp = t >> 5;
  const int v = t & 127, ch = t >> 7;
  const int h = static_cast<int>(blockIdx.x % p.HV);
  const int64_t n = order[blockIdx.x / p.HV];
  const int qh = h / (p.HV / p.HQ);
  const int64_t HV = p.HV;
  int64_t start, end;
  seq_bounds(p, n, start, end);

  // this thread's quarter of state row v: S[n, h, v, 32c .. 32c+32)
  const int64_t sbase = ((n * HV + h) * kHeadDim + v) * kHeadDim + 32 * ch;
  float S[32];
#pragma unroll
  for (int i = 0; i < 32; i += 4) {
    const float4 x = p.state ? *reinterpret_cast<const float4*>(p.state + sbase + i)
                             : make_float4(0.f, 0.f, 0.f, 0.f);
    S[i] = x.x; S[i + 1] = x.y; S[i + 2] = x.z; S[i + 3] = x.w;
  }
  if (end <= start) {  // empty sequence: pass the state through
#pragma unroll
    for (int i = 0; i < 32; i += 4)
      *reinterpret_cast<float4*>(p.new_state + sbase + i) =
          make_float4(S[i], S[i + 1], S[i + 2], S[i + 3]);
    return;
  }
  const uint8_t* a2_seq = a2_in + static_cast<uint64_t>(offs[n]) * HV * kA2Bytes +
                          static_cast<uint64_t>(h) * kA2Bytes;
  const uint64_t a2_chunk_stride = static_cast<uint64_t>(HV) * kA2Bytes;

  auto issue_loads = [&](int64_t cs, int64_t c, int b) {
    fence_async_smem();
    uint8_t* kq = sm + T_OFF_KQ + b * 32768;
    mbar_arrive_expect_tx(&bar_ld[b], 4 * 8192 + 16384);
    const int tok = static_cast<int>(cs);
    tma_load_3d(kq, &maps.k, &bar_ld[b], 0, qh, tok);
    tma_load_3d(kq + 8192, &maps.q, &bar_ld[b], 0, qh, tok);
    tma_load_3d(kq + 16384, &maps.k, &bar_ld[b], 64, qh, tok);
    tma_load_3d(kq + 16384 + 8192, &maps.q, &bar_ld[b], 64, qh, tok);
    tma_load_3d(sm + T_OFF_V + b * 16384, &maps.v, &bar_ld[b], 0, h, tok);
    mbar_arrive_expect_tx(&bar_a2[b], kA2Bytes);
    const uint8_t* src = a2_seq + static_cast<uint64_t>(c) * a2_chunk_stride;
    uint8_t* a2 = sm + T_OFF_A2 + b * 32768;
    bulk_load(a2, src, 16384, &bar_a2[b]);
    bulk_load(a2 + 16384, src + 16384, 8192, &bar_a2[b]);
  };

  if (t == 0) {
    for (int i = 0; i < 5; ++i) mbar_init(&bar_ld[i], 1);
    fence_mbar_init();
  }
  if (warp == 0) tmem_alloc(tmem_slot, kScanTTmemCols);
  // rows 64..127 of the lo part of [T_b; P] stay zero (P enters as hi only)
  for (int i = t; i < 2 * 512; i += kScanTThreads) {
    const int b = i >> 9, q = i & 511;
    reinterpret_cast<uint4*>(sm + T_OFF_A2 + b * 32768 + 16384 + 8192)[q] =
        make_uint4(0u, 0u, 0u, 0u);
  }
  fence_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t lane = tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16);

  auto write_s_operand = [&]() {
    uint32_t hw[16], lw[16];
    split_words<16>(S, hw, lw);
    tmem_st16(lane + TT_S + 16 * ch, hw);
    tmem_st16(lane + TT_S + 64 + 16 * ch, lw);
    tmem_st_wait();
  };
  write_s_operand();

  const float A_log = load_scalar(p.A_log, p.A_log_dtype, h);
  const float dtb = load_scalar(p.dt_bias, p.dt_bias_dtype, h);
  const bool gate_thread = t >= kScanTGateBase && t < kScanTGateBase + kC;
  auto load_gates = [&](int64_t cs, float& ra, float& rb) {
    if (gate_thread) {
      const int64_t tok = cs + (t - kScanTGateBase);
      const bool valid = tok < end;
      ra = valid ? load_scalar(p.a, p.a_dtype, tok * HV + h) : 0.0f;
      rb = valid ? load_scalar(p.b, p.b_dtype, tok * HV + h) : 0.0f;
    }
  };
  // gates of a chunk (warps 4-5): cumulative log decay, then gamma_j and f_j
  auto gates = [&](float ra, float rb, int L, int buf) {
    float* g = sG0 + buf * kC;
    chunk_gates_w01(ra, rb, L, A_log, dtb, g, sBeta0 + buf * kC, kScanTGateBase);
    named_bar_sync(1, 64);
    const int j = t - kScanTGateBase;
    sGam0[buf * kC + j] = ex2(g[j]);
    sF0[buf * kC + j] = (j < L) ? ex2(g[kC - 1] - g[j]) : 0.0f;
  };
  float ra = 0.f, rb = 0.f;
  load_gates(start, ra, rb);
  if (gate_thread) gates(ra, rb, static_cast<int>((end - start) < kC ? (end - start) : kC), 0);
  if (t == 0) issue_loads(start, 0, 0);

  uint32_t mma_phase = 0;
  bool ok = true;
  int64_t c = 0;
#ifdef GDN_PHASE_PROFILE
  long long sphase_last_ = clock64();
#endif
  for (int64_t cs = start; cs < end; cs += kC, ++c) {
    const int L = static_cast<int>((end - cs) < kC ? (end - cs) : kC);
    const int64_t next = cs + kC;
    const int b = static_cast<int>(c & 1);
    const uint32_t ph = static_cast<uint32_t>((c >> 1) & 1);
    const float* sGam = sGam0 + b * kC;
    const float* sF = sF0 + b * kC;
    const uint8_t* kq = sm + T_OFF_KQ + b * 32768;
    const uint8_t* a2 = sm + T_OFF_A2 + b * 32768;
    const uint8_t* vt = sm + T_OFF_V + b * 16384;
    float nra = 0.f, nrb = 0.f;
    if (next < end) load_gates(next, nra, nrb);

    SPHASE(0);  // top: next loads issued
    // ---- D1 = S [K;Q]^T ---------------------------------------------------------------
    ok = mbar_wait(&bar_ld[b], ph);
    SPHASE(1);  // K/Q/V wait
    tc_fence_before();
    if (!__syncthreads_and(ok)) break;  // also: the S operand of every thread is stored
    tc_fence_after();
    SPHASE(10);  // top barrier
    if (warp == 0) {
      __syncwarp();
      const uint64_t bd = desc_kmajor(smem_u32(kq));
#pragma unroll
      for (int s = 0; s < 8; ++s)
        mma_bf16_ts_w(tmem + TT_D1, tmem + TT_S + s * 8,
                    bd + (((s >> 2) * 16384 + (s & 3) * 32) >> 4), ID_T_K, s > 0);
#pragma unroll
      for (int s = 0; s < 8; ++s)
        mma_bf16_ts_w(tmem + TT_D1, tmem + TT_S + 64 + s * 8,
                    bd + (((s >> 2) * 16384 + (s & 3) * 32) >> 4), ID_T_K64, 1);
      mma_commit_w(bar_mma);
    }
    // chunk c+1's tiles into the other buffers (their last users, chunk c-1, are done),
    // from another warp while thread 0 is blocked issuing the MMAs
    if (t == 32 && next < end) issue_loads(next, c + 1, b ^ 1);
    if (gate_thread && next < end)
      gates(nra, nrb, static_cast<int>((end - next) < kC ? (end - next) : kC), b ^ 1);
    SPHASE(2);  // sync + G1 issue + gates
    ok = mbar_wait(bar_mma, mma_phase);
    mma_phase ^= 1;
    tc_fence_after();
    if (!__syncthreads_and(ok)) break;
    SPHASE(3);  // G1 wait

    {
      // X^T row v, columns j in [16c, 16c+16): V[j][v] - gamma_j (KH)^T[v][j]
      float d[16];
      tmem_ld16(lane + TT_D1 + 16 * ch, d);
      tmem_ld_wait();
      float x[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const int j = 16 * ch + i;
        const unsigned short raw =
            *reinterpret_cast<const unsigned short*>(vt + j * 256 + v * 2);
        x[i] = __uint_as_float(static_cast<uint32_t>(raw) << 16) - sGam[j] * d[i];
      }
      uint32_t hw[8], lw[8];
      split_words<8>(x, hw, lw);
      tmem_st8(lane + TT_X + 8 * ch, hw);
      tmem_st8(lane + TT_X + 32 + 8 * ch, lw);
      tmem_st_wait();
    }

    SPHASE(4);  // X build
    // ---- D2 = X^T [T_b; P]^T -----------------------------------------------------------
    ok = mbar_wait(&bar_a2[b], ph);
    tc_fence_before();
    if (!__syncthreads_and(ok)) break;
    tc_fence_after();
    if (warp == 0) {
      __syncwarp();
      const uint64_t bh = desc_kmajor(smem_u32(a2)), bl = desc_kmajor(smem_u32(a2 + 16384));
#pragma unroll
      for (int s = 0; s < 4; ++s)
        mma_bf16_ts_w(tmem + TT_D2, tmem + TT_X + s * 8, bh + ((s * 32) >> 4), ID_T_K, s > 0);
#pragma unroll
      for (int s = 0; s < 4; ++s)
        mma_bf16_ts_w(tmem + TT_D2, tmem + TT_X + 32 + s * 8, bh + ((s * 32) >> 4), ID_T_K64, 1);
#pragma unroll
      for (int s = 0; s < 4; ++s)
        mma_bf16_ts_w(tmem + TT_D2, tmem + TT_X + s * 8, bl + ((s * 32) >> 4), ID_T_K64, 1);
      mma_commit_w(bar_mma);
    }
    SPHASE(5);  // A2 wait + sync + G2 issue
    ok = mbar_wait(bar_mma, mma_phase);
    mma_phase ^= 1;
    tc_fence_after();
    if (!__syncthreads_and(ok)) break;
    SPHASE(6);  // G2 wait
    {
      // U'^T = U^T diag(f) -> operand (over X^T, consumed)
      float u[16];
      tmem_ld16(lane + TT_D2 + 16 * ch, u);
      tmem_ld_wait();
#pragma unroll
      for (int i = 0; i < 16; ++i) u[i] *= sF[16 * ch + i];
      uint32_t hw[8], lw[8];
      split_words<8>(u, hw, lw);
      tmem_st8(lane + TT_X + 8 * ch, hw);
      tmem_st8(lane + TT_X + 32 + 8 * ch, lw);
      tmem_st_wait();
    }
    SPHASE(7);  // U' + O
    // ---- dS = U'^T K (into the S operand columns: G1 is done) ---------------------------
    if (t == 0) bulk_wait_read<1>();  // this chunk's output tile buffer is free again
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 0) {
      __syncwarp();
      const uint64_t bk = desc_mnmajor(smem_u32(kq), 16384);
#pragma unroll
      for (int s = 0; s < 4; ++s)
        mma_bf16_ts_w(tmem + TT_S, tmem + TT_X + s * 8, bk + ((s * 2048) >> 4), ID_T_MN, s > 0);
#pragma unroll
      for (int s = 0; s < 4; ++s)
        mma_bf16_ts_w(tmem + TT_S, tmem + TT_X + 32 + s * 8, bk + ((s * 2048) >> 4), ID_T_MN, 1);
      mma_commit_w(bar_mma);
    }
    {
      // while dS is computed: O^T row v, tokens i in [32c, 32c+32) (D1 and D2 columns
      // that the state-update MMA does not touch)
      float o[16], qv[16];
      tmem_ld16(lane + TT_D2 + 64 + 16 * ch, o);
      tmem_ld16(lane + TT_D1 + 64 + 16 * ch, qv);
      tmem_ld_wait();
      if (L == kC) {
        // full chunk: stage the tile, one TMA store after the next barrier
        __nv_bfloat16* tile = reinterpret_cast<__nv_bfloat16*>(sm + T_OFF_O + b * 16384);
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const int ii = 16 * ch + i;
          tile[ii * kHeadDim + v] = __float2bfloat16_rn(p.scale * fmaf(sGam[ii], qv[i], o[i]));
        }
      } else {
        // partial (last) chunk: only its own tokens; rows past L belong to the next sequence
        __nv_bfloat16* dst = p.out + (cs * HV + h) * kHeadDim + v;
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const int ii = 16 * ch + i;
          if (ii < L)
            dst[static_cast<int64_t>(ii) * HV * kHeadDim] =
                __float2bfloat16_rn(p.scale * fmaf(sGam[ii], qv[i], o[i]));
        }
      }
      fence_async_smem();
    }
    ok = mbar_wait(bar_mma, mma_phase);
    mma_phase ^= 1;
    tc_fence_after();
    if (!__syncthreads_and(ok)) break;
    SPHASE(8);  // sync + G3 issue + O + wait
    {
      float d0[32];
      tmem_ld32(lane + TT_S + 32 * ch, d0);
      tmem_ld_wait();
      const float gl = sGam[kC - 1];
#pragma unroll
      for (int i = 0; i < 32; ++i) S[i] = fmaf(gl, S[i], d0[i]);
    }
    tc_fence_before();
    __syncthreads();  // every thread has read its dS columns before they are overwritten
    tc_fence_after();
    if (t == 0 && L == kC) {
      tma_store_3d(&maps.o, sm + T_OFF_O + b * 16384, 0, h, static_cast<int>(cs));
      bulk_commit();
    }
    write_s_operand();
    SPHASE(9);  // S update + operand
  }

  if (t == 0) bulk_wait_all();  // output stores complete before the block exits
  if (ok) {
#pragma unroll
    for (int i = 0; i < 32; i += 4)
      *reinterpret_cast<float4*>(p.new_state + sbase + i) =
          make_float4(S[i], S[i + 1], S[i + 2], S[i + 3]);
  } else if (t == 0 && p.status) {
    atomicExch(p.status, 1);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, kScanTTmemCols);
}

bool encode_v_map(CUtensorMap* map, const void* base, int64_t T, int HV) {
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) return false;
  const cuuint64_t dims[3] = {static_cast<cuuint64_t>(kHeadDim), static_cast<cuuint64_t>(HV),
                              static_cast<cuuint64_t>(T)};
  const cuuint64_t strides[2] = {static_cast<cuuint64_t>(kHeadDim) * 2,
                                 static_cast<cuuint64_t>(HV) * kHeadDim * 2};
  const cuuint32_t box[3] = {static_cast<cuuint32_t>(kHeadDim), 1, kC};
  const cuuint32_t estr[3] = {1, 1, 1};
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides,
             box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) ==
         CUDA_SUCCESS;
}

}  // namespace

// Workspace: [0, 256) status word; [256, ...) chunk offsets (N + 1 int64), then the
// scan order (N int32); then, 1024-aligned, 24 KB of [T_b; P] per (chunk, v-head).
static size_t head_bytes(int64_t N) {
  return (256 + 8 * static_cast<size_t>(N + 1) + 4 * static_cast<size_t>(N) + 1023) &
         ~size_t(1023);
}

size_t prefill_twophase_workspace_bytes(int64_t T, int64_t N, int HV) {
  const size_t head = head_bytes(N);
  const size_t chunks = static_cast<size_t>((T + kC - 1) / kC + N);
  return head + chunks * static_cast<size_t>(HV) * kA2Bytes;
}

int launch_prefill_twophase(const PrefillParams& p, void* workspace, cudaStream_t stream) {
  if (p.N == 0) return 0;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  int64_t* offs = reinterpret_cast<int64_t*>(ws + 256);
  int32_t* order = reinterpret_cast<int32_t*>(ws + 256 + 8 * (p.N + 1));
  const size_t head = head_bytes(p.N);
  uint8_t* a2 = ws + head;
  ChunkTmaps maps;
  const int64_t Tm = p.T > 0 ? p.T : 1;
  const void* kb = p.T > 0 ? static_cast<const void*>(p.k) : static_cast<const void*>(p.new_state);
  const void* qb = p.T > 0 ? static_cast<const void*>(p.q) : static_cast<const void*>(p.new_state);
  if (!encode_qk_map(&maps.k, kb, Tm, p.HQ) || !encode_qk_map(&maps.q, qb, Tm, p.HQ)) return -2;
  if (cudaFuncSetAttribute(prep_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kPrepSmem) !=
      cudaSuccess)
    return -1;
  chunk_offsets_kernel<<<1, 1024, 0, stream>>>(p, offs);
  scan_order_kernel<<<static_cast<unsigned>((p.N + 255) / 256), 256, 0, stream>>>(p.N, offs,
                                                                                 order);
  const int64_t cap = (p.T + kC - 1) / kC + p.N;
  if (p.T > 0) {
    prep_kernel<<<static_cast<unsigned>(cap * p.HV), kPrepThreads, kPrepSmem, stream>>>(p, maps, offs, a2);
  }
  ScanMaps smaps;
  smaps.k = maps.k;
  smaps.q = maps.q;
  const void* vb = p.T > 0 ? static_cast<const void*>(p.v) : static_cast<const void*>(p.new_state);
  void* ob = p.T > 0 ? static_cast<void*>(p.out) : static_cast<void*>(p.new_state);
  if (!encode_v_map(&smaps.v, vb, Tm, p.HV) || !encode_v_map(&smaps.o, ob, Tm, p.HV)) return -2;
  if (cudaFuncSetAttribute(scan_t_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           kScanTSmem) != cudaSuccess)
    return -1;
  scan_t_kernel<<<static_cast<unsigned>(p.N * p.HV), kScanTThreads, kScanTSmem, stream>>>(
      p, smaps, offs, order, a2);
  return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

}  // namespace gdn

#ifdef GDN_PHASE_PROFILE
extern "C" __attribute__((visibility("default"))) int gdn_debug_prep_cycles(long long* host,
                                                                              int reset) {
  if (cudaMemcpyFromSymbol(host, gdn::g_prep_cycles, sizeof(long long) * 16) != cudaSuccess)
    return -1;
  if (reset) {
    long long z[16] = {0};
    if (cudaMemcpyToSymbol(gdn::g_prep_cycles, z, sizeof(z)) != cudaSuccess) return -1;
  }
  return 0;
}
extern "C" __attribute__((visibility("default"))) int gdn_debug_scan_cycles(long long* host,
                                                                              int reset) {
  if (cudaMemcpyFromSymbol(host, gdn::g_scan_cycles, sizeof(long long) * 16) != cudaSuccess)
    return -1;
  if (reset) {
    long long z[16] = {0};
    if (cudaMemcpyToSymbol(gdn::g_scan_cycles, z, sizeof(z)) != cudaSuccess) return -1;
  }
  return 0;
}
#endif
