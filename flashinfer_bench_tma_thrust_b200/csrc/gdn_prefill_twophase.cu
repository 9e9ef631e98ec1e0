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
//   scan (one block per (sequence, v-head, 64-wide V tile), chunk by chunk):
//     [KH; QH] = [K;Q] H,  X = V - gamma KH,  [U; O'] = [T_b; P] X,
//     O = scale (gamma QH + O'),  H <- gamma_last H + K^T diag(f) U.
//
// The prep phase has (T/64 + N) x HV independent blocks, so the triangular solve
// and the operand construction run at full occupancy instead of on the critical
// path of each sequence; the scan keeps only the state chain and receives
// [T_b; P] with one bulk copy per chunk. P enters the tensor core as hi only (its
// rounding only touches the output, which is bf16), T_b as hi + lo.
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
    if (t == 0) {
      const Operand kq{smem_u32(sm + P_OFF_KQ), 0, false, 0, 0, 16384};
      issue_gemm(tmem + PT_S, kq, kq, ID_KK, 8);
      mma_commit(bar_mma);
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
      if (t == 0) {  // P = M T_b (result rows 0..63)
        const Operand mA{smem_u32(sm + P_OFF_M_HI), smem_u32(sm + P_OFF_M_LO), false, 0, 0, 0};
        const Operand tb{smem_u32(sm + P_OFF_TB_HI), smem_u32(sm + P_OFF_TB_LO), true, 8192,
                         2048, 0};
        issue_gemm(tmem + PT_P, mA, tb, ID_KM, 4);
        mma_commit(bar_mma);
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

// ------------------------------------------------------------------ scan
// Shared memory: KQ tile (32 KB; its Q halves hold X and then diag(f) U),
// H hi/lo (32 KB), [T_b; P] hi/lo (32 KB; lo rows 64..127 stay zero).
// 256 threads: thread t owns TMEM lane / operand row r = t % 128 and the 32
// columns [32 c, 32 c + 32) of it, c = t / 128 (warps w and w + 4 share lanes).
constexpr uint32_t S_OFF_KQ = 0;
constexpr uint32_t S_OFF_X_HI = 8192;
constexpr uint32_t S_OFF_X_LO = 24576;
constexpr uint32_t S_OFF_H_HI = 32768;
constexpr uint32_t S_OFF_H_LO = 49152;
constexpr uint32_t S_OFF_A2_HI = 65536;
constexpr uint32_t S_OFF_A2_LO = 81920;
constexpr uint32_t S_OFF_G = 98304;  // 2 x 64 fp32 (double-buffered by chunk parity)
constexpr uint32_t S_OFF_BETA = 98816;  // 2 x 64 fp32 (written by the gate scan, unused here)
constexpr uint32_t S_OFF_BAR = 99328;
constexpr uint32_t kScanSmem = 99392 + 1024;
constexpr uint32_t kScanTmemCols = 256;
constexpr uint32_t ST_1 = 64, ST_2 = 128, ST_3 = 192;  // columns 0..63 unused
constexpr int kScanThreads = 256;
// Thread that issues the MMAs, TMA and bulk copies: warp 3 (rows 96..127), whose own
// per-chunk work (output rows) is off the state chain, so the cycles it spends
// blocked on MMA issue do not delay the chain's conversions.
constexpr int kIssuer = 96;
// Warps 4-5 (threads 128..191, idle while the state-update MMA runs) load the raw
// gates and compute the next chunk's decays.
constexpr int kGateBase = 128;
constexpr int kHalf = kVT / 2;  // columns per thread

// Split 32 fp32 values into bf16 hi/lo and write them as chunks [c0, c0+4) of
// row `row` of two 128B-swizzled tiles.
__device__ __forceinline__ void store_half_row_split(uint8_t* hi, uint8_t* lo, uint32_t row,
                                                     uint32_t c0, const float* v) {
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    uint32_t hw[4], lw[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      split2(v[c * 8 + 2 * e], v[c * 8 + 2 * e + 1], hw[e], lw[e]);
    }
    const uint32_t off = sw128_chunk(row, c0 + c);
    *reinterpret_cast<uint4*>(hi + off) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
    *reinterpret_cast<uint4*>(lo + off) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
  }
}

__device__ __forceinline__ void tmem_ld32w(uint32_t taddr, float (&r)[32]) {
  tmem_ld32(taddr, r);
  tmem_ld_wait();
}

__global__ void __launch_bounds__(kScanThreads, 2)
    scan_kernel(const PrefillParams p, const __grid_constant__ ChunkTmaps maps,
                const int64_t* __restrict__ offs, const int32_t* __restrict__ order,
                const uint8_t* __restrict__ a2_in) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                           ~uintptr_t(1023));
  float* sG0 = reinterpret_cast<float*>(sm + S_OFF_G);
  float* sBeta0 = reinterpret_cast<float*>(sm + S_OFF_BETA);
  uint64_t* bar_tma = reinterpret_cast<uint64_t*>(sm + S_OFF_BAR);
  uint64_t* bar_a2 = bar_tma + 1;
  uint64_t* bar_mma = bar_tma + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + S_OFF_BAR + 32);

  const int t = threadIdx.x, warp = t >> 5;
  const int r = t & 127;         // row / TMEM lane
  const int ch = t >> 7;         // column half
  const int col0 = ch * kHalf;   // first column owned
  const int64_t unit = blockIdx.x;
  const int vt = static_cast<int>(unit % kTiles);
  const int h = static_cast<int>((unit / kTiles) % p.HV);
  const int64_t n = order[unit / (kTiles * p.HV)];
  const int qh = h / (p.HV / p.HQ);
  const int64_t HV = p.HV;
  int64_t start, end;
  seq_bounds(p, n, start, end);

  // state rows of this tile: S[n, h, vt*64 + v, k]; this thread owns k = r, v in its half
  const int64_t sbase = ((n * p.HV + h) * kHeadDim + vt * kVT + col0) * kHeadDim + r;
  float hrow[kHalf];
#pragma unroll
  for (int v = 0; v < kHalf; ++v) hrow[v] = p.state ? p.state[sbase + v * kHeadDim] : 0.0f;
  if (end <= start) {  // empty sequence: pass the state through
#pragma unroll
    for (int v = 0; v < kHalf; ++v) p.new_state[sbase + v * kHeadDim] = hrow[v];
    return;
  }
  const uint8_t* a2_seq = a2_in + static_cast<uint64_t>(offs[n]) * HV * kA2Bytes +
                          static_cast<uint64_t>(h) * kA2Bytes;
  const uint64_t a2_chunk_stride = static_cast<uint64_t>(HV) * kA2Bytes;

  auto issue_tma = [&](int64_t cs) {
    fence_async_smem();
    mbar_arrive_expect_tx(bar_tma, 4 * 8192);
    const int tok = static_cast<int>(cs);
    tma_load_3d(sm + S_OFF_KQ, &maps.k, bar_tma, 0, qh, tok);
    tma_load_3d(sm + S_OFF_KQ + 8192, &maps.q, bar_tma, 0, qh, tok);
    tma_load_3d(sm + S_OFF_KQ + 16384, &maps.k, bar_tma, 64, qh, tok);
    tma_load_3d(sm + S_OFF_KQ + 16384 + 8192, &maps.q, bar_tma, 64, qh, tok);
  };
  auto issue_a2 = [&](int64_t c) {
    fence_async_smem();
    mbar_arrive_expect_tx(bar_a2, kA2Bytes);
    const uint8_t* src = a2_seq + static_cast<uint64_t>(c) * a2_chunk_stride;
    bulk_load(sm + S_OFF_A2_HI, src, 16384, bar_a2);
    bulk_load(sm + S_OFF_A2_LO, src + 16384, 8192, bar_a2);
  };

  if (t == 0) {
    mbar_init(bar_tma, 1);
    mbar_init(bar_a2, 1);
    mbar_init(bar_mma, 1);
    fence_mbar_init();
  }
  if (warp == 0) tmem_alloc(tmem_slot, kScanTmemCols);
  // the lo half of [T_b; P] has no P rows: rows 64..127 stay zero
  for (int i = t; i < 8192 / 16; i += kScanThreads)
    reinterpret_cast<uint4*>(sm + S_OFF_A2_LO + 8192)[i] = make_uint4(0u, 0u, 0u, 0u);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t trow = tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16) + col0;
  store_half_row_split(sm + S_OFF_H_HI, sm + S_OFF_H_LO, r, ch * 4, hrow);

  const float A_log = load_scalar(p.A_log, p.A_log_dtype, h);
  const float dtb = load_scalar(p.dt_bias, p.dt_bias_dtype, h);
  auto load_gates = [&](int64_t cs, float& ra, float& rb) {
    if (t >= kGateBase && t < kGateBase + kC) {
      const int64_t tok = cs + (t - kGateBase);
      const bool valid = tok < end;
      ra = valid ? load_scalar(p.a, p.a_dtype, tok * HV + h) : 0.0f;
      rb = valid ? load_scalar(p.b, p.b_dtype, tok * HV + h) : 0.0f;
    }
  };

  uint32_t tma_phase = 0, a2_phase = 0, mma_phase = 0;
  bool ok = true;
  float ra = 0.f, rb = 0.f;
  if (t == kIssuer) {
    issue_tma(start);
    issue_a2(0);
  }
  load_gates(start, ra, rb);
  if (t >= kGateBase && t < kGateBase + kC)
    chunk_gates_w01(ra, rb, static_cast<int>((end - start) < kC ? (end - start) : kC), A_log,
                    dtb, sG0, sBeta0, kGateBase);
  __syncthreads();

  int64_t c = 0;
#ifdef GDN_PHASE_PROFILE
  long long sphase_last_ = clock64();
#endif
  for (int64_t cs = start; cs < end; cs += kC, ++c) {
    const int L = static_cast<int>((end - cs) < kC ? (end - cs) : kC);
    const int64_t next = cs + kC;
    const int buf = static_cast<int>(c & 1);
    const float* sG = sG0 + buf * kC;  // gates of this chunk (computed during the previous one)

    // ---- [KH; QH] = [K;Q] H --------------------------------------------------------
    SPHASE(0);  // loop top -> before TMA wait
    ok = mbar_wait(bar_tma, tma_phase);
    tma_phase ^= 1;
    SPHASE(1);  // TMA wait
    sync_before_mma();
    if (!__syncthreads_and(ok)) break;
    if (t == kIssuer) {
      const Operand kq{smem_u32(sm + S_OFF_KQ), 0, false, 0, 0, 16384};
      const Operand hB{smem_u32(sm + S_OFF_H_HI), smem_u32(sm + S_OFF_H_LO), true, 8192, 2048, 0};
      issue_gemm(tmem + ST_1, kq, hB, ID_KM, 8);
      mma_commit(bar_mma);
    }
    uint4 vraw[4];
    if (r < kC) {
      if (r < L) {
        const uint4* src = reinterpret_cast<const uint4*>(
            p.v + ((cs + r) * HV + h) * kHeadDim + vt * kVT + col0);
#pragma unroll
        for (int q = 0; q < 4; ++q) vraw[q] = src[q];
      } else {
#pragma unroll
        for (int q = 0; q < 4; ++q) vraw[q] = make_uint4(0u, 0u, 0u, 0u);
      }
    }
    float nra = 0.f, nrb = 0.f;
    if (next < end) load_gates(next, nra, nrb);
    SPHASE(2);  // G1 issue + V/gate loads
    ok = mbar_wait(bar_mma, mma_phase);
    mma_phase ^= 1;
    tc_fence_after();
    if (!__syncthreads_and(ok)) break;

    const float g_last = sG[kC - 1];
    if (r < kC) {
      // X row j = r: V_j - gamma_j (K H)_j, into the dead Q half of the tile
      float xr[32];
      tmem_ld32w(trow + ST_1, xr);
      const float gam = ex2(sG[r]);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const uint32_t w[4] = {vraw[q].x, vraw[q].y, vraw[q].z, vraw[q].w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          xr[q * 8 + 2 * e] = __uint_as_float(w[e] << 16) - gam * xr[q * 8 + 2 * e];
          xr[q * 8 + 2 * e + 1] = __uint_as_float(w[e] & 0xffff0000u) - gam * xr[q * 8 + 2 * e + 1];
        }
      }
      store_half_row_split(sm + S_OFF_X_HI, sm + S_OFF_X_LO, r, ch * 4, xr);
    }
    SPHASE(3);  // G1 wait + X build

    // ---- [U; O'] = [T_b; P] X ---------------------------------------------------------
    ok = mbar_wait(bar_a2, a2_phase);
    a2_phase ^= 1;
    SPHASE(4);  // A2 wait
    sync_before_mma();
    if (!__syncthreads_and(ok)) break;
    if (t == kIssuer) {
      const Operand a2{smem_u32(sm + S_OFF_A2_HI), smem_u32(sm + S_OFF_A2_LO), false, 0, 0, 0};
      const Operand xb{smem_u32(sm + S_OFF_X_HI), smem_u32(sm + S_OFF_X_LO), true, 8192, 2048, 0};
      issue_gemm(tmem + ST_2, a2, xb, ID_KM, 4);
      mma_commit(bar_mma);
    }
    SPHASE(5);  // G2 issue
    ok = mbar_wait(bar_mma, mma_phase);
    mma_phase ^= 1;
    tc_fence_after();
    if (!__syncthreads_and(ok)) break;
    if (t == kIssuer && next < end) issue_a2(c + 1);  // [T_b; P] of this chunk is consumed
    if (r < kC) {
      // f_j U_j with f_j = e^{Gamma_last - Gamma_j} (0 for padded rows): the state
      // update then reads the raw K tile, dH = K^T diag(f) U
      float u[32];
      tmem_ld32w(trow + ST_2, u);
      const float f = (r < L) ? ex2(g_last - sG[r]) : 0.0f;
#pragma unroll
      for (int v = 0; v < kHalf; ++v) u[v] *= f;
      store_half_row_split(sm + S_OFF_X_HI, sm + S_OFF_X_LO, r, ch * 4, u);
    }
    SPHASE(6);  // G2 wait + U build

    // ---- dH = K^T diag(f) U (into its own TMEM columns, so O' stays readable) -------------
    sync_before_mma();
    if (t == kIssuer) {
      const Operand kt{smem_u32(sm + S_OFF_KQ), 0, true, 16384, 2048, 0};
      const Operand ub{smem_u32(sm + S_OFF_X_HI), smem_u32(sm + S_OFF_X_LO), true, 8192, 2048, 0};
      issue_gemm(tmem + ST_3, kt, ub, ID_MM, 4);
      mma_commit(bar_mma);
    }
    // while the MMA runs: rows 64..127 produce the output, warps 0-1 the gates of the
    // next chunk (into the other gate buffer)
    if (r >= kC) {
      const int i = r - kC;
      float o[32], qhv[32];
      tmem_ld32(trow + ST_2, o);
      tmem_ld32(trow + ST_1, qhv);
      tmem_ld_wait();
      if (i < L) {
        const float gam = ex2(sG[i]);
        __nv_bfloat16* dst = p.out + ((cs + i) * HV + h) * kHeadDim + vt * kVT + col0;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          uint32_t w[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int v0 = q * 8 + 2 * e;
            const float o0 = p.scale * fmaf(gam, qhv[v0], o[v0]);
            const float o1 = p.scale * fmaf(gam, qhv[v0 + 1], o[v0 + 1]);
            w[e] = pack2_rn(o0, o1);
          }
          *reinterpret_cast<uint4*>(dst + q * 8) = make_uint4(w[0], w[1], w[2], w[3]);
        }
      }
    } else if (t >= kGateBase && t < kGateBase + kC && next < end) {
      const int nL = static_cast<int>((end - next) < kC ? (end - next) : kC);
      chunk_gates_w01(nra, nrb, nL, A_log, dtb, sG0 + (buf ^ 1) * kC, sBeta0 + (buf ^ 1) * kC,
                      kGateBase);
    }
    SPHASE(7);  // G3 issue + O + next gates
    ok = mbar_wait(bar_mma, mma_phase);
    mma_phase ^= 1;
    tc_fence_after();
    if (!__syncthreads_and(ok)) break;
    SPHASE(8);  // G3 wait
    if (t == kIssuer && next < end) issue_tma(next);
    {
      // the fp32 state row stays in registers for the whole sequence
      float dh[32];
      tmem_ld32w(trow + ST_3, dh);
      const float gl = ex2(g_last);
#pragma unroll
      for (int v = 0; v < kHalf; ++v) hrow[v] = fmaf(gl, hrow[v], dh[v]);
      store_half_row_split(sm + S_OFF_H_HI, sm + S_OFF_H_LO, r, ch * 4, hrow);
    }
    SPHASE(9);  // H update
  }

  if (ok) {
#pragma unroll
    for (int v = 0; v < kHalf; ++v) p.new_state[sbase + v * kHeadDim] = hrow[v];
  } else if (t == kIssuer && p.status) {
    atomicExch(p.status, 1);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, kScanTmemCols);
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
          cudaSuccess ||
      cudaFuncSetAttribute(scan_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kScanSmem) !=
          cudaSuccess)
    return -1;
  chunk_offsets_kernel<<<1, 1024, 0, stream>>>(p, offs);
  scan_order_kernel<<<static_cast<unsigned>((p.N + 255) / 256), 256, 0, stream>>>(p.N, offs,
                                                                                 order);
  const int64_t cap = (p.T + kC - 1) / kC + p.N;
  if (p.T > 0) {
    prep_kernel<<<static_cast<unsigned>(cap * p.HV), kPrepThreads, kPrepSmem, stream>>>(p, maps, offs, a2);
  }
  scan_kernel<<<static_cast<unsigned>(p.N * p.HV * kTiles), kScanThreads, kScanSmem, stream>>>(p, maps,
                                                                                     offs, order,
                                                                                     a2);
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
