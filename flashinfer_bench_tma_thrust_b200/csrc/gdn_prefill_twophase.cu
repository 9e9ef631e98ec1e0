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
#include <cstdlib>
#include <mutex>

#include "gdn_launch.h"

namespace gdn {
namespace {

using namespace sm100;
using namespace chunk;

constexpr uint32_t kA2Bytes = 24576;     // [T_b; P] image: hi 16 KB | T_b lo 8 KB
constexpr uint32_t kGateBytes = 512;     // gamma_j (64 fp32), then f_j (64 fp32)
constexpr uint32_t kUnitBytes = kA2Bytes + kGateBytes;  // per (chunk, v-head)


// Status word bits (sticky, in the workspace): a bounded wait gave up; cu_seqlens held a
// value outside [0, T] (used clamped) or ranges whose chunks overflow the workspace
// (overlapping sequences: the call then computes nothing and passes states through).
constexpr int kStatusWaitTimeout = 1;
constexpr int kStatusBadSeqlens = 2;

// Capacity of the workspace in (chunk) units per v-head: ceil(T / 64) + N.
__device__ __forceinline__ int64_t unit_capacity(const PrefillParams& p) {
  return (p.T + kC - 1) / kC + p.N;
}

__device__ __forceinline__ void seq_bounds(const PrefillParams& p, int64_t n, int64_t& start,
                                           int64_t& end) {
  start = load_index(p.cu_seqlens, p.cu_dtype, n);
  end = load_index(p.cu_seqlens, p.cu_dtype, n + 1);
  start = start < 0 ? 0 : (start > p.T ? p.T : start);
  end = end < 0 ? 0 : (end > p.T ? p.T : end);
}

// ------------------------------------------------------------------ chunk offsets
// offs[n] = number of 64-token chunks in sequences 0..n-1 (offs[0] = 0). One block.
constexpr int64_t kInlineSortN = 1024;  // scan order computed by this kernel up to here
__global__ void __launch_bounds__(1024) chunk_offsets_kernel(const PrefillParams p,
                                                             int64_t* offs, int32_t* order,
                                                             int64_t* eoffs, int split_q) {
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
      const int64_t rs = load_index(p.cu_seqlens, p.cu_dtype, n);
      const int64_t re = load_index(p.cu_seqlens, p.cu_dtype, n + 1);
      if ((rs < 0 || rs > p.T || re < 0 || re > p.T) && p.status)
        atomicOr(p.status, kStatusBadSeqlens);
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
  if (t == 0 && carry > unit_capacity(p) && p.status) atomicOr(p.status, kStatusBadSeqlens);
  if (p.N <= kInlineSortN) {
    // the scan order (as scan_order_kernel: longest first, ties by index), one sequence
    // per thread over chunk counts held in shared memory; saves that kernel's launch
    __shared__ int64_t s_cnt[kInlineSortN];
    if (t < p.N) s_cnt[t] = offs[t + 1] - offs[t];  // this block's own writes, synced above
    __syncthreads();
    if (t < p.N) {
      const int64_t cn = s_cnt[t];
      int64_t rank = 0;
      for (int64_t m = 0; m < p.N; ++m) {
        const int64_t cm = s_cnt[m];
        rank += (cm > cn || (cm == cn && m < t)) ? 1 : 0;
      }
      order[rank] = static_cast<int32_t>(t);
    }
    if (split_q > 0 && t == 0) {
      // split call: sequence n's first floor(cnt_n split_q / 1024) chunks are "early"
      // (prep before the scan's first part); eoffs = their prefix sums
      int64_t e = 0;
      eoffs[0] = 0;
      for (int64_t n = 0; n < p.N; ++n) {
        e += (s_cnt[n] * split_q) >> 10;
        eoffs[n + 1] = e;
      }
    }
  }
}

// ------------------------------------------------------------------ chunk gates
// One warp per (chunk, v-head), tokens l and l + 32 per lane: the gates (accurate
// softplus / exp / sigmoid), the in-chunk cumulative log2 decay G_j (an inclusive scan
// of each half of the chunk, the first half's total added to the second — the same
// operations in the same order as a two-warp scan) and beta_j. Written into the unit:
// the scan's gates (gamma_j = 2^{G_j}, f_j = 2^{G_last - G_j}) at their place after
// the image, and G_j, beta_j for the prep in the image's first 512 bytes (the prep
// reads them first and overwrites them with T_b later). Taking this off the prep
// blocks removes two block-wide barriers and the gate arithmetic (two warps busy while
// six wait) from the start of every prep block.
__global__ void __launch_bounds__(256) chunk_gates_kernel(const PrefillParams p,
                                                          const int64_t* __restrict__ offs,
                                                          int64_t* __restrict__ table,
                                                          uint8_t* __restrict__ a2_out,
                                                          const int64_t* __restrict__ eoffs,
                                                          longlong2* __restrict__ elist,
                                                          longlong2* __restrict__ llist) {
  const int lane = threadIdx.x & 31;
  const int64_t gw = static_cast<int64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5);
  const int64_t gchunk = gw / p.HV;
  const int h = static_cast<int>(gw % p.HV);
  const int64_t total = offs[p.N];
  if (gchunk >= total || total > unit_capacity(p)) return;
  int64_t lo = 0, hi = p.N;  // the sequence holding the chunk: the last n with offs[n] <= g
  while (lo < hi) {
    const int64_t mid = (lo + hi + 1) >> 1;
    if (offs[mid] <= gchunk) lo = mid;
    else hi = mid - 1;
  }
  int64_t start, end;
  seq_bounds(p, lo, start, end);
  const int64_t cs = start + (gchunk - offs[lo]) * kC;
  const int L = static_cast<int>((end - cs) < kC ? (end - cs) : kC);
  // the chunk table entry for the prep blocks: first token and length; in a split call
  // also the chunk's place in the early or the late unit list
  if (h == 0 && lane == 0) {
    table[gchunk] = cs * 128 + L;
    if (eoffs) {
      const int64_t k = gchunk - offs[lo], spn = eoffs[lo + 1] - eoffs[lo];
      const longlong2 e = make_longlong2(gchunk, cs * 128 + L);
      if (k < spn) elist[eoffs[lo] + k] = e;
      else llist[(offs[lo] - eoffs[lo]) + (k - spn)] = e;
    }
  }
  const float A_log = load_scalar(p.A_log, p.A_log_dtype, h);
  const float dtb = load_scalar(p.dt_bias, p.dt_bias_dtype, h);
  const bool v0 = lane < L, v1 = lane + 32 < L;
  float ra0 = 0.f, rb0 = 0.f, ra1 = 0.f, rb1 = 0.f;
  if (v0) {
    ra0 = load_scalar(p.a, p.a_dtype, (cs + lane) * p.HV + h);
    rb0 = load_scalar(p.b, p.b_dtype, (cs + lane) * p.HV + h);
  }
  if (v1) {
    ra1 = load_scalar(p.a, p.a_dtype, (cs + lane + 32) * p.HV + h);
    rb1 = load_scalar(p.b, p.b_dtype, (cs + lane + 32) * p.HV + h);
  }
  float x0 = v0 ? gate_log_decay(A_log, ra0, dtb) * kLog2e : 0.0f;
  float x1 = v1 ? gate_log_decay(A_log, ra1, dtb) * kLog2e : 0.0f;
  const float b0 = v0 ? gate_beta(rb0) : 0.0f, b1 = v1 ? gate_beta(rb1) : 0.0f;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const float y0 = __shfl_up_sync(0xffffffffu, x0, o);
    const float y1 = __shfl_up_sync(0xffffffffu, x1, o);
    if (lane >= o) {
      x0 += y0;
      x1 += y1;
    }
  }
  x1 += __shfl_sync(0xffffffffu, x0, 31);
  const float glast = __shfl_sync(0xffffffffu, x1, 31);
  uint8_t* unit = a2_out + (static_cast<uint64_t>(gchunk) * p.HV + h) * kUnitBytes;
  float* gp = reinterpret_cast<float*>(unit);
  gp[lane] = x0;
  gp[lane + 32] = x1;
  gp[kC + lane] = b0;
  gp[kC + lane + 32] = b1;
  float* gd = reinterpret_cast<float*>(unit + kA2Bytes);
  gd[lane] = ex2(x0);
  gd[lane + 32] = ex2(x1);
  gd[kC + lane] = v0 ? ex2(glast - x0) : 0.0f;
  gd[kC + lane + 32] = v1 ? ex2(glast - x1) : 0.0f;
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
// 256 threads; thread t owns TMEM lane / row t % 128 and a 32-column half of it. Four
// blocks per SM (64 registers, 52 KB of shared memory, 128 TMEM columns each).
// Shared memory: the K/Q tile (32 KB, TMA) is dead after S; then M hi/lo (rows 0..63 of
// the A operand of P = M T_b: the operand reads 128 rows, the rows after M lo are A's
// and their results are not used), the fp32 A and T of the solve (padded rows, 17 KB
// each), and T_b hi/lo over A once the solve no longer reads it.
constexpr uint32_t P_OFF_KQ = 0;
constexpr uint32_t P_OFF_M_HI = 0;
constexpr uint32_t P_OFF_M_LO = 8192;
constexpr uint32_t P_OFF_AF = 16384;
constexpr uint32_t P_OFF_TF = 33792;
constexpr uint32_t P_OFF_TB_HI = 16384;
constexpr uint32_t P_OFF_TB_LO = 24576;
constexpr uint32_t P_OFF_G = 51200;
constexpr uint32_t P_OFF_BETA = 51456;
constexpr uint32_t P_OFF_BAR = 51712;
constexpr uint32_t kPrepSmem = 51776 + 1024;
constexpr uint32_t kPrepTmemCols = 128;
constexpr uint32_t PT_S = 0, PT_P = 64;
constexpr int kPrepThreads = 256;

template <int mode>
__global__ void __launch_bounds__(kPrepThreads, 4)
    prep_kernel(const PrefillParams p, const __grid_constant__ ChunkTmaps maps,
                const int64_t* __restrict__ offs, const int64_t* __restrict__ table,
                uint8_t* __restrict__ a2_out, const int64_t* __restrict__ eoffs,
                const longlong2* __restrict__ list) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = align_smem<1024>(smem_raw);
  float* sAf = reinterpret_cast<float*>(sm + P_OFF_AF);
  float* sTf = reinterpret_cast<float*>(sm + P_OFF_TF);
  float* sG = reinterpret_cast<float*>(sm + P_OFF_G);
  float* sBeta = reinterpret_cast<float*>(sm + P_OFF_BETA);
  uint64_t* bar_tma = reinterpret_cast<uint64_t*>(sm + P_OFF_BAR);
  uint64_t* bar_mma = bar_tma + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + P_OFF_BAR + 16);

  const int t = threadIdx.x, warp = t >> 5, r = t & 127, c0 = (t >> 7) * 32;
  const int h = static_cast<int>(blockIdx.x % p.HV);
  int64_t gchunk, entry;
  if constexpr (mode == 0) {  // every unit, in chunk order
    gchunk = blockIdx.x / p.HV;
    const int64_t total = offs[p.N];
    entry = gchunk < unit_capacity(p) ? table[gchunk] : 0;
    if (gchunk >= total || total > unit_capacity(p)) return;  // (overflow: nothing written)
  } else {  // split call: the early (mode 1) or late (mode 2) units, from their list
    const int64_t pos = blockIdx.x / p.HV;
    const int64_t total = offs[p.N], ne = eoffs[p.N];
    if (total > unit_capacity(p) || pos >= (mode == 1 ? ne : total - ne)) return;
    const longlong2 e = list[pos];
    gchunk = e.x;
    entry = e.y;
  }
  const int64_t cs = entry >> 7;  // (the chunk's length, entry & 127, is the gates kernel's)
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
  if (t < kC) {  // G_j and beta_j, written into this unit by chunk_gates_kernel
    const float* gp = reinterpret_cast<const float*>(
        a2_out + (static_cast<uint64_t>(gchunk) * p.HV + h) * kUnitBytes);
    sG[t] = gp[t];
    sBeta[t] = gp[kC + t];
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t trow = tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16) + c0;

  // S = [K;Q] K^T: only the K/Q tile (TMA-written) feeds it, so warp 0 issues it as
  // soon as its own wait for the copy returns, with no block-wide barrier; every thread
  // then waits for the MMA's completion before the tile's space is reused
  bool ok = true;
  if (t < 32) {
    ok = mbar_wait(bar_tma, 0);
    if (__all_sync(0xffffffffu, ok)) {
      const Operand kq{smem_u32(sm + P_OFF_KQ), 0, false, 0, 0, 16384};
      issue_gemm(tmem + PT_S, kq, kq, ID_KK, 8);
      mma_commit_w(bar_mma);
    }
  }
  ok = mbar_wait(bar_mma, 0) && ok;
  tc_fence_after();
  {
    {
      // the K/Q tile is dead: M and A reuse its space (after a failed wait this reads
      // stale TMEM, and the barrier below stops the block)
      build_a_m_256<PadLayout>(trow + PT_S, sAf, sG, sBeta, sm + P_OFF_M_HI, sm + P_OFF_M_LO);
    }
    ok = __syncthreads_and(ok);  // (so that thread 0 reports a failure seen by any thread)
    if (ok) {
      solve_tb_256<PadLayout>(sAf, sTf, sBeta, sm + P_OFF_TB_HI, sm + P_OFF_TB_LO);
      sync_before_mma();
      if (t < 32) {  // warp 0 issues  // P = M T_b (result rows 0..63)
        const Operand mA{smem_u32(sm + P_OFF_M_HI), smem_u32(sm + P_OFF_M_LO), false, 0, 0, 0};
        const Operand tb{smem_u32(sm + P_OFF_TB_HI), smem_u32(sm + P_OFF_TB_LO), true, 8192,
                         2048, 0};
        issue_gemm(tmem + PT_P, mA, tb, ID_KM, 4);
        mma_commit_w(bar_mma);
      }
      // meanwhile: the T_b rows of [T_b; P] are the T_b tiles themselves (same swizzled
      // row image): bulk-copy hi to rows 0..63 of the hi part, lo to the lo part
      uint8_t* dst = a2_out + (static_cast<uint64_t>(gchunk) * p.HV + h) * kUnitBytes;
      if (t == 32) {
        bulk_store(dst, sm + P_OFF_TB_HI, 8192);
        bulk_store(dst + 16384, sm + P_OFF_TB_LO, 8192);
        bulk_commit();
      }
      ok = mbar_wait(bar_mma, 1);
      tc_fence_after();
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
    }
  }
  if (t == 32) bulk_wait_all();  // the T_b tiles stay in place until copied
  if (!ok && t == 0 && p.status) atomicOr(p.status, kStatusWaitTimeout);
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, kPrepTmemCols);
}

// ------------------------------------------------------------------ scan: shared pieces
constexpr uint32_t kScanTTmemCols = 512;
constexpr uint32_t ID_T_K = idesc_bf16(128, 128, false, false);   // B K-major
constexpr uint32_t ID_T_MN = idesc_bf16(128, 128, false, true);   // B MN-major
// N = 64: the lo (correction) terms are taken only for the columns that feed the state
// (KH and U); the QH and PX columns reach the bf16 output alone and take hi x hi
constexpr uint32_t ID_T_K64 = idesc_bf16(128, 64, false, false);

struct ScanMaps {
  CUtensorMap k, q, v;
};

// 2n fp32 -> n bf16x2 words, hi and lo parts
template <int NW>
__device__ __forceinline__ void split_words(const float* x, uint32_t (&hi)[NW], uint32_t (&lo)[NW]) {
#pragma unroll
  for (int w = 0; w < NW; ++w) split2(x[2 * w], x[2 * w + 1], hi[w], lo[w]);
}

// ------------------------------------------------------------------ scan: MMA groups
// Each group of the scan's products is issued from one asm block: one elect.sync, the
// accumulate predicates set once, the per-K-step operand offsets as immediates. The
// issuing warp shares its SM sub-partition with four busy state warps; with fewer
// instructions per MMA the group is issued faster when the sub-partition's issue slots
// are contended (a micro-benchmark with four FMA-bound warps beside the issuer: 2.0 K
// cycles for the 16-MMA group against 3.1 K with one elect.sync per MMA). Called by all
// lanes of the issuing warp.

// G1a: D (128 x 128) = A^T-operand in TMEM (thread quarter layout: K step s hi at
// 32 (s/2) + 8 (s%2), lo 16 further) x K-major B tile with two 64-wide K atoms
// (16 KB apart): 8 hi steps at N = 128, 8 lo steps at N = 64.
__device__ __forceinline__ void mma_group_g1a(uint32_t d, uint32_t a, uint64_t b) {
  asm volatile(
      "{\n\t.reg .pred e, pf, pt;\n\t.reg .b64 bb;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "setp.ne.b32 pf, 0, 0;\n\tsetp.eq.b32 pt, 0, 0;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, pf;\n\t"
      "add.s64 bb, %2, 2;\n\t@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%5], bb, %3, pt;\n\t"
      "add.s64 bb, %2, 4;\n\t@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%6], bb, %3, pt;\n\t"
      "add.s64 bb, %2, 6;\n\t@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%7], bb, %3, pt;\n\t"
      "add.s64 bb, %2, 1024;\n\t@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%8], bb, %3, pt;\n\t"
      "add.s64 bb, %2, 1026;\n\t@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%9], bb, %3, pt;\n\t"
      "add.s64 bb, %2, 1028;\n\t@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%10], bb, %3, pt;\n\t"
      "add.s64 bb, %2, 1030;\n\t@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%11], bb, %3, pt;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%12], %2, %4, pt;\n\t"
      "add.s64 bb, %2, 2;\n\t@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%13], bb, %4, pt;\n\t"
      "add.s64 bb, %2, 4;\n\t@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%14], bb, %4, pt;\n\t"
      "add.s64 bb, %2, 6;\n\t@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%15], bb, %4, pt;\n\t"
      "add.s64 bb, %2, 1024;\n\t@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%16], bb, %4, pt;\n\t"
      "add.s64 bb, %2, 1026;\n\t@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%17], bb, %4, pt;\n\t"
      "add.s64 bb, %2, 1028;\n\t@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%18], bb, %4, pt;\n\t"
      "add.s64 bb, %2, 1030;\n\t@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%19], bb, %4, pt;\n\t"
      "}" ::"r"(d), "r"(a), "l"(b), "r"(ID_T_K), "r"(ID_T_K64), "r"(a + 8), "r"(a + 32),
      "r"(a + 40), "r"(a + 64), "r"(a + 72), "r"(a + 96), "r"(a + 104), "r"(a + 16),
      "r"(a + 24), "r"(a + 48), "r"(a + 56), "r"(a + 80), "r"(a + 88), "r"(a + 112),
      "r"(a + 120)
      : "memory");
}

// G2 / G1': D = A x B over a 64-deep K: A in TMEM with each 16-column group holding one
// K step's hi (columns 0..7) and lo (8..15); B a K-major tile (hi; lo for the first 64
// rows only). Three-term split product: 4 x (hi hi, N = 128), 4 x (lo hi, N = 64),
// 4 x (hi lo, N = 64). `acc` = accumulate onto D from the first MMA.
__device__ __forceinline__ void mma_group_x3(uint32_t d, uint32_t a, uint64_t bh, uint64_t bl,
                                             uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred e, p0, pt;\n\t.reg .b64 bb;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "setp.ne.b32 p0, %5, 0;\n\tsetp.eq.b32 pt, 0, 0;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %6, p0;\n\t"
      "add.s64 bb, %2, 2;\n\t@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%8], bb, %6, pt;\n\t"
      "add.s64 bb, %2, 4;\n\t@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%9], bb, %6, pt;\n\t"
      "add.s64 bb, %2, 6;\n\t@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%10], bb, %6, pt;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%11], %2, %7, pt;\n\t"
      "add.s64 bb, %2, 2;\n\t@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%12], bb, %7, pt;\n\t"
      "add.s64 bb, %2, 4;\n\t@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%13], bb, %7, pt;\n\t"
      "add.s64 bb, %2, 6;\n\t@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%14], bb, %7, pt;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %3, %7, pt;\n\t"
      "add.s64 bb, %3, 2;\n\t@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%8], bb, %7, pt;\n\t"
      "add.s64 bb, %3, 4;\n\t@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%9], bb, %7, pt;\n\t"
      "add.s64 bb, %3, 6;\n\t@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%10], bb, %7, pt;\n\t"
      "}" ::"r"(d), "r"(a), "l"(bh), "l"(bl), "r"(0u), "r"(acc), "r"(ID_T_K), "r"(ID_T_K64),
      "r"(a + 16), "r"(a + 32), "r"(a + 48), "r"(a + 8), "r"(a + 24), "r"(a + 40), "r"(a + 56)
      : "memory");
}

// G3: D (128 x 128) = A (layout of mma_group_x3) x MN-major K tile (2048 B per K step):
// 4 x hi, 4 x lo, N = 128, the first MMA overwriting D.
__device__ __forceinline__ void mma_group_g3(uint32_t d, uint32_t a, uint64_t b) {
  asm volatile(
      "{\n\t.reg .pred e, pf, pt;\n\t.reg .b64 bb;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "setp.ne.b32 pf, 0, 0;\n\tsetp.eq.b32 pt, 0, 0;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, pf;\n\t"
      "add.s64 bb, %2, 128;\n\t@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%4], bb, %3, pt;\n\t"
      "add.s64 bb, %2, 256;\n\t@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%5], bb, %3, pt;\n\t"
      "add.s64 bb, %2, 384;\n\t@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%6], bb, %3, pt;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%7], %2, %3, pt;\n\t"
      "add.s64 bb, %2, 128;\n\t@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%8], bb, %3, pt;\n\t"
      "add.s64 bb, %2, 256;\n\t@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%9], bb, %3, pt;\n\t"
      "add.s64 bb, %2, 384;\n\t@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%10], bb, %3, pt;\n\t"
      "}" ::"r"(d), "r"(a), "l"(b), "r"(ID_T_MN), "r"(a + 16), "r"(a + 32), "r"(a + 48),
      "r"(a + 8), "r"(a + 24), "r"(a + 40), "r"(a + 56)
      : "memory");
}

// B_m^T = [K;Q]_{m+1} K_m^T: 8 shared-memory x shared-memory steps (K-major, two K atoms
// 16 KB apart), N = 64, the first MMA overwriting D.
__device__ __forceinline__ void mma_group_b(uint32_t d, uint64_t a, uint64_t b) {
  asm volatile(
      "{\n\t.reg .pred e, pf, pt;\n\t.reg .b64 aa, bb;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "setp.ne.b32 pf, 0, 0;\n\tsetp.eq.b32 pt, 0, 0;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, pf;\n\t"
      "add.s64 aa, %1, 2;\n\tadd.s64 bb, %2, 2;\n\t@e tcgen05.mma.cta_group::1.kind::f16 [%0], aa, bb, %3, pt;\n\t"
      "add.s64 aa, %1, 4;\n\tadd.s64 bb, %2, 4;\n\t@e tcgen05.mma.cta_group::1.kind::f16 [%0], aa, bb, %3, pt;\n\t"
      "add.s64 aa, %1, 6;\n\tadd.s64 bb, %2, 6;\n\t@e tcgen05.mma.cta_group::1.kind::f16 [%0], aa, bb, %3, pt;\n\t"
      "add.s64 aa, %1, 1024;\n\tadd.s64 bb, %2, 1024;\n\t@e tcgen05.mma.cta_group::1.kind::f16 [%0], aa, bb, %3, pt;\n\t"
      "add.s64 aa, %1, 1026;\n\tadd.s64 bb, %2, 1026;\n\t@e tcgen05.mma.cta_group::1.kind::f16 [%0], aa, bb, %3, pt;\n\t"
      "add.s64 aa, %1, 1028;\n\tadd.s64 bb, %2, 1028;\n\t@e tcgen05.mma.cta_group::1.kind::f16 [%0], aa, bb, %3, pt;\n\t"
      "add.s64 aa, %1, 1030;\n\tadd.s64 bb, %2, 1030;\n\t@e tcgen05.mma.cta_group::1.kind::f16 [%0], aa, bb, %3, pt;\n\t"
      "}" ::"r"(d), "l"(a), "l"(b), "r"(ID_KK)
      : "memory");
}

// ------------------------------------------------------------------ scan, pipelined
// The state product of chunk c+1 is split so that most of it leaves the chain:
// with S_{c+1} = g_c S_c + U'_c^T K_c (g_c = gamma_last of chunk c),
//   D1_{c+1} = S_{c+1} [K;Q]_{c+1}^T
//            = (g_c S_c) [K;Q]_{c+1}^T          (G1a: needs only S_c)
//            + U'_c^T ([K;Q]_{c+1} K_c^T)^T     (G1': 64-deep, after U'_c)
// so the chain of one chunk is X_c -> G2_c -> U'_c -> G1'_c -> X_{c+1}; G1a_{c+1}, the
// state product G3_c (dS_c = U'_c^T K_c), the state update and B_c = [K;Q]_{c+1} K_c^T
// (exact bf16 operands) run beside it. G2_c writes its [U^T | (PX)^T] over D1_c
// (the (QH)^T half of D1_c is read for the output before G2's result is consumed).
//
// Warp roles: warps 0-15 (512 threads) own the state: thread t holds row v = t % 128
// and quarter c = t / 128 of every row-sliced quantity (32 state columns, 16 columns of
// X / U / output), and compute everything on CUDA cores; warp 16 issues every MMA and
// every copy and does nothing else, so that an issue that blocks on a full MMA queue
// never delays the state warps. 96 registers per thread (17 warps: at most five share
// an SM sub-partition's register file). The state warps tell the issuer that an
// operand is ready through mbarriers (one arrival per warp); the issuer's commits tell
// the state warps that a product is done.
constexpr int kScanWThreads = 544;
constexpr int kScanWState = 512;          // state threads (warps 0-15)
constexpr uint32_t kStateBar = 1;         // named barrier of the state threads
constexpr uint32_t Q_OFF_KQ = 0;          // 3 x 32 KB
constexpr uint32_t Q_OFF_A2 = 98304;      // 2 x 24 KB: [T_b; P] hi 16 KB | T_b lo 8 KB
constexpr uint32_t Q_OFF_V = 147456;      // 2 x 16 KB: V tile, rows j x 128 v
constexpr uint32_t Q_OFF_B = 180224;      // B_c^T image: hi 16 KB (128 rows) | lo 8 KB (K rows)
constexpr uint32_t Q_OFF_GATES = 204800;  // 2 x (gamma_j, f_j): 2 x 512 B, from the prep
constexpr uint32_t Q_OFF_BAR = 206848;    // 15 mbarriers, TMEM slot
constexpr uint32_t kScanWSmem = 206848 + 512 + 1024;
// operand g S: thread quarter c writes columns [32c, 32c + 32) as 16 hi words then 16 lo
// words (K step s: hi at 32 (s/2) + 8 (s%2), lo 16 further); dS (fp32) from G3
constexpr uint32_t TP_S = 0;
// D1 of even / odd chunks: [(KH)^T | (QH)^T]. Each thread then writes X^T, later U'^T,
// over its own 16 fp32 columns of (KH)^T as 8 hi words followed by 8 lo words (so no
// thread overwrites columns another thread has yet to read); as an A operand, K step s
// is hi at column 16 s and lo at 16 s + 8. B_{c}^T accumulates in the (QH)^T half of
// D1_{c+1}'s buffer, free until G1a_{c+1}.
constexpr uint32_t TP_D1 = 128;  // 2 x 128
constexpr uint32_t TP_GO = 384;  // G2's result [U^T | (PX)^T]

template <int mode>
__global__ void __launch_bounds__(kScanWThreads, 1)
    scan_w_kernel(const PrefillParams p, const __grid_constant__ ScanMaps maps,
                  const int64_t* __restrict__ offs, const int32_t* __restrict__ order,
                  const uint8_t* __restrict__ a2_in, const int64_t* __restrict__ eoffs) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = align_smem<1024>(smem_raw);
  uint64_t* bar_kq = reinterpret_cast<uint64_t*>(sm + Q_OFF_BAR);  // [3] K/Q tiles
  uint64_t* bar_va = bar_kq + 3;                                   // [2] V + [T_b; P]
  uint64_t* bar_g2 = bar_kq + 5;    // commits: G2
  uint64_t* bar_tb = bar_kq + 6;    //          B_c
  uint64_t* bar_ch = bar_kq + 7;    //          D1 complete (G1'; G1a_0 in the prologue)
  uint64_t* bar_g3 = bar_kq + 8;    //          G3
  uint64_t* bar_g1a = bar_kq + 9;   //          G1a
  uint64_t* bar_x = bar_kq + 10;    // state warps: X^T stored
  uint64_t* bar_op = bar_kq + 11;   //              S operand stored, B_c read
  uint64_t* bar_u = bar_kq + 12;    //              U'^T stored
  uint64_t* bar_bi = bar_kq + 13;   //              B_c image stored
  uint64_t* bar_o = bar_kq + 14;    //              chunk's output rows read
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + Q_OFF_BAR + 128);

  const int t = threadIdx.x, warp = t >> 5;
  const bool state_wg = t < kScanWState;
  const bool issuer = warp == kScanWState / 32;
  const int v = t & 127, ch = (t >> 7) & 3;
  const int h = static_cast<int>(blockIdx.x % p.HV);
  const int64_t n = order[blockIdx.x / p.HV];
  const int qh = h / (p.HV / p.HQ);
  const int64_t HV = p.HV;
  int64_t start, end;
  seq_bounds(p, n, start, end);
  // a split call's first part (mode 1) runs the sequence's early chunks, the second part
  // (mode 2) the rest from the state the first part wrote
  int64_t k0 = 0;
  if (mode != 0 && end > start) {  // (mode: compile-time)
    const int64_t spn = eoffs[n + 1] - eoffs[n];
    if (mode == 1) {
      const int64_t e1 = start + spn * kC;
      end = e1 < end ? e1 : end;
    } else {
      k0 = spn;
      start += spn * kC;
    }
  }

  const bool skip = end <= start || offs[p.N] > unit_capacity(p);
  // this thread's quarter of state row v: S[n, h, v, 32c .. 32c+32)
  const int64_t sbase = ((n * HV + h) * kHeadDim + v) * kHeadDim + 32 * ch;
  float S[32];
  if (state_wg) {
#pragma unroll
    for (int i = 0; i < 32; i += 4) {
      const float4 x = p.state ? *reinterpret_cast<const float4*>(p.state + sbase + i)
                               : make_float4(0.f, 0.f, 0.f, 0.f);
      S[i] = x.x; S[i + 1] = x.y; S[i + 2] = x.z; S[i + 3] = x.w;
    }
    // empty sequence, or a workspace overflow (no units were written): pass the state
    // through
    if (skip) {
#pragma unroll
      for (int i = 0; i < 32; i += 4)
        *reinterpret_cast<float4*>(p.new_state + sbase + i) =
            make_float4(S[i], S[i + 1], S[i + 2], S[i + 3]);
    }
  }
  if (skip) return;
  const int64_t nch = (end - start + kC - 1) / kC;

  if (t == 0) {
    for (int i = 0; i < 10; ++i) mbar_init(&bar_kq[i], 1);
    for (int i = 10; i < 15; ++i) mbar_init(&bar_kq[i], kScanWState / 32);
    fence_mbar_init();
  }
  if (issuer) tmem_alloc(tmem_slot, kScanTTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  bool ok = true;

  if (issuer) {
    // ================================ MMA / copy issuer ================================
    const uint8_t* a2_seq = a2_in + static_cast<uint64_t>(offs[n] + k0) * HV * kUnitBytes +
                            static_cast<uint64_t>(h) * kUnitBytes;
    const uint64_t a2_chunk_stride = static_cast<uint64_t>(HV) * kUnitBytes;
    const bool leader = (t & 31) == 0;
    auto issue_kq = [&](int64_t m) {  // chunk m's K/Q tile -> buffer m % 3
      const int bq = static_cast<int>(m % 3);
      uint8_t* kq = sm + Q_OFF_KQ + bq * 32768;
      mbar_arrive_expect_tx(&bar_kq[bq], 4 * 8192);
      const int tok = static_cast<int>(start + m * kC);
      tma_load_3d(kq, &maps.k, &bar_kq[bq], 0, qh, tok);
      tma_load_3d(kq + 8192, &maps.q, &bar_kq[bq], 0, qh, tok);
      tma_load_3d(kq + 16384, &maps.k, &bar_kq[bq], 64, qh, tok);
      tma_load_3d(kq + 16384 + 8192, &maps.q, &bar_kq[bq], 64, qh, tok);
    };
    // chunk m's V tile, [T_b; P] image and gates -> buffer m & 1
    auto issue_va = [&](int64_t m) {
      const int b = static_cast<int>(m & 1);
      mbar_arrive_expect_tx(&bar_va[b], 16384 + kUnitBytes);
      tma_load_3d(sm + Q_OFF_V + b * 16384, &maps.v, &bar_va[b], 0, h,
                  static_cast<int>(start + m * kC));
      const uint8_t* src = a2_seq + static_cast<uint64_t>(m) * a2_chunk_stride;
      uint8_t* a2 = sm + Q_OFF_A2 + b * kA2Bytes;
      bulk_load(a2, src, 16384, &bar_va[b]);
      bulk_load(a2 + 16384, src + 16384, 8192, &bar_va[b]);
      bulk_load(sm + Q_OFF_GATES + b * kGateBytes, src + kA2Bytes, kGateBytes, &bar_va[b]);
    };
    // G1a: D1 (columns d) = (operand columns) [K;Q]^T of the tile kq
    auto issue_g1a = [&](uint32_t d, const uint8_t* kq) {
      mma_group_g1a(tmem + d, tmem + TP_S, desc_kmajor(smem_u32(kq)));
    };
    // B_m^T = [K;Q]_{m+1} K_m^T (exact bf16 operands, one term) into the first 64
    // columns of D1_{m+1}'s buffer (free until G1a_{m+1})
    auto issue_b = [&](int64_t m) -> bool {
      const bool w = mbar_wait_spin(&bar_kq[(m + 1) % 3], static_cast<uint32_t>(((m + 1) / 3) & 1));
      tc_fence_after();
      __syncwarp();
      if (!w) return false;
      const uint8_t* kqm = sm + Q_OFF_KQ + static_cast<int>(m % 3) * 32768;
      const uint8_t* kqm1 = sm + Q_OFF_KQ + static_cast<int>((m + 1) % 3) * 32768;
      mma_group_b(tmem + TP_D1 + 128 * static_cast<uint32_t>((m + 1) & 1) + 64,
                  desc_kmajor(smem_u32(kqm1)), desc_kmajor(smem_u32(kqm)));
      mma_commit_w(bar_tb);
      return true;
    };
    if (leader) {
      issue_kq(0);
      issue_va(0);
      if (nch > 1) {
        issue_kq(1);
        issue_va(1);
      }
    }
    __syncwarp();
    uint32_t ph_x = 0, ph_op = 0, ph_u = 0, ph_bi = 0, ph_g1a = 0;
    // prologue: D1_0 = S_0 [K;Q]_0^T
    ok = mbar_wait_spin(bar_op, ph_op) && ok;
    ph_op ^= 1;
    ok = mbar_wait_spin(&bar_kq[0], 0) && ok;
    tc_fence_after();
    __syncwarp();
    if (ok) {
      issue_g1a(TP_D1, sm + Q_OFF_KQ);
      mma_commit_w(bar_ch);
      if (nch > 1) ok = issue_b(0);
    }
    for (int64_t c = 0; ok && c < nch; ++c) {
      const bool last = c == nch - 1;
      const int b = static_cast<int>(c & 1);
      const uint32_t d1c = TP_D1 + 128 * b, d1n = TP_D1 + 128 * (b ^ 1);
      const uint8_t* kqc = sm + Q_OFF_KQ + static_cast<int>(c % 3) * 32768;
      const uint8_t* kqn = sm + Q_OFF_KQ + static_cast<int>((c + 1) % 3) * 32768;
      const uint8_t* a2 = sm + Q_OFF_A2 + b * kA2Bytes;
      // chunk c+1's V, [T_b; P] and gates into chunk c-1's buffers (chunk 1's were
      // requested with chunk 0's): their readers, X_{c-1} and G2_{c-1}, finished before
      // U'_{c-1} was signalled
      if (leader && c > 0 && c + 1 < nch) issue_va(c + 1);
      __syncwarp();
      // ---- G2_c: D1_c <- X^T [T_b; P]^T = [U^T | (PX)^T] ----------------------------
      ok = mbar_wait_spin(bar_x, ph_x) && ok;
      ph_x ^= 1;
      ok = mbar_wait_spin(&bar_va[b], static_cast<uint32_t>((c >> 1) & 1)) && ok;
      tc_fence_after();
      __syncwarp();
      if (!ok) break;
      {
        mma_group_x3(tmem + TP_GO, tmem + d1c, desc_kmajor(smem_u32(a2)),
                     desc_kmajor(smem_u32(a2 + 16384)), 0u);
        mma_commit_w(bar_g2);
      }
      if (!last) {
        // ---- G1a_{c+1} = (g_c S_c) [K;Q]_{c+1}^T once the operand is stored -------------
        ok = mbar_wait_spin(bar_op, ph_op) && ok;
        ph_op ^= 1;
        tc_fence_after();
        __syncwarp();
        if (!ok) break;
        // chunk c+2's K/Q tile into chunk c-1's buffer (the third one for c = 0): its
        // last reader G3_{c-1} finished before this operand was signalled
        if (leader && c + 2 < nch) issue_kq(c + 2);
        __syncwarp();
        issue_g1a(d1n, kqn);
        mma_commit_w(bar_g1a);
      }
      // ---- U'_c stored: G1'_c onto D1_{c+1}, then G3_c: dS_c = U'^T K_c ----------------
      ok = mbar_wait_spin(bar_u, ph_u) && ok;
      ph_u ^= 1;
      tc_fence_after();
      __syncwarp();
      if (!ok) break;
      if (!last) {
        ok = mbar_wait_spin(bar_bi, ph_bi) && ok;  // the B_c image
        ph_bi ^= 1;
        tc_fence_after();
        __syncwarp();
        if (!ok) break;
        mma_group_x3(tmem + d1n, tmem + d1c, desc_kmajor(smem_u32(sm + Q_OFF_B)),
                     desc_kmajor(smem_u32(sm + Q_OFF_B + 16384)), 1u);
        mma_commit_w(bar_ch);
        // G3 overwrites the operand columns that G1a_{c+1} reads (another accumulator:
        // no implicit order between them)
        ok = mbar_wait_spin(bar_g1a, ph_g1a) && ok;
        ph_g1a ^= 1;
        tc_fence_after();
        __syncwarp();
        if (!ok) break;
      }
      {
        mma_group_g3(tmem + TP_S, tmem + d1c, desc_mnmajor(smem_u32(kqc), 16384));
        mma_commit_w(bar_g3);
      }
      // B_{c+1} for chunk c+1's state-side work (D1_c's buffer is read: U'_c is stored)
      // B_{c+1} overwrites the (QH)^T half of D1_c: after the state warps have read
      // chunk c's output rows
      if (c + 2 < nch) {
        ok = mbar_wait_spin(bar_o, static_cast<uint32_t>(c & 1)) && ok;
        tc_fence_after();
        __syncwarp();
        if (!ok || !issue_b(c + 1)) {
          ok = false;
          break;
        }
      }
    }
  } else if (state_wg) {
    // ================================ state warps ======================================
    const uint32_t lane = tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16);
    const bool lane0 = (t & 31) == 0;
    // this warp's arrival on a ready barrier: every lane's TMEM stores have completed
    // and its shared-memory writes are visible to the tensor core
    auto signal = [&](uint64_t* bar) {
      fence_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane0) mbar_arrive(bar);
    };
    // the S operand: bf16 hi/lo of scale * S (this thread's 32 columns)
    auto write_s_operand = [&](float scale) {
      float hl[32];  // bit images: 16 hi words, then 16 lo words
#pragma unroll
      for (int w = 0; w < 16; ++w) {
        uint32_t hw, lw;
        const float2 gs = mul2(make_float2(scale, scale), make_float2(S[2 * w], S[2 * w + 1]));
        split2(gs.x, gs.y, hw, lw);
        hl[w] = __uint_as_float(hw);
        hl[16 + w] = __uint_as_float(lw);
      }
      tmem_st32(lane + TP_S + 32 * ch, hl);
      tmem_st_wait();
    };
    // prologue: the operand S_0 for D1_0
    write_s_operand(1.0f);
    signal(bar_op);

    uint32_t ph_ch = 0, ph_g2 = 0, ph_tb = 0, ph_g3 = 0;
    float g_prev = 1.0f;  // gamma_last of the previous chunk
    // output rows of the chunk (bf16 pairs), stored once U' is signalled
    uint32_t opk[8];
    int64_t o_cs = 0;
    int o_L = 0;
    auto store_output = [&]() {
      __nv_bfloat16* dst = p.out + (o_cs * HV + h) * kHeadDim + v;
      const int64_t row = HV * kHeadDim;
      dst += static_cast<int64_t>(16 * ch) * row;
      if (o_L == kC) {  // full chunk (uniform): no per-token predicate
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const uint32_t w = opk[i >> 1];
          dst[i * row] =
              __ushort_as_bfloat16(static_cast<unsigned short>((i & 1) ? (w >> 16) : (w & 0xffffu)));
        }
      } else {
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const uint32_t w = opk[i >> 1];
          if (16 * ch + i < o_L)
            dst[i * row] = __ushort_as_bfloat16(
                static_cast<unsigned short>((i & 1) ? (w >> 16) : (w & 0xffffu)));
        }
      }
    };
    for (int64_t c = 0; c < nch; ++c) {
      const int64_t cs = start + c * kC;
      const int L = static_cast<int>((end - cs) < kC ? (end - cs) : kC);
      const bool last = c == nch - 1;
      const int b = static_cast<int>(c & 1);
      const uint32_t d1c = TP_D1 + 128 * b, d1n = TP_D1 + 128 * (b ^ 1);
      // gates of chunk c (from the prep, arrived with the [T_b; P] image)
      const float* sGam = reinterpret_cast<const float*>(sm + Q_OFF_GATES + b * kGateBytes);
      const float* sF = sGam + kC;
      const uint8_t* vt = sm + Q_OFF_V + b * 16384;
      // ---- D1_c complete: X_c^T = V^T - (KH)^T diag(gamma), over (KH)^T ------------------
      ok = mbar_wait(bar_ch, ph_ch) && ok;
      ph_ch ^= 1;
      ok = mbar_wait(&bar_va[b], static_cast<uint32_t>((c >> 1) & 1)) && ok;
      tc_fence_after();
      {
        float d[16];
        tmem_ld16(lane + d1c + 16 * ch, d);
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
        tmem_st8(lane + d1c + 16 * ch, hw);
        tmem_st8(lane + d1c + 16 * ch + 8, lw);
        tmem_st_wait();
      }
      signal(bar_x);

      // ---- beside the chain: S_c = g_{c-1} S_{c-1} + dS_{c-1}; operand g_c S_c; B_c ------
      if (c > 0) {
        ok = mbar_wait(bar_g3, ph_g3) && ok;  // G3_{c-1}: dS_{c-1}
        ph_g3 ^= 1;
        tc_fence_after();
        float d0[32];
        tmem_ld32(lane + TP_S + 32 * ch, d0);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 32; i += 2) {
          const float2 r = fma2(make_float2(g_prev, g_prev), make_float2(S[i], S[i + 1]),
                                make_float2(d0[i], d0[i + 1]));
          S[i] = r.x;
          S[i + 1] = r.y;
        }
      }
      g_prev = sGam[kC - 1];
      if (!last) {
        tc_fence_before();
        // every state thread has read dS_{c-1}
        if (!named_bar_and(kStateBar, kScanWState, ok)) break;
        tc_fence_after();
        write_s_operand(g_prev);
        ok = mbar_wait(bar_tb, ph_tb) && ok;
        ph_tb ^= 1;
        tc_fence_after();
        {
          // row v of B_c^T (the [K;Q]_{c+1} row), columns i in [16c, 16c+16). B_c sits in
          // the (QH)^T half of D1_{c+1}'s buffer, which G1a_{c+1} overwrites: the operand
          // is signalled (and G1a_{c+1} issued) only once every thread holds its B_c row
          float bt[16];
          tmem_ld16(lane + d1n + 64 + 16 * ch, bt);
          tmem_ld_wait();
          signal(bar_op);
          uint32_t hw[8], lw[8];
          split_words<8>(bt, hw, lw);
          uint8_t* bimg = sm + Q_OFF_B;
          *reinterpret_cast<uint4*>(bimg + sw128_chunk(v, 2 * ch)) =
              make_uint4(hw[0], hw[1], hw[2], hw[3]);
          *reinterpret_cast<uint4*>(bimg + sw128_chunk(v, 2 * ch + 1)) =
              make_uint4(hw[4], hw[5], hw[6], hw[7]);
          if (v < kC) {  // lo for the K rows only (the Q rows reach the output alone)
            *reinterpret_cast<uint4*>(bimg + 16384 + sw128_chunk(v, 2 * ch)) =
                make_uint4(lw[0], lw[1], lw[2], lw[3]);
            *reinterpret_cast<uint4*>(bimg + 16384 + sw128_chunk(v, 2 * ch + 1)) =
                make_uint4(lw[4], lw[5], lw[6], lw[7]);
          }
        }
        signal(bar_bi);
      }

      // ---- G2_c done: U'^T = U^T diag(f) over X^T; output rows of chunk c ---------------
      ok = mbar_wait(bar_g2, ph_g2) && ok;
      ph_g2 ^= 1;
      tc_fence_after();
      {
        float u[16];
        tmem_ld16(lane + TP_GO + 16 * ch, u);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 16; i += 2) {
          const float2 r = mul2(make_float2(u[i], u[i + 1]),
                                *reinterpret_cast<const float2*>(sF + 16 * ch + i));
          u[i] = r.x;
          u[i + 1] = r.y;
        }
        uint32_t hw[8], lw[8];
        split_words<8>(u, hw, lw);
        tmem_st8(lane + d1c + 16 * ch, hw);
        tmem_st8(lane + d1c + 16 * ch + 8, lw);
        tmem_st_wait();
      }
      signal(bar_u);
      {
        // O^T row v, tokens i in [16c, 16c+16): scale (gamma_i (QH)^T + (PX)^T), read
        // before B_{c+1} overwrites the (QH)^T half (the issuer waits for bar_o)
        float o[16], qv[16];
        tmem_ld16(lane + TP_GO + 64 + 16 * ch, o);
        tmem_ld16(lane + d1c + 64 + 16 * ch, qv);
        // the gates too: after bar_o the issuer may refill this gate buffer
        float2 gm[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) gm[i] = *reinterpret_cast<const float2*>(sGam + 16 * ch + 2 * i);
        tmem_ld_wait();
        signal(bar_o);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float2 r = mul2(make_float2(p.scale, p.scale),
                                fma2(gm[i],
                                     make_float2(qv[2 * i], qv[2 * i + 1]),
                                     make_float2(o[2 * i], o[2 * i + 1])));
          opk[i] = pack2_rn(r.x, r.y);
        }
        o_cs = cs;
        o_L = L;
      }
      store_output();
    }
    if (ok) {
      ok = mbar_wait(bar_g3, ph_g3);
      tc_fence_after();
    }
    if (named_bar_and(kStateBar, kScanWState, ok)) {
      float d0[32];
      tmem_ld32(lane + TP_S + 32 * ch, d0);
      tmem_ld_wait();
#pragma unroll
      for (int i = 0; i < 32; i += 4)
        *reinterpret_cast<float4*>(p.new_state + sbase + i) =
            make_float4(fmaf(g_prev, S[i], d0[i]), fmaf(g_prev, S[i + 1], d0[i + 1]),
                        fmaf(g_prev, S[i + 2], d0[i + 2]), fmaf(g_prev, S[i + 3], d0[i + 3]));
    } else {
      ok = false;
    }
  }
  if (!ok && p.status) atomicOr(p.status, kStatusWaitTimeout);
  tc_fence_before();
  __syncthreads();
  if (issuer) tmem_dealloc(tmem, kScanTTmemCols);
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

// Workspace: [0, 256) status word; [256, ...) chunk offsets (N + 1 int64), the scan
// order (N int32, padded to 8 B), the chunk table (ceil(T / 64) + N int64); then,
// 1024-aligned, 24.5 KB of [T_b; P] and gates per (chunk, v-head).
static size_t order_bytes(int64_t N) { return (4 * static_cast<size_t>(N) + 7) & ~size_t(7); }
// ... then the early-chunk prefix (N + 1 int64) and, 16-byte aligned, the early and late
// unit lists (16 B per chunk each) of a split call.
struct WsLayout {
  size_t offs, order, table, eoffs, elist, llist, head;
};
static WsLayout ws_layout(int64_t T, int64_t N) {
  const size_t chunks = static_cast<size_t>((T + kC - 1) / kC + N);
  WsLayout w;
  w.offs = 256;
  w.order = w.offs + 8 * static_cast<size_t>(N + 1);
  w.table = w.order + order_bytes(N);
  w.eoffs = w.table + 8 * chunks;
  w.elist = (w.eoffs + 8 * static_cast<size_t>(N + 1) + 15) & ~size_t(15);
  w.llist = w.elist + 16 * chunks;
  w.head = (w.llist + 16 * chunks + 1023) & ~size_t(1023);
  return w;
}
static size_t head_bytes(int64_t T, int64_t N) { return ws_layout(T, N).head; }

// Split calls. When the scan's (sequence, v-head) chains leave SMs idle (one scan block
// per SM), the prep of each sequence's last chunks runs on those SMs while the scan
// works through the first ones: prep (early units, all SMs) -> scan part 1 on the
// caller's stream (dispatched first, as the in-stream successor) || prep (late units) on a
// low-priority side stream, behind an event -> scan part 2 on the caller's stream.
// Only stream order and events between the launches; no kernel waits on another.
struct SplitStreams {
  cudaStream_t side = nullptr;
  cudaEvent_t ev_prep = nullptr, ev_scan = nullptr;
  int sms = 0;
  bool ready = false;
  // held by a split call from its first event record to the final join, so that calls
  // from several host threads (on their own streams and workspaces) never interleave
  // their records and waits on the shared side stream and events
  std::mutex launch;
};
static std::mutex g_split_mutex;
static SplitStreams g_split[64];

// The device's side stream and events, created on the first split call (both events and
// the stream, or nothing: a partial creation is undone and the call runs unsplit).
static SplitStreams* split_streams() {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  std::lock_guard<std::mutex> lock(g_split_mutex);
  SplitStreams& s = g_split[dev];
  if (!s.ready) {
    int lo = 0, hi = 0;
    if (cudaDeviceGetStreamPriorityRange(&lo, &hi) != cudaSuccess ||
        cudaDeviceGetAttribute(&s.sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) {
      cudaGetLastError();
      return nullptr;
    }
    cudaStream_t side = nullptr;
    cudaEvent_t e1 = nullptr, e2 = nullptr;
    const bool ok = cudaStreamCreateWithPriority(&side, cudaStreamNonBlocking, lo) == cudaSuccess &&
                    cudaEventCreateWithFlags(&e1, cudaEventDisableTiming) == cudaSuccess &&
                    cudaEventCreateWithFlags(&e2, cudaEventDisableTiming) == cudaSuccess;
    if (!ok) {
      if (e1) cudaEventDestroy(e1);
      if (side) cudaStreamDestroy(side);
      cudaGetLastError();
      return nullptr;
    }
    s.side = side;
    s.ev_prep = e1;
    s.ev_scan = e2;
    s.ready = true;
  }
  return &s;
}

// Fraction (of 1024) of each sequence's chunks prepped before the scan starts, or 0 for
// no split: the late prep runs on the `idle` SMs during the first scan part and must keep
// ahead of it: (1 - f) P sms / idle <= f S, with S / P ~ 1.4 (scan vs prep time of a call
// on all SMs, measured). Needs >= 8 idle SMs and >= 64 chunks per sequence on average.
static int split_fraction(const PrefillParams& p, int sms) {
  const char* env = getenv("GDN_PREFILL_OVERLAP");
  if (env && env[0] == '0') return 0;
  const int64_t chains = p.N * p.HV, idle = sms - chains;
  if (p.N > kInlineSortN || idle < 8 || p.T < 64 * kC * p.N) return 0;
  const double r = static_cast<double>(sms) / static_cast<double>(idle);
  return static_cast<int>(1024.0 * r / (r + 1.4));
}

size_t prefill_twophase_workspace_bytes(int64_t T, int64_t N, int HV) {
  const size_t head = head_bytes(T, N);
  const size_t chunks = static_cast<size_t>((T + kC - 1) / kC + N);
  return head + chunks * static_cast<size_t>(HV) * kUnitBytes;
}

int prefill_twophase_launches(int64_t T, int64_t N, int HV) {
  if (N <= 0) return 0;
  int dev = -1, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) {
    cudaGetLastError();
    return -1;
  }
  PrefillParams p{};
  p.T = T;
  p.N = N;
  p.HV = HV;
  const int base = N > kInlineSortN ? 4 : 3;  // offsets (+ order), gates, scan (+ prep)
  if (T <= 0) return base - 1;                // no gates or prep launch
  return base + 1 + (split_fraction(p, sms) ? 2 : 0);
}

int launch_prefill_twophase(const PrefillParams& p, void* workspace, cudaStream_t stream) {
  if (p.N == 0) return 0;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  const WsLayout wl = ws_layout(p.T, p.N);
  int64_t* offs = reinterpret_cast<int64_t*>(ws + wl.offs);
  int32_t* order = reinterpret_cast<int32_t*>(ws + wl.order);
  int64_t* table = reinterpret_cast<int64_t*>(ws + wl.table);
  const int64_t cap = (p.T + kC - 1) / kC + p.N;
  int64_t* eoffs = reinterpret_cast<int64_t*>(ws + wl.eoffs);
  longlong2* elist = reinterpret_cast<longlong2*>(ws + wl.elist);
  longlong2* llist = reinterpret_cast<longlong2*>(ws + wl.llist);
  const size_t head = wl.head;
  uint8_t* a2 = ws + head;
  ChunkTmaps maps;
  const int64_t Tm = p.T > 0 ? p.T : 1;
  const void* kb = p.T > 0 ? static_cast<const void*>(p.k) : static_cast<const void*>(p.new_state);
  const void* qb = p.T > 0 ? static_cast<const void*>(p.q) : static_cast<const void*>(p.new_state);
  if (!encode_qk_map(&maps.k, kb, Tm, p.HQ) || !encode_qk_map(&maps.q, qb, Tm, p.HQ)) return -2;
  if (cudaFuncSetAttribute(prep_kernel<0>, cudaFuncAttributeMaxDynamicSharedMemorySize, kPrepSmem) !=
          cudaSuccess ||
      cudaFuncSetAttribute(prep_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, kPrepSmem) !=
          cudaSuccess ||
      cudaFuncSetAttribute(prep_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, kPrepSmem) !=
          cudaSuccess)
    return -1;
  SplitStreams* ss = p.T > 0 ? split_streams() : nullptr;
  const int split_q = ss ? split_fraction(p, ss->sms) : 0;
  chunk_offsets_kernel<<<1, 1024, 0, stream>>>(p, offs, order, eoffs, split_q);
  if (p.N > kInlineSortN)
    scan_order_kernel<<<static_cast<unsigned>((p.N + 255) / 256), 256, 0, stream>>>(p.N, offs,
                                                                                   order);
  if (p.T > 0) {
    chunk_gates_kernel<<<static_cast<unsigned>((cap * p.HV + 7) / 8), 256, 0, stream>>>(
        p, offs, table, a2, split_q ? eoffs : nullptr, elist, llist);
    if (!split_q)
      prep_kernel<0><<<static_cast<unsigned>(cap * p.HV), kPrepThreads, kPrepSmem, stream>>>(
          p, maps, offs, table, a2, eoffs, elist);
  }
  ScanMaps smaps;
  smaps.k = maps.k;
  smaps.q = maps.q;
  const void* vb = p.T > 0 ? static_cast<const void*>(p.v) : static_cast<const void*>(p.new_state);
  if (!encode_v_map(&smaps.v, vb, Tm, p.HV)) return -2;
  for (auto fn : {scan_w_kernel<0>, scan_w_kernel<1>, scan_w_kernel<2>})
    if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, kScanWSmem) !=
        cudaSuccess)
      return -1;
  const unsigned scan_grid = static_cast<unsigned>(p.N * p.HV);
  if (!split_q) {
    scan_w_kernel<0><<<scan_grid, kScanWThreads, kScanWSmem, stream>>>(p, smaps, offs, order,
                                                                      a2, eoffs);
    return cudaGetLastError() == cudaSuccess ? 0 : -1;
  }
  // early units (at most cap * f of them), then the first scan part on the caller's
  // stream while the late units (at most cap (1 - f) + N) are prepped on the side stream
  std::lock_guard<std::mutex> split_lock(ss->launch);
  const int64_t n_early = cap * split_q / 1024 + 1;
  const int64_t n_late = cap - cap * split_q / 1024 + p.N + 1;
  prep_kernel<1><<<static_cast<unsigned>(n_early * p.HV), kPrepThreads, kPrepSmem, stream>>>(
      p, maps, offs, table, a2, eoffs, elist);
  if (cudaEventRecord(ss->ev_prep, stream) != cudaSuccess ||
      cudaStreamWaitEvent(ss->side, ss->ev_prep, 0) != cudaSuccess)
    return -1;
  scan_w_kernel<1><<<scan_grid, kScanWThreads, kScanWSmem, stream>>>(p, smaps, offs, order,
                                                                    a2, eoffs);
  prep_kernel<2><<<static_cast<unsigned>(n_late * p.HV), kPrepThreads, kPrepSmem, ss->side>>>(
      p, maps, offs, table, a2, eoffs, llist);
  if (cudaEventRecord(ss->ev_scan, ss->side) != cudaSuccess ||
      cudaStreamWaitEvent(stream, ss->ev_scan, 0) != cudaSuccess)
    return -1;
  PrefillParams p2 = p;
  p2.state = p.new_state;  // the second part continues from the first part's states
  scan_w_kernel<2><<<scan_grid, kScanWThreads, kScanWSmem, stream>>>(p2, smaps, offs, order,
                                                                    a2, eoffs);
  return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

}  // namespace gdn

