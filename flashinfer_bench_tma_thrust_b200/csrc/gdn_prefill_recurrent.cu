// gdn_prefill_recurrent.cu — token-sequential varlen GDN prefill (SIMT).
//
// The recurrence of gdn/prefill/baseline/triton/kernel.py:63-98, organised
// like the reference's production prefill (gdn/prefill/solution/triton/
// kernel.py:99-209): one thread block per (sequence, v-head, 32-row V tile)
// walks every token of its sequence with the state tile in registers.
// Each warp owns 8 state rows; each lane holds 4 consecutive K elements of
// those rows (32 fp32 registers). The next token's q/k/v/gates are loaded
// before the current token is processed so their latency overlaps the math.
//
// This kernel is the independent cross-check for the chunked tensor-core
// prefill at sizes the CPU oracle cannot reach; it is not the fast path.
#include "gdn_common.cuh"
#include "gdn_launch.h"

namespace gdn {

namespace {

constexpr int kRowsPerWarp = 8;
constexpr int kTileRows = 4 * kRowsPerWarp;  // 32 rows per block
constexpr int kTiles = kHeadDim / kTileRows;  // 4 V tiles per head

struct TokenIn {
  float4 q, k;
  float v;  // lane i < 8: v_in of row i of this warp
  float a, b;
};

__device__ __forceinline__ TokenIn load_token(const PrefillParams& p, int64_t t, int h, int qh,
                                              int row0, int lane) {
  TokenIn in;
  const int64_t qk_off = (t * p.HQ + qh) * kHeadDim + lane * 4;
  in.q = load_bf16x4(p.q + qk_off);
  in.k = load_bf16x4(p.k + qk_off);
  in.v = 0.0f;
  if (lane < kRowsPerWarp) {
    const unsigned short raw = reinterpret_cast<const unsigned short*>(
        p.v)[(t * p.HV + h) * kHeadDim + row0 + lane];
    in.v = __uint_as_float(static_cast<uint32_t>(raw) << 16);
  }
  in.a = load_scalar(p.a, p.a_dtype, t * p.HV + h);
  in.b = load_scalar(p.b, p.b_dtype, t * p.HV + h);
  return in;
}

}  // namespace

__global__ void __launch_bounds__(128) prefill_recurrent_kernel(PrefillParams p) {
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int64_t unit = blockIdx.x;  // (n, h, tile)
  const int tile = static_cast<int>(unit % kTiles);
  const int h = static_cast<int>((unit / kTiles) % p.HV);
  const int64_t n = unit / (kTiles * p.HV);
  const int qh = h / (p.HV / p.HQ);
  const int row0 = tile * kTileRows + warp * kRowsPerWarp;

  int64_t start = load_index(p.cu_seqlens, p.cu_dtype, n);
  int64_t end = load_index(p.cu_seqlens, p.cu_dtype, n + 1);
  start = start < 0 ? 0 : (start > p.T ? p.T : start);
  end = end < 0 ? 0 : (end > p.T ? p.T : end);

  const int64_t srow = ((n * p.HV + h) * kHeadDim + row0) * kHeadDim + lane * 4;
  float4 s[kRowsPerWarp];
#pragma unroll
  for (int i = 0; i < kRowsPerWarp; ++i)
    s[i] = p.state ? *reinterpret_cast<const float4*>(p.state + srow + i * kHeadDim)
                   : make_float4(0.f, 0.f, 0.f, 0.f);

  const float A_log = load_scalar(p.A_log, p.A_log_dtype, h);
  const float dtb = load_scalar(p.dt_bias, p.dt_bias_dtype, h);

  if (end > start) {
    TokenIn cur = load_token(p, start, h, qh, row0, lane);
    for (int64_t t = start; t < end; ++t) {
      TokenIn nxt = cur;
      if (t + 1 < end) nxt = load_token(p, t + 1, h, qh, row0, lane);
      const float g = expf(gate_log_decay(A_log, cur.a, dtb));
      const float beta = gate_beta(cur.b);
      const float kq = warp_sum(cur.q.x * cur.k.x + cur.q.y * cur.k.y + cur.q.z * cur.k.z +
                                cur.q.w * cur.k.w);
      float o_lane = 0.0f;
#pragma unroll
      for (int i = 0; i < kRowsPerWarp; ++i) {
        float sk = s[i].x * cur.k.x + s[i].y * cur.k.y + s[i].z * cur.k.z + s[i].w * cur.k.w;
        float sq = s[i].x * cur.q.x + s[i].y * cur.q.y + s[i].z * cur.q.z + s[i].w * cur.q.w;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
          sk += __shfl_xor_sync(0xffffffffu, sk, o);
          sq += __shfl_xor_sync(0xffffffffu, sq, o);
        }
        const float vin = __shfl_sync(0xffffffffu, cur.v, i);
        const float delta = beta * (vin - g * sk);
        s[i].x = fmaf(g, s[i].x, delta * cur.k.x);
        s[i].y = fmaf(g, s[i].y, delta * cur.k.y);
        s[i].z = fmaf(g, s[i].z, delta * cur.k.z);
        s[i].w = fmaf(g, s[i].w, delta * cur.k.w);
        if (lane == i) o_lane = p.scale * fmaf(g, sq, delta * kq);
      }
      if (lane < kRowsPerWarp)
        p.out[(t * p.HV + h) * kHeadDim + row0 + lane] = __float2bfloat16_rn(o_lane);
      cur = nxt;
    }
  }
#pragma unroll
  for (int i = 0; i < kRowsPerWarp; ++i)
    *reinterpret_cast<float4*>(p.new_state + srow + i * kHeadDim) = s[i];
}

int launch_prefill_recurrent(const PrefillParams& p, cudaStream_t stream) {
  const int64_t units = p.N * p.HV * kTiles;
  if (units == 0) return 0;
  prefill_recurrent_kernel<<<static_cast<unsigned>(units), 128, 0, stream>>>(p);
  return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

}  // namespace gdn
