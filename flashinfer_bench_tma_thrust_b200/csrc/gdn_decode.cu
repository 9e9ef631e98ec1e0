// gdn_decode.cu — fused single-token GDN decode for sm_100a.
//
// Math (reference: gdn/decode/baseline/triton/kernel.py:57-100; production
// Triton kernel gdn/decode/solution/triton/kernel.py:23-82). Per (b, v-head h)
// with k-last state S[v][k]:
//   g = exp(-exp(A_log) softplus(a + dt_bias)), beta = sigmoid(b)
//   for each row v:   old   = g * (S[v,:] . k)
//                     delta = beta * (v_in[v] - old)
//                     S'[v,:] = g * S[v,:] + delta * k
//                     o[v]  = scale * (S'[v,:] . q) = scale * (g * (S[v,:] . q) + delta * (k . q))
//
// Every v-row is an independent 512-byte unit once the per-head scalars
// (g, beta, k.q) are known, so the work is a pure stream: one warp covers a
// row with one 16-byte load per lane, both dot products reduce with warp
// shuffles, and the updated row goes back with one 16-byte store per lane.
// The state is read once and written once; nothing is staged through shared
// memory. Rows of one head are split over several thread blocks when the batch
// is small so that all 148 SMs get work.
#include "gdn_common.cuh"
#include "gdn_launch.h"

namespace gdn {

// State element access: fp32 (the reference layout) or bf16 (reduced-precision
// option: half the HBM bytes, fp32 math, rounded to bf16 on store).
template <typename S>
struct StateIO;
template <>
struct StateIO<float> {
  static __device__ __forceinline__ float4 load(const void* base, int64_t idx) {
    return ld_stream_f4(static_cast<const float*>(base) + idx);
  }
  static __device__ __forceinline__ void store(void* base, int64_t idx, float4 v) {
    st_stream_f4(static_cast<float*>(base) + idx, v);
  }
};
template <>
struct StateIO<__nv_bfloat16> {
  static __device__ __forceinline__ float4 load(const void* base, int64_t idx) {
    uint2 raw;
    asm volatile("ld.global.cs.v2.u32 {%0,%1}, [%2];"
                 : "=r"(raw.x), "=r"(raw.y)
                 : "l"(static_cast<const __nv_bfloat16*>(base) + idx));
    return make_float4(__uint_as_float(raw.x << 16), __uint_as_float(raw.x & 0xffff0000u),
                       __uint_as_float(raw.y << 16), __uint_as_float(raw.y & 0xffff0000u));
  }
  static __device__ __forceinline__ void store(void* base, int64_t idx, float4 v) {
    const __nv_bfloat162 a = __floats2bfloat162_rn(v.x, v.y);
    const __nv_bfloat162 b = __floats2bfloat162_rn(v.z, v.w);
    const uint32_t ua = *reinterpret_cast<const uint32_t*>(&a);
    const uint32_t ub = *reinterpret_cast<const uint32_t*>(&b);
    asm volatile("st.global.cs.v2.u32 [%0], {%1,%2};" ::"l"(static_cast<__nv_bfloat16*>(base) +
                                                            idx),
                 "r"(ua), "r"(ub)
                 : "memory");
  }
};

// ROWS: rows each warp keeps in flight (loads issued back to back before any
// reduction) — the memory-level parallelism knob.
template <int ROWS, typename S = float>
__global__ void __launch_bounds__(128) decode_kernel(DecodeParams p) {
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int64_t head = blockIdx.x / p.splits;       // flattened (b, h)
  const int split = blockIdx.x - head * p.splits;   // which row block of the head
  const int64_t bi = head / p.HV;
  const int h = static_cast<int>(head - bi * p.HV);
  const int qh = h / (p.HV / p.HQ);

  // Per-head scalars (every thread computes the same values; loads broadcast).
  const float A_log = load_scalar(p.A_log, p.A_log_dtype, h);
  const float dtb = load_scalar(p.dt_bias, p.dt_bias_dtype, h);
  const float a = load_scalar(p.a, p.a_dtype, head);
  const float bb = load_scalar(p.b, p.b_dtype, head);
  const float g = expf(gate_log_decay(A_log, a, dtb));
  const float beta = gate_beta(bb);

  const int64_t qk_off = (bi * p.HQ + qh) * kHeadDim + lane * 4;
  const float4 q = load_bf16x4(p.q + qk_off);
  const float4 k = load_bf16x4(p.k + qk_off);
  const float kq = warp_sum(q.x * k.x + q.y * k.y + q.z * k.z + q.w * k.w);

  const int rows_per_warp = p.rows_per_warp;
  const int row0 = (split * 4 + warp) * rows_per_warp;
  const int64_t vrow_base = head * kHeadDim;  // row index into v / out
  // lane r holds v_in for row row0 + r (rows_per_warp <= 32)
  float v_lane = 0.0f;
  if (lane < rows_per_warp) {
    const unsigned short raw =
        reinterpret_cast<const unsigned short*>(p.v)[vrow_base + row0 + lane];
    v_lane = __uint_as_float(static_cast<uint32_t>(raw) << 16);
  }
  float o_lane = 0.0f;

  const int64_t state_base = (vrow_base + row0) * kHeadDim + lane * 4;
  const void* src_state = p.state_any ? p.state_any : static_cast<const void*>(p.state);
  void* dst_state = p.new_state_any ? p.new_state_any : static_cast<void*>(p.new_state);

  for (int r0 = 0; r0 < rows_per_warp; r0 += ROWS) {
    float4 s[ROWS];
    if (src_state) {
#pragma unroll
      for (int i = 0; i < ROWS; ++i)
        s[i] = StateIO<S>::load(src_state, state_base + (r0 + i) * kHeadDim);
    } else {
#pragma unroll
      for (int i = 0; i < ROWS; ++i) s[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int i = 0; i < ROWS; ++i) {
      float sk = s[i].x * k.x + s[i].y * k.y + s[i].z * k.z + s[i].w * k.w;
      float sq = s[i].x * q.x + s[i].y * q.y + s[i].z * q.z + s[i].w * q.w;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        sk += __shfl_xor_sync(0xffffffffu, sk, o);
        sq += __shfl_xor_sync(0xffffffffu, sq, o);
      }
      const float vin = __shfl_sync(0xffffffffu, v_lane, r0 + i);
      const float delta = beta * (vin - g * sk);
      float4 n;
      n.x = fmaf(g, s[i].x, delta * k.x);
      n.y = fmaf(g, s[i].y, delta * k.y);
      n.z = fmaf(g, s[i].z, delta * k.z);
      n.w = fmaf(g, s[i].w, delta * k.w);
      StateIO<S>::store(dst_state, state_base + (r0 + i) * kHeadDim, n);
      if (lane == r0 + i) o_lane = p.scale * fmaf(g, sq, delta * kq);
    }
  }
  if (lane < rows_per_warp) p.out[vrow_base + row0 + lane] = __float2bfloat16_rn(o_lane);
}

template <typename S>
int launch_decode_t(const DecodeParams& p_in, cudaStream_t stream) {
  DecodeParams p = p_in;
  const int64_t heads = p.B * p.HV;
  if (heads == 0) return 0;
  // Choose how many thread blocks share one head (splits * 4 warps * rows_per_warp = 128):
  // at large batch one block per head (32 rows per warp); at small batch split the
  // head's rows so that the grid covers the SMs several times over.
  int splits = 1;
  const int64_t target_blocks = 148 * 4;
  while (splits < 8 && heads * splits < target_blocks) splits *= 2;
  p.splits = splits;
  p.rows_per_warp = kHeadDim / (4 * splits);
  const dim3 grid(static_cast<unsigned>(heads * splits));
  if (p.rows_per_warp >= 8) {
    decode_kernel<8, S><<<grid, 128, 0, stream>>>(p);
  } else {
    decode_kernel<4, S><<<grid, 128, 0, stream>>>(p);
  }
  return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

int launch_decode(const DecodeParams& p, cudaStream_t stream) {
  return p.state_bf16 ? launch_decode_t<__nv_bfloat16>(p, stream)
                      : launch_decode_t<float>(p, stream);
}

}  // namespace gdn
