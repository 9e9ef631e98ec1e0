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
#include <cuda_fp16.h>
#include <algorithm>

#include "gdn_common.cuh"
#include "gdn_launch.h"
#include "sm100_umma.cuh"

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
  // Choose how many thread blocks share one head (splits * 4 warps * rows_per_warp = 128).
  // Short blocks keep the end of the grid from idling SMs while the last long blocks
  // stream: measured on B200 (state GB/s by batch), four blocks per head (8 rows per
  // warp) up to 16384 heads (B = 512 at 32 v-heads) and two beyond are best, e.g. at
  // B = 256 6.65 TB/s against 6.20 with one block per head. A bf16 state (half the
  // bytes per row) is best with one block per head (5.8 TB/s against 4.9 with four).
  // At small batch the split grows until the grid covers the SMs several times over.
  int splits = sizeof(S) == 4 ? (heads <= 16384 ? 4 : 2) : 1;
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

namespace gdn {

// ---------------------------------------------------------------- fp8 state option
// State rows stored as FP8 E4M3 with one fp32 scale per row (S[v][k] = fp8[v][k] *
// scale[v]): 132 bytes per 128-element row instead of 512. The row is dequantised,
// updated in fp32 exactly as in decode_kernel, the output is read from the fp32 row,
// and the new row is requantised with scale = max|row| / 448 (E4M3's largest finite
// value), round to nearest, saturating.
namespace {

__device__ __forceinline__ float4 fp8x4_to_f4(uint32_t w, float s) {
  float4 r;
  uint32_t lo2, hi2;  // two halves -> two f16x2 pairs
  asm("{\n\t.reg .b16 a, b;\n\tmov.b32 {a, b}, %2;\n\t"
      "cvt.rn.f16x2.e4m3x2 %0, a;\n\tcvt.rn.f16x2.e4m3x2 %1, b;\n\t}"
      : "=r"(lo2), "=r"(hi2)
      : "r"(w));
  const __half2 h01 = *reinterpret_cast<const __half2*>(&lo2);
  const __half2 h23 = *reinterpret_cast<const __half2*>(&hi2);
  const float2 f01 = __half22float2(h01), f23 = __half22float2(h23);
  r.x = f01.x * s;
  r.y = f01.y * s;
  r.z = f23.x * s;
  r.w = f23.y * s;
  return r;
}

__device__ __forceinline__ uint32_t f4_to_fp8x4(float4 v, float inv_s) {
  uint16_t a, b;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(a) : "f"(v.y * inv_s), "f"(v.x * inv_s));
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(b) : "f"(v.w * inv_s), "f"(v.z * inv_s));
  return static_cast<uint32_t>(a) | (static_cast<uint32_t>(b) << 16);
}

// One warp handles 4 rows per step: lane = 8 * sub + seg, sub = row in the group,
// seg = 16-element segment; a 16-byte load brings 16 E4M3 codes. Dot products and
// the row maximum reduce over the 8 lanes of a row (3 shuffles). G groups of 4 rows
// are loaded before any is processed (memory-level parallelism).
template <int G>
__global__ void __launch_bounds__(128) decode_fp8_kernel(DecodeParams p, const float* scale_in,
                                                          float* scale_out) {
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int sub = lane >> 3, seg = lane & 7;
  const int64_t head = blockIdx.x / p.splits;
  const int split = blockIdx.x - head * p.splits;
  const int64_t bi = head / p.HV;
  const int h = static_cast<int>(head - bi * p.HV);
  const int qh = h / (p.HV / p.HQ);
  const float A_log = load_scalar(p.A_log, p.A_log_dtype, h);
  const float dtb = load_scalar(p.dt_bias, p.dt_bias_dtype, h);
  const float g = expf(gate_log_decay(A_log, load_scalar(p.a, p.a_dtype, head), dtb));
  const float beta = gate_beta(load_scalar(p.b, p.b_dtype, head));
  const int64_t qk_off = (bi * p.HQ + qh) * kHeadDim + seg * 16;
  float qf[16], kf[16];
#pragma unroll
  for (int i = 0; i < 16; i += 4) {
    const float4 q4 = load_bf16x4(p.q + qk_off + i), k4 = load_bf16x4(p.k + qk_off + i);
    qf[i] = q4.x; qf[i + 1] = q4.y; qf[i + 2] = q4.z; qf[i + 3] = q4.w;
    kf[i] = k4.x; kf[i + 1] = k4.y; kf[i + 2] = k4.z; kf[i + 3] = k4.w;
  }
  float kq = 0.f;
#pragma unroll
  for (int i = 0; i < 16; ++i) kq = fmaf(qf[i], kf[i], kq);
#pragma unroll
  for (int o = 1; o < 8; o <<= 1) kq += __shfl_xor_sync(0xffffffffu, kq, o);
  const int rows_per_warp = p.rows_per_warp;
  const int row0 = (split * 4 + warp) * rows_per_warp;
  const int64_t vrow_base = head * kHeadDim;
  const uint4* src = static_cast<const uint4*>(p.state_any);
  uint4* dst = static_cast<uint4*>(p.new_state_any);
  for (int r0 = 0; r0 < rows_per_warp; r0 += 4 * G) {
    uint4 cw[G];
    float sc[G], vin[G];
#pragma unroll
    for (int gi = 0; gi < G; ++gi) {
      const int64_t row = vrow_base + row0 + r0 + 4 * gi + sub;
      if (src) {
        asm volatile("ld.global.cs.v4.u32 {%0,%1,%2,%3}, [%4];"
                     : "=r"(cw[gi].x), "=r"(cw[gi].y), "=r"(cw[gi].z), "=r"(cw[gi].w)
                     : "l"(src + row * 8 + seg));
        sc[gi] = scale_in[row];
      } else {
        cw[gi] = make_uint4(0u, 0u, 0u, 0u);
        sc[gi] = 0.f;
      }
      const unsigned short raw = reinterpret_cast<const unsigned short*>(p.v)[row];
      vin[gi] = __uint_as_float(static_cast<uint32_t>(raw) << 16);
    }
#pragma unroll
    for (int gi = 0; gi < G; ++gi) {
      float s[16];
      const uint32_t w[4] = {cw[gi].x, cw[gi].y, cw[gi].z, cw[gi].w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float4 f = fp8x4_to_f4(w[e], sc[gi]);
        s[4 * e] = f.x; s[4 * e + 1] = f.y; s[4 * e + 2] = f.z; s[4 * e + 3] = f.w;
      }
      float sk = 0.f, sq = 0.f;
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        sk = fmaf(s[i], kf[i], sk);
        sq = fmaf(s[i], qf[i], sq);
      }
#pragma unroll
      for (int o = 1; o < 8; o <<= 1) {
        sk += __shfl_xor_sync(0xffffffffu, sk, o);
        sq += __shfl_xor_sync(0xffffffffu, sq, o);
      }
      const float delta = beta * (vin[gi] - g * sk);
      float m = 0.f;
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        s[i] = fmaf(g, s[i], delta * kf[i]);
        m = fmaxf(m, fabsf(s[i]));
      }
#pragma unroll
      for (int o = 1; o < 8; o <<= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
      const float nsc = m > 0.f ? m * (1.0f / 448.0f) : 1.0f;
      const float inv = 1.0f / nsc;
      uint4 ow;
      ow.x = f4_to_fp8x4(make_float4(s[0], s[1], s[2], s[3]), inv);
      ow.y = f4_to_fp8x4(make_float4(s[4], s[5], s[6], s[7]), inv);
      ow.z = f4_to_fp8x4(make_float4(s[8], s[9], s[10], s[11]), inv);
      ow.w = f4_to_fp8x4(make_float4(s[12], s[13], s[14], s[15]), inv);
      const int64_t row = vrow_base + row0 + r0 + 4 * gi + sub;
      asm volatile("st.global.cs.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(dst + row * 8 + seg),
                   "r"(ow.x), "r"(ow.y), "r"(ow.z), "r"(ow.w)
                   : "memory");
      if (seg == 0) {
        scale_out[row] = nsc;
        p.out[row] = __float2bfloat16_rn(p.scale * fmaf(g, sq, delta * kq));
      }
    }
  }
}


// One head (128 rows) of the fp8 state in shared memory: codes, row scales, v.
constexpr uint32_t kFp8Codes = kHeadDim * kHeadDim;         // 16384 bytes
// + 128 fp32 scales, 128 bf16 v, the head's q and k rows (128 bf16 each)
constexpr uint32_t kFp8StageBytes = kFp8Codes + 512 + 256 + 512;
constexpr int kFp8Stages = 2;
constexpr uint32_t kFp8Smem = kFp8Stages * kFp8StageBytes + 64;

// Three-input maximum (one instruction on sm_100).
__device__ __forceinline__ float max3f(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// Streaming fp8-state decode: a persistent block walks over heads (b, h) and keeps the
// next head's codes, scales and v arriving in shared memory by bulk copy (one mbarrier
// per stage) while it computes the current one, so that every SM has tens of KB of
// loads in flight without holding them in registers. Warp w covers rows 32w..32w+31 in
// 8 steps of 4 rows (lane = 8 sub + seg: 16 codes of row 4 step + sub per lane). The
// row scale multiplies the two dot products once and the update's decay factor once
// (S = c s: S.k = s (c.k), g S + d k = (g s) c + d k); products run as packed f32x2
// operations. New codes, scales and outputs go straight to global memory. A bounded
// wait that gives up marks that head's outputs and scales NaN and ends the block.
template <bool HAS_STATE>
__global__ void __launch_bounds__(128, 4) decode_fp8_stream_kernel(DecodeParams p,
                                                                   const float* scale_in,
                                                                   float* scale_out,
                                                                   int64_t heads) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = sm100::align_smem<128>(smem_raw);
  uint64_t* bar = reinterpret_cast<uint64_t*>(sm + kFp8Stages * kFp8StageBytes);
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const int sub = lane >> 3, seg = lane & 7;
  const int64_t stride = gridDim.x;
  const uint8_t* codes_g = static_cast<const uint8_t*>(p.state_any);
  uint4* dst = static_cast<uint4*>(p.new_state_any);
  if (t == 0) {
    for (int s = 0; s < kFp8Stages; ++s) sm100::mbar_init(&bar[s], 1);
    sm100::fence_mbar_init();
  }
  __syncthreads();
  auto issue = [&](int64_t hd, int s) {  // thread 0: head hd -> stage s
    uint8_t* st = sm + s * kFp8StageBytes;
    sm100::mbar_arrive_expect_tx(&bar[s], (HAS_STATE ? kFp8Codes + 512 : 0) + 768);
    if (HAS_STATE) {
      sm100::bulk_load(st, codes_g + hd * kFp8Codes, kFp8Codes, &bar[s]);
      sm100::bulk_load(st + kFp8Codes, scale_in + hd * kHeadDim, 512, &bar[s]);
    }
    sm100::bulk_load(st + kFp8Codes + 512, p.v + hd * kHeadDim, 256, &bar[s]);
    const int64_t qrow = (hd / p.HV * p.HQ + (hd % p.HV) / (p.HV / p.HQ)) * kHeadDim;
    sm100::bulk_load(st + kFp8Codes + 768, p.q + qrow, 256, &bar[s]);
    sm100::bulk_load(st + kFp8Codes + 1024, p.k + qrow, 256, &bar[s]);
  };
  // the gate inputs of the block's first head; later heads' are loaded one head ahead
  float ga = 0.f, gb = 0.f, gA = 0.f, gd = 0.f;
  if (static_cast<int64_t>(blockIdx.x) < heads) {
    const int h0 = static_cast<int>(blockIdx.x % p.HV);
    ga = load_scalar(p.a, p.a_dtype, blockIdx.x);
    gb = load_scalar(p.b, p.b_dtype, blockIdx.x);
    gA = load_scalar(p.A_log, p.A_log_dtype, h0);
    gd = load_scalar(p.dt_bias, p.dt_bias_dtype, h0);
  }
  if (t == 0) {
    for (int s = 0; s < kFp8Stages; ++s) {
      const int64_t hd = blockIdx.x + s * stride;
      if (hd < heads) issue(hd, s);
    }
  }
  int it = 0;
  for (int64_t head = blockIdx.x; head < heads; head += stride, ++it) {
    const int s = it % kFp8Stages;
    const uint32_t parity = static_cast<uint32_t>((it / kFp8Stages) & 1);
    const float g = expf(gate_log_decay(gA, ga, gd));
    const float beta = gate_beta(gb);
    {  // the next head's gate inputs, consumed one iteration later
      const int64_t nh = head + stride;
      if (nh < heads) {
        const int h1 = static_cast<int>(nh % p.HV);
        ga = load_scalar(p.a, p.a_dtype, nh);
        gb = load_scalar(p.b, p.b_dtype, nh);
        gA = load_scalar(p.A_log, p.A_log_dtype, h1);
        gd = load_scalar(p.dt_bias, p.dt_bias_dtype, h1);
      }
    }
    const bool ok = sm100::mbar_wait(&bar[s], parity);
    if (!__all_sync(0xffffffffu, ok)) {
      // the copies did not arrive: this head's results are marked invalid
      const int64_t row = head * kHeadDim + (kHeadDim / 4) * warp + lane;
      scale_out[row] = __int_as_float(0x7fc00000);
      p.out[row] = __float2bfloat16_rn(__int_as_float(0x7fc00000));
      break;
    }
    // this lane's q/k segment from the stage
    const uint8_t* stq = sm + s * kFp8StageBytes + kFp8Codes + 768;
    float2 qf[8], kf[8];
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const uint4 qw = *reinterpret_cast<const uint4*>(stq + seg * 32 + 16 * i);
      const uint4 kw = *reinterpret_cast<const uint4*>(stq + 256 + seg * 32 + 16 * i);
      const uint32_t qa[4] = {qw.x, qw.y, qw.z, qw.w}, ka[4] = {kw.x, kw.y, kw.z, kw.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        qf[4 * i + e] = make_float2(__uint_as_float(qa[e] << 16), __uint_as_float(qa[e] & 0xffff0000u));
        kf[4 * i + e] = make_float2(__uint_as_float(ka[e] << 16), __uint_as_float(ka[e] & 0xffff0000u));
      }
    }
    float2 kq2 = make_float2(0.f, 0.f);
#pragma unroll
    for (int i = 0; i < 8; ++i) kq2 = sm100::fma2(qf[i], kf[i], kq2);
    float kq = kq2.x + kq2.y;
#pragma unroll
    for (int o = 1; o < 8; o <<= 1) kq += __shfl_xor_sync(0xffffffffu, kq, o);
    const uint8_t* st = sm + s * kFp8StageBytes;
    const float* ssc = reinterpret_cast<const float*>(st + kFp8Codes);
    const unsigned short* sv = reinterpret_cast<const unsigned short*>(st + kFp8Codes + 512);
#pragma unroll 2
    for (int step = 0; step < kHeadDim / 16; ++step) {
      const int r = (kHeadDim / 4) * warp + 4 * step + sub;  // row within the head
      const float vin = __uint_as_float(static_cast<uint32_t>(sv[r]) << 16);
      float2 c[8];
      float cs = 0.f;
      if (HAS_STATE) {
        const uint4 cw = *reinterpret_cast<const uint4*>(st + r * kHeadDim + seg * 16);
        const uint32_t w[4] = {cw.x, cw.y, cw.z, cw.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          uint32_t lo2, hi2;
          asm("{\n\t.reg .b16 a, b;\n\tmov.b32 {a, b}, %2;\n\t"
              "cvt.rn.f16x2.e4m3x2 %0, a;\n\tcvt.rn.f16x2.e4m3x2 %1, b;\n\t}"
              : "=r"(lo2), "=r"(hi2)
              : "r"(w[e]));
          c[2 * e] = __half22float2(*reinterpret_cast<const __half2*>(&lo2));
          c[2 * e + 1] = __half22float2(*reinterpret_cast<const __half2*>(&hi2));
        }
        cs = ssc[r];
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) c[i] = make_float2(0.f, 0.f);
      }
      // two independent accumulator chains per dot product (instruction-level parallelism)
      float2 sk2[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
      float2 sq2[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        sk2[i & 1] = sm100::fma2(c[i], kf[i], sk2[i & 1]);
        sq2[i & 1] = sm100::fma2(c[i], qf[i], sq2[i & 1]);
      }
      float sk = (sk2[0].x + sk2[0].y) + (sk2[1].x + sk2[1].y);
      float sq = (sq2[0].x + sq2[0].y) + (sq2[1].x + sq2[1].y);
#pragma unroll
      for (int o = 1; o < 8; o <<= 1) {
        sk += __shfl_xor_sync(0xffffffffu, sk, o);
        sq += __shfl_xor_sync(0xffffffffu, sq, o);
      }
      sk *= cs;
      sq *= cs;
      const float delta = beta * (vin - g * sk);
      // new row n = (g s) c + d k = gs (c + r k) with r = d / gs: one packed FMA per
      // pair; gs is kept >= 1e-30 (a smaller one changes n by at most 1e-30 |c|), and the
      // row maximum and the quantisation scale carry the factor gs
      const float gs = fmaxf(g * cs, 1e-30f);
      const float rr = __fdividef(delta, gs);
      const float2 r2 = make_float2(rr, rr);
      float mm[2] = {0.f, 0.f};
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        c[i] = sm100::fma2(r2, kf[i], c[i]);
        mm[i & 1] = max3f(mm[i & 1], fabsf(c[i].x), fabsf(c[i].y));
      }
      float m = fmaxf(mm[0], mm[1]);
#pragma unroll
      for (int o = 1; o < 8; o <<= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
      const float nsc = m > 0.f ? gs * m * (1.0f / 448.0f) : 1.0f;
      const float inv = m > 0.f ? __fdividef(448.0f, m) : 1.0f;
      uint32_t ow[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 a = sm100::mul2(c[2 * e], make_float2(inv, inv));
        const float2 b = sm100::mul2(c[2 * e + 1], make_float2(inv, inv));
        uint16_t lo, hi;
        asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(lo) : "f"(a.y), "f"(a.x));
        asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(hi) : "f"(b.y), "f"(b.x));
        ow[e] = static_cast<uint32_t>(lo) | (static_cast<uint32_t>(hi) << 16);
      }
      const int64_t row = head * kHeadDim + r;
      asm volatile("st.global.cs.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(dst + row * 8 + seg),
                   "r"(ow[0]), "r"(ow[1]), "r"(ow[2]), "r"(ow[3])
                   : "memory");
      if (seg == 0) {
        scale_out[row] = nsc;
        p.out[row] = __float2bfloat16_rn(p.scale * fmaf(g, sq, delta * kq));
      }
    }
    __syncthreads();  // every warp is done with stage s
    if (t == 0 && head + kFp8Stages * stride < heads) issue(head + kFp8Stages * stride, s);
  }
}

}  // namespace

int launch_decode_fp8(const DecodeParams& p_in, const float* scale_in, float* scale_out,
                      cudaStream_t stream) {
  DecodeParams p = p_in;
  const int64_t heads = p.B * p.HV;
  if (heads == 0) return 0;
  const auto a16 = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15u) == 0; };
  const bool bulk_ok = a16(p.v) && a16(p.q) && a16(p.k) &&
                       (!p.state_any || (a16(p.state_any) && a16(scale_in)));
  if (heads < 148 * 4 || !bulk_ok) {
    // small batch: rows of a head split over several blocks so that all SMs get work
    int splits = 1;
    while (splits < 8 && heads * splits < 148 * 4) splits *= 2;
    p.splits = splits;
    p.rows_per_warp = kHeadDim / (4 * splits);
    const dim3 grid(static_cast<unsigned>(heads * splits));
    if (p.rows_per_warp >= 16)
      decode_fp8_kernel<4><<<grid, 128, 0, stream>>>(p, scale_in, scale_out);
    else
      decode_fp8_kernel<1><<<grid, 128, 0, stream>>>(p, scale_in, scale_out);
  } else {
    // persistent streaming blocks, as many as fit on the GPU at once
    static int blocks_per_sm[2] = {0, 0}, sms = 0;
    const bool has = p.state_any != nullptr;
    const int nthr = 128;
    auto fn = has ? decode_fp8_stream_kernel<true> : decode_fp8_stream_kernel<false>;
    const int key = has;
    if (!blocks_per_sm[key]) {
      int dev = 0;
      if (cudaGetDevice(&dev) != cudaSuccess ||
          cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
          cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, kFp8Smem + 128) !=
              cudaSuccess ||
          cudaOccupancyMaxActiveBlocksPerMultiprocessor(&blocks_per_sm[key], fn, nthr,
                                                        kFp8Smem + 128) != cudaSuccess)
        return -1;
    }
    const int64_t grid = std::min<int64_t>(heads, static_cast<int64_t>(sms) * blocks_per_sm[key]);
    fn<<<static_cast<unsigned>(grid), nthr, kFp8Smem + 128, stream>>>(p, scale_in, scale_out,
                                                                      heads);
  }
  return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

}  // namespace gdn
