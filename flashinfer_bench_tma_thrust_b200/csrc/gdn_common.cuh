// gdn_common.cuh — device helpers shared by the GDN kernels (sm_100a).
//
// Gate math follows the reference decode/prefill baselines
// (gdn/decode/baseline/triton/kernel.py:57-59, gdn/prefill/baseline/triton/kernel.py:49-51):
//   g    = exp(-exp(A_log) * softplus(a + dt_bias)),  softplus(x) = x > 20 ? x : log1p(exp(x))
//   beta = sigmoid(b)
// computed in fp32 with the full-precision CUDA math functions (no fast-math).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace gdn {

constexpr int kHeadDim = 128;  // D = K = V, fixed by the trace definitions

enum DType : int { kF32 = 0, kBF16 = 1, kI32 = 2, kI64 = 3 };

// Load element i of a gate/parameter vector stored as fp32 or bf16.
__device__ __forceinline__ float load_scalar(const void* p, int dtype, int64_t i) {
  if (dtype == kBF16) {
    const unsigned short raw = reinterpret_cast<const unsigned short*>(p)[i];
    return __uint_as_float(static_cast<uint32_t>(raw) << 16);
  }
  return reinterpret_cast<const float*>(p)[i];
}

// Load element i of cu_seqlens (int32 or int64).
__device__ __forceinline__ int64_t load_index(const void* p, int dtype, int64_t i) {
  if (dtype == kI64) return reinterpret_cast<const int64_t*>(p)[i];
  return static_cast<int64_t>(reinterpret_cast<const int32_t*>(p)[i]);
}

__device__ __forceinline__ float softplus_ref(float x) {
  // torch.nn.functional.softplus with beta=1, threshold=20.
  return x > 20.0f ? x : log1pf(expf(x));
}

// log(g) = -exp(A_log) * softplus(a + dt_bias). Kept in log space for the
// chunked kernel, exponentiated for the recurrent ones.
__device__ __forceinline__ float gate_log_decay(float A_log, float a, float dt_bias) {
  return -expf(A_log) * softplus_ref(a + dt_bias);
}

__device__ __forceinline__ float gate_beta(float b) { return 1.0f / (1.0f + expf(-b)); }

// Four consecutive bf16 values (8 bytes, 8-byte aligned) -> float4.
__device__ __forceinline__ float4 load_bf16x4(const __nv_bfloat16* p) {
  const uint2 raw = *reinterpret_cast<const uint2*>(p);
  float4 r;
  r.x = __uint_as_float(raw.x << 16);
  r.y = __uint_as_float(raw.x & 0xffff0000u);
  r.z = __uint_as_float(raw.y << 16);
  r.w = __uint_as_float(raw.y & 0xffff0000u);
  return r;
}

__device__ __forceinline__ float warp_sum(float x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}

// Streaming 128-bit global load/store of state rows: each state element is
// touched exactly once per launch, so keep it out of L1 and mark it first to
// evict in L2.
__device__ __forceinline__ float4 ld_stream_f4(const float* p) {
  float4 r;
  asm volatile("ld.global.cs.v4.f32 {%0,%1,%2,%3}, [%4];"
               : "=f"(r.x), "=f"(r.y), "=f"(r.z), "=f"(r.w)
               : "l"(p));
  return r;
}

__device__ __forceinline__ void st_stream_f4(float* p, float4 v) {
  asm volatile("st.global.cs.v4.f32 [%0], {%1,%2,%3,%4};" ::"l"(p), "f"(v.x), "f"(v.y),
               "f"(v.z), "f"(v.w)
               : "memory");
}

}  // namespace gdn
