// gdn_launch.h — internal (C++) launch parameters shared between the C ABI
// layer (gdn_capi.cu) and the kernel translation units.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace gdn {

struct DecodeParams {
  const __nv_bfloat16* q;  // [B, HQ, D]
  const __nv_bfloat16* k;  // [B, HQ, D]
  const __nv_bfloat16* v;  // [B, HV, D]
  const float* state;      // [B, HV, D, D] or nullptr
  const void* A_log;
  const void* a;
  const void* dt_bias;
  const void* b;
  int A_log_dtype, a_dtype, dt_bias_dtype, b_dtype;
  float scale;
  __nv_bfloat16* out;  // [B, HV, D]
  float* new_state;    // [B, HV, D, D]
  int64_t B;
  int HQ, HV;
  int splits;         // thread blocks per head (set by the launcher)
  int rows_per_warp;  // set by the launcher
  int state_bf16;             // 1: state / new_state are bf16 (state_any / new_state_any)
  const void* state_any;      // bf16 state (or nullptr)
  void* new_state_any;        // bf16 new state
};

struct PrefillParams {
  const __nv_bfloat16* q;  // [T, HQ, D]
  const __nv_bfloat16* k;  // [T, HQ, D]
  const __nv_bfloat16* v;  // [T, HV, D]
  const float* state;      // [N, HV, D, D] or nullptr
  const void* A_log;
  const void* a;  // [T, HV]
  const void* dt_bias;
  const void* b;  // [T, HV]
  int A_log_dtype, a_dtype, dt_bias_dtype, b_dtype;
  const void* cu_seqlens;  // [N+1]
  int cu_dtype;
  float scale;
  __nv_bfloat16* out;  // [T, HV, D]
  float* new_state;    // [N, HV, D, D]
  int64_t T, N;
  int HQ, HV;
  int* status;  // chunked kernel: set to 1 if a bounded wait gave up (sticky)
};

int launch_decode(const DecodeParams& p, cudaStream_t stream);
int launch_decode_fp8(const DecodeParams& p, const float* scale_in, float* scale_out,
                      cudaStream_t stream);
int launch_prefill_recurrent(const PrefillParams& p, cudaStream_t stream);
int launch_prefill_chunked(const PrefillParams& p, cudaStream_t stream);
size_t prefill_twophase_workspace_bytes(int64_t T, int64_t N, int HV);
int launch_prefill_twophase(const PrefillParams& p, void* workspace, cudaStream_t stream);
// kernel launches a two-phase call of these sizes makes on the current device (split
// calls included), or -1 if the device cannot be queried
int prefill_twophase_launches(int64_t T, int64_t N, int HV);

}  // namespace gdn
