// gdn_capi.cu — the extern "C" boundary declared in include/gdn_b200.h.
//
// Validates arguments on the host (no device reads, no synchronisation),
// fills the internal launch parameters and returns a status code. No C++
// exception escapes: every entry point is noexcept-by-construction.
#include <math.h>

#include "gdn_b200.h"
#include "gdn_launch.h"

namespace {

constexpr int kAbiVersion = 1;

bool gate_dtype_ok(int dt) { return dt == GDN_DTYPE_F32 || dt == GDN_DTYPE_BF16; }

int check_heads(int32_t HQ, int32_t HV, int32_t D) {
  if (D != 128) return GDN_ERR_UNSUPPORTED_SHAPE;
  if (HQ <= 0 || HV <= 0 || HV % HQ != 0) return GDN_ERR_UNSUPPORTED_SHAPE;
  return GDN_OK;
}

float resolve_scale(float scale, int32_t D) {
  // Reference: `if scale is None or scale == 0.0: scale = 1/sqrt(K)`
  // (gdn/decode/baseline/triton/kernel.py:52-53). Negative or NaN is treated the same.
  if (!(scale > 0.0f)) return 1.0f / sqrtf(static_cast<float>(D));
  return scale;
}

int launch_status(int rc) { return rc == 0 ? GDN_OK : GDN_ERR_CUDA; }

int fill_prefill(gdn::PrefillParams* p, const void* q, const void* k, const void* v,
                 const float* state, const void* A_log, int A_log_dtype, const void* a,
                 int a_dtype, const void* dt_bias, int dt_bias_dtype, const void* b, int b_dtype,
                 const void* cu_seqlens, int cu_dtype, float scale, void* out, float* new_state,
                 int64_t T, int64_t N, int32_t HQ, int32_t HV, int32_t D) {
  if (T < 0 || N < 0) return GDN_ERR_INVALID_ARG;
  int rc = check_heads(HQ, HV, D);
  if (rc != GDN_OK) return rc;
  if (!gate_dtype_ok(A_log_dtype) || !gate_dtype_ok(a_dtype) || !gate_dtype_ok(dt_bias_dtype) ||
      !gate_dtype_ok(b_dtype))
    return GDN_ERR_UNSUPPORTED_DTYPE;
  if (cu_dtype != GDN_DTYPE_I32 && cu_dtype != GDN_DTYPE_I64) return GDN_ERR_UNSUPPORTED_DTYPE;
  if (N == 0) return GDN_OK;
  if (!cu_seqlens || !A_log || !dt_bias || !new_state) return GDN_ERR_INVALID_ARG;
  if (T > 0 && (!q || !k || !v || !a || !b || !out)) return GDN_ERR_INVALID_ARG;
  *p = gdn::PrefillParams{};
  p->q = static_cast<const __nv_bfloat16*>(q);
  p->k = static_cast<const __nv_bfloat16*>(k);
  p->v = static_cast<const __nv_bfloat16*>(v);
  p->state = state;
  p->A_log = A_log;
  p->a = a;
  p->dt_bias = dt_bias;
  p->b = b;
  p->A_log_dtype = A_log_dtype;
  p->a_dtype = a_dtype;
  p->dt_bias_dtype = dt_bias_dtype;
  p->b_dtype = b_dtype;
  p->cu_seqlens = cu_seqlens;
  p->cu_dtype = cu_dtype;
  p->scale = resolve_scale(scale, D);
  p->out = static_cast<__nv_bfloat16*>(out);
  p->new_state = new_state;
  p->T = T;
  p->N = N;
  p->HQ = HQ;
  p->HV = HV;
  return GDN_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

constexpr size_t kChunkedWorkspaceBytes = 256;  // fused path: status word (sticky error flag)

}  // namespace

extern "C" {

int gdn_abi_version(void) { return kAbiVersion; }

const char* gdn_status_string(int status) {
  switch (status) {
    case GDN_OK: return "ok";
    case GDN_ERR_INVALID_ARG: return "invalid argument (null pointer or negative size)";
    case GDN_ERR_UNSUPPORTED_SHAPE: return "unsupported shape (need D == 128 and HV % HQ == 0)";
    case GDN_ERR_UNSUPPORTED_DTYPE: return "unsupported dtype code for an argument";
    case GDN_ERR_CUDA: return "CUDA launch or runtime error";
    case GDN_ERR_WORKSPACE: return "workspace missing or too small";
    case GDN_ERR_DEVICE: return "device is not an sm_100 (B200) class GPU";
    default: return "unknown status";
  }
}

int gdn_decode_fwd(const void* q, const void* k, const void* v, const float* state,
                   const void* A_log, int A_log_dtype, const void* a, int a_dtype,
                   const void* dt_bias, int dt_bias_dtype, const void* b, int b_dtype,
                   float scale, void* out, float* new_state, int64_t B, int32_t HQ,
                   int32_t HV, int32_t D, void* stream) {
  if (B < 0) return GDN_ERR_INVALID_ARG;
  int rc = check_heads(HQ, HV, D);
  if (rc != GDN_OK) return rc;
  if (!gate_dtype_ok(A_log_dtype) || !gate_dtype_ok(a_dtype) || !gate_dtype_ok(dt_bias_dtype) ||
      !gate_dtype_ok(b_dtype))
    return GDN_ERR_UNSUPPORTED_DTYPE;
  if (B == 0) return GDN_OK;
  if (!q || !k || !v || !A_log || !a || !dt_bias || !b || !out || !new_state)
    return GDN_ERR_INVALID_ARG;
  gdn::DecodeParams p{};
  p.q = static_cast<const __nv_bfloat16*>(q);
  p.k = static_cast<const __nv_bfloat16*>(k);
  p.v = static_cast<const __nv_bfloat16*>(v);
  p.state = state;
  p.A_log = A_log;
  p.a = a;
  p.dt_bias = dt_bias;
  p.b = b;
  p.A_log_dtype = A_log_dtype;
  p.a_dtype = a_dtype;
  p.dt_bias_dtype = dt_bias_dtype;
  p.b_dtype = b_dtype;
  p.scale = resolve_scale(scale, D);
  p.out = static_cast<__nv_bfloat16*>(out);
  p.new_state = new_state;
  p.B = B;
  p.HQ = HQ;
  p.HV = HV;
  return launch_status(gdn::launch_decode(p, static_cast<cudaStream_t>(stream)));
}

int gdn_decode_fwd_bf16state(const void* q, const void* k, const void* v, const void* state,
                             const void* A_log, int A_log_dtype, const void* a, int a_dtype,
                             const void* dt_bias, int dt_bias_dtype, const void* b, int b_dtype,
                             float scale, void* out, void* new_state, int64_t B, int32_t HQ,
                             int32_t HV, int32_t D, void* stream) {
  if (B < 0) return GDN_ERR_INVALID_ARG;
  int rc = check_heads(HQ, HV, D);
  if (rc != GDN_OK) return rc;
  if (!gate_dtype_ok(A_log_dtype) || !gate_dtype_ok(a_dtype) || !gate_dtype_ok(dt_bias_dtype) ||
      !gate_dtype_ok(b_dtype))
    return GDN_ERR_UNSUPPORTED_DTYPE;
  if (B == 0) return GDN_OK;
  if (!q || !k || !v || !A_log || !a || !dt_bias || !b || !out || !new_state)
    return GDN_ERR_INVALID_ARG;
  gdn::DecodeParams p{};
  p.q = static_cast<const __nv_bfloat16*>(q);
  p.k = static_cast<const __nv_bfloat16*>(k);
  p.v = static_cast<const __nv_bfloat16*>(v);
  p.state_bf16 = 1;
  p.state_any = state;
  p.new_state_any = new_state;
  p.A_log = A_log;
  p.a = a;
  p.dt_bias = dt_bias;
  p.b = b;
  p.A_log_dtype = A_log_dtype;
  p.a_dtype = a_dtype;
  p.dt_bias_dtype = dt_bias_dtype;
  p.b_dtype = b_dtype;
  p.scale = resolve_scale(scale, D);
  p.out = static_cast<__nv_bfloat16*>(out);
  p.B = B;
  p.HQ = HQ;
  p.HV = HV;
  return launch_status(gdn::launch_decode(p, static_cast<cudaStream_t>(stream)));
}

int gdn_decode_fwd_fp8state(const void* q, const void* k, const void* v, const void* state,
                            const float* state_scale, const void* A_log, int A_log_dtype,
                            const void* a, int a_dtype, const void* dt_bias, int dt_bias_dtype,
                            const void* b, int b_dtype, float scale, void* out, void* new_state,
                            float* new_state_scale, int64_t B, int32_t HQ, int32_t HV,
                            int32_t D, void* stream) {
  if (B < 0) return GDN_ERR_INVALID_ARG;
  int rc = check_heads(HQ, HV, D);
  if (rc != GDN_OK) return rc;
  if (!gate_dtype_ok(A_log_dtype) || !gate_dtype_ok(a_dtype) || !gate_dtype_ok(dt_bias_dtype) ||
      !gate_dtype_ok(b_dtype))
    return GDN_ERR_UNSUPPORTED_DTYPE;
  if (B == 0) return GDN_OK;
  if (!q || !k || !v || !A_log || !a || !dt_bias || !b || !out || !new_state ||
      !new_state_scale || (state && !state_scale))
    return GDN_ERR_INVALID_ARG;
  gdn::DecodeParams p{};
  p.q = static_cast<const __nv_bfloat16*>(q);
  p.k = static_cast<const __nv_bfloat16*>(k);
  p.v = static_cast<const __nv_bfloat16*>(v);
  p.state_any = state;
  p.new_state_any = new_state;
  p.A_log = A_log;
  p.a = a;
  p.dt_bias = dt_bias;
  p.b = b;
  p.A_log_dtype = A_log_dtype;
  p.a_dtype = a_dtype;
  p.dt_bias_dtype = dt_bias_dtype;
  p.b_dtype = b_dtype;
  p.scale = resolve_scale(scale, D);
  p.out = static_cast<__nv_bfloat16*>(out);
  p.B = B;
  p.HQ = HQ;
  p.HV = HV;
  return launch_status(
      gdn::launch_decode_fp8(p, state_scale, new_state_scale, static_cast<cudaStream_t>(stream)));
}

int gdn_prefill_recurrent_fwd(const void* q, const void* k, const void* v, const float* state,
                              const void* A_log, int A_log_dtype, const void* a, int a_dtype,
                              const void* dt_bias, int dt_bias_dtype, const void* b,
                              int b_dtype, const void* cu_seqlens, int cu_dtype, float scale,
                              void* out, float* new_state, int64_t T, int64_t N, int32_t HQ,
                              int32_t HV, int32_t D, void* stream) {
  gdn::PrefillParams p;
  int rc = fill_prefill(&p, q, k, v, state, A_log, A_log_dtype, a, a_dtype, dt_bias,
                        dt_bias_dtype, b, b_dtype, cu_seqlens, cu_dtype, scale, out, new_state, T,
                        N, HQ, HV, D);
  if (rc != GDN_OK || N == 0) return rc;
  return launch_status(gdn::launch_prefill_recurrent(p, static_cast<cudaStream_t>(stream)));
}

size_t gdn_prefill_chunked_workspace_size(int64_t T, int64_t N, int32_t HV) {
  if (T < 0 || N < 0 || HV <= 0) return kChunkedWorkspaceBytes;
  const size_t two = gdn::prefill_twophase_workspace_bytes(T, N, HV);
  return two > kChunkedWorkspaceBytes ? two : kChunkedWorkspaceBytes;
}

int gdn_prefill_chunked_fwd(const void* q, const void* k, const void* v, const float* state,
                            const void* A_log, int A_log_dtype, const void* a, int a_dtype,
                            const void* dt_bias, int dt_bias_dtype, const void* b, int b_dtype,
                            const void* cu_seqlens, int cu_dtype, float scale, void* out,
                            float* new_state, int64_t T, int64_t N, int32_t HQ, int32_t HV,
                            int32_t D, void* workspace, size_t workspace_bytes, void* stream) {
  gdn::PrefillParams p;
  int rc = fill_prefill(&p, q, k, v, state, A_log, A_log_dtype, a, a_dtype, dt_bias,
                        dt_bias_dtype, b, b_dtype, cu_seqlens, cu_dtype, scale, out, new_state, T,
                        N, HQ, HV, D);
  if (rc != GDN_OK || N == 0) return rc;
  if (T > 0x7fffffffLL) return GDN_ERR_UNSUPPORTED_SHAPE;  // TMA coordinates are 32-bit
  if (!workspace || workspace_bytes < kChunkedWorkspaceBytes) return GDN_ERR_WORKSPACE;
  if (T > 0 && (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(out)))
    return GDN_ERR_INVALID_ARG;
  p.status = static_cast<int*>(workspace);
  // two-phase (parallel prep + state scan) when the workspace holds the per-chunk
  // [T_b; P] images, otherwise the fused single-kernel path (256 bytes)
  if (workspace_bytes >= gdn::prefill_twophase_workspace_bytes(T, N, HV))
    rc = gdn::launch_prefill_twophase(p, workspace, static_cast<cudaStream_t>(stream));
  else
    rc = gdn::launch_prefill_chunked(p, static_cast<cudaStream_t>(stream));
  if (rc == -2) return GDN_ERR_CUDA;
  return launch_status(rc);
}

int gdn_prefill_chunked_launches(int64_t T, int64_t N, int32_t HV, size_t workspace_bytes) {
  if (T < 0 || N < 0 || HV <= 0) return GDN_ERR_INVALID_ARG;
  if (N == 0) return 0;
  if (workspace_bytes < kChunkedWorkspaceBytes) return GDN_ERR_WORKSPACE;
  if (workspace_bytes < gdn::prefill_twophase_workspace_bytes(T, N, HV)) return 1;
  const int n = gdn::prefill_twophase_launches(T, N, HV);
  return n < 0 ? GDN_ERR_CUDA : n;
}

int gdn_prefill_chunked_status(const void* workspace, int* host_status, void* stream) {
  if (!workspace || !host_status) return GDN_ERR_INVALID_ARG;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (cudaMemcpyAsync(host_status, workspace, sizeof(int), cudaMemcpyDeviceToHost, st) !=
          cudaSuccess ||
      cudaStreamSynchronize(st) != cudaSuccess)
    return GDN_ERR_CUDA;
  return GDN_OK;
}

}  // extern "C"
