// Bench-only comparator (test / measurement infrastructure, never linked into the
// product): a C entry point over the reference's own decode kernel family "v10"
// (gdn/kernels/cute_cpp/gdn_decode_v10.cuh, launchers at :1066-1170), compiled from
// the reference checkout's header where it lies by oracle/build_ref.py into
// oracle/_ref/libref_v10.so. Tensors as the reference's packaged CUDA solution passes
// them (gdn/decode/solution/cuda/kernel.py:496-531): q/k [B, HQ, 128], v [B, HV, 128],
// a/b [B, HV] bf16, A_log/dt_bias fp32, state/new_state [B, HV, 128, 128] fp32,
// out [B, HV, 128] bf16, all contiguous; int strides as the reference computes them.
#include "gdn_decode_v10.cuh"

extern "C" __attribute__((visibility("default"))) int ref_v10_decode(
    int variant, const void* q, const void* k, const void* v, const void* state,
    const void* A_log, const void* a, const void* dt_bias, const void* b, void* out,
    void* new_state, float scale, int B, int HQ, int HV, int block_v, void* stream) {
  const int D = 128;
  auto fn = variant == 1 ? gdn::gdn_decode_v10_launch_tma : gdn::gdn_decode_v10_launch_cute;
  fn(q, k, v, state, A_log, a, dt_bias, b, out, new_state, scale, B, HV, D,
     /*q*/ HQ * D, D, /*k*/ HQ * D, D, /*v*/ HV * D, D,
     /*state*/ HV * D * D, D * D, D, /*a*/ HV, /*b*/ HV, /*out*/ HV * D, D,
     /*new_state*/ HV * D * D, D * D, D, block_v, static_cast<cudaStream_t>(stream));
  return static_cast<int>(cudaGetLastError());
}
