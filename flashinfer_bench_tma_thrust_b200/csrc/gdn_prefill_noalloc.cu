// gdn_prefill_noalloc.cu — chunked prefill for callers that cannot allocate.
//
// The chunked prefill needs a small scratch buffer (its status word). The
// regular entry point takes it from the caller. Some callers have no way to
// provide one: a serving engine that reserves its whole memory budget at start-up
// and forbids allocations afterwards (a cudaMalloc in the middle of a step can
// fail once the pool owns the device memory, and it can synchronise the device,
// stalling every stream), or host code reaching this library through a thin FFI
// that has no CUDA allocator of its own. For them this entry point uses a
// fixed-size scratch array compiled into the library: every GPU that loads the
// library holds kNoAllocScratchBytes of device memory for it until the process
// exits, and no call allocates anything.
#include <mutex>

#include "gdn_b200.h"

namespace {

constexpr size_t kNoAllocScratchBytes = 4096;  // stated maximum scratch for one call
constexpr size_t kFusedScratchBytes = 256;     // what the fused single-kernel path needs
constexpr int kMaxDevices = 64;

// The scratch itself. In host code this name is only a stand-in for the device
// symbol, not a device address: its address must come from cudaGetSymbolAddress.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_setup_mutex;
void* g_scratch_ptr[kMaxDevices] = {};

// Per-device set-up, done once on the first call for that device (with that
// device current): resolve the device address of the scratch array.
int scratch_for_current_device(void** out) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return GDN_ERR_CUDA;
  std::lock_guard<std::mutex> lock(g_setup_mutex);
  if (!g_scratch_ptr[dev]) {
    void* ptr = nullptr;
    if (cudaGetSymbolAddress(&ptr, g_noalloc_scratch) != cudaSuccess || !ptr) return GDN_ERR_CUDA;
    g_scratch_ptr[dev] = ptr;
  }
  *out = g_scratch_ptr[dev];
  return GDN_OK;
}

}  // namespace

extern "C" int gdn_prefill_chunked_fwd_noalloc(
    const void* q, const void* k, const void* v, const float* state, const void* A_log,
    int A_log_dtype, const void* a, int a_dtype, const void* dt_bias, int dt_bias_dtype,
    const void* b, int b_dtype, const void* cu_seqlens, int cu_dtype, float scale, void* out,
    float* new_state, int64_t T, int64_t N, int32_t HQ, int32_t HV, int32_t D, void* stream) {
  // Given less workspace than its two-phase path needs, gdn_prefill_chunked_fwd runs
  // the fused single-kernel path, whose scratch is the 256-byte status word.
  const size_t need = kFusedScratchBytes;
  if (need > kNoAllocScratchBytes) return GDN_ERR_WORKSPACE;
  void* scratch = nullptr;
  const int rc = scratch_for_current_device(&scratch);
  if (rc != GDN_OK) return rc;
  // The array keeps whatever the previous call left in it; the status word must
  // start at zero for this call. A memset enqueued on the stream allocates nothing.
  if (cudaMemsetAsync(scratch, 0, need, static_cast<cudaStream_t>(stream)) != cudaSuccess)
    return GDN_ERR_CUDA;
  return gdn_prefill_chunked_fwd(q, k, v, state, A_log, A_log_dtype, a, a_dtype, dt_bias,
                                 dt_bias_dtype, b, b_dtype, cu_seqlens, cu_dtype, scale, out,
                                 new_state, T, N, HQ, HV, D, scratch, kNoAllocScratchBytes,
                                 stream);
}
