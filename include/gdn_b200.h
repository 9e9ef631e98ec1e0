/*
 * gdn_b200.h — C ABI of the B200 (sm_100a) Gated Delta Net operators.
 *
 * Every entry point takes plain device pointers, sizes and a cudaStream_t passed
 * as void*, launches asynchronously on that stream and returns a status code
 * (GDN_OK or a negative GDN_ERR_*). No exception crosses this boundary and no
 * entry point synchronises the host with the device.
 *
 * Tensors are dense row-major (C-contiguous). Shapes use the names of the
 * reference's trace definitions (gdn/trace_definitions/gdn_{decode,prefill}_
 * qk4_v8_d128_k_last.json): q/k [.., HQ, D], v [.., HV, D], state k-last
 * [.., HV, V=D, K=D] fp32. D must be 128 and HV a multiple of HQ (GVA: v-head h
 * reads q/k head h / (HV/HQ)).
 *
 * The reference binds its kernels through torch-typed pybind wrappers
 * (gdn/decode/solution/cuda/kernel.py:295-364) and through void C launchers
 * with raw pointers (gdn/gdn_kernels.cu:26-170); these functions replace both
 * with one status-returning C interface.
 */
#ifndef GDN_B200_H
#define GDN_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define GDN_API __attribute__((visibility("default")))
#else
#define GDN_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes. */
#define GDN_OK 0
#define GDN_ERR_INVALID_ARG (-1)      /* null pointer where one is required, negative size */
#define GDN_ERR_UNSUPPORTED_SHAPE (-2)/* D != 128, HV not a multiple of HQ, ... */
#define GDN_ERR_UNSUPPORTED_DTYPE (-3)/* dtype code not accepted for that argument */
#define GDN_ERR_CUDA (-4)             /* a CUDA runtime call or a kernel launch failed */
#define GDN_ERR_WORKSPACE (-5)        /* workspace null or smaller than required */
#define GDN_ERR_DEVICE (-6)           /* device is not sm_100 class */

/* Element type codes for arguments that accept more than one type. */
#define GDN_DTYPE_F32 0
#define GDN_DTYPE_BF16 1
#define GDN_DTYPE_I32 2
#define GDN_DTYPE_I64 3

/* Version of this ABI; bumped on any signature change. */
GDN_API int gdn_abi_version(void);

/* Human-readable text for a status code (static storage). */
GDN_API const char* gdn_status_string(int status);

/*
 * Single-token decode: one recurrent step for B sequences.
 *
 * Replaces the solution entry kernel(q,k,v,state,A_log,a,dt_bias,b,scale)
 * of gdn/decode/solution/triton/kernel.py:85-135 (same math as the PyTorch
 * baseline gdn/decode/baseline/triton/kernel.py:27-100).
 *
 *   q, k      bf16 [B, HQ, D]       (the reference's [B, 1, HQ, D])
 *   v         bf16 [B, HV, D]
 *   state     fp32 [B, HV, D, D] k-last, or NULL for a zero initial state
 *   A_log     [HV]    dtype A_log_dtype   (F32 or BF16)
 *   a         [B, HV] dtype a_dtype       (F32 or BF16)
 *   dt_bias   [HV]    dtype dt_bias_dtype (F32 or BF16)
 *   b         [B, HV] dtype b_dtype       (F32 or BF16)
 *   scale     output scale; <= 0 selects 1/sqrt(D) (reference: None or 0.0)
 *   out       bf16 [B, HV, D]
 *   new_state fp32 [B, HV, D, D] k-last. May alias `state` (in-place update):
 *             every element is read and then written by the same thread.
 *
 * B == 0 is a no-op returning GDN_OK. Offsets are 64-bit (B up to 2^31-1).
 */
GDN_API int gdn_decode_fwd(const void* q, const void* k, const void* v, const float* state,
                   const void* A_log, int A_log_dtype, const void* a, int a_dtype,
                   const void* dt_bias, int dt_bias_dtype, const void* b, int b_dtype,
                   float scale, void* out, float* new_state, int64_t B, int32_t HQ,
                   int32_t HV, int32_t D, void* stream);

/*
 * Decode with a bf16 recurrent state (reduced-precision option, reported
 * separately from the fp32 path): state / new_state are bf16 [B, HV, D, D]
 * k-last; the math is fp32 and the new state is rounded to bf16 on store, which
 * halves the state bytes streamed through HBM. Counterpart of the reference's
 * gdn_decode_kernel_v10_bf16 (gdn/kernels/cute_cpp/gdn_decode_v10.cuh:517-659).
 * Other arguments as gdn_decode_fwd; new_state may alias state.
 */
GDN_API int gdn_decode_fwd_bf16state(const void* q, const void* k, const void* v,
                                     const void* state, const void* A_log, int A_log_dtype,
                                     const void* a, int a_dtype, const void* dt_bias,
                                     int dt_bias_dtype, const void* b, int b_dtype, float scale,
                                     void* out, void* new_state, int64_t B, int32_t HQ,
                                     int32_t HV, int32_t D, void* stream);

/*
 * Decode with an FP8 (E4M3) recurrent state and one fp32 scale per state row
 * (reduced-precision option, reported separately): state / new_state uint8
 * [B, HV, D, D] k-last holding E4M3 codes, state_scale / new_state_scale fp32
 * [B, HV, D] with S[v][k] = code[v][k] * scale[v]. fp32 math; the new row is
 * requantised with scale = max|row| / 448. Counterpart of the reference's
 * gdn_decode_kernel_v10_fp8 (gdn/kernels/cute_cpp/gdn_decode_v10.cuh:666-862).
 * state may be NULL (zeros); new_state / new_state_scale may alias the inputs.
 */
GDN_API int gdn_decode_fwd_fp8state(const void* q, const void* k, const void* v,
                                    const void* state, const float* state_scale,
                                    const void* A_log, int A_log_dtype, const void* a,
                                    int a_dtype, const void* dt_bias, int dt_bias_dtype,
                                    const void* b, int b_dtype, float scale, void* out,
                                    void* new_state, float* new_state_scale, int64_t B,
                                    int32_t HQ, int32_t HV, int32_t D, void* stream);

/*
 * Variable-length prefill over cu_seqlens-packed sequences, token-sequential
 * recurrence (one thread block per sequence, v-head and 32-row V tile, the
 * state tile held in registers across the whole sequence).
 *
 * Same semantics as gdn/prefill/baseline/triton/kernel.py:18-100; the
 * structure of gdn/prefill/solution/triton/kernel.py:99-209. Kept as an
 * independent second implementation to cross-check the chunked kernel at
 * sizes the CPU oracle cannot reach.
 *
 *   q, k        bf16 [T, HQ, D];  v bf16 [T, HV, D]
 *   state       fp32 [N, HV, D, D] k-last or NULL (zeros)
 *   a, b        [T, HV] (F32 or BF16);  A_log, dt_bias [HV] (F32 or BF16)
 *   cu_seqlens  [N+1] int32 or int64 (cu_dtype), device memory
 *   out         bf16 [T, HV, D];  new_state fp32 [N, HV, D, D]
 *
 * A sequence with end <= start copies its initial state through (zeros when
 * state is NULL), as the reference does (baseline kernel.py:68-71). Token
 * indices are clamped to [0, T] so a malformed cu_seqlens cannot read or write
 * outside the buffers. new_state must not alias state.
 */
GDN_API int gdn_prefill_recurrent_fwd(const void* q, const void* k, const void* v, const float* state,
                              const void* A_log, int A_log_dtype, const void* a, int a_dtype,
                              const void* dt_bias, int dt_bias_dtype, const void* b,
                              int b_dtype, const void* cu_seqlens, int cu_dtype, float scale,
                              void* out, float* new_state, int64_t T, int64_t N, int32_t HQ,
                              int32_t HV, int32_t D, void* stream);

/*
 * Variable-length prefill, chunked tensor-core kernel (the fast path).
 *
 * Replaces the solution entry kernel(q,k,v,state,A_log,a,dt_bias,b,cu_seqlens,
 * scale) of gdn/prefill/solution/triton/kernel.py:272-347 and the reference's
 * chunked tcgen05 prototype entry gdn/prefill/solution/cuda/chunked_proto.py:
 * 2671-2709 (which drives a CUTLASS GEMM through ctypes from a Python loop
 * over chunks); semantics of gdn/prefill/baseline/triton/kernel.py:18-100.
 * Arguments as gdn_prefill_recurrent_fwd, plus:
 *
 *   workspace        device memory, 16-byte aligned, zeroed once by the caller
 *                    before its first use. With at least
 *                    gdn_prefill_chunked_workspace_size(T, N, HV) bytes the call
 *                    runs the two-phase path (a parallel prep kernel over all
 *                    (chunk, v-head) pairs writes 24.5 KB per pair — the [T_b; P]
 *                    operand image and the chunk's gates — then the state scan);
 *                    with less, but at least 256 bytes, it runs the fused
 *                    single-kernel path. The first 4 bytes are a sticky status
 *                    word, a bit set (read it with gdn_prefill_chunked_status):
 *                    bit 0 = one of a kernel's bounded waits gave up (that call's
 *                    outputs are invalid); bit 1 = cu_seqlens held a value outside
 *                    [0, T] (used clamped) or overlapping ranges whose chunks
 *                    overflow the two-phase workspace (that call computed nothing
 *                    and passed the states through). Calls that share a workspace
 *                    must be stream-ordered.
 *
 * q, k, v and out must be 16-byte aligned (q/k are read by TMA); T < 2^31.
 * Stream-ordered launches, no host synchronisation (two-phase path: chunk offsets,
 * chunk gates, prep, scan; fused path: one kernel). When the (sequence, v-head) scan
 * chains leave at least 8 SMs idle and sequences average 64+ chunks, the two-phase call
 * is split: the prep of each sequence's last chunks runs on a low-priority side stream
 * of the library (one per device, created on the first such call, with two events)
 * concurrently with the first part of the scan, joined back into `stream` by an event
 * before the scan's second part; environment variable GDN_PREFILL_OVERLAP=0 turns this
 * off. The side stream and its events are created by the first split call on a device:
 * make that call before any stream capture on that device. Split calls from several host
 * threads are safe (a per-device lock orders their event records and waits). The work runs in fp32 on the state
 * with tensor-core products carried as bf16 hi/lo pairs (about 16 significant bits).
 */
GDN_API size_t gdn_prefill_chunked_workspace_size(int64_t T, int64_t N, int32_t HV);

GDN_API int gdn_prefill_chunked_fwd(const void* q, const void* k, const void* v,
                                    const float* state, const void* A_log, int A_log_dtype,
                                    const void* a, int a_dtype, const void* dt_bias,
                                    int dt_bias_dtype, const void* b, int b_dtype,
                                    const void* cu_seqlens, int cu_dtype, float scale, void* out,
                                    float* new_state, int64_t T, int64_t N, int32_t HQ,
                                    int32_t HV, int32_t D, void* workspace,
                                    size_t workspace_bytes, void* stream);

/* Number of kernel launches a gdn_prefill_chunked_fwd call with these sizes and this
 * workspace size makes on the current device: 1 on the fused path; on the two-phase path
 * 4 (5 above 1024 sequences), plus 2 when the call is split (see above), fewer when
 * T = 0. No counterpart in the reference (a diagnostic; launches nothing). Returns a
 * negative status code on bad sizes or if the device cannot be queried. */
GDN_API int gdn_prefill_chunked_launches(int64_t T, int64_t N, int32_t HV,
                                         size_t workspace_bytes);

/* Copy the workspace status word (the bit set above) to *host_status (synchronises
 * `stream`). Clearing it is the caller's: it is the workspace's first 4 bytes. */
GDN_API int gdn_prefill_chunked_status(const void* workspace, int* host_status, void* stream);

/*
 * Chunked prefill that allocates nothing. No counterpart in the reference.
 *
 * For callers that cannot hand the library device memory: a serving engine
 * whose memory pool owns the whole device and forbids allocations during a
 * step (a cudaMalloc there can fail or synchronise the device), or an FFI
 * caller without a CUDA allocator. Same arguments as gdn_prefill_chunked_fwd
 * minus the workspace; the scratch is a 4096-byte array compiled into the
 * library, held on every GPU that loads it until the process exits.
 *
 * - The first call on a device (with that device current) looks up the
 *   array's device address once; make that first call before any stream
 *   capture on that device.
 * - Runs the fused single-kernel path, whose scratch is 256 bytes for any T,
 *   N and HV; returns GDN_ERR_WORKSPACE if a call would need more than 4096.
 * - All calls share the one array, which keeps the previous call's contents;
 *   each call zeroes the part it uses with a memset on `stream`. Calls whose
 *   work overlaps on the GPU (different streams without ordering) race on it.
 * - The status word is not readable from outside; outputs are valid unless a
 *   bounded wait inside the kernel gave up.
 * - Calls no cudaMalloc, cudaFree or other allocating routine.
 */
GDN_API int gdn_prefill_chunked_fwd_noalloc(const void* q, const void* k, const void* v,
                                            const float* state, const void* A_log,
                                            int A_log_dtype, const void* a, int a_dtype,
                                            const void* dt_bias, int dt_bias_dtype,
                                            const void* b, int b_dtype, const void* cu_seqlens,
                                            int cu_dtype, float scale, void* out,
                                            float* new_state, int64_t T, int64_t N, int32_t HQ,
                                            int32_t HV, int32_t D, void* stream);

/*
 * Diagnostics. Known-answer check of the tensor-core path the chunked prefill
 * is built on (no counterpart in the reference): D[128x64] fp32 = A[128x128] x
 * B[128x64], bf16 row-major inputs, staged in shared memory in the K-major
 * (0) or MN-major (1) 128B-swizzled layout and multiplied with tcgen05.mma
 * into TMEM. *status (device int, caller zeroes it) becomes 1 if the
 * completion wait timed out.
 */
GDN_API int gdn_selftest_umma(const void* A, const void* B, float* D, int a_mn_major,
                              int b_mn_major, int* status, void* stream);

/*
 * Diagnostics. Known-answer check of the tensor-core product with A read from
 * tensor memory (no counterpart in the reference): D[128x128] fp32 =
 * A[128x128] x B[128x128], bf16 row-major inputs ([m][k] and [k][n]); A is
 * stored into TMEM row by row (two bf16 per 32-bit column), B in shared memory.
 */
GDN_API int gdn_selftest_umma_ts(const void* A, const void* B, float* D, int* status,
                                 void* stream);

/*
 * Diagnostics. The bounded mbarrier wait used by every kernel here, run on a
 * barrier that nothing arrives on (no counterpart in the reference): the wait
 * gives up after about one second, *status (device int) becomes 1 and
 * *waited_ns (device int64) holds the time waited; the context stays usable.
 */
GDN_API int gdn_selftest_wait_timeout(int* status, long long* waited_ns, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* GDN_B200_H */
