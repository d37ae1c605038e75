/*
 * cudalab_gemv.h -- C ABI of the B200 (sm_100a) weight-only quantized GEMV
 * library libcudalab_gemv.so.
 *
 * Operators
 *   INT4 (W4A16):  y[n] = sum_k (scale[n, k/128] * q[n,k]) * x[k]
 *       W_packed uint8 [N, K/2], two 4-bit two's-complement values per byte,
 *       low nibble = element k = 2b, high nibble = element 2b+1;
 *       scale fp16 [N, K/128]; x fp16 [K]; y fp16 [N]; K % 128 == 0.
 *   INT8:          y[n] = sum_k (scale[n] * W_q[n,k]) * x[k]
 *       W_q int8 [N, K]; scale fp32 [N]; x fp16 [K]; y fp16 [N].
 *   Both accumulate in fp32 and round once to fp16 at the end.
 *
 * Conventions
 *   - All pointers are device pointers of one CUDA device (the current one),
 *     row-major and contiguous.  Buffers are owned by the caller; no entry point
 *     allocates device memory or synchronises the stream (except the timing
 *     entry points, which synchronise on purpose).
 *   - `stream` is a cudaStream_t passed as void* (NULL = legacy default stream).
 *   - Every entry point returns CL_OK (0) or a CL_ERR_* status; the message of
 *     the last failure on the calling thread is available from cl_last_error().
 *   - A vectorised variant whose alignment contract is not met (W or x base not
 *     16-byte aligned, or INT8 K % 16 != 0) runs the scalar baseline kernel
 *     instead, so its output is bit-identical to the "*_baseline" variant.
 */
#ifndef CUDALAB_GEMV_H_
#define CUDALAB_GEMV_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ---- */
#define CL_OK 0
#define CL_ERR_UNKNOWN_VARIANT 1 /* variant name not in the registry */
#define CL_ERR_INVALID_ARGUMENT 2 /* null pointer, N/K out of contract, ... */
#define CL_ERR_CUDA 3 /* a CUDA runtime call failed (launch, event, ...) */
#define CL_ERR_BUFFER_TOO_SMALL 4 /* output text buffer too short */
#define CL_ERR_DEVICE_TIMEOUT 5 /* a bounded device-side wait expired */

/* ---- launch flags ---- */
/* Launch with programmatic stream serialization: the GEMV starts streaming its
 * weights and scales while the previous kernel in the stream finishes, and
 * waits for that kernel before it reads x or writes y.  Only valid when W and
 * scale are not written by the kernel immediately before it (static weights). */
#define CL_LAUNCH_PDL 1u
/* Together with CL_LAUNCH_PDL: x is not written by the kernel immediately
 * before this GEMV either (e.g. several projections of one activation, or
 * independent GEMVs issued back to back).  The tensor-core variants then read
 * x and compute before waiting on the preceding kernel and wait only before
 * storing y.  Ignored by variants that do not use it. */
#define CL_LAUNCH_INPUTS_READY 2u
/* Together with CL_LAUNCH_PDL | CL_LAUNCH_INPUTS_READY: y is not read or
 * written by any kernel that may still be running when this GEMV starts
 * (independent output buffers, e.g. the q / k / v projections of one
 * activation, or a stream of independent GEMVs).  The tensor-core variants
 * then store y without waiting; one CTA still waits for the preceding kernel,
 * so the GEMV completes after it and the stream's completion order (and what
 * later kernels may rely on) is unchanged.  Ignored by the sharded entry
 * points and by variants that do not use it. */
#define CL_LAUNCH_OUTPUTS_FREE 4u

/* ---- variant list selectors ---- */
#define CL_VARIANTS_NORMAL 0 /* dispatchable variants */
#define CL_VARIANTS_ALL 1 /* including quarantined ones */
#define CL_VARIANTS_QUARANTINED 2 /* quarantined only */

/* Library version string, e.g. "cudalab-b200 0.1.0 (sm_100a)". */
const char* cl_version(void);

/* Message of the last failing call on this thread ("" if none). */
const char* cl_last_error(void);

/* Reads (and optionally clears) the bounded-wait status word of the current
 * device: 0 = no device-side wait expired since the last clear. */
int cl_device_status(int clear, int* status_out);

/* No counterpart in the reference (its kernels never wait on device-side
 * events).  Sets the bound of every device-side wait of later launches, in SM
 * clock cycles (default 4e9, about two seconds at 2 GHz; cycles <= 0 restores
 * it), process-wide, and writes the previous bound to *previous (may be
 * NULL).  A wait that runs out records CL_ERR_DEVICE_TIMEOUT-class status
 * codes in cl_device_status and its kernel returns; a short bound lets a test
 * make a wait expire without holding the GPU. */
int cl_set_wait_budget(int64_t cycles, int64_t* previous);

/* ---- INT4 W4A16 ---- */

/* Replaces the pybind entry points `forward` / `forward_into` of
 * kernels/int4gemv/bindings.cpp:145-176 (reference interface
 * `int4gemv_forward_into(name, Wp, scale, x, out)`); tensor-level checks
 * (dims, dtypes, devices, contiguity) stay in the Python host wrapper, which
 * applies them in the reference order before calling this function. */
int cl_int4gemv(const char* variant, const uint8_t* W_packed, const void* scale, const void* x,
                void* out, int64_t N, int64_t K, void* stream);

/* Same with launch flags (CL_LAUNCH_*). */
int cl_int4gemv_ex(const char* variant, const uint8_t* W_packed, const void* scale,
                   const void* x, void* out, int64_t N, int64_t K, void* stream, uint32_t flags);

/* Batched form (no reference counterpart: the reference's operator is M = 1;
 * its sharded 70B-class configuration uses M in {1, 4, 16}): X fp16 [M, K] ->
 * Y fp16 [M, N], both row-major and contiguous, M >= 1.  The tensor-core
 * variants dequantise each weight once per 16 activation rows; the other
 * variants run once per row.  Row m of Y equals cl_int4gemv_ex on row m of X
 * up to the fp32 summation order of the variant. */
int cl_int4gemv_batched(const char* variant, const uint8_t* W_packed, const void* scale,
                        const void* X, void* Y, int64_t M, int64_t N, int64_t K, void* stream,
                        uint32_t flags);

/* Replaces `native_timing` of kernels/int4gemv/bindings.cpp:180-253: `warmup`
 * untimed launches, then `n_windows` windows of `launches_per_window`
 * back-to-back launches bracketed by CUDA events on `stream`; writes the
 * per-launch microseconds of each window to per_window_us[n_windows]. */
int cl_int4gemv_native_timing(const char* variant, const uint8_t* W_packed, const void* scale,
                              const void* x, void* out, int64_t N, int64_t K, int64_t warmup,
                              int64_t n_windows, int64_t launches_per_window, void* stream,
                              uint32_t flags, double* per_window_us);

/* Replaces `variants` / `all_variants` / `quarantined_variants` of
 * kernels/int4gemv/bindings.cpp:258-285: writes the sorted names, separated by
 * '\n' and NUL-terminated, into buf[buf_len]; *needed receives the size
 * required including the terminator. */
int cl_int4gemv_list_variants(int which, char* buf, size_t buf_len, size_t* needed);

/* ---- RMSNorm and the fused RMSNorm -> INT4 GEMV ----
 *
 * RMSNorm of fp16 rows with the arithmetic of the reference's rmsnorm_ref
 * (cudalab/reference.py:41-45) and its v4 kernel (kernels/rmsnorm/
 * rmsnorm_v4.cu:84-108): v = mean(x^2) accumulated in fp32, r = 1 / sqrt(v +
 * eps) (correctly rounded here), y = fp16((x * r) * w).
 *
 * cl_rmsnorm_f16 replaces the fp16 path of `forward_into` of the reference's
 * rmsnorm operator (kernels/rmsnorm/bindings.cpp:43-55, 110): X, Y fp16
 * [M, H], weight fp16 [H]; H a multiple of 8 and at most 3 * 2^20, pointers
 * 16-byte aligned, eps finite and >= 0 (bindings.cpp:40).
 *
 * cl_int4gemv_rmsnorm has no reference counterpart: Y[m] = W * RMSNorm(X[m],
 * norm_weight) in one launch per 16 rows (the decoder step "norm, then the
 * quantised projection").  Each CTA reduces the whole activation row and
 * normalises the words it stages, so the normalised activations never go to
 * memory.  W_packed / scale / K as for cl_int4gemv; X fp16 [M, K] and Y fp16
 * [M, N] contiguous; norm_weight fp16 [K]; X, W_packed and norm_weight
 * 16-byte aligned.  The result equals cl_rmsnorm_f16 followed by
 * cl_int4gemv_batched with variant int4gemv_mma_w8c2 (same geometry), bit for
 * bit.  Variants: int4gemv_rmsnorm (geometry per call) and
 * int4gemv_rmsnorm_w2 / _w4 / _w8 / _w8c2 / _w16 (fixed geometry; all give
 * the same bits).  norm_weight is read like W_packed: possibly before the
 * preceding kernel on the stream has completed (under CL_LAUNCH_PDL), so it
 * must not be written by that kernel. */
int cl_rmsnorm_f16(const void* X, const void* weight, float eps, void* Y, int64_t M, int64_t H,
                   void* stream, uint32_t flags);
int cl_int4gemv_rmsnorm(const char* variant, const uint8_t* W_packed, const void* scale,
                        const void* X, const void* norm_weight, float eps, void* Y, int64_t M,
                        int64_t N, int64_t K, void* stream, uint32_t flags);

/* ---- INT8 ---- */

/* Replaces `forward` / `forward_into` of kernels/qgemv/bindings.cpp:66-115
 * (W_q int8 [N,K], scale fp32 [N], x fp16 [K], out fp16 [N]). */
int cl_qgemv(const char* variant, const int8_t* W_q, const float* scale, const void* x, void* out,
             int64_t N, int64_t K, void* stream);

int cl_qgemv_ex(const char* variant, const int8_t* W_q, const float* scale, const void* x,
                void* out, int64_t N, int64_t K, void* stream, uint32_t flags);

/* Batched INT8 (same contract as cl_int4gemv_batched). */
int cl_qgemv_batched(const char* variant, const int8_t* W_q, const float* scale, const void* X,
                     void* Y, int64_t M, int64_t N, int64_t K, void* stream, uint32_t flags);

/* Replaces `native_timing` of kernels/qgemv/bindings.cpp (same contract as
 * cl_int4gemv_native_timing). */
int cl_qgemv_native_timing(const char* variant, const int8_t* W_q, const float* scale,
                           const void* x, void* out, int64_t N, int64_t K, int64_t warmup,
                           int64_t n_windows, int64_t launches_per_window, void* stream,
                           uint32_t flags, double* per_window_us);

/* Replaces `variants` / `all_variants` / `quarantined_variants` of
 * kernels/qgemv/bindings.cpp:281-306. */
int cl_qgemv_list_variants(int which, char* buf, size_t buf_len, size_t* needed);

/* ---- dense GEMV (fp16 or fp32 weights and activations) ----
 * y[n] = sum_k W[n, k] * x[k], fp32 accumulation, one rounding to the
 * element type at the end; W [N, K] row-major, x [K], y [N], all of element
 * type `dtype` (CL_DTYPE_F16 / CL_DTYPE_F32).  Replace `forward` /
 * `forward_into` / `native_timing` / the variant lists of
 * kernels/gemv/bindings.cpp:136-336 (tensor-level checks of
 * bindings.cpp:86-125 are made by the host wrapper).  Variants: gemv_baseline,
 * gemv_vec4_row, gemv_warp_vec4, gemv_splitk4 (quarantined, as in the
 * reference), gemv_mma (fp16: tensor cores; fp32: CUDA cores).  A vectorised
 * variant whose alignment contract is not met (W or x not 16-byte aligned, K
 * not a multiple of the elements per 16 bytes; gemv_mma fp16: of 32) runs the
 * baseline kernel and returns its bits. */
#define CL_DTYPE_F16 0
#define CL_DTYPE_F32 1
int cl_gemv_ex(const char* variant, const void* W, const void* x, void* out, int64_t N, int64_t K,
               int dtype, void* stream, uint32_t flags);
int cl_gemv(const char* variant, const void* W, const void* x, void* out, int64_t N, int64_t K,
            int dtype, void* stream);
int cl_gemv_native_timing(const char* variant, const void* W, const void* x, void* out, int64_t N,
                          int64_t K, int dtype, int64_t warmup, int64_t n_windows,
                          int64_t launches_per_window, void* stream, uint32_t flags,
                          double* per_window_us);
int cl_gemv_list_variants(int which, char* buf, size_t buf_len, size_t* needed);

/* ---- quantisation on the device ----
 * Replace the offline torch quantisers quantize_w of
 * cudalab/int4gemv_quantize.py:61-114 (INT4: group 128, scale fp16 =
 * fp32 amax / 7, q = clamp(round_half_even(W / scale), -7, 7), packed two per
 * byte, low nibble = even k) and cudalab/qgemv_quantize.py:33-64 (INT8: scale
 * fp32 = row amax / 127, q = clamp(round_half_even(W / scale), -127, 127)),
 * byte for byte.  W is fp16 [N, K], row-major, finite; W is 8-byte aligned
 * for INT4. */
int cl_int4gemv_quantize(const void* W, int64_t N, int64_t K, uint8_t* W_packed, void* scale,
                         void* stream);
int cl_qgemv_quantize(const void* W, int64_t N, int64_t K, int8_t* W_q, float* scale,
                      void* stream);

/* ---- row-sharded GEMV over the GPUs of one node (one process per GPU) ----
 *
 * Rows of W are split into contiguous shards, one per rank; x is replicated;
 * every rank ends the step holding all N_total rows of y.  Replaces the
 * "local GEMV, then NCCL all-gather of y" step of the reference's sharded
 * configuration (70B-class MLP shapes; the reference has no multi-GPU code,
 * so there is no reference entry point): here the all-gather is fused into
 * the GEMV epilogue, each CTA storing its rows into every rank's y buffer
 * over NVLink peer mappings and the ranks completing the step through a flag
 * block (no multicast objects are used). */
#define CL_MAX_PEERS 8
#define CL_IPC_HANDLE_BYTES 64
#define CL_PEER_FLAG_BYTES 64 /* size of one rank's flag block (zeroed at allocation) */

/* Allocates `bytes` of device memory on the current device, zero-filled, and
 * writes its CUDA IPC handle (CL_IPC_HANDLE_BYTES bytes) to ipc_handle.  Setup
 * only: the GEMV entry points never allocate. */
int cl_peer_alloc(size_t bytes, void** ptr, void* ipc_handle);
/* Maps another process's cl_peer_alloc buffer into this process. */
int cl_peer_open(const void* ipc_handle, void** peer_ptr);
int cl_peer_close(void* peer_ptr);
int cl_peer_free(void* ptr);

/* One step of the sharded INT4 GEMV on this rank.
 *   W_shard [N_shard, K/2], scale_shard [N_shard, K/128]: rows
 *     [row0, row0 + N_shard) of the full matrix; x fp16 [M, K], 1 <= M <= 16
 *     (the same on every rank).
 *   y_peers[2 * world]: every rank's two y buffers ([M, N_total] halves) as
 *     pointers valid in this process, parity-0 buffers of ranks 0..world-1
 *     first, then the parity-1 buffers (own rank: local pointers).
 *   flag_peers[world]: every rank's flag block (CL_PEER_FLAG_BYTES, zero
 *     before the first step).
 * Step e (1, 2, ... counted on the device, so the call can be captured into a
 * CUDA graph) writes the parity (e & 1) buffers.  All ranks must issue the
 * same steps in the same order.  A rank that waits more than about two
 * seconds for another records status 5 (cl_device_status) instead of
 * hanging; the group must then be set up again. */
int cl_int4gemv_sharded(const char* variant, const uint8_t* W_shard, const void* scale_shard,
                        const void* x, int64_t M, void* const* y_peers, void* const* flag_peers,
                        int rank, int world, int64_t row0, int64_t N_shard, int64_t N_total,
                        int64_t K, void* stream, uint32_t flags);
/* No counterpart in the reference.  The fused step of cl_int4gemv_sharded on
 * one GPU, for callers that may not allocate device memory: code whose host
 * framework (a serving runtime, a plugin host) owns every device allocation
 * and hands it only the tensors it computes on, or code that runs under a
 * fixed device-memory budget that forbids further allocations.  Such callers
 * cannot make the flag block
 * that cl_peer_alloc provides; here it lives in a fixed 256-byte array inside
 * the library (one per GPU that loads it, held until the process exits), so
 * the call allocates nothing.  The caller passes W_packed [N, K/2], scale
 * [N, K/128], x [M, K] and y [M, N] (fp16, 1 <= M <= 16; larger M is rejected
 * with CL_ERR_INVALID_ARGUMENT); y receives W x, the same bits as
 * cl_int4gemv_ex / cl_int4gemv_batched with the same variant family.  The
 * scratch is one flag block whatever N, K and M are.  The first call on a
 * device looks up the array's device address; so does the first call after
 * the device's context changed (e.g. after cudaDeviceReset, which loads the
 * library's device code again at a new address).  Make that first call on
 * each device (and the first after a context change) before any stream
 * capture begins.  Every call clears
 * the block on `stream` before its kernel.  All calls share the one block:
 * calls that overlap on the GPU (other streams, other threads) race and must
 * be serialised by the caller. */
int cl_int4gemv_fused_noalloc(const char* variant, const uint8_t* W_packed, const void* scale,
                              const void* x, int64_t M, void* y, int64_t N, int64_t K,
                              void* stream, uint32_t flags);
/* Same for INT8 (W_shard int8 [N_shard, K], scale_shard fp32 [N_shard], K % 64 == 0). */
int cl_qgemv_sharded(const char* variant, const int8_t* W_shard, const float* scale_shard,
                     const void* x, int64_t M, void* const* y_peers, void* const* flag_peers,
                     int rank, int world, int64_t row0, int64_t N_shard, int64_t N_total,
                     int64_t K, void* stream, uint32_t flags);

#ifdef __cplusplus
} /* extern "C" */
#endif

#endif /* CUDALAB_GEMV_H_ */
