// C ABI of libcudalab_gemv.so (declarations: include/cudalab_gemv.h).
//
// Plain pointers and sizes only.  This layer owns: the variant registry
// lookup, the pointer/size contract checks that do not need tensor metadata,
// status codes + a per-thread error message, and the native launch-loop timer.
// Tensor-level checks (dims, dtypes, devices, contiguity) are made by the host
// wrapper before the call, in the order of the reference extension.
#include <cuda.h>  // CUcontext / CUresult types; the driver functions come via the runtime
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/cudalab_gemv.h"
#include "gemv_launch.h"
#include "gemv_quantize.h"

namespace {

thread_local std::string g_last_error;

int fail(int code, const std::string& msg) {
    g_last_error = msg;
    return code;
}

int cuda_fail(cudaError_t e, const char* what) {
    return fail(CL_ERR_CUDA, std::string(what) + ": " + cudaGetErrorName(e) + " (" +
                                 cudaGetErrorString(e) + ")");
}

const clb::VariantDesc* find(const clb::VariantDesc* table, int n, const char* name) {
    if (name == nullptr) return nullptr;
    for (int i = 0; i < n; ++i)
        if (std::strcmp(table[i].name, name) == 0) return &table[i];
    return nullptr;
}

std::string unknown_msg(const char* op, const clb::VariantDesc* table, int n, const char* name) {
    std::vector<std::string> names;
    for (int i = 0; i < n; ++i)
        if (!table[i].quarantined) names.emplace_back(table[i].name);
    std::sort(names.begin(), names.end());
    std::string s = std::string("unknown ") + op + " variant '" + (name ? name : "(null)") +
                    "'; available: ";
    for (auto& v : names) s += v + " ";
    return s;
}

int list_variants(const clb::VariantDesc* table, int n, int which, char* buf, size_t len,
                  size_t* needed) {
    std::vector<std::string> names;
    for (int i = 0; i < n; ++i) {
        const bool q = table[i].quarantined;
        if (which == CL_VARIANTS_NORMAL && q) continue;
        if (which == CL_VARIANTS_QUARANTINED && !q) continue;
        names.emplace_back(table[i].name);
    }
    std::sort(names.begin(), names.end());
    std::string joined;
    for (size_t i = 0; i < names.size(); ++i) {
        if (i) joined += '\n';
        joined += names[i];
    }
    if (needed) *needed = joined.size() + 1;
    if (which != CL_VARIANTS_NORMAL && which != CL_VARIANTS_ALL && which != CL_VARIANTS_QUARANTINED)
        return fail(CL_ERR_INVALID_ARGUMENT, "list_variants: unknown selector");
    if (buf == nullptr || len < joined.size() + 1)
        return fail(CL_ERR_BUFFER_TOO_SMALL, "list_variants: buffer too small");
    std::memcpy(buf, joined.c_str(), joined.size() + 1);
    return CL_OK;
}

// Shared argument checks.  is_int4 adds the group-size contract K % 128 == 0;
// `scale` may be null only for the dense GEMV (pass its W instead).
int check_args(const char* op, const void* W, const void* scale, const void* x, const void* out,
               int64_t N, int64_t K, bool is_int4) {
    if (N <= 0) return fail(CL_ERR_INVALID_ARGUMENT, std::string(op) + ": N must be > 0");
    if (K <= 0) return fail(CL_ERR_INVALID_ARGUMENT, std::string(op) + ": K must be > 0");
    if (is_int4 && (K % 128) != 0)
        return fail(CL_ERR_INVALID_ARGUMENT,
                    std::string(op) + ": K must be divisible by 128 (group_size=128)");
    if (N > (int64_t)1 << 31)
        return fail(CL_ERR_INVALID_ARGUMENT, std::string(op) + ": N exceeds 2^31 rows");
    if (!W || !scale || !x || !out)
        return fail(CL_ERR_INVALID_ARGUMENT, std::string(op) + ": null device pointer");
    return CL_OK;
}

int run(const clb::VariantDesc* table, int n, const char* op, const char* variant, const void* W,
        const void* scale, const void* x, void* out, int64_t N, int64_t K, void* stream,
        uint32_t flags, bool is_int4) {
    const clb::VariantDesc* v = find(table, n, variant);
    if (!v) return fail(CL_ERR_UNKNOWN_VARIANT, unknown_msg(op, table, n, variant));
    const int rc = check_args(op, W, scale, x, out, N, K, is_int4);
    if (rc != CL_OK) return rc;
    const clb::GemvArgs a{W, scale, x, out, N, K, 1, K, N};
    cudaError_t e = v->fn(a, static_cast<cudaStream_t>(stream), flags);
    if (e != cudaSuccess) return cuda_fail(e, "kernel launch");
    return CL_OK;
}

// Batched: X [M, K] -> Y [M, N], both row-major and contiguous; the
// tensor-core kernels take up to 16 activation rows per launch.
int run_batched(const clb::VariantDesc* table, int n, const char* op, const char* variant,
                const void* W, const void* scale, const void* X, void* Y, int64_t M, int64_t N,
                int64_t K, void* stream, uint32_t flags, bool is_int4) {
    const clb::VariantDesc* v = find(table, n, variant);
    if (!v) return fail(CL_ERR_UNKNOWN_VARIANT, unknown_msg(op, table, n, variant));
    if (M <= 0) return fail(CL_ERR_INVALID_ARGUMENT, std::string(op) + ": M must be > 0");
    const int rc = check_args(op, W, scale, X, Y, N, K, is_int4);
    if (rc != CL_OK) return rc;
    constexpr int64_t kPass = 16;
    for (int64_t m0 = 0; m0 < M; m0 += kPass) {
        const clb::GemvArgs a{W, scale, static_cast<const uint16_t*>(X) + m0 * K,
                              static_cast<uint16_t*>(Y) + m0 * N, N, K,
                              std::min<int64_t>(kPass, M - m0), K, N};
        cudaError_t e = v->fn(a, static_cast<cudaStream_t>(stream), flags);
        if (e != cudaSuccess) return cuda_fail(e, "kernel launch");
    }
    return CL_OK;
}

int timing(const clb::VariantDesc* table, int n, const char* op, const char* variant,
           const void* W, const void* scale, const void* x, void* out, int64_t N, int64_t K,
           int64_t warmup, int64_t n_windows, int64_t lpw, void* stream_v, uint32_t flags,
           double* per_window_us, bool is_int4) {
    const clb::VariantDesc* v = find(table, n, variant);
    if (!v) return fail(CL_ERR_UNKNOWN_VARIANT, unknown_msg(op, table, n, variant));
    if (warmup < 0) return fail(CL_ERR_INVALID_ARGUMENT, "warmup must be >= 0");
    if (n_windows < 1) return fail(CL_ERR_INVALID_ARGUMENT, "n_windows must be >= 1");
    if (lpw < 1) return fail(CL_ERR_INVALID_ARGUMENT, "launches_per_window must be >= 1");
    if (!per_window_us) return fail(CL_ERR_INVALID_ARGUMENT, "per_window_us is null");
    int rc = check_args(op, W, scale, x, out, N, K, is_int4);
    if (rc != CL_OK) return rc;
    cudaStream_t s = static_cast<cudaStream_t>(stream_v);
    const clb::GemvArgs a{W, scale, x, out, N, K, 1, K, N};
    for (int64_t i = 0; i < warmup; ++i) {
        cudaError_t e = v->fn(a, s, flags);
        if (e != cudaSuccess) return cuda_fail(e, "warmup launch");
    }
    cudaError_t e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) return cuda_fail(e, "warmup synchronize");
    cudaEvent_t ev0, ev1;
    if ((e = cudaEventCreate(&ev0)) != cudaSuccess) return cuda_fail(e, "event create");
    if ((e = cudaEventCreate(&ev1)) != cudaSuccess) {
        cudaEventDestroy(ev0);
        return cuda_fail(e, "event create");
    }
    rc = CL_OK;
    for (int64_t w = 0; w < n_windows && rc == CL_OK; ++w) {
        if ((e = cudaEventRecord(ev0, s)) != cudaSuccess) { rc = cuda_fail(e, "event record"); break; }
        for (int64_t i = 0; i < lpw; ++i) {
            e = v->fn(a, s, flags);
            if (e != cudaSuccess) { rc = cuda_fail(e, "timed launch"); break; }
        }
        if (rc != CL_OK) break;
        if ((e = cudaEventRecord(ev1, s)) != cudaSuccess) { rc = cuda_fail(e, "event record"); break; }
        if ((e = cudaEventSynchronize(ev1)) != cudaSuccess) { rc = cuda_fail(e, "event sync"); break; }
        float ms = 0.f;
        if ((e = cudaEventElapsedTime(&ms, ev0, ev1)) != cudaSuccess) { rc = cuda_fail(e, "elapsed"); break; }
        per_window_us[w] = (double)ms * 1e3 / (double)lpw;
    }
    cudaEventDestroy(ev0);
    cudaEventDestroy(ev1);
    return rc;
}

const clb::ShardedVariantDesc* find_sharded(const clb::ShardedVariantDesc* t, int n,
                                             const char* name) {
    if (name == nullptr) return nullptr;
    for (int i = 0; i < n; ++i)
        if (std::strcmp(t[i].name, name) == 0) return &t[i];
    return nullptr;
}

int run_sharded(const clb::ShardedVariantDesc* table, int n, const char* op, const char* variant,
                const void* W, const void* scale, const void* x, int64_t M, void* const* y_peers,
                void* const* flag_peers, int rank, int world, int64_t row0, int64_t N_shard,
                int64_t N_total, int64_t K, void* stream, uint32_t flags, bool is_int4) {
    const std::string o(op);
    const clb::ShardedVariantDesc* v = find_sharded(table, n, variant);
    if (!v) {
        std::string m = "unknown " + o + " sharded variant '" + (variant ? variant : "(null)") +
                        "'; available: ";
        for (int i = 0; i < n; ++i) m += std::string(table[i].name) + " ";
        return fail(CL_ERR_UNKNOWN_VARIANT, m);
    }
    int rc = check_args(op, W, scale, x, y_peers, N_shard, K, is_int4);
    if (rc != CL_OK) return rc;
    if (M < 1 || M > 16)
        return fail(CL_ERR_INVALID_ARGUMENT, o + "_sharded: M must be in [1, 16]");
    if (world < 1 || world > CL_MAX_PEERS)
        return fail(CL_ERR_INVALID_ARGUMENT, o + "_sharded: world must be in [1, 8]");
    if (rank < 0 || rank >= world)
        return fail(CL_ERR_INVALID_ARGUMENT, o + "_sharded: rank out of range");
    if (row0 < 0 || N_total <= 0 || row0 + N_shard > N_total)
        return fail(CL_ERR_INVALID_ARGUMENT, o + "_sharded: shard rows outside [0, N_total)");
    if (!is_int4 && (K % 64) != 0)
        return fail(CL_ERR_INVALID_ARGUMENT, o + "_sharded: K must be divisible by 64");
    if ((reinterpret_cast<uintptr_t>(W) | reinterpret_cast<uintptr_t>(x)) & 15u)
        return fail(CL_ERR_INVALID_ARGUMENT, o + "_sharded: W and x must be 16-byte aligned");
    if (!flag_peers) return fail(CL_ERR_INVALID_ARGUMENT, o + "_sharded: null flag pointers");
    clb::PeerArgs pa{};
    for (int p = 0; p < world; ++p) {
        if (!y_peers[p] || !y_peers[world + p] || !flag_peers[p])
            return fail(CL_ERR_INVALID_ARGUMENT, o + "_sharded: null peer pointer");
        pa.y[0][p] = y_peers[p];
        pa.y[1][p] = y_peers[world + p];
        pa.flag[p] = static_cast<unsigned*>(flag_peers[p]);
    }
    pa.row0 = row0;
    pa.rank = rank;
    pa.world = world;
    const clb::GemvArgs a{W, scale, x, nullptr, N_shard, K, M, K, N_total};
    cudaError_t e = v->fn(a, pa, static_cast<cudaStream_t>(stream), flags);
    if (e != cudaSuccess) {
        char ctx[160];
        std::snprintf(ctx, sizeof ctx, "sharded kernel launch (rank %d/%d, rows %lld+%lld of %lld, K %lld)",
                      rank, world, (long long)row0, (long long)N_shard, (long long)N_total,
                      (long long)K);
        return cuda_fail(e, ctx);
    }
    return CL_OK;
}

// ---- the fused single-GPU step without an allocated flag block ----
//
// Scratch of cl_int4gemv_fused_noalloc: one flag block (CL_PEER_FLAG_BYTES of
// arrival epochs, CTA ticket and step counter), the only memory besides its
// inputs and outputs that the fused kernel touches.  It is a file-scope
// device array, so it costs no allocation; every GPU that loads the library
// holds these 256 bytes until the process exits.  Host code must not hand
// `g_noalloc_flags` to a kernel: on the host the name stands for a host-side
// copy, so its device address is looked up once per device.
constexpr size_t kNoAllocScratchBytes = 256;
static_assert(kNoAllocScratchBytes >= CL_PEER_FLAG_BYTES, "room for one flag block");
static __device__ __align__(256) unsigned char g_noalloc_flags[kNoAllocScratchBytes];

constexpr int kNoAllocMaxDevices = 64;
std::mutex g_noalloc_mu;
struct NoAllocSlot {
    void* addr = nullptr;
    unsigned long long ctx_id = 0;  // context the address belongs to (0: unknown)
};
NoAllocSlot g_noalloc_slot[kNoAllocMaxDevices];

// Unique id of the calling thread's current CUDA context, 0 when the driver
// cannot tell.  The two driver functions are fetched through the runtime, so
// the library keeps no link-time dependency on the driver library.
unsigned long long current_context_id() {
    using GetCurrent = CUresult (*)(CUcontext*);
    using GetId = CUresult (*)(CUcontext, unsigned long long*);
    static GetCurrent get_current = nullptr;
    static GetId get_id = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            get_current = reinterpret_cast<GetCurrent>(p);
        p = nullptr;
        if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            get_id = reinterpret_cast<GetId>(p);
    });
    CUcontext ctx = nullptr;
    unsigned long long id = 0;
    if (!get_current || !get_id || get_current(&ctx) != CUDA_SUCCESS || ctx == nullptr ||
        get_id(ctx, &id) != CUDA_SUCCESS)
        return 0;
    return id;
}

// Device address of the flag block on the current device.  Set-up happens on
// the first call per device, with that device current, and again whenever
// the device's current context differs from the one the address was looked
// up in (after a cudaDeviceReset the runtime loads the library's module into
// a new context, at a new address); when the context id cannot be read the
// address is looked up on every call.
int noalloc_flag_block(void** out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_fail(e, "int4gemv_fused_noalloc: cudaGetDevice");
    if (dev < 0 || dev >= kNoAllocMaxDevices)
        return fail(CL_ERR_INVALID_ARGUMENT,
                    "int4gemv_fused_noalloc: device ordinal must be below 64");
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    NoAllocSlot& slot = g_noalloc_slot[dev];
    const unsigned long long ctx = slot.addr ? current_context_id() : 0;
    if (slot.addr == nullptr || ctx == 0 || ctx != slot.ctx_id) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_noalloc_flags);
        if (e != cudaSuccess)
            return cuda_fail(e, "int4gemv_fused_noalloc: cudaGetSymbolAddress(flag block)");
        slot.addr = p;
        slot.ctx_id = current_context_id();  // the lookup made the context current
    }
    *out = slot.addr;
    return CL_OK;
}

}  // namespace

extern "C" {

const char* cl_version(void) { return "cudalab-b200 0.1.0 (sm_100a)"; }

const char* cl_last_error(void) { return g_last_error.c_str(); }

int cl_device_status(int clear, int* status_out) {
    if (!status_out) return fail(CL_ERR_INVALID_ARGUMENT, "status_out is null");
    cudaError_t e = clb::read_device_status(clear, status_out);
    if (e != cudaSuccess) return cuda_fail(e, "read device status");
    return CL_OK;
}

int cl_set_wait_budget(int64_t cycles, int64_t* previous) {
    const long long prev = clb::set_wait_budget((long long)cycles);
    if (previous) *previous = (int64_t)prev;
    return CL_OK;
}

// ---- INT4 ----
int cl_int4gemv_ex(const char* variant, const uint8_t* W_packed, const void* scale, const void* x,
                   void* out, int64_t N, int64_t K, void* stream, uint32_t flags) {
    int n = 0;
    const clb::VariantDesc* t = clb::int4_variants(&n);
    return run(t, n, "int4gemv", variant, W_packed, scale, x, out, N, K, stream, flags, true);
}

int cl_int4gemv(const char* variant, const uint8_t* W_packed, const void* scale, const void* x,
                void* out, int64_t N, int64_t K, void* stream) {
    return cl_int4gemv_ex(variant, W_packed, scale, x, out, N, K, stream, 0u);
}

int cl_int4gemv_batched(const char* variant, const uint8_t* W_packed, const void* scale,
                        const void* X, void* Y, int64_t M, int64_t N, int64_t K, void* stream,
                        uint32_t flags) {
    int n = 0;
    const clb::VariantDesc* t = clb::int4_variants(&n);
    return run_batched(t, n, "int4gemv", variant, W_packed, scale, X, Y, M, N, K, stream, flags,
                       true);
}

int cl_int4gemv_native_timing(const char* variant, const uint8_t* W_packed, const void* scale,
                              const void* x, void* out, int64_t N, int64_t K, int64_t warmup,
                              int64_t n_windows, int64_t launches_per_window, void* stream,
                              uint32_t flags, double* per_window_us) {
    int n = 0;
    const clb::VariantDesc* t = clb::int4_variants(&n);
    return timing(t, n, "int4gemv", variant, W_packed, scale, x, out, N, K, warmup, n_windows,
                  launches_per_window, stream, flags, per_window_us, true);
}

int cl_int4gemv_list_variants(int which, char* buf, size_t buf_len, size_t* needed) {
    int n = 0;
    const clb::VariantDesc* t = clb::int4_variants(&n);
    return list_variants(t, n, which, buf, buf_len, needed);
}

// ---- RMSNorm and the fused RMSNorm -> INT4 GEMV ----
int cl_rmsnorm_f16(const void* X, const void* weight, float eps, void* Y, int64_t M, int64_t H,
                   void* stream, uint32_t flags) {
    if (M <= 0) return fail(CL_ERR_INVALID_ARGUMENT, "rmsnorm: M must be > 0");
    if (H <= 0) return fail(CL_ERR_INVALID_ARGUMENT, "rmsnorm: H must be > 0");
    if (H % 8 != 0) return fail(CL_ERR_INVALID_ARGUMENT, "rmsnorm: H must be a multiple of 8");
    if (H > 3 * ((int64_t)1 << 20))
        return fail(CL_ERR_INVALID_ARGUMENT, "rmsnorm: H exceeds 3 * 2^20 halves");
    if (M > INT32_MAX) return fail(CL_ERR_INVALID_ARGUMENT, "rmsnorm: M exceeds 2^31 - 1 rows");
    if (!(eps >= 0.f) || !std::isfinite(eps))
        return fail(CL_ERR_INVALID_ARGUMENT, "rmsnorm: eps must be finite and >= 0");
    if (!X || !weight || !Y) return fail(CL_ERR_INVALID_ARGUMENT, "rmsnorm: null device pointer");
    cudaError_t e = clb::launch_rmsnorm_f16(X, weight, eps, Y, M, H,
                                            static_cast<cudaStream_t>(stream), flags);
    if (e != cudaSuccess) return cuda_fail(e, "rmsnorm launch");
    return CL_OK;
}

int cl_int4gemv_rmsnorm(const char* variant, const uint8_t* W_packed, const void* scale,
                        const void* X, const void* norm_weight, float eps, void* Y, int64_t M,
                        int64_t N, int64_t K, void* stream, uint32_t flags) {
    int n = 0;
    const clb::VariantDesc* t = clb::int4_rmsnorm_variants(&n);
    const char* op = "int4gemv_rmsnorm";
    const clb::VariantDesc* v = find(t, n, variant);
    if (!v) return fail(CL_ERR_UNKNOWN_VARIANT, unknown_msg(op, t, n, variant));
    if (M <= 0) return fail(CL_ERR_INVALID_ARGUMENT, std::string(op) + ": M must be > 0");
    const int rc = check_args(op, W_packed, scale, X, Y, N, K, true);
    if (rc != CL_OK) return rc;
    if (!norm_weight) return fail(CL_ERR_INVALID_ARGUMENT, std::string(op) + ": null norm weight");
    if (!(eps >= 0.f) || !std::isfinite(eps))
        return fail(CL_ERR_INVALID_ARGUMENT, std::string(op) + ": eps must be finite and >= 0");
    constexpr int64_t kPass = 16;
    for (int64_t m0 = 0; m0 < M; m0 += kPass) {
        clb::GemvArgs a{W_packed, scale, static_cast<const uint16_t*>(X) + m0 * K,
                        static_cast<uint16_t*>(Y) + m0 * N, N, K,
                        std::min<int64_t>(kPass, M - m0), K, N};
        a.norm_w = norm_weight;
        a.norm_eps = eps;
        cudaError_t e = v->fn(a, static_cast<cudaStream_t>(stream), flags);
        if (e != cudaSuccess) return cuda_fail(e, "kernel launch");
    }
    return CL_OK;
}

// ---- INT8 ----
int cl_qgemv_ex(const char* variant, const int8_t* W_q, const float* scale, const void* x,
                void* out, int64_t N, int64_t K, void* stream, uint32_t flags) {
    int n = 0;
    const clb::VariantDesc* t = clb::int8_variants(&n);
    return run(t, n, "qgemv", variant, W_q, scale, x, out, N, K, stream, flags, false);
}

int cl_qgemv(const char* variant, const int8_t* W_q, const float* scale, const void* x, void* out,
             int64_t N, int64_t K, void* stream) {
    return cl_qgemv_ex(variant, W_q, scale, x, out, N, K, stream, 0u);
}

int cl_qgemv_batched(const char* variant, const int8_t* W_q, const float* scale, const void* X,
                     void* Y, int64_t M, int64_t N, int64_t K, void* stream, uint32_t flags) {
    int n = 0;
    const clb::VariantDesc* t = clb::int8_variants(&n);
    return run_batched(t, n, "qgemv", variant, W_q, scale, X, Y, M, N, K, stream, flags, false);
}

int cl_qgemv_native_timing(const char* variant, const int8_t* W_q, const float* scale,
                           const void* x, void* out, int64_t N, int64_t K, int64_t warmup,
                           int64_t n_windows, int64_t launches_per_window, void* stream,
                           uint32_t flags, double* per_window_us) {
    int n = 0;
    const clb::VariantDesc* t = clb::int8_variants(&n);
    return timing(t, n, "qgemv", variant, W_q, scale, x, out, N, K, warmup, n_windows,
                  launches_per_window, stream, flags, per_window_us, false);
}

int cl_qgemv_list_variants(int which, char* buf, size_t buf_len, size_t* needed) {
    int n = 0;
    const clb::VariantDesc* t = clb::int8_variants(&n);
    return list_variants(t, n, which, buf, buf_len, needed);
}

// ---- quantisation ----
static const clb::VariantDesc* gemv_table(int dtype, int* n) {
    if (dtype != CL_DTYPE_F16 && dtype != CL_DTYPE_F32) return nullptr;
    return clb::gemv_variants(dtype, n);
}

int cl_gemv_ex(const char* variant, const void* W, const void* x, void* out, int64_t N, int64_t K,
               int dtype, void* stream, uint32_t flags) {
    int n = 0;
    const clb::VariantDesc* t = gemv_table(dtype, &n);
    if (!t) return fail(CL_ERR_INVALID_ARGUMENT, "gemv: dtype must be CL_DTYPE_F16 or CL_DTYPE_F32");
    return run(t, n, "gemv", variant, W, W, x, out, N, K, stream, flags, false);
}

int cl_gemv(const char* variant, const void* W, const void* x, void* out, int64_t N, int64_t K,
            int dtype, void* stream) {
    return cl_gemv_ex(variant, W, x, out, N, K, dtype, stream, 0u);
}

int cl_gemv_native_timing(const char* variant, const void* W, const void* x, void* out, int64_t N,
                          int64_t K, int dtype, int64_t warmup, int64_t n_windows,
                          int64_t launches_per_window, void* stream, uint32_t flags,
                          double* per_window_us) {
    int n = 0;
    const clb::VariantDesc* t = gemv_table(dtype, &n);
    if (!t) return fail(CL_ERR_INVALID_ARGUMENT, "gemv: dtype must be CL_DTYPE_F16 or CL_DTYPE_F32");
    return timing(t, n, "gemv", variant, W, W, x, out, N, K, warmup, n_windows,
                  launches_per_window, stream, flags, per_window_us, false);
}

int cl_gemv_list_variants(int which, char* buf, size_t buf_len, size_t* needed) {
    int n = 0;
    const clb::VariantDesc* t = clb::gemv_variants(CL_DTYPE_F16, &n);  // same names for fp32
    return list_variants(t, n, which, buf, buf_len, needed);
}

int cl_int4gemv_quantize(const void* W, int64_t N, int64_t K, uint8_t* W_packed, void* scale,
                         void* stream) {
    if (N <= 0 || K <= 0) return fail(CL_ERR_INVALID_ARGUMENT, "int4gemv_quantize: N, K must be > 0");
    if (K % 128 != 0)
        return fail(CL_ERR_INVALID_ARGUMENT,
                    "int4gemv_quantize: K must be divisible by 128 (group_size=128)");
    if (!W || !W_packed || !scale)
        return fail(CL_ERR_INVALID_ARGUMENT, "int4gemv_quantize: null device pointer");
    if (reinterpret_cast<uintptr_t>(W) & 7u)
        return fail(CL_ERR_INVALID_ARGUMENT, "int4gemv_quantize: W must be 8-byte aligned");
    cudaError_t e = clb::launch_int4_quantize(W, N, K, W_packed, scale,
                                              static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "int4gemv_quantize launch");
    return CL_OK;
}

int cl_qgemv_quantize(const void* W, int64_t N, int64_t K, int8_t* W_q, float* scale,
                      void* stream) {
    if (N <= 0 || K <= 0) return fail(CL_ERR_INVALID_ARGUMENT, "qgemv_quantize: N, K must be > 0");
    if (N > ((int64_t)1 << 31) - 1)
        return fail(CL_ERR_INVALID_ARGUMENT, "qgemv_quantize: N exceeds 2^31 - 1 rows");
    if (!W || !W_q || !scale)
        return fail(CL_ERR_INVALID_ARGUMENT, "qgemv_quantize: null device pointer");
    cudaError_t e = clb::launch_int8_quantize(W, N, K, W_q, scale,
                                              static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "qgemv_quantize launch");
    return CL_OK;
}

// ---- peer buffers and the row-sharded GEMV ----
int cl_peer_alloc(size_t bytes, void** ptr, void* ipc_handle) {
    if (!ptr || !ipc_handle || bytes == 0)
        return fail(CL_ERR_INVALID_ARGUMENT, "peer_alloc: null output or zero size");
    static_assert(sizeof(cudaIpcMemHandle_t) == CL_IPC_HANDLE_BYTES, "IPC handle size");
    void* p = nullptr;
    cudaError_t e = cudaMalloc(&p, bytes);
    if (e != cudaSuccess) return cuda_fail(e, "peer_alloc: cudaMalloc");
    if ((e = cudaMemset(p, 0, bytes)) != cudaSuccess) {
        cudaFree(p);
        return cuda_fail(e, "peer_alloc: cudaMemset");
    }
    cudaIpcMemHandle_t h;
    if ((e = cudaIpcGetMemHandle(&h, p)) != cudaSuccess) {
        cudaFree(p);
        return cuda_fail(e, "peer_alloc: cudaIpcGetMemHandle");
    }
    std::memcpy(ipc_handle, &h, sizeof(h));
    *ptr = p;
    return CL_OK;
}

int cl_peer_open(const void* ipc_handle, void** peer_ptr) {
    if (!ipc_handle || !peer_ptr) return fail(CL_ERR_INVALID_ARGUMENT, "peer_open: null pointer");
    cudaIpcMemHandle_t h;
    std::memcpy(&h, ipc_handle, sizeof(h));
    cudaError_t e = cudaIpcOpenMemHandle(peer_ptr, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) return cuda_fail(e, "peer_open: cudaIpcOpenMemHandle");
    return CL_OK;
}

int cl_peer_close(void* peer_ptr) {
    if (!peer_ptr) return fail(CL_ERR_INVALID_ARGUMENT, "peer_close: null pointer");
    cudaError_t e = cudaIpcCloseMemHandle(peer_ptr);
    if (e != cudaSuccess) return cuda_fail(e, "peer_close: cudaIpcCloseMemHandle");
    return CL_OK;
}

int cl_peer_free(void* ptr) {
    if (!ptr) return fail(CL_ERR_INVALID_ARGUMENT, "peer_free: null pointer");
    cudaError_t e = cudaFree(ptr);
    if (e != cudaSuccess) return cuda_fail(e, "peer_free: cudaFree");
    return CL_OK;
}

int cl_int4gemv_sharded(const char* variant, const uint8_t* W_shard, const void* scale_shard,
                        const void* x, int64_t M, void* const* y_peers, void* const* flag_peers,
                        int rank,
                        int world, int64_t row0, int64_t N_shard, int64_t N_total, int64_t K,
                        void* stream, uint32_t flags) {
    int n = 0;
    const clb::ShardedVariantDesc* t = clb::int4_sharded_variants(&n);
    return run_sharded(t, n, "int4gemv", variant, W_shard, scale_shard, x, M, y_peers, flag_peers,
                       rank, world, row0, N_shard, N_total, K, stream, flags, true);
}

int cl_int4gemv_fused_noalloc(const char* variant, const uint8_t* W_packed, const void* scale,
                              const void* x, int64_t M, void* y, int64_t N, int64_t K,
                              void* stream, uint32_t flags) {
    int n = 0;
    const clb::ShardedVariantDesc* t = clb::int4_sharded_variants(&n);
    // Every check of the launch first, so that a rejected call leaves the
    // stream untouched.
    if (!find_sharded(t, n, variant))
        return fail(CL_ERR_UNKNOWN_VARIANT, std::string("int4gemv_fused_noalloc: unknown variant '") +
                                                (variant ? variant : "(null)") + "'");
    int rc = check_args("int4gemv_fused_noalloc", W_packed, scale, x, y, N, K, true);
    if (rc != CL_OK) return rc;
    if (M < 1 || M > 16)
        return fail(CL_ERR_INVALID_ARGUMENT,
                    "int4gemv_fused_noalloc: M must be in [1, 16] (larger batches: call again "
                    "per 16 rows)");
    if ((reinterpret_cast<uintptr_t>(W_packed) | reinterpret_cast<uintptr_t>(x)) & 15u)
        return fail(CL_ERR_INVALID_ARGUMENT,
                    "int4gemv_fused_noalloc: W_packed and x must be 16-byte aligned");
    void* flag = nullptr;
    rc = noalloc_flag_block(&flag);
    if (rc != CL_OK) return rc;
    // The block keeps the previous call's contents: start every call from zero.
    cudaError_t e = cudaMemsetAsync(flag, 0, CL_PEER_FLAG_BYTES, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "int4gemv_fused_noalloc: clearing the flag block");
    void* ys[2] = {y, y};  // one rank: both step parities write the caller's y
    void* fs[1] = {flag};
    return run_sharded(t, n, "int4gemv", variant, W_packed, scale, x, M, ys, fs, 0, 1, 0, N, N, K,
                       stream, flags, true);
}

int cl_qgemv_sharded(const char* variant, const int8_t* W_shard, const float* scale_shard,
                     const void* x, int64_t M, void* const* y_peers, void* const* flag_peers,
                     int rank,
                     int world, int64_t row0, int64_t N_shard, int64_t N_total, int64_t K,
                     void* stream, uint32_t flags) {
    int n = 0;
    const clb::ShardedVariantDesc* t = clb::int8_sharded_variants(&n);
    return run_sharded(t, n, "qgemv", variant, W_shard, scale_shard, x, M, y_peers, flag_peers,
                       rank, world, row0, N_shard, N_total, K, stream, flags, false);
}

}  // extern "C"
