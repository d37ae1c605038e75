// Dense GEMV, y[n] = sum_k W[n, k] * x[k] with fp16 or fp32 weights and
// activations, fp32 accumulation and one final rounding to the element type:
// the reference's third operator (contract: kernels/gemv/gemv_common.h:1-40 of
// the reference; variants kernels/gemv/gemv_baseline.cu, gemv_vec4_row.cu,
// gemv_warp_vec4.cu, gemv_splitk4.cu).
//
// Variants (same names as the reference's registry):
//   gemv_baseline   one 256-thread CTA per row, element loads strided over the
//                   CTA, fp32 FMA, fixed reduction tree.  No alignment
//                   contract.  It is also the fallback of every vectorised
//                   variant, so a fallback reproduces it bit for bit.
//   gemv_vec4_row   one CTA per row, 16-byte loads (8 halves / 4 floats).
//   gemv_warp_vec4  one warp per row (8 rows per CTA), 16-byte loads.
//   gemv_splitk4    one CTA per row, K cut into four contiguous quarters
//                   summed by 64 threads each, quarters added in order.  Kept
//                   out of the normal list as in the reference (its kernel
//                   there used a process-wide workspace; this one needs none).
//   gemv_mma        fp16: the tensor-core kernel of gemv_mma.cuh with dense
//                   weights (exact fp16 products, fp32 accumulation);
//                   fp32: one warp per row with eight 16-byte loads in flight
//                   per lane, or one CTA per row for a few long rows (tensor
//                   cores would round fp32 operands to tf32).
// Vectorised contract: W and x 16-byte aligned and K a multiple of the
// elements per 16 bytes (gemv_mma fp16: K a multiple of 32); otherwise the
// baseline kernel runs.  Every kernel waits for the preceding grid before it
// touches memory, so programmatic dependent launch is safe with any of them.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "gemv_common.cuh"
#include "gemv_launch.h"

namespace clb {
namespace {

constexpr int kRowThreads = 256;

__device__ __forceinline__ float to_f(__half v) { return __half2float(v); }
__device__ __forceinline__ float to_f(float v) { return v; }
__device__ __forceinline__ void from_f(float v, __half* out) { *out = __float2half_rn(v); }
__device__ __forceinline__ void from_f(float v, float* out) { *out = v; }

// Elements of one 16-byte vector, multiplied into acc in index order.
__device__ __forceinline__ float dot16(uint4 w, uint4 x, float acc, __half) {
    const __half2* wh = reinterpret_cast<const __half2*>(&w);
    const __half2* xh = reinterpret_cast<const __half2*>(&x);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float2 a = __half22float2(wh[i]);
        const float2 b = __half22float2(xh[i]);
        acc = __fmaf_rn(a.x, b.x, acc);
        acc = __fmaf_rn(a.y, b.y, acc);
    }
    return acc;
}
__device__ __forceinline__ float dot16(uint4 w, uint4 x, float acc, float) {
    acc = __fmaf_rn(__uint_as_float(w.x), __uint_as_float(x.x), acc);
    acc = __fmaf_rn(__uint_as_float(w.y), __uint_as_float(x.y), acc);
    acc = __fmaf_rn(__uint_as_float(w.z), __uint_as_float(x.z), acc);
    acc = __fmaf_rn(__uint_as_float(w.w), __uint_as_float(x.w), acc);
    return acc;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Sum over a 256-thread CTA: each warp's xor tree, then the eight warp sums
// in warp order by thread 0.
__device__ __forceinline__ float cta_sum(float v, float* red) {
    v = warp_sum(v);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    float s = 0.f;
    if (threadIdx.x == 0) {
#pragma unroll
        for (int w = 0; w < kRowThreads / 32; ++w) s += red[w];
    }
    return s;
}

template <class T>
__global__ void __launch_bounds__(kRowThreads)
    dense_scalar_kernel(const T* __restrict__ W, const T* __restrict__ x, T* __restrict__ y,
                        int64_t K) {
    pdl_wait_prior_grids();
    __shared__ float red[kRowThreads / 32];
    const T* w = W + (int64_t)blockIdx.x * K;
    float acc = 0.f;
    for (int64_t k = threadIdx.x; k < K; k += kRowThreads) acc = __fmaf_rn(to_f(w[k]), to_f(x[k]), acc);
    const float s = cta_sum(acc, red);
    if (threadIdx.x == 0) from_f(s, y + blockIdx.x);
}

template <class T>
__global__ void __launch_bounds__(kRowThreads)
    dense_vec_row_kernel(const T* __restrict__ W, const T* __restrict__ x, T* __restrict__ y,
                         int64_t K) {
    pdl_wait_prior_grids();
    __shared__ float red[kRowThreads / 32];
    constexpr int kPer = 16 / sizeof(T);
    const int64_t nv = K / kPer;
    const uint4* w = reinterpret_cast<const uint4*>(W + (int64_t)blockIdx.x * K);
    const uint4* xv = reinterpret_cast<const uint4*>(x);
    float acc = 0.f;
#pragma unroll 4
    for (int64_t i = threadIdx.x; i < nv; i += kRowThreads)
        acc = dot16(ldg_stream16(w + i, policy_evict_first()), __ldg(xv + i), acc, T{});
    const float s = cta_sum(acc, red);
    if (threadIdx.x == 0) from_f(s, y + blockIdx.x);
}

// One warp per row; kDepth independent 16-byte loads per lane in flight.
template <class T, int kDepth>
__global__ void __launch_bounds__(kRowThreads)
    dense_warp_kernel(const T* __restrict__ W, const T* __restrict__ x, T* __restrict__ y,
                      int64_t N, int64_t K) {
    pdl_wait_prior_grids();
    constexpr int kPer = 16 / sizeof(T);
    const int lane = threadIdx.x & 31;
    const int64_t row = (int64_t)blockIdx.x * (kRowThreads / 32) + (threadIdx.x >> 5);
    if (row >= N) return;
    const int64_t nv = K / kPer;
    const uint4* w = reinterpret_cast<const uint4*>(W + row * K);
    const uint4* xv = reinterpret_cast<const uint4*>(x);
    const uint64_t pol = policy_evict_first();
    float acc = 0.f;
    int64_t i = lane;
    for (; i + 32 * (kDepth - 1) < nv; i += 32 * kDepth) {
        uint4 wv[kDepth];
#pragma unroll
        for (int d = 0; d < kDepth; ++d) wv[d] = ldg_stream16(w + i + 32 * d, pol);
#pragma unroll
        for (int d = 0; d < kDepth; ++d) acc = dot16(wv[d], __ldg(xv + i + 32 * d), acc, T{});
    }
    for (; i < nv; i += 32) acc = dot16(ldg_stream16(w + i, pol), __ldg(xv + i), acc, T{});
    acc = warp_sum(acc);
    if (lane == 0) from_f(acc, y + row);
}

// K in four contiguous quarters (K % 4 == 0), 64 threads each.
template <class T>
__global__ void __launch_bounds__(kRowThreads)
    dense_splitk4_kernel(const T* __restrict__ W, const T* __restrict__ x, T* __restrict__ y,
                         int64_t K) {
    pdl_wait_prior_grids();
    __shared__ float red[kRowThreads / 32];
    const int64_t q = K / 4;
    const int part = threadIdx.x >> 6, j = threadIdx.x & 63;
    const T* w = W + (int64_t)blockIdx.x * K + part * q;
    const T* xs = x + part * q;
    float acc = 0.f;
    for (int64_t k = j; k < q; k += 64) acc = __fmaf_rn(to_f(w[k]), to_f(xs[k]), acc);
    acc = warp_sum(acc);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
    __syncthreads();
    if (threadIdx.x == 0) {
        const float s0 = red[0] + red[1], s1 = red[2] + red[3];
        const float s2 = red[4] + red[5], s3 = red[6] + red[7];
        from_f(((s0 + s1) + s2) + s3, y + blockIdx.x);
    }
}

template <class Kern, class... Args>
cudaError_t launch_pdl(Kern kernel, dim3 grid, cudaStream_t s, unsigned flags, Args... args) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(kRowThreads);
    cfg.stream = s;
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr.val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = (flags & 1u) ? &attr : nullptr;
    cfg.numAttrs = (flags & 1u) ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kernel, args...);
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

template <class T>
bool vec_ok(const GemvArgs& a) {
    return aligned16(a.W) && aligned16(a.x) && a.K % (16 / (int64_t)sizeof(T)) == 0;
}

template <class T>
cudaError_t run_scalar(const GemvArgs& a, cudaStream_t s, unsigned flags) {
    return launch_pdl(dense_scalar_kernel<T>, dim3((unsigned)a.N), s, flags,
                      static_cast<const T*>(a.W), static_cast<const T*>(a.x),
                      static_cast<T*>(a.y), a.K);
}

template <class T>
cudaError_t run_vec_row(const GemvArgs& a, cudaStream_t s, unsigned flags) {
    if (!vec_ok<T>(a)) return run_scalar<T>(a, s, flags);
    return launch_pdl(dense_vec_row_kernel<T>, dim3((unsigned)a.N), s, flags,
                      static_cast<const T*>(a.W), static_cast<const T*>(a.x),
                      static_cast<T*>(a.y), a.K);
}

template <class T, int kDepth>
cudaError_t run_warp(const GemvArgs& a, cudaStream_t s, unsigned flags) {
    if (!vec_ok<T>(a)) return run_scalar<T>(a, s, flags);
    const dim3 grid((unsigned)((a.N + kRowThreads / 32 - 1) / (kRowThreads / 32)));
    return launch_pdl(dense_warp_kernel<T, kDepth>, grid, s, flags, static_cast<const T*>(a.W),
                      static_cast<const T*>(a.x), static_cast<T*>(a.y), a.N, a.K);
}

template <class T>
cudaError_t run_splitk4(const GemvArgs& a, cudaStream_t s, unsigned flags) {
    if (a.K % 4 != 0) return run_scalar<T>(a, s, flags);
    return launch_pdl(dense_splitk4_kernel<T>, dim3((unsigned)a.N), s, flags,
                      static_cast<const T*>(a.W), static_cast<const T*>(a.x),
                      static_cast<T*>(a.y), a.K);
}

// fp32 production path: one warp per row with eight loads in flight, except
// for few long rows (N <= 2048, K >= 2048), where a warp per row leaves most
// of the GPU idle and a whole CTA per row streams them (measured on B200:
// 1024 x 4096 in 4.75 instead of 9.17 us).
cudaError_t run_f32_auto(const GemvArgs& a, cudaStream_t s, unsigned flags) {
    if (a.N <= 2048 && a.K >= 2048) return run_vec_row<float>(a, s, flags);
    return run_warp<float, 8>(a, s, flags);
}

const VariantDesc kF16Variants[] = {
    {"gemv_baseline", run_scalar<__half>, false},
    {"gemv_mma", launch_gemv_f16_mma, false},
    {"gemv_splitk4", run_splitk4<__half>, true},
    {"gemv_vec4_row", run_vec_row<__half>, false},
    {"gemv_warp_vec4", run_warp<__half, 1>, false},
};

const VariantDesc kF32Variants[] = {
    {"gemv_baseline", run_scalar<float>, false},
    {"gemv_mma", run_f32_auto, false},
    {"gemv_splitk4", run_splitk4<float>, true},
    {"gemv_vec4_row", run_vec_row<float>, false},
    {"gemv_warp_vec4", run_warp<float, 1>, false},
};

}  // namespace

cudaError_t launch_f16_scalar(const void* W, const void*, const void* x, void* y, int64_t N,
                              int64_t K, cudaStream_t s, unsigned flags) {
    const GemvArgs a{W, nullptr, x, y, N, K, 1, K, N};
    return run_scalar<__half>(a, s, flags);
}

const VariantDesc* gemv_variants(int dtype, int* count) {
    if (dtype == 0) {
        *count = (int)(sizeof(kF16Variants) / sizeof(kF16Variants[0]));
        return kF16Variants;
    }
    *count = (int)(sizeof(kF32Variants) / sizeof(kF32Variants[0]));
    return kF32Variants;
}

}  // namespace clb
