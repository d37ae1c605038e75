// Kernels and launchers of the weight-only quantized GEMV library (sm_100a).
//
// Variants (names are the dispatch keys of the C ABI):
//   int4gemv_baseline      scalar reference-role kernel, one warp per row, byte
//                          loads; also the fallback of every vectorised INT4
//                          variant whose alignment contract is not met, so a
//                          fallback result is bit-identical to this variant.
//   int4gemv_ldg           register-direct 16-byte streaming loads (L1
//                          no-allocate, L2 evict-first), one-tile prefetch,
//                          fp16 exact dequant + mixed fma.rn.f32.f16.
//   int4gemv_bulk          persistent one-CTA-per-SM kernel; a producer warp
//                          streams 16 KiB weight tiles through a shared-memory
//                          ring with cp.async.bulk + mbarriers; same math.
//   int4gemv_*_f32x2       the same two pipelines with exact fp32 dequant and
//                          packed fma.rn.f32x2 math.
//   qgemv_*                the INT8 row-scaled counterparts.
#include <cuda_runtime.h>

#include <algorithm>
#include <map>
#include <mutex>
#include <utility>

#include "gemv_launch.h"
#include "gemv_vector.cuh"
#include "gemv_mma.cuh"

namespace clb {

// ---------------------------------------------------------------------------
// Scalar kernels (baseline + fallback).  One warp per output row, 8 rows per
// 256-thread block; each lane walks the row with a 32-byte stride.  Per term:
// dequantised weight (q * s) rounded to fp32, then one fma with x.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) int4gemv_scalar_kernel(const uint8_t* __restrict__ Wp,
                                                              const __half* __restrict__ scale,
                                                              const __half* __restrict__ x,
                                                              __half* __restrict__ y, int64_t N,
                                                              int64_t K) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t row = (int64_t)blockIdx.x * 8 + warp;
    if (row >= N) return;
    const int64_t rb = K >> 1;
    const uint8_t* wr = Wp + row * rb;
    const __half* sr = scale + row * (K >> 7);
    float acc = 0.f;
    for (int64_t b = lane; b < rb; b += 32) {
        const uint32_t byte = wr[b];
        const float s = __half2float(sr[b >> 6]);  // both nibbles of a byte share a group
        const int lo = (int)(byte << 28) >> 28;    // sign-extended element 2b
        const int hi = (int)(byte << 24) >> 28;    // sign-extended element 2b+1
        const float w0 = __fmul_rn((float)lo, s);
        const float w1 = __fmul_rn((float)hi, s);
        acc = __fmaf_rn(w0, __half2float(x[2 * b]), acc);
        acc = __fmaf_rn(w1, __half2float(x[2 * b + 1]), acc);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0) y[row] = __float2half_rn(acc);
}

__global__ void __launch_bounds__(256) qgemv_scalar_kernel(const int8_t* __restrict__ Wq,
                                                           const float* __restrict__ scale,
                                                           const __half* __restrict__ x,
                                                           __half* __restrict__ y, int64_t N,
                                                           int64_t K) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t row = (int64_t)blockIdx.x * 8 + warp;
    if (row >= N) return;
    const int8_t* wr = Wq + row * K;
    const float s = scale[row];
    float acc = 0.f;
    for (int64_t k = lane; k < K; k += 32) {
        const float w = __fmul_rn((float)wr[k], s);
        acc = __fmaf_rn(w, __half2float(x[k]), acc);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0) y[row] = __float2half_rn(acc);
}

// ---------------------------------------------------------------------------
// Host side: device properties, geometry, launch helpers.
// ---------------------------------------------------------------------------
namespace {

constexpr int kMaxDevices = 64;

int sm_count(int dev) {
    static int cache[kMaxDevices] = {0};
    if (dev < 0 || dev >= kMaxDevices) return 148;
    if (cache[dev] == 0) {
        int v = 0;
        if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v <= 0)
            v = 148;
        cache[dev] = v;
    }
    return cache[dev];
}

// Opt a kernel into more than 48 KiB of dynamic shared memory, once per
// device and kernel.
template <class K>
cudaError_t ensure_smem_attr(K kernel, int dev, int bytes) {
    static std::mutex mu;
    static std::map<std::pair<const void*, int>, int> done;
    if (bytes <= 48 * 1024) return cudaSuccess;
    std::lock_guard<std::mutex> lock(mu);
    const auto key = std::make_pair(reinterpret_cast<const void*>(kernel), dev);
    auto it = done.find(key);
    if (it != done.end() && it->second >= bytes) return cudaSuccess;
    // request the largest dynamic size this kernel can ever use: the opt-in
    // limit of the device minus the kernel's static shared memory
    int optin = 0;
    cudaError_t e = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    if (e != cudaSuccess) return e;
    cudaFuncAttributes fa{};
    if ((e = cudaFuncGetAttributes(&fa, kernel)) != cudaSuccess) return e;
    const int want = optin - (int)fa.sharedSizeBytes;
    if (want < bytes) return cudaErrorInvalidValue;
    e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, want);
    if (e == cudaSuccess) done[key] = want;
    return e;
}

// Slice / tile geometry of the vectorised kernels (see gemv_vector.cuh).
GemvGeom make_geom(int64_t N, int64_t K, bool int4, bool bulk, int num_sms) {
    GemvGeom g{};
    g.N = N;
    g.K = K;
    g.row_bytes = int4 ? K / 2 : K;
    int64_t sb = kMaxSliceBytes;
    while (sb > kChunkBytes && (g.row_bytes % sb) != 0) sb >>= 1;
    g.slice_bytes = (int32_t)sb;
    g.n_slices = (int32_t)(g.row_bytes / sb);
    g.chunks = (int32_t)(sb / kChunkBytes);
    g.thread_rows = kConsumerThreads / g.chunks;
    g.tile_rows = kRowsPerThread * g.thread_rows;
    g.groups = int4 ? (int32_t)(K / 128) : 1;
    const int64_t scale_row_bytes = int4 ? (int64_t)g.groups * 2 : 4;
    int64_t ctas = std::min<int64_t>(N, (int64_t)num_sms * (bulk ? 1 : 2));
    const int64_t max_rows_by_scale = std::max<int64_t>(1, kScaleSmemBytes / scale_row_bytes);
    ctas = std::max<int64_t>(ctas, (N + max_rows_by_scale - 1) / max_rows_by_scale);
    g.ctas = (int32_t)ctas;
    g.rows_base = (int32_t)(N / ctas);
    g.rows_rem = (int32_t)(N % ctas);
    const int64_t max_rows = g.rows_base + (g.rows_rem > 0 ? 1 : 0);
    g.scale_smem = (int32_t)(max_rows * scale_row_bytes);
    if (bulk) {
        const int64_t stage_rows = std::min<int64_t>(g.tile_rows, max_rows);
        int64_t stage = stage_rows * sb;
        stage = (stage + 127) & ~int64_t(127);
        g.stage_bytes = (int32_t)stage;
        g.stages = (int32_t)std::min<int64_t>(kMaxStages, kRingBytes / stage);
        g.ring_bytes = kRingBytes;
    } else {
        g.stage_bytes = 0;
        g.stages = 1;
        g.ring_bytes = 0;
    }
    return g;
}

template <class Kern, class... Args>
cudaError_t launch(Kern kernel, dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                   unsigned flags, Args... args) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    cfg.numAttrs = 0;
    if (flags & 1u) {
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
    }
    return cudaLaunchKernelEx(&cfg, kernel, args...);
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

cudaError_t launch_int4_scalar(const void* W, const void* scale, const void* x, void* y, int64_t N,
                               int64_t K, cudaStream_t s, unsigned flags) {
    const dim3 grid((unsigned)((N + 7) / 8));
    return launch(int4gemv_scalar_kernel, grid, dim3(256), 0, s, flags,
                  static_cast<const uint8_t*>(W), static_cast<const __half*>(scale),
                  static_cast<const __half*>(x), static_cast<__half*>(y), N, K);
}

cudaError_t launch_int8_scalar(const void* W, const void* scale, const void* x, void* y, int64_t N,
                               int64_t K, cudaStream_t s, unsigned flags) {
    const dim3 grid((unsigned)((N + 7) / 8));
    return launch(qgemv_scalar_kernel, grid, dim3(256), 0, s, flags,
                  static_cast<const int8_t*>(W), static_cast<const float*>(scale),
                  static_cast<const __half*>(x), static_cast<__half*>(y), N, K);
}

template <class Fmt, class Math, bool kBulk>
cudaError_t launch_vec(const void* W, const void* scale, const void* x, void* y, int64_t N,
                       int64_t K, cudaStream_t s, unsigned flags) {
    constexpr bool kInt4 = Fmt::kGroupScale;
    // Alignment contract of the 16-byte paths; otherwise run the scalar
    // kernel, whose output the baseline variant reproduces bit for bit.
    const bool ok = aligned16(W) && aligned16(x) && (kInt4 ? (K % 32 == 0) : (K % 16 == 0));
    if (!ok) {
        return kInt4 ? launch_int4_scalar(W, scale, x, y, N, K, s, flags)
                     : launch_int8_scalar(W, scale, x, y, N, K, s, flags);
    }
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    const GemvGeom g = make_geom(N, K, kInt4, kBulk, sm_count(dev));
    const int smem = smem_total(g);
    auto kernel = gemv_vec_kernel<Fmt, Math, kBulk>;
    e = ensure_smem_attr(kernel, dev, smem);
    if (e != cudaSuccess) return e;
    const dim3 grid((unsigned)g.ctas);
    const dim3 block(kBulk ? kConsumerThreads + 32 : kConsumerThreads);
    using S = typename Fmt::Scale;
    return launch(kernel, grid, block, (size_t)smem, s, flags, static_cast<const uint8_t*>(W),
                  static_cast<const S*>(scale), static_cast<const __half*>(x),
                  static_cast<__half*>(y), g);
}

// Geometry of the tensor-core kernels (see gemv_mma.cuh).  Returns false when
// the staged activations do not fit in shared memory (K beyond ~100k).
// ctas_per_sm: CTAs of one GEMV per SM before tiles are shared (1 for 8-warp
// CTAs; 2 for 4-warp CTAs keeps the warps of one GEMV per SM unchanged).
bool make_mma_geom(int64_t N, int64_t K, bool int4, int num_sms, int ctas_per_sm, MmaGeom& g) {
    g = MmaGeom{};
    g.N = N;
    g.K = K;
    g.row_bytes = int4 ? K / 2 : K;
    g.blocks = (int32_t)(g.row_bytes / 64);
    g.n_kc = (g.blocks + kMmaChunkBlocks - 1) / kMmaChunkBlocks;
    const int64_t tiles = (N + 15) / 16;
    int64_t ctas = std::min<int64_t>(tiles, (int64_t)num_sms * ctas_per_sm);
    for (;;) {
        const int64_t per = (tiles + ctas - 1) / ctas;
        if (per * g.n_kc <= kMmaPartialMax || ctas >= tiles) break;
        ctas = std::min<int64_t>(tiles, ctas + std::max<int64_t>(1, ctas / 8));
    }
    g.ctas = (int32_t)ctas;
    g.tiles_base = (int32_t)(tiles / ctas);
    g.tiles_rem = (int32_t)(tiles % ctas);
    const int64_t max_tiles = g.tiles_base + (g.tiles_rem > 0 ? 1 : 0);
    g.max_rows = (int32_t)std::min<int64_t>(16 * max_tiles, N);
    g.max_items = (int32_t)(max_tiles * g.n_kc);
    if (g.max_items > kMmaPartialMax) return false;
    g.xs_bytes = (int32_t)(K * 2);
    return mma_smem_total(g) <= 226 * 1024;  // 1 KiB left for static shared memory
}

template <class Fmt, int kWarps, int kCtasPerSm, bool kPeer>
cudaError_t launch_mma_impl(const void* W, const void* scale, const void* x, void* y, int64_t N,
                            int64_t K, cudaStream_t s, unsigned flags, const PeerOut& po) {
    constexpr bool kInt4 = Fmt::kGroupScale;
    const bool ok = aligned16(W) && aligned16(x) && (kInt4 ? (K % 128 == 0) : (K % 64 == 0));
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    MmaGeom g;
    if constexpr (kPeer) {
        // the sharded entry points check this contract before launching
        if (!ok) return cudaErrorMisalignedAddress;
        if (!make_mma_geom(N, K, kInt4, sm_count(dev), kCtasPerSm, g))
            return cudaErrorInvalidConfiguration;
    } else if (!ok || !make_mma_geom(N, K, kInt4, sm_count(dev), kCtasPerSm, g)) {
        return kInt4 ? launch_int4_scalar(W, scale, x, y, N, K, s, flags)
                     : launch_int8_scalar(W, scale, x, y, N, K, s, flags);
    }
    g.early_x = (flags & 3u) == 3u ? 1 : 0;
    const int smem = mma_smem_total(g);
    const bool all_full = (g.blocks % kMmaChunkBlocks) == 0;
    auto kernel = all_full ? gemv_mma_kernel<Fmt, kWarps, true, kPeer>
                           : gemv_mma_kernel<Fmt, kWarps, false, kPeer>;
    if (smem > 48 * 1024) {
        e = ensure_smem_attr(kernel, dev, smem);
        if (e != cudaSuccess) return e;
    }
    using S = typename Fmt::Scale;
    return launch(kernel, dim3((unsigned)g.ctas), dim3(32 * kWarps), (size_t)smem, s, flags,
                  static_cast<const uint8_t*>(W), static_cast<const S*>(scale),
                  static_cast<const __half*>(x), static_cast<__half*>(y), g, po);
}

template <class Fmt, int kWarps, int kCtasPerSm>
cudaError_t launch_mma(const void* W, const void* scale, const void* x, void* y, int64_t N,
                       int64_t K, cudaStream_t s, unsigned flags) {
    return launch_mma_impl<Fmt, kWarps, kCtasPerSm, false>(W, scale, x, y, N, K, s, flags,
                                                           PeerOut{});
}

template <class Fmt, int kWarps, int kCtasPerSm>
cudaError_t launch_mma_sharded(const void* W, const void* scale, const void* x,
                               const PeerArgs& pa, int64_t N_shard, int64_t K, cudaStream_t s,
                               unsigned flags) {
    if (pa.world < 1 || pa.world > kMaxPeers || pa.rank < 0 || pa.rank >= pa.world)
        return cudaErrorInvalidValue;
    PeerOut po{};
    for (int p = 0; p < pa.world; ++p) {
        po.y[0][p] = static_cast<__half*>(pa.y[0][p]);
        po.y[1][p] = static_cast<__half*>(pa.y[1][p]);
        po.flag[p] = pa.flag[p];
    }
    po.row0 = pa.row0;
    po.rank = pa.rank;
    po.world = pa.world;
    return launch_mma_impl<Fmt, kWarps, kCtasPerSm, true>(W, scale, x, nullptr, N_shard, K, s,
                                                          flags, po);
}

// Geometry chosen per call (measured on B200 with L2-cold pools):
//  * independent GEMVs (CL_LAUNCH_PDL | CL_LAUNCH_INPUTS_READY): 4-warp CTAs,
//    one per SM per GEMV, so up to four GEMVs overlap on an SM; 8-warp CTAs
//    once K > 16384 (the staged activations then limit co-residency);
//  * chained or plain launches: 8-warp CTAs, two per SM per GEMV (shorter
//    per-GEMV latency), one per SM for K <= 2048.
template <class Fmt>
cudaError_t launch_mma_auto(const void* W, const void* scale, const void* x, void* y, int64_t N,
                            int64_t K, cudaStream_t s, unsigned flags) {
    if ((flags & 3u) == 3u)
        return K <= 16384 ? launch_mma<Fmt, 4, 1>(W, scale, x, y, N, K, s, flags)
                          : launch_mma<Fmt, 8, 1>(W, scale, x, y, N, K, s, flags);
    return K <= 2048 ? launch_mma<Fmt, 8, 1>(W, scale, x, y, N, K, s, flags)
                     : launch_mma<Fmt, 8, 2>(W, scale, x, y, N, K, s, flags);
}

template <class Fmt>
cudaError_t launch_mma_sharded_auto(const void* W, const void* scale, const void* x,
                                    const PeerArgs& pa, int64_t N, int64_t K, cudaStream_t s,
                                    unsigned flags) {
    if ((flags & 3u) == 3u)
        return K <= 16384 ? launch_mma_sharded<Fmt, 4, 1>(W, scale, x, pa, N, K, s, flags)
                          : launch_mma_sharded<Fmt, 8, 1>(W, scale, x, pa, N, K, s, flags);
    return K <= 2048 ? launch_mma_sharded<Fmt, 8, 1>(W, scale, x, pa, N, K, s, flags)
                     : launch_mma_sharded<Fmt, 8, 2>(W, scale, x, pa, N, K, s, flags);
}

const VariantDesc kInt4Variants[] = {
    {"int4gemv_baseline", launch_int4_scalar, false},
    {"int4gemv_bulk", launch_vec<Int4Fmt, MathF16, true>, false},
    {"int4gemv_bulk_f32x2", launch_vec<Int4Fmt, MathF32x2, true>, false},
    {"int4gemv_ldg", launch_vec<Int4Fmt, MathF16, false>, false},
    {"int4gemv_ldg_f32x2", launch_vec<Int4Fmt, MathF32x2, false>, false},
    {"int4gemv_mma", launch_mma_auto<MmaInt4>, false},
    {"int4gemv_mma_w4", launch_mma<MmaInt4, 4, 1>, false},
    {"int4gemv_mma_w8", launch_mma<MmaInt4, 8, 1>, false},
    {"int4gemv_mma_w8c2", launch_mma<MmaInt4, 8, 2>, false},
    {"int4gemv_mma_w16", launch_mma<MmaInt4, 16, 1>, false},
};

const VariantDesc kInt8Variants[] = {
    {"qgemv_baseline", launch_int8_scalar, false},
    {"qgemv_bulk", launch_vec<Int8Fmt, MathF16, true>, false},
    {"qgemv_bulk_f32x2", launch_vec<Int8Fmt, MathF32x2, true>, false},
    {"qgemv_ldg", launch_vec<Int8Fmt, MathF16, false>, false},
    {"qgemv_ldg_f32x2", launch_vec<Int8Fmt, MathF32x2, false>, false},
    {"qgemv_mma", launch_mma_auto<MmaInt8>, false},
    {"qgemv_mma_w4", launch_mma<MmaInt8, 4, 1>, false},
    {"qgemv_mma_w8", launch_mma<MmaInt8, 8, 1>, false},
    {"qgemv_mma_w8c2", launch_mma<MmaInt8, 8, 2>, false},
    {"qgemv_mma_w16", launch_mma<MmaInt8, 16, 1>, false},
};

}  // namespace

const ShardedVariantDesc kInt4Sharded[] = {
    {"int4gemv_mma", launch_mma_sharded_auto<MmaInt4>},
    {"int4gemv_mma_w4", launch_mma_sharded<MmaInt4, 4, 1>},
    {"int4gemv_mma_w8", launch_mma_sharded<MmaInt4, 8, 1>},
    {"int4gemv_mma_w8c2", launch_mma_sharded<MmaInt4, 8, 2>},
};

const ShardedVariantDesc kInt8Sharded[] = {
    {"qgemv_mma", launch_mma_sharded_auto<MmaInt8>},
    {"qgemv_mma_w4", launch_mma_sharded<MmaInt8, 4, 1>},
    {"qgemv_mma_w8", launch_mma_sharded<MmaInt8, 8, 1>},
    {"qgemv_mma_w8c2", launch_mma_sharded<MmaInt8, 8, 2>},
};

const VariantDesc* int4_variants(int* count) {
    *count = (int)(sizeof(kInt4Variants) / sizeof(kInt4Variants[0]));
    return kInt4Variants;
}

const VariantDesc* int8_variants(int* count) {
    *count = (int)(sizeof(kInt8Variants) / sizeof(kInt8Variants[0]));
    return kInt8Variants;
}

const ShardedVariantDesc* int4_sharded_variants(int* count) {
    *count = (int)(sizeof(kInt4Sharded) / sizeof(kInt4Sharded[0]));
    return kInt4Sharded;
}

const ShardedVariantDesc* int8_sharded_variants(int* count) {
    *count = (int)(sizeof(kInt8Sharded) / sizeof(kInt8Sharded[0]));
    return kInt8Sharded;
}

cudaError_t read_device_status(int clear, int* status) {
    int v = 0, m = 0;
    cudaError_t e = cudaMemcpyFromSymbol(&v, g_status, sizeof(int));

    if (e != cudaSuccess) return e;
    if (clear) {
        const int zero = 0;
        e = cudaMemcpyToSymbol(g_status, &zero, sizeof(int));

        if (e != cudaSuccess) return e;
    }
    *status = v ? v : m;
    return cudaSuccess;
}

}  // namespace clb
