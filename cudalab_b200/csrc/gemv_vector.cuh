// Vectorised weight-only GEMV kernels for sm_100a (INT4 group-scaled and INT8
// row-scaled), y[n] = sum_k dequant(W)[n,k] * x[k], fp32 accumulation, fp16 out.
//
// Work decomposition (both staging modes):
//   * Each CTA owns a contiguous, balanced range of rows.
//   * A row of W (RB bytes) is cut into slices of SB bytes (SB = largest power
//     of two <= 4 KiB dividing RB).  A slice is C = SB/16 chunks of 16 bytes.
//   * A tile is R_t = 4*P rows x SB bytes = 16 KiB, P = 256/C.  Consumer thread
//     t owns chunk c = t % C of rows p, p+P, p+2P, p+3P (p = t / C), so the 16
//     bytes it reads from shared memory are contiguous across the warp, and the
//     activations of its chunk (32 or 16 halves) sit in registers and are reused
//     for its 4 rows.
//   * Tiles run row-block outer, slice inner: a thread's 4 row partial sums stay
//     in registers across all slices and are reduced across the C threads of a
//     row once per row-block (warp butterfly + a shared-memory pass when C > 32).
//   * Group scales (INT4) or row scales (INT8) of the CTA's rows are staged into
//     shared memory once, at kernel start, overlapping the first weight fetches.
//
// Staging modes:
//   kBulk = true : a producer warp streams tiles through a ring of shared-memory
//                  stages with cp.async.bulk (TMA engine) + mbarriers, L2
//                  evict-first.  One CTA per SM, persistent over its rows.
//   kBulk = false: consumers load their own 16-byte chunks straight into
//                  registers (ld.global.nc, L1 no-allocate, L2 evict-first) with
//                  a one-tile register prefetch.
//
// Programmatic dependent launch: weights and scales are fetched before
// griddepcontrol.wait; activations are read and outputs written after it, so a
// GEMV launched with the programmatic-serialization attribute overlaps its
// weight stream with the tail of the preceding kernel without ever observing
// that kernel's activations early.
#pragma once

#include "gemv_common.cuh"

namespace clb {

struct GemvGeom {
    int64_t N;            // rows
    int64_t K;            // logical reduction length
    int64_t row_bytes;    // RB: bytes of W per row
    int32_t slice_bytes;  // SB
    int32_t n_slices;     // RB / SB
    int32_t chunks;       // C = SB / 16
    int32_t thread_rows;  // P = 256 / C
    int32_t tile_rows;    // R_t = 4 P
    int32_t rows_base;    // rows per CTA (first rows_rem CTAs get one more)
    int32_t rows_rem;
    int32_t stages;       // ring stages (bulk only)
    int32_t stage_bytes;  // bytes per ring stage (bulk only)
    int32_t groups;       // K / 128 for INT4, 1 for INT8
    int32_t scale_smem;   // bytes of the staged scale block
    int32_t ring_bytes;   // bytes reserved for the ring (0 for register-direct)
    int32_t ctas;         // grid size
    long long wait_cycles;  // bound of every mbarrier wait (SM cycles)
};

// ---------------------------------------------------------------------------
// Formats
// ---------------------------------------------------------------------------
struct Int4Fmt {
    static constexpr int kElems = 32;  // elements per 16-byte chunk
    static constexpr bool kGroupScale = true;
    using Scale = __half;
};
struct Int8Fmt {
    static constexpr int kElems = 16;
    static constexpr bool kGroupScale = false;
    using Scale = float;
};

struct MathF16 {};    // exact fp16 dequant + mixed fma.rn.f32.f16
struct MathF32x2 {};  // exact fp32 dequant + packed fma.rn.f32x2

template <class Fmt, class Math>
struct XRegs;

// ---- INT4, mixed precision -------------------------------------------------
template <>
struct XRegs<Int4Fmt, MathF16> {
    __half2 h[16];  // h[j] = (x[2j], x[2j+1]) of the 32-element chunk

    __device__ __forceinline__ void load(const __half* xk) {
        const uint4* p = reinterpret_cast<const uint4*>(xk);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const uint4 v = __ldg(p + j);
            h[4 * j + 0] = u32_as_h2(v.x);
            h[4 * j + 1] = u32_as_h2(v.y);
            h[4 * j + 2] = u32_as_h2(v.z);
            h[4 * j + 3] = u32_as_h2(v.w);
        }
    }

    __device__ __forceinline__ float dot(const uint4 wv) const {
        const uint32_t w[4] = {wv.x, wv.y, wv.z, wv.w};
        float a0 = 0.f, a1 = 0.f;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            __half2 q[4];
            int4x8_to_h2(w[i], q);  // (n0,n4) (n1,n5) (n2,n6) (n3,n7)
            const __half2 x01 = h[4 * i], x23 = h[4 * i + 1];
            const __half2 x45 = h[4 * i + 2], x67 = h[4 * i + 3];
            a0 = fma_h(__low2half(q[0]), __low2half(x01), a0);
            a1 = fma_h(__low2half(q[1]), __high2half(x01), a1);
            a0 = fma_h(__low2half(q[2]), __low2half(x23), a0);
            a1 = fma_h(__low2half(q[3]), __high2half(x23), a1);
            a0 = fma_h(__high2half(q[0]), __low2half(x45), a0);
            a1 = fma_h(__high2half(q[1]), __high2half(x45), a1);
            a0 = fma_h(__high2half(q[2]), __low2half(x67), a0);
            a1 = fma_h(__high2half(q[3]), __high2half(x67), a1);
        }
        return a0 + a1;
    }
};

// ---- INT4, packed fp32 -----------------------------------------------------
template <>
struct XRegs<Int4Fmt, MathF32x2> {
    unsigned long long xp[16];  // xp[j] = (x[2j], x[2j+1]) as fp32 pair

    __device__ __forceinline__ void load(const __half* xk) {
        const uint4* p = reinterpret_cast<const uint4*>(xk);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const uint4 v = __ldg(p + j);
            const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const float2 f = __half22float2(u32_as_h2(u[e]));
                xp[4 * j + e] = f2_pack(f.x, f.y);
            }
        }
    }

    __device__ __forceinline__ float dot(const uint4 wv) const {
        // biases of nibble positions 0..4: 2^(23-4p) + 8
        constexpr float B0 = 8388608.f + 8.f, B1 = 524288.f + 8.f, B2 = 32768.f + 8.f;
        constexpr float B3 = 2048.f + 8.f, B4 = 128.f + 8.f;
        const unsigned long long nb01 = f2_pack(-B0, -B1);
        const unsigned long long nb23 = f2_pack(-B2, -B3);
        const unsigned long long nb45 = f2_pack(-B4, -B2);
        const unsigned long long nb67 = f2_pack(-B3, -B4);
        const uint32_t w[4] = {wv.x, wv.y, wv.z, wv.w};
        unsigned long long acc_a = 0ull, acc_b = 0ull;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint32_t lo = w[i], hi = w[i] >> 12;  // hi: nibbles 3..7 at positions 0..4
            const unsigned long long q01 =
                f2_add(f2_pack(nib_to_biased_f32<0>(lo), nib_to_biased_f32<1>(lo)), nb01);
            const unsigned long long q23 =
                f2_add(f2_pack(nib_to_biased_f32<2>(lo), nib_to_biased_f32<3>(lo)), nb23);
            const unsigned long long q45 =
                f2_add(f2_pack(nib_to_biased_f32<4>(lo), nib_to_biased_f32<2>(hi)), nb45);
            const unsigned long long q67 =
                f2_add(f2_pack(nib_to_biased_f32<3>(hi), nib_to_biased_f32<4>(hi)), nb67);
            acc_a = f2_fma(q01, xp[4 * i + 0], acc_a);
            acc_b = f2_fma(q23, xp[4 * i + 1], acc_b);
            acc_a = f2_fma(q45, xp[4 * i + 2], acc_a);
            acc_b = f2_fma(q67, xp[4 * i + 3], acc_b);
        }
        float a0, a1, b0, b1;
        f2_unpack(acc_a, a0, a1);
        f2_unpack(acc_b, b0, b1);
        return (a0 + a1) + (b0 + b1);
    }
};

// ---- INT8, mixed precision -------------------------------------------------
template <>
struct XRegs<Int8Fmt, MathF16> {
    __half2 h[8];  // h[j] = (x[2j], x[2j+1]) of the 16-element chunk

    __device__ __forceinline__ void load(const __half* xk) {
        const uint4* p = reinterpret_cast<const uint4*>(xk);
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            const uint4 v = __ldg(p + j);
            h[4 * j + 0] = u32_as_h2(v.x);
            h[4 * j + 1] = u32_as_h2(v.y);
            h[4 * j + 2] = u32_as_h2(v.z);
            h[4 * j + 3] = u32_as_h2(v.w);
        }
    }

    __device__ __forceinline__ float dot(const uint4 wv) const {
        const uint32_t w[4] = {wv.x, wv.y, wv.z, wv.w};
        float a0 = 0.f, a1 = 0.f;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            __half2 q[2];
            int8x4_to_h2(w[i], q);  // (b0,b1) (b2,b3)
            const __half2 x01 = h[2 * i], x23 = h[2 * i + 1];
            a0 = fma_h(__low2half(q[0]), __low2half(x01), a0);
            a1 = fma_h(__high2half(q[0]), __high2half(x01), a1);
            a0 = fma_h(__low2half(q[1]), __low2half(x23), a0);
            a1 = fma_h(__high2half(q[1]), __high2half(x23), a1);
        }
        return a0 + a1;
    }
};

// ---- INT8, packed fp32 -----------------------------------------------------
template <>
struct XRegs<Int8Fmt, MathF32x2> {
    unsigned long long xp[8];

    __device__ __forceinline__ void load(const __half* xk) {
        const uint4* p = reinterpret_cast<const uint4*>(xk);
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            const uint4 v = __ldg(p + j);
            const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const float2 f = __half22float2(u32_as_h2(u[e]));
                xp[4 * j + e] = f2_pack(f.x, f.y);
            }
        }
    }

    __device__ __forceinline__ float dot(const uint4 wv) const {
        // byte at bits 0..7 -> 2^23 + u, at bits 8..15 -> 2^15 + u (u = b + 128)
        constexpr float B0 = 8388608.f + 128.f, B1 = 32768.f + 128.f;
        const unsigned long long nb = f2_pack(-B0, -B1);
        const uint32_t w[4] = {wv.x, wv.y, wv.z, wv.w};
        unsigned long long acc_a = 0ull, acc_b = 0ull;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint32_t lo = w[i], hi = w[i] >> 16;
            const float f0 = __uint_as_float(lop3_sel_xor(lo, 0x000000FFu, 0x4B000080u));
            const float f1 = __uint_as_float(lop3_sel_xor(lo, 0x0000FF00u, 0x47008000u));
            const float f2 = __uint_as_float(lop3_sel_xor(hi, 0x000000FFu, 0x4B000080u));
            const float f3 = __uint_as_float(lop3_sel_xor(hi, 0x0000FF00u, 0x47008000u));
            acc_a = f2_fma(f2_add(f2_pack(f0, f1), nb), xp[2 * i + 0], acc_a);
            acc_b = f2_fma(f2_add(f2_pack(f2, f3), nb), xp[2 * i + 1], acc_b);
        }
        float a0, a1, b0, b1;
        f2_unpack(acc_a, a0, a1);
        f2_unpack(acc_b, b0, b1);
        return (a0 + a1) + (b0 + b1);
    }
};

// ---------------------------------------------------------------------------
// Shared-memory layout: [ring | scales | red[2][8][4] f32 | full[16] | empty[16]]
// ---------------------------------------------------------------------------
__host__ __device__ inline int red_offset(const GemvGeom& g) {
    return g.ring_bytes + ((g.scale_smem + 15) & ~15);
}
__host__ __device__ inline int bar_offset(const GemvGeom& g) {
    return red_offset(g) + 2 * kConsumerWarps * 4 * 4;
}
__host__ __device__ inline int smem_total(const GemvGeom& g) {
    return bar_offset(g) + 2 * kMaxStages * 8;
}

__device__ __forceinline__ void cta_rows(const GemvGeom& g, int64_t& r0, int& nrows) {
    const int b = blockIdx.x;
    r0 = (int64_t)b * g.rows_base + (b < g.rows_rem ? b : g.rows_rem);
    nrows = g.rows_base + (b < g.rows_rem ? 1 : 0);
}

// Stage this CTA's scales (all groups of rows [r0, r0+nrows)) into shared
// memory with the consumer threads.  Head/tail in 2-byte (INT4) or 4-byte
// (INT8) units, body in 16-byte streaming loads.
template <class Fmt>
__device__ __forceinline__ void stage_scales(const typename Fmt::Scale* scale, const GemvGeom& g,
                                             int64_t r0, int nrows, uint8_t* s_dst, int tid,
                                             uint64_t pol) {
    using S = typename Fmt::Scale;
    const int64_t first = r0 * g.groups;
    const int64_t count = (int64_t)nrows * g.groups;
    const S* src = scale + first;
    S* dst = reinterpret_cast<S*>(s_dst);
    const uintptr_t a = reinterpret_cast<uintptr_t>(src);
    int64_t head = (int64_t)(((16 - (a & 15)) & 15) / sizeof(S));
    if ((a % sizeof(S)) != 0) head = count;  // not even element aligned: scalar
    if (head > count) head = count;
    for (int64_t i = tid; i < head; i += kConsumerThreads) dst[i] = src[i];
    const int64_t body = ((count - head) * (int64_t)sizeof(S)) / 16;
    // destination of the body may be unaligned for 16-byte stores: copy via
    // 4-byte pieces when the head shifted it off alignment.
    const bool dst_aligned = ((head * (int64_t)sizeof(S)) & 15) == 0;
    for (int64_t v = tid; v < body; v += kConsumerThreads) {
        const uint4 q = ldg_stream16(reinterpret_cast<const uint8_t*>(src + head) + 16 * v, pol);
        uint8_t* d = reinterpret_cast<uint8_t*>(dst + head) + 16 * v;
        if (dst_aligned) {
            *reinterpret_cast<uint4*>(d) = q;
        } else {
            // head*sizeof(S) is even, so 2-byte stores are always legal
            const uint32_t u[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                reinterpret_cast<uint16_t*>(d)[2 * e] = (uint16_t)(u[e] & 0xFFFF);
                reinterpret_cast<uint16_t*>(d)[2 * e + 1] = (uint16_t)(u[e] >> 16);
            }
        }
    }
    const int64_t done = head + body * 16 / (int64_t)sizeof(S);
    for (int64_t i = done + tid; i < count; i += kConsumerThreads) dst[i] = src[i];
}

// Multi-value butterfly: reduce 4 values over the 32 lanes of a warp; lane L
// ends with the full sum of value (L>>4 & 1)*2 + (L>>3 & 1).
__device__ __forceinline__ float warp_reduce4(float v0, float v1, float v2, float v3, int lane) {
    const bool u = (lane & 16) != 0;
    float a0 = u ? v2 : v0, a1 = u ? v3 : v1;
    const float b0 = u ? v0 : v2, b1 = u ? v1 : v3;
    a0 += __shfl_xor_sync(0xffffffffu, b0, 16);
    a1 += __shfl_xor_sync(0xffffffffu, b1, 16);
    const bool t = (lane & 8) != 0;
    float c = t ? a1 : a0;
    const float d = t ? a0 : a1;
    c += __shfl_xor_sync(0xffffffffu, d, 8);
    c += __shfl_xor_sync(0xffffffffu, c, 4);
    c += __shfl_xor_sync(0xffffffffu, c, 2);
    c += __shfl_xor_sync(0xffffffffu, c, 1);
    return c;
}

// ---------------------------------------------------------------------------
// The kernel.
// ---------------------------------------------------------------------------
template <class Fmt, class Math, bool kBulk>
__global__ void __launch_bounds__(kBulk ? kConsumerThreads + 32 : kConsumerThreads, 2)
gemv_vec_kernel(const uint8_t* __restrict__ W, const typename Fmt::Scale* __restrict__ scale,
                const __half* __restrict__ x, __half* __restrict__ y, const GemvGeom g) {
    extern __shared__ __align__(128) uint8_t smem[];
    uint8_t* ring = smem;
    uint8_t* s_scale = smem + g.ring_bytes;
    float* red = reinterpret_cast<float*>(smem + red_offset(g));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + bar_offset(g));
    const uint32_t full0 = smem_u32(bars);
    const uint32_t empty0 = smem_u32(bars + kMaxStages);

    int64_t r0;
    int nrows;
    cta_rows(g, r0, nrows);
    const int tid = threadIdx.x;
    const int warp = tid >> 5, lane = tid & 31;
    const uint64_t pol = policy_evict_first();
    const int n_rb = (nrows + g.tile_rows - 1) / g.tile_rows;
    const int total_iters = n_rb * g.n_slices;

    if constexpr (kBulk) {
        if (tid == 0) {
            for (int s = 0; s < g.stages; ++s) {
                mbar_init(full0 + 8 * s, 1);
                mbar_init(empty0 + 8 * s, kConsumerWarps);
            }
            fence_barrier_init();
        }
        __syncthreads();
    }
    // Let the next kernel in the stream start staging its own weights as soon
    // as every CTA of this grid is resident.
    pdl_allow_dependents();

    if constexpr (kBulk) {
        if (warp == kConsumerWarps) {
            // ---------------- producer warp ----------------
            int issued = 0;
            for (int it = 0; it < total_iters; ++it) {
                const int st = it % g.stages;
                const int rb = it / g.n_slices, sl = it % g.n_slices;
                const int rows_here = min(g.tile_rows, nrows - rb * g.tile_rows);
                const uint32_t bytes = (uint32_t)rows_here * (uint32_t)g.slice_bytes;
                int ok = 1;
                if (lane == 0) {
                    if (it >= g.stages) {
                        const uint32_t par = (uint32_t)((it / g.stages) - 1) & 1u;
                        if (!mbar_wait_bounded(empty0 + 8 * st, par, g.wait_cycles)) ok = 0;
                    }
                    if (ok) mbar_arrive_expect_tx(full0 + 8 * st, bytes);
                }
                ok = __shfl_sync(0xffffffffu, ok, 0);
                if (!ok) {
                    // stop issuing; the consumers time out on their own waits
                    if (lane == 0) record_status(kStatusTimeoutEmpty);
                    break;
                }
                issued = it + 1;
                {
                    const uint32_t dst = smem_u32(ring + (size_t)st * g.stage_bytes);
                    const int64_t row0 = r0 + (int64_t)rb * g.tile_rows;
                    if (g.n_slices == 1) {
                        if (lane == 0)
                            bulk_g2s(dst, W + row0 * g.row_bytes, bytes, full0 + 8 * st, pol);
                    } else {
                        for (int r = lane; r < rows_here; r += 32)
                            bulk_g2s(dst + (uint32_t)r * (uint32_t)g.slice_bytes,
                                     W + (row0 + r) * g.row_bytes + (int64_t)sl * g.slice_bytes,
                                     (uint32_t)g.slice_bytes, full0 + 8 * st, pol);
                    }
                }
                __syncwarp();
            }
            // Every copy this CTA issued must land before the CTA may exit.
            if (lane == 0) {
                const int used = issued < g.stages ? issued : g.stages;
                for (int st = 0; st < used; ++st) {
                    const int last = st + ((issued - 1 - st) / g.stages) * g.stages;
                    const uint32_t par = (uint32_t)(last / g.stages) & 1u;
                    if (!mbar_wait_bounded(full0 + 8 * st, par, g.wait_cycles))
                        record_status(kStatusTimeoutDrain);
                }
            }
            return;
        }
    }

    // ---------------- consumers ----------------
    stage_scales<Fmt>(scale, g, r0, nrows, s_scale, tid, pol);
    consumer_sync();

    const int C = g.chunks, P = g.thread_rows;
    const int c = tid % C, p = tid / C;
    const __half* sc4 = reinterpret_cast<const __half*>(s_scale);
    const float* sc8 = reinterpret_cast<const float*>(s_scale);

    // Register-direct mode: prefetch the first tile's weights before waiting
    // on the preceding grid (weights never depend on it).
    uint4 wnext[kRowsPerThread];
    auto fetch = [&](int it, uint4 (&dst)[kRowsPerThread]) {
        const int rb = it / g.n_slices, sl = it % g.n_slices;
        const int rows_here = min(g.tile_rows, nrows - rb * g.tile_rows);
#pragma unroll
        for (int i = 0; i < kRowsPerThread; ++i) {
            const int lr = p + P * i;
            if (lr < rows_here) {
                const int64_t row = r0 + (int64_t)rb * g.tile_rows + lr;
                dst[i] = ldg_stream16(
                    W + row * g.row_bytes + (int64_t)sl * g.slice_bytes + kChunkBytes * c, pol);
            } else {
                dst[i] = make_uint4(0u, 0u, 0u, 0u);
            }
        }
    };
    if constexpr (!kBulk) {
        if (total_iters > 0) fetch(0, wnext);
    }

    pdl_wait_prior_grids();

    XRegs<Fmt, Math> xr;
    if (g.n_slices == 1) xr.load(x + (int64_t)Fmt::kElems * c);

    bool failed = false;
    int it = 0;
    for (int rb = 0; rb < n_rb; ++rb) {
        const int rows_here = min(g.tile_rows, nrows - rb * g.tile_rows);
        float acc[kRowsPerThread] = {0.f, 0.f, 0.f, 0.f};
        for (int sl = 0; sl < g.n_slices; ++sl, ++it) {
            const int64_t k0 =
                (int64_t)sl * g.slice_bytes * (Fmt::kElems / kChunkBytes) + (int64_t)Fmt::kElems * c;
            if (g.n_slices > 1) xr.load(x + k0);
            uint4 wv[kRowsPerThread];
            const int st = kBulk ? it % g.stages : 0;
            if constexpr (kBulk) {
                const uint32_t par = (uint32_t)(it / g.stages) & 1u;
                if (!failed && !mbar_wait_bounded(full0 + 8 * st, par, g.wait_cycles)) {
                    record_status(kStatusTimeoutFull);
                    failed = true;
                }
                const uint32_t base = smem_u32(ring + (size_t)st * g.stage_bytes) +
                                      (uint32_t)(kChunkBytes * c);
#pragma unroll
                for (int i = 0; i < kRowsPerThread; ++i) {
                    const int lr = p + P * i;
                    wv[i] = (!failed && lr < rows_here)
                                ? lds16(base + (uint32_t)lr * (uint32_t)g.slice_bytes)
                                : make_uint4(0u, 0u, 0u, 0u);
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(empty0 + 8 * st);
            } else {
#pragma unroll
                for (int i = 0; i < kRowsPerThread; ++i) wv[i] = wnext[i];
                if (it + 1 < total_iters) fetch(it + 1, wnext);
            }
#pragma unroll
            for (int i = 0; i < kRowsPerThread; ++i) {
                const int lr = p + P * i;
                if (lr < rows_here) {
                    const float d = xr.dot(wv[i]);
                    if constexpr (Fmt::kGroupScale) {
                        const int lrow = rb * g.tile_rows + lr;
                        const float s =
                            __half2float(sc4[(int64_t)lrow * g.groups + (int)(k0 >> 7)]);
                        acc[i] = fmaf(s, d, acc[i]);
                    } else {
                        acc[i] += d;
                    }
                }
            }
        }
        // ---- reduce the row partials over the C threads of each row ----
        const int64_t row0 = r0 + (int64_t)rb * g.tile_rows;
        if (C >= 32) {
            const float v = warp_reduce4(acc[0], acc[1], acc[2], acc[3], lane);
            float* rbuf = red + (rb & 1) * kConsumerWarps * 4;
            if ((lane & 7) == 0) rbuf[warp * 4 + (lane >> 3)] = v;
            consumer_sync();
            if (tid < rows_here) {
                const int lr = tid, pp = lr % P, i = lr / P;
                const int wpr = C >> 5;  // warps per row-lane
                float s = 0.f;
                for (int w = pp * wpr; w < (pp + 1) * wpr; ++w) s += rbuf[w * 4 + i];
                if constexpr (!Fmt::kGroupScale) s *= sc8[rb * g.tile_rows + lr];
                if (!failed) y[row0 + lr] = __float2half_rn(s);
            }
        } else {
#pragma unroll
            for (int i = 0; i < kRowsPerThread; ++i)
                for (int o = C >> 1; o > 0; o >>= 1)
                    acc[i] += __shfl_xor_sync(0xffffffffu, acc[i], o);
            if (c == 0) {
#pragma unroll
                for (int i = 0; i < kRowsPerThread; ++i) {
                    const int lr = p + P * i;
                    if (lr < rows_here) {
                        float s = acc[i];
                        if constexpr (!Fmt::kGroupScale) s *= sc8[rb * g.tile_rows + lr];
                        if (!failed) y[row0 + lr] = __float2half_rn(s);
                    }
                }
            }
        }
    }
}

}  // namespace clb
