// INT4 weight-only GEMV / small-batch GEMM on the 5th-generation tensor cores
// (tcgen05 + Tensor Memory + TMA) for sm_100a:
//   Y[m, n] = sum_k (s[n, k/128] * q[n, k]) * X[m, k],  1 <= M <= 16.
//
// Roles and data flow of one CTA (a tile of 128 weight rows, one K split):
//   * control thread (warp 8, lane 0): streams the tile's weights two scale
//     groups at a time (128 rows x 128 bytes, 128-byte swizzle) with a 2-D
//     TMA copy into a ring of shared-memory stages (L2 evict-first), and
//     issues the MMAs;
//   * 256 row threads (warps 0-7; warps w and w + 4 share TMEM lanes
//     32 (w & 3) .. +31 = tile rows, one thread per row and half group): per
//     group, read their 32 bytes of the row from the stage, dequantise them
//     exactly (lop3 + add.f16x2 per two values) and store the 64 fp16 values
//     into a TMEM A buffer with tcgen05.st; stage the group's activations
//     (16 columns x 128 k, fp16, prefetched one group ahead) into shared
//     memory; after the group's MMAs, read their 8 accumulator columns back
//     with tcgen05.ld and add s[n, group] * D[n, m] into their row sums in
//     registers.
//   * MMA: tcgen05.mma.cta_group::1.kind::f16, M = 128 (weight rows, A in
//     TMEM), N = 16 (activation rows, zero past M, B in shared memory,
//     K-major, no swizzle), K = 16; eight per group into one accumulator,
//     the first one overwriting it.  Products of fp16 values are exact; the
//     group's sum is rounded to fp32, scaled (one rounding) and added to the
//     row sum (one rounding) -- the same per-term rounding budget as the
//     register-fed kernels.
// The dequantised values leave registers through tcgen05.st (one instruction
// per 64 columns), so the per-weight issue cost is the dequantisation itself;
// MMAs are issued by one thread and run on the tensor cores beside it.
//
// Pipelines (every barrier is waited on at most one phase behind, so parity
// waits are unambiguous):
//   w_full[kTcStages]  weight stage landed (TMA transaction count); a stage
//                      is refilled once the MMA thread has seen both of its
//                      groups dequantised;
//   a_full[kTcABufs]   A buffer + activation tile of a group written (one
//                      arrival per row thread, a group after it was stored);
//   a_free[kTcABufs]   the group's MMAs completed (tcgen05.commit): the
//                      buffer may be rewritten kTcABufs groups later.  A
//                      commit tracks every earlier MMA of its thread, so the
//                      same wait shows the accumulators of older groups
//                      complete: group g's accumulator (one of kTcDBufs) is
//                      read kTcDBufs groups later, just before the row threads
//                      release the group that reuses it, and the MMA round
//                      trip never stalls them.
//
// Tensor Memory: 256 columns per CTA (A: 3 x 64, D: 4 x 16), allocated only after
// the programmatic-dependent-launch wait (so a kernel that may still hold
// TMEM has completed) and released before any cluster barrier, so no CTA
// ever waits on another CTA while it holds TMEM.  Every mbarrier wait is
// bounded (MmaGeom-style wait_cycles); on expiry the CTA records status 6,
// stops issuing work, waits (bounded) for its own copies and MMAs, frees its
// TMEM and returns.
//
// K splits (S > 1, a cluster of S CTAs per tile) sum their partial row sums
// in split order through distributed shared memory; S depends on the shape
// and the SM count only, so results do not depend on flags.
#pragma once

#include <cuda.h>

#include "gemv_mma.cuh"

namespace clb {

constexpr int kTcRows = 128;                              // weight rows per tile (MMA M)
constexpr int kTcN = 16;                                  // MMA N (activation rows, padded)
constexpr int kTcGroupK = 128;                            // k per scale group
constexpr int kTcStageGroups = 2;                         // scale groups per weight stage
constexpr int kTcStages = 4;                              // weight stages in shared memory
constexpr int kTcStageBytes = kTcRows * kTcStageGroups * (kTcGroupK / 2);  // 16 KiB
constexpr int kTcABufs = 3;                               // TMEM A buffers / activation tiles
constexpr int kTcDBufs = 4;                               // TMEM accumulators
constexpr int kTcXBytes = kTcN * kTcGroupK * 2;           // 4 KiB: 16 x 128 fp16
constexpr int kTcTmemCols = 256;
static_assert(kTcABufs * 64 + kTcDBufs * 16 <= kTcTmemCols, "TMEM columns");
constexpr int kTcRowWarps = 8;                            // two per TMEM lane quarter
constexpr int kTcRowThreads = 32 * kTcRowWarps;
constexpr int kTcThreads = kTcRowThreads + 32;            // + 1 control warp
constexpr int kTcMaxSplits = 8;
constexpr int kStatusTimeoutTc = 6;  // a tensor-core pipeline wait expired

struct TcGeom {
    int64_t N, K;
    int64_t x_stride, y_stride;  // elements between activation rows of X / Y
    int32_t M;                   // activation rows (1..16)
    int32_t groups;              // K / 128
    int32_t splits;              // K splits (cluster size when > 1)
    int32_t gsplit;              // groups per split (the last split may have fewer)
    long long wait_cycles;       // bound of every mbarrier wait (SM cycles)
    int32_t wait_first;          // wait for the preceding kernel before any global access
};

// Shared memory: [weight stages | activation tiles | split row sums | barriers]
__host__ __device__ inline int tc_x_off() { return kTcStages * kTcStageBytes; }
__host__ __device__ inline int tc_rsum_off() { return tc_x_off() + kTcABufs * kTcXBytes; }
__host__ __device__ inline int tc_bar_off(const TcGeom& g) {
    return tc_rsum_off() + (g.splits > 1 ? kTcRows * kTcN * 4 : 0);
}
// At least 80 KiB, so that at most two CTAs share an SM: two CTAs' TMEM
// (2 x 256 columns) always fits, and an allocation never has to wait.
__host__ __device__ inline int tc_smem_total(const TcGeom& g) {
    const int need = tc_bar_off(g) + 128 + 1024;  // barriers and flags; 1 KiB to align stages
    return need < 80 * 1024 ? 80 * 1024 : need;
}

// Instruction descriptor of tcgen05.mma kind::f16: D fp32 (bits 4-5 = 1), A and
// B fp16 (bits 7-9, 10-12 = 0), both K-major (bits 15, 16 = 0), N >> 3 at bit
// 17, M >> 4 at bit 24.
constexpr uint32_t kTcIdesc = (1u << 4) | ((uint32_t)(kTcN >> 3) << 17) |
                              ((uint32_t)(kTcRows >> 4) << 24);

// Shared-memory matrix descriptor, K-major without swizzle: 8-row x 16-byte
// core matrices; LBO = bytes between the two K halves of a K = 16 step,
// SBO = bytes between 8-row groups; version 1 (bits 46-47).
__device__ __forceinline__ uint64_t tc_smem_desc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
    return (uint64_t)((addr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
           ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46);
}

__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[tmem] x B[smem desc], one elected thread.
__device__ __forceinline__ void tc_mma(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                       uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %3, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %4, {%5, %6, %7, %8}, p;\n\t}"
        ::"r"(d_tmem), "r"(a_tmem), "l"(b_desc), "r"(accumulate), "r"(kTcIdesc), "r"(0u), "r"(0u),
        "r"(0u), "r"(0u)
        : "memory");
}

// Arrive once on `bar` when every tcgen05 operation this thread issued so far
// has completed.
__device__ __forceinline__ void tc_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     bar)
                 : "memory");
}

// 2-D TMA load of one box into shared memory, completing on `bar`.
__device__ __forceinline__ void tc_tma_2d(uint32_t dst, const CUtensorMap* map, int x, int y,
                                          uint32_t bar, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        ".L2::cache_hint [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar), "l"(policy)
        : "memory");
}

// 32 consecutive 32-bit columns of this thread's TMEM lane.
__device__ __forceinline__ void tc_st32(uint32_t taddr, const uint32_t (&v)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {"
        "%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "
        "%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(
            taddr),
        "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]),
        "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]),
        "r"(v[15]), "r"(v[16]), "r"(v[17]), "r"(v[18]), "r"(v[19]), "r"(v[20]), "r"(v[21]),
        "r"(v[22]), "r"(v[23]), "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]), "r"(v[28]),
        "r"(v[29]), "r"(v[30]), "r"(v[31])
        : "memory");
}

// 8 consecutive 32-bit columns of this thread's TMEM lane (waits for them).
__device__ __forceinline__ void tc_ld8(uint32_t taddr, float (&d)[8]) {
    uint32_t r[8];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7])
        : "r"(taddr)
        : "memory");
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 8; ++i) d[i] = __uint_as_float(r[i]);
}

// The same read split in two: the load is issued, other work follows, and the
// wait makes the registers valid (they are passed through it, so no use can
// move above it).
__device__ __forceinline__ void tc_ld8_issue(uint32_t taddr, uint32_t (&r)[8]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7])
        : "r"(taddr)
        : "memory");
}
__device__ __forceinline__ void tc_ld8_wait(uint32_t (&r)[8]) {
    asm volatile("tcgen05.wait::ld.sync.aligned;"
                 : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]),
                   "+r"(r[6]), "+r"(r[7])
                 :
                 : "memory");
}

__device__ __forceinline__ void tc_wait_st() {
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Row threads: record an expired wait and decide, uniformly across the warp
// (tcgen05.ld / st are warp-collective), whether to stop.
__device__ __forceinline__ bool tc_stop(bool ok, volatile int* fail) {
    if (!ok) {
        record_status(kStatusTimeoutTc);
        *fail = 1;
    }
    return __any_sync(0xffffffffu, !ok || *fail != 0);
}

// A 32-bit word of CTA `rank`'s shared memory at the offset of `local`.
__device__ __forceinline__ uint32_t ld_cluster_u32(uint32_t local, uint32_t rank) {
    uint32_t ra, v;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(ra) : "r"(local), "r"(rank));
    asm volatile("ld.shared::cluster.u32 %0, [%1];" : "=r"(v) : "r"(ra) : "memory");
    return v;
}

template <bool kPeer>
__global__ void __launch_bounds__(kTcThreads, 1)
gemv_tc_int4_kernel(const __grid_constant__ CUtensorMap wmap, const __half* __restrict__ scale,
                    const __half* __restrict__ x, __half* __restrict__ y, const TcGeom g,
                    const PeerOut po) {
    extern __shared__ uint8_t smem_raw[];
    // stages need 1 KiB alignment (TMA swizzle pattern); the rest follows
    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    const uint32_t s_base = smem_u32(smem);
    const uint32_t s_x = s_base + tc_x_off();
    float* rsum = reinterpret_cast<float*>(smem + tc_rsum_off());
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + tc_bar_off(g));
    const uint32_t b_wfull = smem_u32(bars);             // kTcStages: weight stage landed
    const uint32_t b_afull = b_wfull + 8 * kTcStages;    // kTcABufs: A + x tile written
    const uint32_t b_afree = b_afull + 8 * kTcABufs;     // kTcABufs: their MMAs completed
    volatile uint32_t* s_tmem =
        reinterpret_cast<volatile uint32_t*>(bars + kTcStages + 2 * kTcABufs);
    volatile int* s_fail = reinterpret_cast<volatile int*>(s_tmem + 1);
    volatile unsigned* s_epoch = reinterpret_cast<volatile unsigned*>(s_tmem + 2);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int split = g.splits > 1 ? (int)cluster_rank() : 0;
    const int tile = blockIdx.x / g.splits;
    const int64_t row0 = (int64_t)tile * kTcRows;
    const int g0 = split * g.gsplit;
    const int G = min(g.gsplit, g.groups - g0);
    const int n_stage_uses = (G + kTcStageGroups - 1) / kTcStageGroups;
    const bool mma_thread = warp == kTcRowWarps && lane == 0;

    pdl_allow_dependents();
    // Without the caller's CL_LAUNCH_PDL: launched early all the same, but no
    // global access before the preceding kernel has completed (stream order).
    if (g.wait_first) pdl_wait_prior_grids();
    if (tid == 0) {
        for (int i = 0; i < kTcStages; ++i) mbar_init(b_wfull + 8 * i, 1);
        for (int j = 0; j < kTcABufs; ++j) {
            mbar_init(b_afull + 8 * j, kTcRowThreads);
            mbar_init(b_afree + 8 * j, 1);
        }
        *s_fail = 0;
        fence_barrier_init();
    }
    __syncthreads();

    // Weights never depend on the preceding kernel: the first stages are
    // requested before waiting on it.  Stage use u holds groups 2u, 2u + 1.
    const uint64_t pol = policy_evict_first();
    int issued = 0;  // stage uses requested (control thread)
    auto request = [&](int u) {
        const int st = u % kTcStages;
        const uint32_t bar = b_wfull + 8 * st;
        mbar_arrive_expect_tx(bar, kTcStageBytes);
        tc_tma_2d(s_base + st * kTcStageBytes, &wmap,
                  (g0 + kTcStageGroups * u) * (kTcGroupK / 2), (int)row0, bar, pol);
    };
    if (mma_thread)
        for (; issued < min(kTcStages, n_stage_uses); ++issued) request(issued);
    pdl_wait_prior_grids();
    // Tensor Memory only after the preceding kernel has completed.
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_u32(const_cast<uint32_t*>(s_tmem))),
                     "r"(kTcTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    if constexpr (kPeer) {
        if (tid == 0) *s_epoch = *reinterpret_cast<volatile unsigned*>(po.flag[po.rank] + kStep) + 1u;
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *s_tmem;
    const uint32_t t_d0 = tmem + kTcABufs * 64;  // accumulators, 16 columns each

    // Row warp w: TMEM lanes 32 (w & 3) .. +31 (tile rows), half h = w >> 2 of
    // each group (bytes 32 h .. 32 h + 31 of a row's 64, A columns 32 h ..
    // 32 h + 31) and of the activation columns (m = 8 h .. 8 h + 7).
    const int quarter = warp & 3, half = (warp >> 2) & 1;
    float yacc[8];
#pragma unroll
    for (int m = 0; m < 8; ++m) yacc[m] = 0.f;

    if (warp < kTcRowWarps) {
        // ---------------- row threads ----------------
        const int r = 32 * quarter + lane;                   // tile row = TMEM lane
        const int64_t row = row0 + r;
        const int64_t srow = row < g.N ? row : g.N - 1;      // rows past N read scales of N-1
        const __half* srow_p = scale + srow * g.groups + g0;
        const uint32_t lane_base = (uint32_t)(32 * quarter) << 16;
        // this thread's 16-byte piece of each activation tile: entry u =
        // (n, k8), n = u >> 4 activation row, k8 = u & 15 eight-k block
        const int un = tid >> 4, uk8 = tid & 15;
        auto load_x = [&](int gi) {
            uint4 v = make_uint4(0u, 0u, 0u, 0u);
            if (un < g.M)
                v = __ldg(reinterpret_cast<const uint4*>(
                    x + un * g.x_stride + (int64_t)(g0 + gi) * kTcGroupK + 8 * uk8));
            return v;
        };
        const uint32_t x_off = (uint32_t)((((2 * uk8 + (un >> 3)) << 3) + (un & 7)) << 4);
        // sums of group h (accumulator h % kTcDBufs); the caller has seen a
        // commit issued after group h's MMAs, so they are complete
        auto drain = [&](int h, float s) {
            float d[8];
            tc_ld8(t_d0 + lane_base + (uint32_t)(kTcN * (h % kTcDBufs) + 8 * half), d);
#pragma unroll
            for (int m = 0; m < 8; ++m) yacc[m] = fmaf(s, d[m], yacc[m]);
        };
        // Software pipeline across groups: group gi's TMEM store is waited for
        // (and gi released to the MMA thread) at the start of iteration gi + 1,
        // and the accumulator read of group gi - kTcDBufs is issued before the
        // dequantisation and waited for after it, so neither TMEM round trip
        // stalls the thread.
        // Every thread arrives and every thread polls: measured faster here
        // than one elected lane per warp with a warp barrier.
        auto release = [&](int h) {
            tc_wait_st();
            fence_proxy_async_smem();
            tc_fence_before();
            mbar_arrive(b_afull + 8 * (h % kTcABufs));
        };
        auto wait_commit = [&](int h) -> bool {
            return mbar_wait_bounded(b_afree + 8 * (h % kTcABufs), (uint32_t)(h / kTcABufs) & 1u,
                                     g.wait_cycles);
        };
        uint4 xv = load_x(0);
        // scale of group gi - kTcDBufs, loaded one iteration ahead and kept as
        // fp16 until its use, so the load's latency is not paid where it is issued
        __half s_lag = __float2half(0.f);
        int released = 0;   // groups released to the MMA thread
        for (int gi = 0; gi < G; ++gi) {
            const int j = gi % kTcABufs;
            const int lagged = gi - kTcDBufs;
            const uint4 xv_next = gi + 1 < G ? load_x(gi + 1) : make_uint4(0u, 0u, 0u, 0u);
            const __half s_lag_next = lagged + 1 >= 0 ? srow_p[lagged + 1] : __float2half(0.f);
            if (gi >= 1) {
                release(gi - 1);
                released = gi;
            }
            const int use = gi / kTcStageGroups, st = use % kTcStages;
            if ((gi % kTcStageGroups) == 0 &&
                tc_stop(mbar_wait_bounded(b_wfull + 8 * st, (uint32_t)(use / kTcStages) & 1u,
                                        g.wait_cycles),
                        s_fail))
                break;
            // this thread's 32 bytes of the row's group: 16-byte piece p (0..7)
            // of row r sits at piece p ^ (r & 7) (TMA 128-byte swizzle)
            uint32_t wq[8];
            {
                const uint32_t rowp = s_base + st * kTcStageBytes + r * (kTcStageGroups * 64);
                const int p0 = 4 * (gi % kTcStageGroups) + 2 * half;
#pragma unroll
                for (int c = 0; c < 2; ++c) {
                    const uint4 v = lds16(rowp + (((p0 + c) ^ (r & 7)) << 4));
                    wq[4 * c + 0] = v.x;
                    wq[4 * c + 1] = v.y;
                    wq[4 * c + 2] = v.z;
                    wq[4 * c + 3] = v.w;
                }
            }
            // A buffer j and activation tile j are free once the MMAs of
            // group gi - kTcABufs completed (and with them those of every
            // earlier group: a commit tracks all prior MMAs of its thread)
            const bool free_ok = gi < kTcABufs || wait_commit(gi - kTcABufs);
            if (tc_stop(free_ok, s_fail)) break;
            tc_fence_after();
            // group gi - kTcDBufs (complete: gi - kTcABufs is later): read its
            // accumulator now, add it after the dequantisation
            uint32_t dr[8];
            if (lagged >= 0)
                tc_ld8_issue(t_d0 + lane_base + (uint32_t)(kTcN * (lagged % kTcDBufs) + 8 * half),
                             dr);
            // exact dequantisation: word w (k = 8w .. 8w + 7 of this half) ->
            // columns 4w .. 4w + 3 holding (k0, k4) (k1, k5) (k2, k6) (k3, k7)
            uint32_t a[32];
#pragma unroll
            for (int w = 0; w < 8; ++w) {
                const uint32_t hw = wq[w] >> 8;
                a[4 * w + 0] = nib_pair_lo(wq[w]);
                a[4 * w + 1] = nib_pair_hi(wq[w]);
                a[4 * w + 2] = nib_pair_lo(hw);
                a[4 * w + 3] = nib_pair_hi(hw);
            }
            tc_st32(tmem + lane_base + (uint32_t)(64 * j + 32 * half), a);
            // activation tile j: core matrix (k8, n >> 3) of 8 rows x 16 bytes
            // at ((2 k8 + (n >> 3)) * 8 + (n & 7)) * 16, halves in the same
            // (k0, k4) (k1, k5) ... order as A
            {
                uint4 p;
                p.x = prmt_i<0x5410u>(xv.x, xv.z);
                p.y = prmt_i<0x7632u>(xv.x, xv.z);
                p.z = prmt_i<0x5410u>(xv.y, xv.w);
                p.w = prmt_i<0x7632u>(xv.y, xv.w);
                asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(
                                 s_x + j * kTcXBytes + x_off),
                             "r"(p.x), "r"(p.y), "r"(p.z), "r"(p.w)
                             : "memory");
            }
            xv = xv_next;
            // the accumulator of group gi - kTcDBufs is reused by group gi,
            // released to the MMA thread only after this read
            if (lagged >= 0) {
                tc_ld8_wait(dr);
                const float sl = __half2float(s_lag);
#pragma unroll
                for (int m = 0; m < 8; ++m) yacc[m] = fmaf(sl, __uint_as_float(dr[m]), yacc[m]);
            }
            s_lag = s_lag_next;
        }
        // the last group, then the last groups' sums once its MMAs completed
        if (G > 0 && !__any_sync(0xffffffffu, *s_fail != 0)) {
            release(G - 1);
            released = G;
        }
        if (G > 0 && released == G && !__any_sync(0xffffffffu, *s_fail != 0)) {
            if (!tc_stop(wait_commit(G - 1), s_fail)) {
                tc_fence_after();
                for (int h = max(0, G - kTcDBufs); h < G; ++h)
                    drain(h, __half2float(srow_p[h]));
            }
        }
        // no tcgen05.st of this thread may still be in flight when TMEM is freed
        tc_wait_st();
    } else if (mma_thread) {
        // ---------------- MMAs and weight refills ----------------
        int committed = 0;
        for (int gi = 0; gi < G; ++gi) {
            const int j = gi % kTcABufs;
            if (!mbar_wait_bounded(b_afull + 8 * j, (uint32_t)(gi / kTcABufs) & 1u,
                                   g.wait_cycles)) {
                record_status(kStatusTimeoutTc);
                *s_fail = 1;
            }
            if (*s_fail) break;
            tc_fence_after();
            const uint32_t a_t = tmem + (uint32_t)(64 * j);
            const uint32_t d_t = t_d0 + (uint32_t)(kTcN * (gi % kTcDBufs));
            const uint32_t xb = s_x + j * kTcXBytes;
#pragma unroll
            for (int kk = 0; kk < kTcGroupK / 16; ++kk)
                tc_mma(d_t, a_t + 8 * kk, tc_smem_desc(xb + 512 * kk, 256, 128), kk > 0 ? 1u : 0u);
            tc_commit(b_afree + 8 * j);
            committed = gi + 1;
            // the stage of groups gi - 1, gi was read before a_full arrived
            if ((gi % kTcStageGroups) == kTcStageGroups - 1 || gi == G - 1) {
                if (issued < n_stage_uses) request(issued++);
            }
        }
        if (*s_fail) {
            // drain: every requested stage and the last committed MMAs
            // (bounded again; the CTA returns either way)
            for (int q = max(0, issued - kTcStages); q < issued; ++q)
                mbar_wait_bounded(b_wfull + 8 * (q % kTcStages), (uint32_t)(q / kTcStages) & 1u,
                                  g.wait_cycles);
            if (committed > 0)
                mbar_wait_bounded(b_afree + 8 * ((committed - 1) % kTcABufs),
                                  (uint32_t)((committed - 1) / kTcABufs) & 1u, g.wait_cycles);
        }
    }

    // every tcgen05 operation of this CTA has completed: release TMEM before
    // any wait on other CTAs
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                     "r"(kTcTmemCols)
                     : "memory");
    }
    const bool failed = *s_fail != 0;
    const unsigned epoch = kPeer ? *s_epoch : 0u;
    auto store = [&](int64_t r, int m, float v) {
        const __half h = __float2half_rn(v);
        if constexpr (kPeer) {
            const int64_t off = m * g.y_stride + po.row0 + r;
#pragma unroll
            for (int p = 0; p < kMaxPeers; ++p)
                if (p < po.world) ((epoch & 1) ? po.y[1][p] : po.y[0][p])[off] = h;
        } else {
            y[m * g.y_stride + r] = h;
        }
    };
    const int my_row = 32 * quarter + lane;
    if (g.splits == 1) {
        if (warp < kTcRowWarps && !failed && row0 + my_row < g.N) {
#pragma unroll
            for (int m = 0; m < 8; ++m)
                if (8 * half + m < g.M) store(row0 + my_row, 8 * half + m, yacc[m]);
        }
    } else {
        if (warp < kTcRowWarps) {
#pragma unroll
            // [activation row][tile row]: a warp writes, and a split later
            // reads, contiguous runs of one activation row
            for (int m = 0; m < 8; ++m) rsum[(8 * half + m) * kTcRows + my_row] = yacc[m];
        }
        cluster_sync_all();
        // split s finishes activation rows [s * mspan, (s + 1) * mspan) of the
        // tile's rows (sums in split order), eight consecutive tile rows per
        // thread: one 16-byte store per destination where it is aligned, so
        // every rank's buffer receives whole 256-byte runs of a row of Y
        const int64_t left = g.N - row0;
        const int nrows = left < kTcRows ? (int)left : kTcRows;
        const int mspan = (g.M + g.splits - 1) / g.splits;
        const int mlo = min(g.M, split * mspan), mhi = min(g.M, mlo + mspan);
        const int nvec = (nrows + 7) / 8;
        bool any_fail = false;
        const uint32_t fail_addr = smem_u32(const_cast<int*>(s_fail));
        for (int sp = 0; sp < g.splits; ++sp) any_fail |= ld_cluster_u32(fail_addr, sp) != 0u;
        if (!any_fail) {
            // every thread sums (row, activation row) elements over the
            // splits into a staged copy in the weight-stage area (idle now),
            // then eight rows at a time go out
            __half* staged = reinterpret_cast<__half*>(smem);
            for (int idx = tid; idx < (mhi - mlo) * nrows; idx += kTcThreads) {
                const int mm = idx / nrows, rr = idx - mm * nrows;
                float v = 0.f;
                for (int sp = 0; sp < g.splits; ++sp)
                    v += ld_cluster_f32(rsum + (mlo + mm) * kTcRows + rr, sp);
                staged[mm * kTcRows + rr] = __float2half_rn(v);
            }
            __syncthreads();
            for (int idx = tid; idx < (mhi - mlo) * nvec; idx += kTcThreads) {
                const int mm = idx / nvec, r8 = 8 * (idx - mm * nvec);
                const int cnt = min(8, nrows - r8);
                const __half* src = staged + mm * kTcRows + r8;
                const uint4 v8 = *reinterpret_cast<const uint4*>(src);
                auto put = [&](__half* dst) {
                    if (cnt == 8 && (reinterpret_cast<uintptr_t>(dst) & 15u) == 0) {
                        *reinterpret_cast<uint4*>(dst) = v8;
                    } else {
                        for (int i = 0; i < cnt; ++i) dst[i] = src[i];
                    }
                };
                const int m = mlo + mm;
                if constexpr (kPeer) {
                    const int64_t off = m * g.y_stride + po.row0 + row0 + r8;
#pragma unroll
                    for (int p = 0; p < kMaxPeers; ++p)
                        if (p < po.world) put(((epoch & 1) ? po.y[1][p] : po.y[0][p]) + off);
                } else {
                    put(y + m * g.y_stride + row0 + r8);
                }
            }
        }
        // no CTA leaves while the others may still read its row sums
        cluster_sync_all();
    }
    if constexpr (kPeer) {
        __syncthreads();
        if (tid == 0) peer_arrive_and_wait(po, epoch, g.wait_cycles);
    }
}

}  // namespace clb
