// Tensor-core weight-only GEMV / small-batch GEMM for sm_100a (INT4
// group-scaled, INT8 row-scaled, and dense fp16 weights),
// Y[m, n] = sum_k (s * q[n, k]) * X[m, k] for M = 1..16 activation rows.
//
// Why tensor cores at M = 1: on the CUDA cores the exact dequantisation plus
// an fp32 multiply-add costs 4+ issued instructions per weight element
// (measured with ncu), which caps the kernel below the HBM roofline.  Here
// the dequantised fp16 values feed `mma.sync.m16n8k16` (exact fp16 x fp16
// products, fp32 accumulation), so the multiply-adds leave the issue stream
// and the dequantisation (one lop3 + one add.f16x2 per two elements) is
// nearly all that remains.  With M > 1 the same dequantised A fragments are
// reused for every activation row, so the cost per weight barely grows.
//
// Decomposition
//   * Rows form 16-row mma tiles; a row is cut into 64-byte blocks (INT4: one
//     128-wide scale group; INT8: 64 elements) and blocks into chunks of 4.
//   * The grid is (row groups) x (K splits).  A row group is a balanced,
//     contiguous range of tiles; a K split is a contiguous range of chunks.
//     With more than one split, the splits of a row group form a thread-block
//     cluster and their partial row sums are added through distributed
//     shared memory in split order (deterministic).  Splits are used when the
//     row tiles alone cannot fill the GPU or the activations of the whole K
//     range do not fit in shared memory.
//   * An item = (tile, chunk) = 16 rows x 256 bytes.  Warp w processes items
//     w, w+kWarps, ... in (tile, chunk) order.  Lane (g, t) loads its A
//     fragments directly from global memory: 16 bytes of row g and of row g+8
//     per block, which for a warp is 16 rows x 64 contiguous bytes -- whole
//     32-byte sectors, no shared-memory staging.  Two items per warp are in
//     flight (register double buffer, L2 evict-first), the first two issued
//     before waiting on the preceding kernel.
//   * Item partials land in shared memory; tiles are processed in rounds so
//     that the partial buffer is reused, and each round's rows are summed in
//     chunk order (deterministic) and stored.
//
// Batch columns
//   * M = 1 (kNB = 0): INT4 block q of an item is fed through batch column q
//     (the other lanes read a zero region), so the accumulators keep the four
//     groups apart and the group scales are applied once per item.  INT8 uses
//     column 0 and applies the row scale at the very end.
//   * M = 2..16 (kNB = 1 or 2 column blocks of 8): column c of block j is
//     activation row 8j + c.  INT4 blocks get a fresh accumulator that is
//     scaled by the group scale into the item's output; INT8 accumulates all
//     blocks and applies the row scale at the end.
//
// Fragment / k-permutation (m16n8k16, row.col): lane (g, t) holds A rows g and
// g+8 at k-positions {2t, 2t+1, 2t+8, 2t+9}.  The k order inside a step is
// free as long as A and B agree.  INT4: the 16 bytes lane t reads for a block
// are 32 consecutive elements k0..k0+31 (4 words of 8 nibbles); step 2w uses
// nibble pairs (0,4) and (1,5) of word w, step 2w+1 pairs (2,6) and (3,7) --
// exactly what one lop3 yields -- and the activations are staged in shared
// memory in that permuted order.  INT8: step j uses word j, byte pairs (0,1)
// and (2,3), i.e. natural order.  fp16: step s uses words 2s and 2s+1 (the
// weights need no conversion), natural order too.
#pragma once

#include "gemv_common.cuh"

namespace clb {

constexpr int kMmaChunkBlocks = 4;  // 64-byte blocks per item row
constexpr int kMmaMaxM = 16;        // activation rows per launch
constexpr int kMmaMaxSplits = 8;    // portable cluster size

struct MmaGeom {
    int64_t N, K;
    int64_t row_bytes;            // bytes of one weight row
    int64_t x_stride, y_stride;   // elements between activation rows of X / Y
    int32_t blocks;               // 64-byte blocks per row
    int32_t n_kc;                 // chunks per row
    int32_t M;                    // activation rows (1..16)
    int32_t groups;               // row groups; grid = groups * splits
    int32_t tiles_base, tiles_rem;  // tiles per row group (balanced)
    int32_t splits;               // K splits (cluster size when > 1)
    int32_t kc_split;             // chunks per split (the last split may have fewer)
    int32_t seg_chunks;           // chunks per segment (one warp, one partial slot)
    int32_t round_tiles;          // tiles per round of the partial buffer
    int32_t xs_words;             // staged 16-byte words per activation row
    int32_t part_floats;          // partial buffer size
    int32_t max_rows;             // rows of the largest row group
    int32_t early_x;              // x is not written by the preceding kernel
    int32_t free_y;               // y is not accessed by any kernel still in flight
    long long wait_cycles;        // bound of the peer-flag wait (SM cycles)
    const __half* norm_w;         // RMSNorm weight [K] (fused-prologue kernels)
    float norm_eps;
    int32_t norm_units;           // RMSNorm unit sums per row of one split (0: no RMSNorm)
    int32_t wait_first;           // wait for the preceding kernel before any global access
};

constexpr int kZeroRegion = 256;  // bytes of zeros ahead of the staged activations

// Shared memory: [zeros | activations | item partials | INT8 row scales |
// row sums of this split (splits > 1) | RMSNorm unit sums (fused RMSNorm)]
__host__ __device__ inline int mma_xs_off() { return kZeroRegion; }
__host__ __device__ inline int mma_part_off(const MmaGeom& g) {
    return kZeroRegion + g.M * g.xs_words * 16;
}
__host__ __device__ inline int mma_sc_off(const MmaGeom& g) {
    return mma_part_off(g) + g.part_floats * 4;
}
__host__ __device__ inline int mma_rsum_off(const MmaGeom& g) {
    return mma_sc_off(g) + ((g.max_rows * 4 + 15) & ~15);
}
__host__ __device__ inline int mma_unit_off(const MmaGeom& g) {
    return mma_rsum_off(g) + (g.splits > 1 ? g.max_rows * g.M * 4 : 0);
}
__host__ __device__ inline int mma_smem_total(const MmaGeom& g) {
    return mma_unit_off(g) + g.M * g.norm_units * 4;
}

__device__ __forceinline__ void mma_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                          uint32_t a3, uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// The first step of an accumulator chain: d = a b + (+0), the zero taken from
// one loop-invariant register instead of zeroing d before every chain.
__device__ __forceinline__ void mma_16816_z(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                            uint32_t a3, uint32_t b0, uint32_t b1) {
    const float z = 0.f;
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%10,%10,%10,%10};"
        : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(z));
}

__device__ __forceinline__ uint32_t h2_as_u32(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }

// Nibbles 0 and 4 of w as an exact half2 (q0, q4): the lop3 gives
// 1024 + (q + 8) per half (exponent of 1024, unit ulp) and one add with an
// immediate removes the bias ...
__device__ __forceinline__ uint32_t nib_pair_lo(uint32_t w) {
    return h2_as_u32(__hadd2(u32_as_h2(lop3_sel_xor_i<0x000F000Fu, 0x64086408u>(w)),
                             h2_const(kH_m1032)));
}
// ... and nibbles 1 and 5 as (q1, q5): they sit at mantissa bits 4..7, so the
// exponent of 64 (ulp 1/16, i.e. 1 at bit 4) reads them as 64 + (q + 8).
// Neither form needs a constant register besides the lop3 pattern.
__device__ __forceinline__ uint32_t nib_pair_hi(uint32_t w) {
    return h2_as_u32(__hadd2(u32_as_h2(lop3_sel_xor_i<0x00F000F0u, 0x54805480u>(w)),
                             h2_const(kH_m72)));
}

// Formats.  kAcc: independent accumulators per item at M = 1 (block q uses
// accumulator q % kAcc), so kAcc dependent mma chains run side by side.  INT4
// block q only writes batch column q, so adding the accumulators of blocks
// with the same column parity is exact (the other terms are zeros) and the
// result does not depend on kAcc.
struct MmaInt4 {
    static constexpr int kKind = 0;  // layout id for the host geometry
    static constexpr int kKAlign = 128;  // K multiple for whole 64-byte blocks / groups
    static constexpr bool kGroupScale = true;
    static constexpr bool kRowScale = false;
    static constexpr bool kDense = false;
    static constexpr int kBlockWords = 16;  // 16-byte words of activations per block
    static constexpr int kAcc = 4;
    using Scale = __half;
};
struct MmaInt8 {
    static constexpr int kKind = 1;  // layout id for the host geometry
    static constexpr int kKAlign = 64;  // K multiple for whole 64-byte blocks / groups
    static constexpr bool kGroupScale = false;
    static constexpr bool kRowScale = true;
    static constexpr bool kDense = false;
    static constexpr int kBlockWords = 8;
    static constexpr int kAcc = 2;
    using Scale = float;
};
// Dense fp16 weights (no scale): a 64-byte block is 32 halves, lane t of a
// quad holds halves 8t .. 8t+7 of its rows, and mma step s takes halves
// 4s .. 4s+3 as k-slots (2t, 2t+1, 2t+8, 2t+9), so the activations keep
// their natural order.
struct MmaF16 {
    static constexpr int kKind = 2;  // layout id for the host geometry
    static constexpr int kKAlign = 32;  // K multiple for whole 64-byte blocks / groups
    static constexpr bool kGroupScale = false;
    static constexpr bool kRowScale = false;
    static constexpr bool kDense = true;
    static constexpr int kBlockWords = 4;
    static constexpr int kAcc = 2;
    using Scale = float;  // unused
};

// ---- cluster helpers (splits > 1) ----
__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\t"
                 "barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ float ld_cluster_f32(const float* local, uint32_t rank) {
    uint32_t a = smem_u32(local), ra;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(ra) : "r"(a), "r"(rank));
    float v;
    asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(ra) : "memory");
    return v;
}

// ---------------------------------------------------------------------------
// Row-sharded GEMV with the all-gather fused into the epilogue.
//
// Every rank owns a contiguous shard of the rows of W.  Instead of writing its
// y rows locally and running a separate all-gather, the kernel stores its rows
// straight into the y buffer of every rank (peer pointers over NVLink), so
// the exchange overlaps the other CTAs' compute.  Each rank's flag block
// holds: [0, kMaxPeers) the last step each rank has completed writing into
// this rank's buffers, [kTicket] the CTA arrival counter of the running step,
// [kStep] the last step this rank completed.  Per step:
//   0. after the preceding kernel completed, the CTA reads the step number
//      e = flag[kStep] + 1 (so a captured graph replays correctly);
//   1. it stores its rows into y[e & 1] of every rank, syncs, fences at
//      system scope and takes a ticket;
//   2. the CTA holding the last ticket resets the ticket, fences, and writes
//      e into slot [rank] of every rank's flag block (release);
//   3. that CTA waits (bounded) until every slot of its own flag block is at
//      least e (acquire), then records flag[kStep] = e; when the grid
//      completes, y[e & 1] holds all rows.
// A rank can run at most one step ahead of another (step e+1 cannot complete
// before every rank started it, i.e. finished step e), so with two y buffers
// alternating by step parity a buffer is never rewritten while a lagging
// rank still reads it.  Only plain peer loads and stores are used.
// ---------------------------------------------------------------------------
constexpr int kMaxPeers = 8;
constexpr int kFlagWords = 16;  // words per rank's flag block
constexpr int kTicket = kMaxPeers;
constexpr int kStep = kMaxPeers + 1;

struct PeerOut {
    __half* y[2][kMaxPeers];    // y buffers of every rank, by step parity and rank
    unsigned* flag[kMaxPeers];  // flag block of every rank, by rank
    int64_t row0;               // first row of this rank's shard in y
    int rank, world;
};

// Ticket of a CTA: acquire-release at GPU scope (every CTA of the grid is on
// this GPU).
__device__ __forceinline__ unsigned ticket_acq_rel_gpu(unsigned* p) {
    unsigned prev;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(prev) : "l"(p) : "memory");
    return prev;
}

// Called by thread 0 of every CTA after a CTA barrier that follows the CTA's
// peer stores.  The ticket is a release at GPU scope (through the barrier it
// covers the whole CTA's stores) and, for the last CTA, an acquire of every
// other CTA's release; the last CTA's system-scope fence and the strong flag
// stores after it (a release pattern: one fence for all peers, not one per
// peer as st.release would imply) then order all of them before each peer's
// acquire of its flag: causality order is transitive across the two scopes,
// so one system fence per step replaces one per CTA.  Loops run over the
// compile-time peer slots so that `po` stays in the parameter space (no
// local copy).
__device__ __forceinline__ void peer_arrive_and_wait(const PeerOut& po, unsigned epoch,
                                                     long long budget) {
    unsigned* mine = po.flag[po.rank];
    const unsigned prev = ticket_acq_rel_gpu(mine + kTicket);
    if (prev != gridDim.x - 1) return;
    atomicExch(mine + kTicket, 0u);
    __threadfence_system();
#pragma unroll
    for (int p = 0; p < kMaxPeers; ++p)
        if (p < po.world) st_relaxed_sys(po.flag[p] + po.rank, epoch);
    const long long t0 = clock64();
    bool ok = true;
    for (int q = 0; q < po.world && ok; ++q) {
        while ((int)(ld_acquire_sys(mine + q) - epoch) < 0) {
            if (clock64() - t0 > budget) {
                record_status(kStatusTimeoutPeer);
                ok = false;
                break;
            }
            __nanosleep(64);
        }
    }
    atomicExch(mine + kStep, epoch);
}

// ---------------------------------------------------------------------------
// Items.
// ---------------------------------------------------------------------------

// One item = 16 rows x up to 4 blocks: the fragments (rows g, g+8) and the
// INT4 group scales of those rows, two per word (block 2i in the low half of
// word i).  M = 1 uses word 0 only: the scales of the two blocks (columns)
// the lane holds; M > 1 all four blocks' scales.
struct MmaItemRegs {
    uint4 wa[kMmaChunkBlocks], wb[kMmaChunkBlocks];
    uint32_t sa[2], sb[2];
};

__device__ __forceinline__ float scale_at(const uint32_t (&s)[2], int q) {
    const uint32_t w = s[q >> 1];
    return __half2float(__ushort_as_half((unsigned short)((q & 1) ? (w >> 16) : (w & 0xFFFFu))));
}

__device__ __forceinline__ uint32_t pack_halves(__half lo, __half hi) {
    return (uint32_t)__half_as_ushort(lo) | ((uint32_t)__half_as_ushort(hi) << 16);
}

// Where one item's loads start, as 64-byte block indices into W (and group
// indices into the INT4 scales, the same numbers) of rows a = g and b = g + 8,
// and the item's first block within the row.  Consecutive chunks of a row are
// 4 blocks apart, so walking a segment only steps the indices.  Rows beyond
// the group re-read its last row (L2 hit; their results are never stored),
// so no load is predicated.  The launch keeps N * blocks below 2^32.
struct MmaFetchPtr {
    uint32_t ea, eb;
    int blk0;
};

__device__ __forceinline__ MmaFetchPtr mma_fetch_ptr(const MmaGeom& g, int64_t r0, int nrows,
                                                     int kc0, int tile, int kc, int gq) {
    const int last = nrows - 1;
    const int64_t ra = r0 + min(16 * tile + gq, last);
    const int64_t rb = r0 + min(16 * tile + gq + 8, last);
    MmaFetchPtr p;
    p.blk0 = kMmaChunkBlocks * (kc0 + kc);
    p.ea = (uint32_t)(ra * g.blocks + p.blk0);
    p.eb = (uint32_t)(rb * g.blocks + p.blk0);
    return p;
}

__device__ __forceinline__ void mma_fetch_step(MmaFetchPtr& p) {
    p.ea += kMmaChunkBlocks;
    p.eb += kMmaChunkBlocks;
    p.blk0 += kMmaChunkBlocks;
}

// Issue the loads of one item in a matrix whose rows are whole chunks (row
// bytes a multiple of 256) with 8-byte aligned scale rows.  wl = W + 16 t (the
// lane's 16 bytes of a block); sl = the INT4 scales, advanced by 2 (t & 1) at
// M = 1 (the lane's first block).  The scales come as one 4-byte (M = 1) or
// 8-byte (M > 1) load per row.
template <class Fmt, int kNB>
__device__ __forceinline__ void mma_fetch(MmaItemRegs& r, const MmaFetchPtr& p,
                                          const uint8_t* wl, const __half* sl, uint64_t pol) {
    const uint8_t* pa = wl + 64 * (size_t)p.ea;
    const uint8_t* pb = wl + 64 * (size_t)p.eb;
#pragma unroll
    for (int q = 0; q < kMmaChunkBlocks; ++q) {
        r.wa[q] = ldg_stream16(pa + 64 * q, pol);
        r.wb[q] = ldg_stream16(pb + 64 * q, pol);
    }
    if constexpr (Fmt::kGroupScale) {
        const __half* sa = sl + p.ea;
        const __half* sb = sl + p.eb;
        if constexpr (kNB == 0) {
            r.sa[0] = __ldg(reinterpret_cast<const unsigned int*>(sa));
            r.sb[0] = __ldg(reinterpret_cast<const unsigned int*>(sb));
        } else {
            const uint2 va = __ldg(reinterpret_cast<const uint2*>(sa));
            const uint2 vb = __ldg(reinterpret_cast<const uint2*>(sb));
            r.sa[0] = va.x;
            r.sa[1] = va.y;
            r.sb[0] = vb.x;
            r.sb[1] = vb.y;
        }
    }
}

// Issue the loads of one item (tile, chunk kc of the split) in a matrix with a
// short last chunk per row: blocks past the row end re-read the row's last
// block (the staged activations are zero there, so they add exact zeros).
// Rows beyond the group re-read its last row.
template <class Fmt, int kNB>
__device__ __forceinline__ void mma_fetch_ragged(MmaItemRegs& r, const uint8_t* W,
                                                 const typename Fmt::Scale* scale,
                                                 const MmaGeom& g, int64_t r0, int nrows, int kc0,
                                                 int tile, int kc, int gq, int t, uint64_t pol) {
    const int last = nrows - 1;
    const int64_t ra = r0 + min(16 * tile + gq, last);
    const int64_t rb = r0 + min(16 * tile + gq + 8, last);
    const int blk0 = kMmaChunkBlocks * (kc0 + kc);
    const uint8_t* pa = W + ra * g.row_bytes + 16 * t;
    const uint8_t* pb = W + rb * g.row_bytes + 16 * t;
#pragma unroll
    for (int q = 0; q < kMmaChunkBlocks; ++q) {
        const int blk = min(blk0 + q, g.blocks - 1);
        r.wa[q] = ldg_stream16(pa + 64 * blk, pol);
        r.wb[q] = ldg_stream16(pb + 64 * blk, pol);
    }
    if constexpr (Fmt::kGroupScale) {
        const __half* sa = reinterpret_cast<const __half*>(scale) + ra * g.blocks;
        const __half* sb = reinterpret_cast<const __half*>(scale) + rb * g.blocks;
        if constexpr (kNB == 0) {
            // lane (g, t) needs the scales of blocks 2(t&1), 2(t&1)+1 of rows g, g+8
            const int b0 = min(blk0 + 2 * (t & 1), g.blocks - 1);
            const int b1 = min(blk0 + 2 * (t & 1) + 1, g.blocks - 1);
            r.sa[0] = pack_halves(sa[b0], sa[b1]);
            r.sb[0] = pack_halves(sb[b0], sb[b1]);
        } else {
            int blk[kMmaChunkBlocks];
#pragma unroll
            for (int q = 0; q < kMmaChunkBlocks; ++q) blk[q] = min(blk0 + q, g.blocks - 1);
            r.sa[0] = pack_halves(sa[blk[0]], sa[blk[1]]);
            r.sa[1] = pack_halves(sa[blk[2]], sa[blk[3]]);
            r.sb[0] = pack_halves(sb[blk[0]], sb[blk[1]]);
            r.sb[1] = pack_halves(sb[blk[2]], sb[blk[3]]);
        }
    }
}

// Running sums of one segment (consecutive chunks of one tile, computed by one
// warp).  M = 1: v[0][0] / v[0][1] = rows g / g + 8 of this lane's columns;
// M > 1: rows g, g+8 x columns 8j + 2t, 8j + 2t + 1 (mma accumulator layout).
template <int kNB>
struct MmaAcc {
    float v[kNB == 0 ? 1 : kNB][4];
};

template <int kNB>
__device__ __forceinline__ void mma_acc_zero(MmaAcc<kNB>& a) {
#pragma unroll
    for (int j = 0; j < (kNB == 0 ? 1 : kNB); ++j) a.v[j][0] = a.v[j][1] = a.v[j][2] = a.v[j][3] = 0.f;
}

// Store a finished segment's sums into slot `slot` of the partial buffer
// (16 rows x max(M, 1) floats, row-major) and reset them.
template <class Fmt, int kNB>
__device__ __forceinline__ void mma_flush(MmaAcc<kNB>& acc, const MmaGeom& g, int gq, int t,
                                          float* part, int slot) {
    if constexpr (kNB == 0) {
        float a = acc.v[0][0], b = acc.v[0][1];
        if constexpr (Fmt::kGroupScale) {
            // lane t < 2 holds the scaled sums of columns (blocks) 2t, 2t + 1;
            // lanes t >= 2 hold the zero columns
            if (t >= 2) a = b = 0.f;
            a += __shfl_xor_sync(0xffffffffu, a, 1);
            b += __shfl_xor_sync(0xffffffffu, b, 1);
        }
        if (t == 0) {
            float* pp = part + slot * 16;
            pp[gq] = a;
            pp[gq + 8] = b;
        }
    } else {
        float* pp = part + slot * 16 * g.M;
#pragma unroll
        for (int j = 0; j < kNB; ++j) {
            const int c = 8 * j + 2 * t;
            if (c < g.M) {
                pp[gq * g.M + c] = acc.v[j][0];
                pp[(gq + 8) * g.M + c] = acc.v[j][2];
            }
            if (c + 1 < g.M) {
                pp[gq * g.M + c + 1] = acc.v[j][1];
                pp[(gq + 8) * g.M + c + 1] = acc.v[j][3];
            }
        }
    }
    mma_acc_zero<kNB>(acc);
}

// Compute one item and add it to the segment's sums.
//   xs: staged activations of this split (row m at xs + m * xs_words), zero
//       past the row end, so the blocks a short last chunk re-reads add
//       exact zeros;
//   lb0: the item's first block relative to the split.
template <class Fmt, int kNB>
__device__ __forceinline__ void mma_item(const MmaItemRegs& r, const uint4* xs, const uint4* zero,
                                         int lb0, const MmaGeom& g, int gq, int t,
                                         MmaAcc<kNB>& sacc) {
    constexpr int kBlk = Fmt::kBlockWords;
    if constexpr (kNB == 0 && Fmt::kGroupScale) {
        // INT4, one activation row.  Block q goes through its own accumulator
        // and only column q of it is read; columns are independent dot
        // products, so the other columns may hold anything.  Lane (g, t)
        // therefore supplies block g & 3's activations for every block: one
        // set of four 16-byte loads per item, no zero region.  The staged
        // layout is [chunk][word w][block][lane t] (16 bytes each), so the 16
        // distinct entries a warp reads for one w are 256 contiguous bytes.
        static_assert(Fmt::kAcc == kMmaChunkBlocks, "one accumulator per block");
        const uint4* xb = xs + (lb0 >> 2) * 64 + (gq & 3) * 4 + t;
        float acc[kMmaChunkBlocks][4];
#pragma unroll
        for (int w = 0; w < 4; ++w) {
            const uint4 bb = xb[16 * w];  // (x0,x4) (x1,x5) (x2,x6) (x3,x7) of word w
#pragma unroll
            for (int q = 0; q < kMmaChunkBlocks; ++q) {
                const uint32_t ua = w == 0 ? r.wa[q].x : w == 1 ? r.wa[q].y
                                                     : w == 2 ? r.wa[q].z : r.wa[q].w;
                const uint32_t ub = w == 0 ? r.wb[q].x : w == 1 ? r.wb[q].y
                                                     : w == 2 ? r.wb[q].z : r.wb[q].w;
                const uint32_t ha = ua >> 8, hb = ub >> 8;
                if (w == 0)
                    mma_16816_z(acc[q], nib_pair_lo(ua), nib_pair_lo(ub), nib_pair_hi(ua),
                                nib_pair_hi(ub), bb.x, bb.y);
                else
                    mma_16816(acc[q], nib_pair_lo(ua), nib_pair_lo(ub), nib_pair_hi(ua),
                              nib_pair_hi(ub), bb.x, bb.y);
                mma_16816(acc[q], nib_pair_lo(ha), nib_pair_lo(hb), nib_pair_hi(ha),
                          nib_pair_hi(hb), bb.z, bb.w);
            }
        }
        // lane t < 2 holds columns 2t, 2t + 1: blocks 0 / 1 (t = 0) or 2 / 3
        // (t = 1).  (These are the values the zero-column form summed with
        // exact zeros; the segment sum below starts from +0, so the results
        // are the same bits.)
        const bool odd = (t & 1) != 0;
        const float e0 = odd ? acc[2][0] : acc[0][0];
        const float e1 = odd ? acc[3][1] : acc[1][1];
        const float e2 = odd ? acc[2][2] : acc[0][2];
        const float e3 = odd ? acc[3][3] : acc[1][3];
        const float sa0 = scale_at(r.sa, 0), sa1 = scale_at(r.sa, 1);
        const float sb0 = scale_at(r.sb, 0), sb1 = scale_at(r.sb, 1);
        sacc.v[0][0] += fmaf(sa1, e1, sa0 * e0);
        sacc.v[0][1] += fmaf(sb1, e3, sb0 * e2);
    } else if constexpr (kNB == 0) {
        float acc[Fmt::kAcc][4];
#pragma unroll
        for (int i = 0; i < Fmt::kAcc; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
#pragma unroll
        for (int q = 0; q < kMmaChunkBlocks; ++q) {
            const int col = Fmt::kGroupScale ? q : 0;
            const uint4* bp = gq == col ? xs + (lb0 + q) * kBlk : zero;
            const uint32_t ua[4] = {r.wa[q].x, r.wa[q].y, r.wa[q].z, r.wa[q].w};
            const uint32_t ub[4] = {r.wb[q].x, r.wb[q].y, r.wb[q].z, r.wb[q].w};
            if constexpr (Fmt::kGroupScale) {
#pragma unroll
                for (int w = 0; w < 4; ++w) {
                    const uint4 bb = bp[w * 4 + t];  // (x0,x4) (x1,x5) (x2,x6) (x3,x7)
                    const uint32_t ha = ua[w] >> 8, hb = ub[w] >> 8;
                    mma_16816(acc[q % Fmt::kAcc], nib_pair_lo(ua[w]), nib_pair_lo(ub[w]),
                              nib_pair_hi(ua[w]), nib_pair_hi(ub[w]), bb.x, bb.y);
                    mma_16816(acc[q % Fmt::kAcc], nib_pair_lo(ha), nib_pair_lo(hb),
                              nib_pair_hi(ha), nib_pair_hi(hb), bb.z, bb.w);
                }
            } else if constexpr (Fmt::kDense) {
                const uint4 bb = bp[t];  // x[8t .. 8t + 8) of the block
                mma_16816(acc[q % Fmt::kAcc], ua[0], ub[0], ua[1], ub[1], bb.x, bb.y);
                mma_16816(acc[q % Fmt::kAcc], ua[2], ub[2], ua[3], ub[3], bb.z, bb.w);
            } else {
#pragma unroll
                for (int jj = 0; jj < 2; ++jj) {
                    const uint4 bb = bp[2 * t + jj];  // x[16t + 8jj .. +8)
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        __half2 qa[2], qb[2];
                        int8x4_to_h2(ua[2 * jj + h], qa);
                        int8x4_to_h2(ub[2 * jj + h], qb);
                        mma_16816(acc[q % Fmt::kAcc], h2_as_u32(qa[0]), h2_as_u32(qb[0]),
                                  h2_as_u32(qa[1]), h2_as_u32(qb[1]), h ? bb.z : bb.x,
                                  h ? bb.w : bb.y);
                    }
                }
            }
        }
        if constexpr (Fmt::kGroupScale) {
            // lane t < 2 holds columns (blocks) 2t (even accumulators, entries
            // 0 / 2) and 2t + 1 (odd accumulators, entries 1 / 3)
            static_assert(Fmt::kAcc % 2 == 0, "column parity per accumulator");
            float e0 = acc[0][0], e2 = acc[0][2], e1 = acc[1][1], e3 = acc[1][3];
#pragma unroll
            for (int i = 2; i < Fmt::kAcc; i += 2) {
                e0 += acc[i][0];
                e2 += acc[i][2];
                e1 += acc[i + 1][1];
                e3 += acc[i + 1][3];
            }
            const float sa0 = scale_at(r.sa, 0), sa1 = scale_at(r.sa, 1);
            const float sb0 = scale_at(r.sb, 0), sb1 = scale_at(r.sb, 1);
            sacc.v[0][0] += fmaf(sa1, e1, sa0 * e0);
            sacc.v[0][1] += fmaf(sb1, e3, sb0 * e2);
        } else {
            static_assert(Fmt::kAcc == 2, "INT8 / fp16 sum their two accumulators");
            sacc.v[0][0] += acc[0][0] + acc[1][0];
            sacc.v[0][1] += acc[0][2] + acc[1][2];
        }
    } else {
        // column c of column block j is activation row 8j + c
        const uint4* bp[kNB];
#pragma unroll
        for (int j = 0; j < kNB; ++j)
            bp[j] = 8 * j + gq < g.M ? xs + (8 * j + gq) * g.xs_words : nullptr;
        float (&out)[kNB][4] = sacc.v;
#pragma unroll
        for (int q = 0; q < kMmaChunkBlocks; ++q) {
            const uint4* bq[kNB];
#pragma unroll
            for (int j = 0; j < kNB; ++j) bq[j] = bp[j] ? bp[j] + (lb0 + q) * kBlk : zero;
            const uint32_t ua[4] = {r.wa[q].x, r.wa[q].y, r.wa[q].z, r.wa[q].w};
            const uint32_t ub[4] = {r.wb[q].x, r.wb[q].y, r.wb[q].z, r.wb[q].w};
            if constexpr (Fmt::kGroupScale) {
                float bacc[kNB][4];
#pragma unroll
                for (int w = 0; w < 4; ++w) {
                    uint4 bb[kNB];
#pragma unroll
                    for (int j = 0; j < kNB; ++j) bb[j] = bq[j][w * 4 + t];
                    const uint32_t a0 = nib_pair_lo(ua[w]), a1 = nib_pair_lo(ub[w]);
                    const uint32_t a2 = nib_pair_hi(ua[w]), a3 = nib_pair_hi(ub[w]);
#pragma unroll
                    for (int j = 0; j < kNB; ++j) {
                        if (w == 0)
                            mma_16816_z(bacc[j], a0, a1, a2, a3, bb[j].x, bb[j].y);
                        else
                            mma_16816(bacc[j], a0, a1, a2, a3, bb[j].x, bb[j].y);
                    }
                    const uint32_t ha = ua[w] >> 8, hb = ub[w] >> 8;
                    const uint32_t c0 = nib_pair_lo(ha), c1 = nib_pair_lo(hb);
                    const uint32_t c2 = nib_pair_hi(ha), c3 = nib_pair_hi(hb);
#pragma unroll
                    for (int j = 0; j < kNB; ++j)
                        mma_16816(bacc[j], c0, c1, c2, c3, bb[j].z, bb[j].w);
                }
                const float sa = scale_at(r.sa, q), sb = scale_at(r.sb, q);
#pragma unroll
                for (int j = 0; j < kNB; ++j) {
                    out[j][0] = fmaf(sa, bacc[j][0], out[j][0]);
                    out[j][1] = fmaf(sa, bacc[j][1], out[j][1]);
                    out[j][2] = fmaf(sb, bacc[j][2], out[j][2]);
                    out[j][3] = fmaf(sb, bacc[j][3], out[j][3]);
                }
            } else if constexpr (Fmt::kDense) {
                uint4 bb[kNB];
#pragma unroll
                for (int j = 0; j < kNB; ++j) bb[j] = bq[j][t];
#pragma unroll
                for (int j = 0; j < kNB; ++j) {
                    mma_16816(out[j], ua[0], ub[0], ua[1], ub[1], bb[j].x, bb[j].y);
                    mma_16816(out[j], ua[2], ub[2], ua[3], ub[3], bb[j].z, bb[j].w);
                }
            } else {
#pragma unroll
                for (int jj = 0; jj < 2; ++jj) {
                    uint4 bb[kNB];
#pragma unroll
                    for (int j = 0; j < kNB; ++j) bb[j] = bq[j][2 * t + jj];
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        __half2 qa[2], qb[2];
                        int8x4_to_h2(ua[2 * jj + h], qa);
                        int8x4_to_h2(ub[2 * jj + h], qb);
#pragma unroll
                        for (int j = 0; j < kNB; ++j)
                            mma_16816(out[j], h2_as_u32(qa[0]), h2_as_u32(qb[0]),
                                      h2_as_u32(qa[1]), h2_as_u32(qb[1]),
                                      h ? bb[j].z : bb[j].x, h ? bb[j].w : bb[j].y);
                    }
                }
            }
        }
    }
}

// A warp's position: segment (tile, seg) and chunk j inside it.  Segments of
// a CTA are dealt to its warps round-robin in (tile, seg) order; a segment is
// G consecutive chunks of one tile (fewer for the last one).
struct MmaSegCursor {
    int tile, seg, j;
};

__device__ __forceinline__ int seg_len(int seg, int G, int n_kc) { return min(G, n_kc - seg * G); }

__device__ __forceinline__ void seg_normalize(MmaSegCursor& c, int n_seg) {
    while (c.seg >= n_seg) {
        c.seg -= n_seg;
        ++c.tile;
    }
}

// ---------------------------------------------------------------------------
// RMSNorm of activation rows (the fused prologue and the standalone kernel).
//
// Formula of the reference (cudalab/reference.py:41-45, kernels/rmsnorm/
// rmsnorm_v4.cu:84-108): v = mean(x^2) in fp32, r = 1 / sqrt(v + eps),
// y = fp16((x * r) * w), each product rounded to fp32.  r is taken correctly
// rounded here (the reference's rsqrtf is within 2 ulp of it).
//
// The fp32 sum of squares has one fixed order, shared by the fused kernel
// (whatever its geometry and K split) and the standalone kernel, so both
// produce the same r bit for bit:
//   word partial  the 8 squares of a 16-byte word: even and odd elements in
//                 two fp32 lanes (fma, element order), then even + odd;
//   unit sum      the 32 word partials of a unit (256 halves starting at a
//                 multiple of 256) added by an xor butterfly (16, 8, 4, 2, 1);
//   row sum       lane l of a warp adds units l, l + 32, ... in order, then an
//                 xor butterfly over the 32 lanes.
// Words past the row end count as zeros (adding +0 changes no bits).  A unit
// is what one warp of the staging loop holds at once, so the fused kernel
// takes the unit sums from the words it stages, and a K split exchanges them
// through distributed shared memory.
// ---------------------------------------------------------------------------
constexpr int kNormUnitWords = 32;  // 16-byte words per unit
constexpr int kNormUnitHalves = 8 * kNormUnitWords;

__device__ __forceinline__ unsigned long long f2_bits(float2 v) {
    return ((unsigned long long)__float_as_uint(v.y) << 32) | __float_as_uint(v.x);
}
__device__ __forceinline__ float2 bits_f2(unsigned long long b) {
    return make_float2(__uint_as_float((uint32_t)b), __uint_as_float((uint32_t)(b >> 32)));
}
__device__ __forceinline__ unsigned long long h2_f2_bits(uint32_t h) {
    return f2_bits(__half22float2(*reinterpret_cast<const __half2*>(&h)));
}

// Word partial of a 16-byte word of halves.
__device__ __forceinline__ float sq_word(const uint4& v) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
    unsigned long long acc = 0ull;  // (+0, +0)
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const unsigned long long f = h2_f2_bits(w[i]);
        asm("fma.rn.f32x2 %0, %1, %1, %0;" : "+l"(acc) : "l"(f));
    }
    const float2 a = bits_f2(acc);
    return a.x + a.y;
}

__device__ __forceinline__ float warp_xor_sum(float v) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
    return v;
}

__device__ __forceinline__ float inv_rms(float sum_sq, int64_t K, float eps) {
    return __frsqrt_rn(__fdiv_rn(sum_sq, (float)K) + eps);
}

// Unit sums of one row of K halves (16-byte aligned) into s_unit[0 ..
// ceil(K / 256)), by a block of kWarps warps: warp w takes units w, w + kWarps,
// ..., four at a time (loads first, then the four butterflies interleaved).
template <int kWarps>
__device__ __forceinline__ void row_unit_sums(const __half* __restrict__ row, int64_t K,
                                              float* s_unit) {
    constexpr int kBatch = 4;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t words = K / 8;
    const int n_units = (int)((K + kNormUnitHalves - 1) / kNormUnitHalves);
    const uint4* p = reinterpret_cast<const uint4*>(row);
    for (int u0 = warp; u0 < n_units; u0 += kWarps * kBatch) {
        uint4 v[kBatch];
#pragma unroll
        for (int b = 0; b < kBatch; ++b) {
            const int64_t q = (int64_t)(u0 + b * kWarps) * kNormUnitWords + lane;
            v[b] = q < words ? __ldg(p + q) : make_uint4(0u, 0u, 0u, 0u);
        }
        float su[kBatch];
#pragma unroll
        for (int b = 0; b < kBatch; ++b) su[b] = sq_word(v[b]);
#pragma unroll
        for (int off = 16; off > 0; off >>= 1)
#pragma unroll
            for (int b = 0; b < kBatch; ++b) su[b] += __shfl_xor_sync(0xffffffffu, su[b], off);
        if (lane == 0) {
#pragma unroll
            for (int b = 0; b < kBatch; ++b)
                if (u0 + b * kWarps < n_units) s_unit[u0 + b * kWarps] = su[b];
        }
    }
}

// Row sum from its unit sums (one warp; every lane returns it).
__device__ __forceinline__ float row_sum_of_units(const float* s_unit, int n_units, int lane) {
    float s = 0.f;
    for (int u = lane; u < n_units; u += 32) s += s_unit[u];
    return warp_xor_sum(s);
}

// fp16((x * r) * w) of the 8 halves of one 16-byte word: both products
// rounded to fp32 (packed multiplies, one rounding per element), then to
// fp16.  Elementwise, so x and w may be permuted alike.
__device__ __forceinline__ uint4 norm_word(const uint4& xv, const uint4& wv, float r) {
    const uint32_t xi[4] = {xv.x, xv.y, xv.z, xv.w};
    const uint32_t wi[4] = {wv.x, wv.y, wv.z, wv.w};
    const unsigned long long rr = f2_bits(make_float2(r, r));
    uint32_t o[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        unsigned long long t;
        asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(t) : "l"(h2_f2_bits(xi[i])), "l"(rr));
        asm("mul.rn.f32x2 %0, %0, %1;" : "+l"(t) : "l"(h2_f2_bits(wi[i])));
        const float2 p = bits_f2(t);
        o[i] = h2_as_u32(__floats2half2_rn(p.x, p.y));
    }
    return make_uint4(o[0], o[1], o[2], o[3]);
}

// ---------------------------------------------------------------------------
// The kernel.
// ---------------------------------------------------------------------------

// kNB <= 1 (M <= 8): 16 / kWarps CTAs fit on an SM (room for the next
// kernels' CTAs under programmatic dependent launch).  kNB = 2: one CTA per
// SM (more registers for the second column block).
// kPeer: y is ignored; rows go to every rank's buffer in `po` (see PeerOut).
// kNorm: the activation rows are RMSNorm'ed (g.norm_w, g.norm_eps) as they
// are staged.
template <class Fmt, int kWarps, int kNB, bool kAllFull, bool kPeer, bool kNorm = false>
__global__ void __launch_bounds__(32 * kWarps, kNB <= 1 ? 16 / kWarps : 1)
gemv_mma_kernel(const uint8_t* __restrict__ W, const typename Fmt::Scale* __restrict__ scale,
                const __half* __restrict__ x, __half* __restrict__ y, const MmaGeom g,
                const PeerOut po) {
    constexpr int kThreads = 32 * kWarps;
    extern __shared__ __align__(128) uint8_t smem[];
    uint4* xs4 = reinterpret_cast<uint4*>(smem + mma_xs_off());
    float* part = reinterpret_cast<float*>(smem + mma_part_off(g));
    float* sc8 = reinterpret_cast<float*>(smem + mma_sc_off(g));
    float* rsum = reinterpret_cast<float*>(smem + mma_rsum_off(g));
    __shared__ unsigned s_epoch;

    // ---- this CTA's rows and K range ----
    const int split = g.splits > 1 ? (int)cluster_rank() : 0;
    const int grp = blockIdx.x / g.splits;
    const int n_tiles = g.tiles_base + (grp < g.tiles_rem ? 1 : 0);
    const int64_t r0 =
        16 * ((int64_t)grp * g.tiles_base + (grp < g.tiles_rem ? grp : g.tiles_rem));
    const int64_t left = g.N - r0;
    const int nrows = left < 16 * n_tiles ? (int)left : 16 * n_tiles;
    const int kc0 = split * g.kc_split;
    const int n_kc = min(g.kc_split, g.n_kc - kc0);
    const int lblocks = min(kMmaChunkBlocks * (kc0 + n_kc), g.blocks) - kMmaChunkBlocks * kc0;
    const int M = kNB == 0 ? 1 : g.M;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int gq = lane >> 2, t = lane & 3;
    const uint64_t pol = policy_evict_first();

    pdl_allow_dependents();
    // Without the caller's CL_LAUNCH_PDL the launch still overlaps the
    // preceding kernel's tail, but touches no global memory before that
    // kernel has completed: the result is that of stream order.
    if (g.wait_first) pdl_wait_prior_grids();
    // Segments of this warp: w, w + kWarps, ... in (tile, seg) order, each
    // walked chunk by chunk.  Weights and scales never depend on the preceding
    // kernel: the first two items are requested before waiting on it.
    // `f` / `fp`: the next item to fetch and where its loads start; the item
    // in a register buffer is computed two items after it was fetched.
    // M = 1 has one chunk per segment (known at compile time).
    const int G = kNB == 0 ? 1 : g.seg_chunks;
    const int n_seg = (n_kc + G - 1) / G;
    auto seg_last = [&](const MmaSegCursor& c) {
        return kNB == 0 || c.j + 1 == seg_len(c.seg, G, n_kc);
    };
    MmaSegCursor f{0, warp, 0};
    seg_normalize(f, n_seg);
    const uint8_t* wl = W + 16 * t;
    const __half* sl =
        reinterpret_cast<const __half*>(scale) + (kNB == 0 && Fmt::kGroupScale ? 2 * (t & 1) : 0);
    MmaFetchPtr fp{};
    if (kAllFull && f.tile < n_tiles) fp = mma_fetch_ptr(g, r0, nrows, kc0, f.tile, f.seg * G, gq);
    // fetch item f, then step to the warp's next item (a new segment: the
    // indices are recomputed)
    auto fetch_next = [&](MmaItemRegs& r) {
        if constexpr (kAllFull) {
            mma_fetch<Fmt, kNB>(r, fp, wl, sl, pol);
        } else {
            mma_fetch_ragged<Fmt, kNB>(r, W, scale, g, r0, nrows, kc0, f.tile, f.seg * G + f.j, gq,
                                       t, pol);
        }
        if (!seg_last(f)) {
            ++f.j;
            if constexpr (kAllFull) mma_fetch_step(fp);
            return;
        }
        f.j = 0;
        const int tile = f.tile;
        f.seg += kWarps;
        seg_normalize(f, n_seg);
        if constexpr (kAllFull) {
            if (f.tile == tile) {  // same rows: step the indices
                const int d = kMmaChunkBlocks * (kc0 + f.seg * G) - fp.blk0;
                fp.ea += d;
                fp.eb += d;
                fp.blk0 += d;
            } else if (f.tile < n_tiles) {
                fp = mma_fetch_ptr(g, r0, nrows, kc0, f.tile, f.seg * G, gq);
            }
        }
    };
    MmaItemRegs ra, rb;
    MmaSegCursor ca = f;
    if (f.tile < n_tiles) fetch_next(ra);
    MmaSegCursor cb = f;
    if (f.tile < n_tiles) fetch_next(rb);
    if constexpr (Fmt::kRowScale) {
        for (int r = tid; r < nrows; r += kThreads)
            sc8[r] = reinterpret_cast<const float*>(scale)[r0 + r];
    }
    if (tid < kZeroRegion / 4) reinterpret_cast<uint32_t*>(smem)[tid] = 0u;

    // Activations of this split: INT4 in the permuted step order, INT8 as is,
    // zeros from the row end to the end of the last chunk.
    const int valid = lblocks * Fmt::kBlockWords;
    const int words = n_kc * kMmaChunkBlocks * Fmt::kBlockWords;
    const int64_t k_first = (int64_t)kMmaChunkBlocks * kc0 * Fmt::kBlockWords * 8;
    // word q of a row: its place in the staged row, and its halves in that order
    auto stage_at = [&](int qq) -> int {
        if constexpr (Fmt::kGroupScale) {
            const int blk = qq >> 4, tt = (qq >> 2) & 3, w = qq & 3;
            if constexpr (kNB == 0)  // [chunk][w][block in chunk][lane] (mma_item)
                return (blk >> 2) * 64 + w * 16 + (blk & 3) * 4 + tt;
            else
                return (blk * 4 + w) * 4 + tt;
        } else {
            return qq;
        }
    };
    auto stage_order = [&](const uint4& v) -> uint4 {
        if constexpr (Fmt::kGroupScale) {
            // entry (blk, w, tt): step 2w (x0, x4, x1, x5), step 2w+1 (x2, x6, x3, x7)
            uint4 e;
            e.x = prmt_i<0x5410u>(v.x, v.z);
            e.y = prmt_i<0x7632u>(v.x, v.z);
            e.z = prmt_i<0x5410u>(v.y, v.w);
            e.w = prmt_i<0x7632u>(v.y, v.w);
            return e;
        } else {
            return v;
        }
    };
    // Fused RMSNorm.  One activation row (kNB = 0): the row's unit sums are
    // taken first, straight from global memory, and the staging loop then
    // normalises in registers (the norm weight words loaded beside x).
    // Several rows: the staging loop takes the unit sums of the words it
    // holds (the 32 lanes of a warp hold one unit of one row at a time: words
    // is a multiple of 32), a K split exchanges them through distributed
    // shared memory, and a pass over the staged words normalises them in
    // place, walking words q = tid, tid + kThreads, ... of the norm weight
    // (kNormBatch loads in flight) and applying each to every row.  The norm
    // weight, like W, is never written by the preceding kernel.
    constexpr bool kNormRow = kNorm && kNB == 0;
    constexpr bool kNormRows = kNorm && kNB != 0;
    constexpr int kNormBatch = !kNormRows ? 1 : (kNB == 1 || kWarps > 8) ? 4 : 8;  // registers
    static_assert(!kNorm || (kMmaChunkBlocks * Fmt::kBlockWords) % kNormUnitWords == 0,
                  "a chunk is whole RMSNorm units");
    float* s_unit = reinterpret_cast<float*>(smem + mma_unit_off(g));
    __shared__ float s_inv[kNorm ? kMmaMaxM : 1];
    const int n_units = (int)((g.K + kNormUnitHalves - 1) / kNormUnitHalves);
    uint4 nw[kNormBatch];
    const uint4* nw_src = reinterpret_cast<const uint4*>(g.norm_w + k_first);
    auto load_norm_w = [&](int qb) {
#pragma unroll
        for (int b = 0; b < kNormBatch; ++b) {
            const int q = qb + b * kThreads;
            nw[b] = q < valid ? __ldg(nw_src + q) : make_uint4(0u, 0u, 0u, 0u);
        }
    };

    // Without the caller's promise that x is not produced by the preceding
    // kernel, x may only be read after that kernel has completed.
    if (!g.early_x) pdl_wait_prior_grids();
    if constexpr (kNormRow) {
        row_unit_sums<kWarps>(x, g.K, s_unit);
        __syncthreads();
        if (warp == 0) {
            const float s = row_sum_of_units(s_unit, n_units, lane);
            if (lane == 0) s_inv[0] = inv_rms(s, g.K, g.norm_eps);
        }
        __syncthreads();
    }
    // (row m, word q) pairs are walked in order, kStageBatch loads in flight
    // per thread before their stores.
    constexpr int kStageBatch = 4;
    {
        const float r_row = kNormRow ? s_inv[0] : 0.f;
        int m = 0, q = tid;
        while (m < M && q >= words) {
            q -= words;
            ++m;
        }
        while (m < M) {
            uint4 v[kStageBatch];
            uint4 vw[kNormRow ? kStageBatch : 1];
            int qs[kStageBatch], ms[kStageBatch];
#pragma unroll
            for (int u = 0; u < kStageBatch; ++u) {
                ms[u] = m;
                qs[u] = q;
                v[u] = make_uint4(0u, 0u, 0u, 0u);
                if (m < M && q < valid) {
                    v[u] = __ldg(reinterpret_cast<const uint4*>(x + m * g.x_stride + k_first) + q);
                    if constexpr (kNormRow) vw[u] = __ldg(nw_src + q);
                }
                q += kThreads;
                while (m < M && q >= words) {
                    q -= words;
                    ++m;
                }
            }
            if constexpr (kNormRows) {
                // the batch's unit sums, butterflies interleaved (words past
                // the last row are zeros; their sums are not stored)
                float su[kStageBatch];
#pragma unroll
                for (int u = 0; u < kStageBatch; ++u) su[u] = sq_word(v[u]);
#pragma unroll
                for (int off = 16; off > 0; off >>= 1)
#pragma unroll
                    for (int u = 0; u < kStageBatch; ++u)
                        su[u] += __shfl_xor_sync(0xffffffffu, su[u], off);
                if (lane == 0) {
#pragma unroll
                    for (int u = 0; u < kStageBatch; ++u)
                        if (ms[u] < M) s_unit[ms[u] * g.norm_units + (qs[u] >> 5)] = su[u];
                }
            }
#pragma unroll
            for (int u = 0; u < kStageBatch; ++u) {
                if (ms[u] >= M) break;  // uniform across the warp
                if constexpr (kNormRow) {
                    if (qs[u] < valid) v[u] = norm_word(v[u], vw[u], r_row);
                }
                xs4[ms[u] * g.xs_words + stage_at(qs[u])] = stage_order(v[u]);
            }
        }
    }
    if constexpr (kNormRows) load_norm_w(tid);
    __syncthreads();
    if constexpr (kNormRows) {
        // 1 / RMS of every row from all its unit sums (every split's, in
        // order), then the staged words normalised in place.
        if (g.splits > 1) cluster_sync_all();
        for (int m = warp; m < M; m += kWarps) {
            float s = 0.f;
            for (int u = lane; u < n_units; u += 32) {
                const int sp = u / g.norm_units;
                const float* a = s_unit + m * g.norm_units + (u - sp * g.norm_units);
                s += g.splits > 1 ? ld_cluster_f32(a, (uint32_t)sp) : *a;
            }
            s = warp_xor_sum(s);
            if (lane == 0) s_inv[m] = inv_rms(s, g.K, g.norm_eps);
        }
        __syncthreads();
        for (int qb = tid; qb < valid; qb += kNormBatch * kThreads) {
            if (qb != tid) load_norm_w(qb);
#pragma unroll
            for (int b = 0; b < kNormBatch; ++b) {
                const int q = qb + b * kThreads;
                if (q >= valid) break;
                const uint4 wq = stage_order(nw[b]);
                uint4* e = xs4 + stage_at(q);
                for (int m = 0; m < M; ++m, e += g.xs_words) *e = norm_word(*e, wq, s_inv[m]);
            }
        }
        __syncthreads();
    }

    const uint4* zero4 = reinterpret_cast<const uint4*>(smem);
    const int RT = g.round_tiles;
    const int n_rounds = (n_tiles + RT - 1) / RT;
    int rnd = 0, tile_end = min(RT, n_tiles);
    bool ready = false;  // the preceding kernel has been waited for (stores allowed)
    unsigned epoch = 0;

    // Store of a finished value (local y, or every rank's y).
    auto store = [&](int r, int m, float s) {
        const __half h = __float2half_rn(s);
        if constexpr (kPeer) {
            const int64_t off = m * g.y_stride + po.row0 + r0 + r;
#pragma unroll
            for (int p = 0; p < kMaxPeers; ++p)
                if (p < po.world) ((epoch & 1) ? po.y[1][p] : po.y[0][p])[off] = h;
        } else {
            y[m * g.y_stride + r0 + r] = h;
        }
    };
    // y may be read or written by the preceding kernel: store only after it.
    // With free_y (y untouched by every kernel still in flight) the stores do
    // not wait; CTA 0 alone waits for the preceding kernel, at its very end,
    // so that this grid still completes after it (completion order, and with
    // it the visibility guarantees of the stream, stay transitive).
    auto make_ready = [&]() {
        if (g.early_x && !(kPeer == false && g.free_y)) pdl_wait_prior_grids();
        if constexpr (kPeer) {
            // the step number, written by the preceding step's last CTA (complete now)
            if (tid == 0)
                s_epoch = *reinterpret_cast<volatile unsigned*>(po.flag[po.rank] + kStep) + 1u;
            __syncthreads();
            epoch = s_epoch;
        }
        ready = true;
    };
    // End of a round: sum the round's rows over their chunks (in chunk order)
    // and store them (one split) or keep them for the cluster sum.
    auto end_round = [&]() {
        __syncthreads();
        const int tile0 = rnd * RT;
        const int row_lo = 16 * tile0, row_hi = min(16 * tile_end, nrows);
        if (g.splits == 1 && !ready) make_ready();
        for (int m = 0; m < M; ++m) {
            for (int r = row_lo + tid; r < row_hi; r += kThreads) {
                const float* pp = part + ((r >> 4) - tile0) * n_seg * 16 * M + (r & 15) * M + m;
                float s = 0.f;
                for (int sg = 0; sg < n_seg; ++sg) s += pp[sg * 16 * M];
                if (g.splits == 1) {
                    if constexpr (Fmt::kRowScale) s *= sc8[r];
                    store(r, m, s);
                } else {
                    rsum[r * M + m] = s;
                }
            }
        }
        __syncthreads();
        ++rnd;
        tile_end = min((rnd + 1) * RT, n_tiles);
    };

    // Ping-pong over two register buffers: compute one item while the other
    // loads.  A segment's last item stores the segment's sums.  Every warp
    // passes exactly n_rounds round ends.
    MmaAcc<kNB> sacc;
    mma_acc_zero<kNB>(sacc);
    for (;;) {
        while (rnd < n_rounds && !(ca.tile < tile_end)) end_round();
        if (rnd >= n_rounds) break;
        {
            const int lb0 = kMmaChunkBlocks * (ca.seg * G + ca.j);
            mma_item<Fmt, kNB>(ra, xs4, zero4, lb0, g, gq, t, sacc);
            if (seg_last(ca))
                mma_flush<Fmt, kNB>(sacc, g, gq, t, part, (ca.tile - rnd * RT) * n_seg + ca.seg);
        }
        ca = f;
        if (f.tile < n_tiles) fetch_next(ra);
        while (rnd < n_rounds && !(cb.tile < tile_end)) end_round();
        if (rnd >= n_rounds) break;
        {
            const int lb0 = kMmaChunkBlocks * (cb.seg * G + cb.j);
            mma_item<Fmt, kNB>(rb, xs4, zero4, lb0, g, gq, t, sacc);
            if (seg_last(cb))
                mma_flush<Fmt, kNB>(sacc, g, gq, t, part, (cb.tile - rnd * RT) * n_seg + cb.seg);
        }
        cb = f;
        if (f.tile < n_tiles) fetch_next(rb);
    }

    if (g.splits > 1) {
        // Sum the splits' row sums in split order through distributed shared
        // memory; split s finishes rows [s * span, (s + 1) * span).
        make_ready();
        cluster_sync_all();
        const int span = (nrows + g.splits - 1) / g.splits;
        const int lo = min(nrows, split * span), hi = min(nrows, lo + span);
        for (int m = 0; m < M; ++m) {
            for (int r = lo + tid; r < hi; r += kThreads) {
                float s = 0.f;
                for (int sp = 0; sp < g.splits; ++sp) s += ld_cluster_f32(rsum + r * M + m, sp);
                if constexpr (Fmt::kRowScale) s *= sc8[r];
                store(r, m, s);
            }
        }
        // no CTA leaves while the others may still read its row sums
        cluster_sync_all();
    }
    if constexpr (kPeer) {
        __syncthreads();
        if (tid == 0) peer_arrive_and_wait(po, epoch, g.wait_cycles);
    } else {
        if (g.free_y && blockIdx.x == 0) pdl_wait_prior_grids();
    }
}

}  // namespace clb
