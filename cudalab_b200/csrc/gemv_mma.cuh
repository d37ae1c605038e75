// Tensor-core weight-only GEMV for sm_100a (INT4 group-scaled, INT8 row-scaled).
//
// Why tensor cores at M = 1: on the CUDA cores the exact dequantisation plus
// an fp32 multiply-add costs 4+ issued instructions per weight element
// (measured with ncu), which caps the kernel below the HBM roofline.  Here
// the dequantised fp16 values feed `mma.sync.m16n8k16` (exact fp16 x fp16
// products, fp32 accumulation), so the multiply-adds leave the issue stream
// and the dequantisation (one lop3 + one fma.f16x2 per two elements) is
// nearly all that remains.
//
// Decomposition
//   * Each CTA owns a balanced, contiguous range of 16-row mma tiles (only the
//     matrix's last tile can be partial; its missing rows are never fetched).  A row is cut into 64-byte blocks (INT4: one 128-wide
//     scale group; INT8: 64 elements) and blocks into chunks of 4.
//   * An item = (tile, chunk) = 16 rows x 256 bytes.  Warp w processes items
//     w, w+8, ... .  Lane (g, t) loads its A fragments directly from global
//     memory: 16 bytes of row g and of row g+8 per block, which for a warp is
//     16 rows x 64 contiguous bytes -- whole 32-byte sectors, no shared-memory
//     staging, no bank conflicts, no per-copy engine overhead.  Two items per
//     warp are in flight (register double buffer, L2 evict-first), the first
//     two issued before waiting on the preceding kernel.
//   * Every block gets a fresh accumulator, scaled by its group scale (INT4)
//     and summed into per-row fp32 partials; partials of an item land in
//     shared memory and are summed per row, in chunk order, at the end
//     (deterministic).
//
// Fragment / k-permutation (m16n8k16, row.col): lane (g, t) holds A rows g and
// g+8 at k-positions {2t, 2t+1, 2t+8, 2t+9}.  The k order inside a step is
// free as long as A and B agree.  INT4: the 16 bytes lane t reads for a block
// are 32 consecutive elements k0..k0+31 (4 words of 8 nibbles); step 2w uses
// nibble pairs (0,4) and (1,5) of word w, step 2w+1 pairs (2,6) and (3,7) --
// exactly what one lop3 yields -- and the activation vector is staged in
// shared memory in that permuted order once per CTA.  INT8: step j uses word
// j, byte pairs (0,1) and (2,3), i.e. natural order.
#pragma once

#include "gemv_common.cuh"

namespace clb {

constexpr int kMmaChunkBlocks = 4;   // 64-byte blocks per item row
constexpr int kMmaPartialMax = 512;  // items per CTA (partials buffer)

struct MmaGeom {
    int64_t N, K;
    int64_t row_bytes;  // RB
    int32_t blocks;     // NB = RB / 64
    int32_t n_kc;       // chunks per row = ceil(NB / 4)
    int32_t tiles_base, tiles_rem, ctas;  // 16-row tiles per CTA (balanced)
    int32_t xs_bytes;   // staged activations (K halves)
    int32_t max_items;  // items of the largest CTA
    int32_t max_rows;   // rows of the largest CTA
    int32_t early_x;    // x is not written by the preceding kernel: read it before the PDL wait
};

// Shared memory: [256 B of zeros | activations | item partials | INT8 row scales]
__host__ __device__ inline int mma_part_off(const MmaGeom& g) {
    return 256 + ((g.xs_bytes + 15) & ~15);
}
__host__ __device__ inline int mma_sc_off(const MmaGeom& g) {
    return mma_part_off(g) + g.max_items * 16 * 4;
}
__host__ __device__ inline int mma_smem_total(const MmaGeom& g) {
    return mma_sc_off(g) + g.max_rows * 4;
}

__device__ __forceinline__ void mma_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                          uint32_t a3, uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t h2_as_u32(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }

// Nibbles 0 and 4 of w as an exact half2 (q0, q4) ...
__device__ __forceinline__ uint32_t nib_pair_lo(uint32_t w) {
    return h2_as_u32(__hfma2(u32_as_h2(lop3_sel_xor_i<0x000F000Fu, 0x64086408u>(w)),
                             h2_const(kH_one), h2_const(kH_m1032)));
}
// ... and nibbles 1 and 5 as (q1, q5).
__device__ __forceinline__ uint32_t nib_pair_hi(uint32_t w) {
    return h2_as_u32(__hfma2(u32_as_h2(lop3_sel_xor_i<0x00F000F0u, 0x64806480u>(w)),
                             h2_const(kH_1_16), h2_const(kH_m72)));
}

__device__ __forceinline__ uint2 lds8(uint32_t addr) {
    uint2 v;
    asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(addr));
    return v;
}

// Formats.  kAcc: independent accumulators per item (blocks of even / odd
// index), which halves the length of the dependent mma chain.
struct MmaInt4 {
    static constexpr int kSteps = 8;  // k-steps per 64-byte block (128 elements)
    static constexpr bool kGroupScale = true;
    static constexpr int kBlockWords = 16;  // uint4 words of x per block
    static constexpr int kAcc = 2;
    using Scale = __half;
};
struct MmaInt8 {
    static constexpr int kSteps = 4;  // 64 elements
    static constexpr bool kGroupScale = false;
    static constexpr int kBlockWords = 8;
    static constexpr int kAcc = 2;
    using Scale = float;
};
// Accumulate one 64-byte block (index q inside its item) of rows g (wa) and
// g+8 (wb).  `bp` points at the block's staged activations for the lanes of
// the batch column that this block feeds, and at a zero region for every
// other lane, so all lanes load unconditionally.  One 16-byte load covers two
// k-steps.
template <class Fmt>
__device__ __forceinline__ void mma_block(const uint4 wa, const uint4 wb, const uint4* bp, int t,
                                          int q, float (&acc)[Fmt::kAcc][4]) {
    const uint32_t ua[4] = {wa.x, wa.y, wa.z, wa.w};
    const uint32_t ub[4] = {wb.x, wb.y, wb.z, wb.w};
    if constexpr (Fmt::kGroupScale) {
#pragma unroll
        for (int w = 0; w < 4; ++w) {
            const uint4 bb = bp[w * 4 + t];  // (x0,x4) (x1,x5) (x2,x6) (x3,x7) of word w
            const uint32_t ha = ua[w] >> 8, hb = ub[w] >> 8;
            // operands of one step are produced back to back, in quad order
            mma_16816(acc[q & 1], nib_pair_lo(ua[w]), nib_pair_lo(ub[w]), nib_pair_hi(ua[w]),
                      nib_pair_hi(ub[w]), bb.x, bb.y);
            mma_16816(acc[q & 1], nib_pair_lo(ha), nib_pair_lo(hb), nib_pair_hi(ha),
                      nib_pair_hi(hb), bb.z, bb.w);
        }
    } else {
#pragma unroll
        for (int jj = 0; jj < 2; ++jj) {
            const uint4 bb = bp[2 * t + jj];  // x[16t + 8jj .. +8): steps 2jj and 2jj+1
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int j = 2 * jj + h;
                __half2 qa[2], qb[2];
                int8x4_to_h2(ua[j], qa);
                int8x4_to_h2(ub[j], qb);
                mma_16816(acc[q & 1], h2_as_u32(qa[0]), h2_as_u32(qb[0]), h2_as_u32(qa[1]),
                          h2_as_u32(qb[1]), h ? bb.z : bb.x, h ? bb.w : bb.y);
            }
        }
    }
}

// One item = 16 rows x up to 4 blocks: the fragments (rows g, g+8) and, for
// INT4, the group scales of those rows.
struct MmaItemRegs {
    uint4 wa[kMmaChunkBlocks], wb[kMmaChunkBlocks];
    __half sa[2], sb[2];  // INT4: scales of the two blocks (columns) this lane holds
};

// Position of a warp's current item: tile, chunk and the derived row data.
struct MmaCursor {
    int tile, kc;
};

__device__ __forceinline__ void cursor_advance(MmaCursor& c, int step, int n_kc) {
    c.kc += step;
    while (c.kc >= n_kc) {
        c.kc -= n_kc;
        ++c.tile;
    }
}

// Issue the loads of one item.  Rows beyond the CTA's range re-read the
// CTA's last row (L2 hit; their results are never stored), so no load is
// predicated.  kAllFull: every chunk of a row has 4 blocks (row bytes a
// multiple of 256); otherwise blocks past the row end re-read its last block.
template <class Fmt, bool kAllFull>
__device__ __forceinline__ void mma_fetch(MmaItemRegs& r, const uint8_t* W,
                                          const typename Fmt::Scale* scale, const MmaGeom& g,
                                          int64_t r0, int nrows, MmaCursor c, int gq, int t,
                                          uint64_t pol) {
    const int last = nrows - 1;
    const int64_t ra = r0 + min(16 * c.tile + gq, last);
    const int64_t rb = r0 + min(16 * c.tile + gq + 8, last);
    const int blk0 = kMmaChunkBlocks * c.kc;
    const uint8_t* pa = W + ra * g.row_bytes + 16 * t;
    const uint8_t* pb = W + rb * g.row_bytes + 16 * t;
#pragma unroll
    for (int q = 0; q < kMmaChunkBlocks; ++q) {
        const int blk = kAllFull ? blk0 + q : min(blk0 + q, g.blocks - 1);
        r.wa[q] = ldg_stream16(pa + 64 * blk, pol);
        r.wb[q] = ldg_stream16(pb + 64 * blk, pol);
    }
    if constexpr (Fmt::kGroupScale) {
        // lane (g, t) needs the scales of blocks 2(t&1), 2(t&1)+1 of rows g, g+8
        const int b0 = blk0 + 2 * (t & 1);
        const int b1 = kAllFull ? b0 + 1 : min(b0 + 1, g.blocks - 1);
        const __half* sa = reinterpret_cast<const __half*>(scale) + ra * g.blocks;
        const __half* sb = reinterpret_cast<const __half*>(scale) + rb * g.blocks;
        const int b0c = kAllFull ? b0 : min(b0, g.blocks - 1);
        r.sa[0] = sa[b0c];
        r.sa[1] = sa[b1];
        r.sb[0] = sb[b0c];
        r.sb[1] = sb[b1];
    }
}

// Compute one item and store its two row partials (rows g, g+8 of the tile).
// INT4: block q of the item is fed through batch column q, so the
// accumulators keep the four blocks' sums apart (columns 2t, 2t+1 in lane t;
// a block's column is non-zero only in the accumulator of its parity); the
// group scales are applied once per item, then the two lanes holding a row's
// columns are combined.  INT8: all blocks share column 0 (the row scale is
// applied at the very end).
template <class Fmt, bool kFull>
__device__ __forceinline__ void mma_item_t(const MmaItemRegs& r, const uint4* xs,
                                           const uint4* zero, MmaCursor c,
                                           const MmaGeom& g, int gq, int t, float* part) {
    const int nb =
        kFull ? kMmaChunkBlocks : min(kMmaChunkBlocks, g.blocks - kMmaChunkBlocks * c.kc);
    constexpr int kBlk = Fmt::kBlockWords;  // uint4 per block of staged activations
    const int blk0 = kMmaChunkBlocks * c.kc;
    const uint4* xbase = xs + blk0 * kBlk;
    float acc[Fmt::kAcc][4];
#pragma unroll
    for (int i = 0; i < Fmt::kAcc; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
#pragma unroll
    for (int q = 0; q < kMmaChunkBlocks; ++q) {
        if (kFull || q < nb) {
            const int col = Fmt::kGroupScale ? q : 0;
            const uint4* bp = gq == col ? xbase + q * kBlk : zero;
            mma_block<Fmt>(r.wa[q], r.wb[q], bp, t, q, acc);
        }
    }
    float acc_a, acc_b;
    if constexpr (Fmt::kGroupScale) {
        // lane t < 2 holds columns (blocks) 2t (even accumulator, entries 0 / 2)
        // and 2t + 1 (odd accumulator, entries 1 / 3); lanes t >= 2 hold zero columns
        const float sa0 = __half2float(r.sa[0]), sa1 = __half2float(r.sa[1]);
        const float sb0 = __half2float(r.sb[0]), sb1 = __half2float(r.sb[1]);
        acc_a = fmaf(sa1, acc[1][1], sa0 * acc[0][0]);
        acc_b = fmaf(sb1, acc[1][3], sb0 * acc[0][2]);
        if (t >= 2) acc_a = acc_b = 0.f;
        acc_a += __shfl_xor_sync(0xffffffffu, acc_a, 1);
        acc_b += __shfl_xor_sync(0xffffffffu, acc_b, 1);
    } else {
        acc_a = acc[0][0] + acc[1][0];
        acc_b = acc[0][2] + acc[1][2];
    }
    if (t == 0) {
        float* pp = part + (c.tile * g.n_kc + c.kc) * 16;
        pp[gq] = acc_a;
        pp[gq + 8] = acc_b;
    }
}

template <class Fmt, bool kAllFull>
__device__ __forceinline__ void mma_item(const MmaItemRegs& r, const uint4* xs, const uint4* zero,
                                         MmaCursor c, const MmaGeom& g, int gq, int t,
                                         float* part) {
    if (kAllFull || kMmaChunkBlocks * c.kc + kMmaChunkBlocks <= g.blocks)
        mma_item_t<Fmt, true>(r, xs, zero, c, g, gq, t, part);
    else
        mma_item_t<Fmt, false>(r, xs, zero, c, g, gq, t, part);
}

constexpr int kZeroRegion = 256;  // bytes of zeros ahead of the staged activations

// ---------------------------------------------------------------------------
// Row-sharded GEMV with the all-gather fused into the epilogue.
//
// Every rank owns a contiguous shard of the rows of W.  Instead of writing its
// y rows locally and running a separate all-gather, each CTA stores its rows
// straight into the y buffer of every rank (peer pointers over NVLink), so
// the exchange overlaps the other CTAs' compute.  Each rank's flag block
// holds: [0, kMaxPeers) the last step each rank has completed writing into
// this rank's buffers, [kTicket] the CTA arrival counter of the running step,
// [kStep] the last step this rank completed.  Per step:
//   0. after the preceding kernel completed, the CTA reads the step number
//      e = flag[kStep] + 1 (so a captured graph replays correctly);
//   1. it stores its rows into y[e & 1] of every rank, fences at system scope,
//      syncs and takes a ticket;
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

// Called by thread 0 of every CTA after a CTA barrier that follows the CTA's
// peer stores: the system-scope fence before the ticket publishes the whole
// CTA's stores (cumulativity through the barrier); the last CTA's fence and
// release stores publish every CTA's stores (through the ticket atomics).
// Loops run over the compile-time peer slots so that `po` stays in the
// parameter space (no local copy).
__device__ __forceinline__ void peer_arrive_and_wait(const PeerOut& po, unsigned epoch) {
    unsigned* mine = po.flag[po.rank];
    __threadfence_system();
    const unsigned prev = atomicAdd(mine + kTicket, 1u);
    if (prev != gridDim.x - 1) return;
    atomicExch(mine + kTicket, 0u);
    __threadfence_system();
#pragma unroll
    for (int p = 0; p < kMaxPeers; ++p)
        if (p < po.world) st_release_sys(po.flag[p] + po.rank, epoch);
    const long long t0 = clock64();
    bool ok = true;
    for (int q = 0; q < po.world && ok; ++q) {
        while ((int)(ld_acquire_sys(mine + q) - epoch) < 0) {
            if (clock64() - t0 > kWaitTimeoutCycles) {
                record_status(kStatusTimeoutPeer);
                ok = false;
                break;
            }
            __nanosleep(64);
        }
    }
    atomicExch(mine + kStep, epoch);
}

// kPeer: y is ignored; rows go to every rank's buffer in `po` (see PeerOut).
template <class Fmt, int kWarps, bool kAllFull, bool kPeer>
__global__ void __launch_bounds__(32 * kWarps, 16 / kWarps)
gemv_mma_kernel(const uint8_t* __restrict__ W, const typename Fmt::Scale* __restrict__ scale,
                const __half* __restrict__ x, __half* __restrict__ y, const MmaGeom g,
                const PeerOut po) {
    constexpr int kThreads = 32 * kWarps;
    extern __shared__ __align__(128) uint8_t smem[];
    uint8_t* xs = smem + kZeroRegion;
    float* part = reinterpret_cast<float*>(smem + mma_part_off(g));
    float* sc8 = reinterpret_cast<float*>(smem + mma_sc_off(g));

    // Whole 16-row tiles per CTA; only the matrix's last tile can be partial.
    const int b = blockIdx.x;
    const int n_tiles = g.tiles_base + (b < g.tiles_rem ? 1 : 0);
    const int64_t r0 = 16 * ((int64_t)b * g.tiles_base + (b < g.tiles_rem ? b : g.tiles_rem));
    const int64_t left = g.N - r0;
    const int nrows = left < 16 * n_tiles ? (int)left : 16 * n_tiles;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int gq = lane >> 2, t = lane & 3;
    const uint64_t pol = policy_evict_first();

    pdl_allow_dependents();
    // Items of this warp: w, w + kWarps, ... in (tile, chunk) order.  Weights
    // and scales never depend on the preceding kernel: the first two items
    // are requested before waiting on it.
    MmaCursor c0{0, warp};
    cursor_advance(c0, 0, g.n_kc);
    MmaCursor c1 = c0;
    cursor_advance(c1, kWarps, g.n_kc);
    MmaItemRegs ra, rb;
    if (c0.tile < n_tiles) mma_fetch<Fmt, kAllFull>(ra, W, scale, g, r0, nrows, c0, gq, t, pol);
    if (c1.tile < n_tiles) mma_fetch<Fmt, kAllFull>(rb, W, scale, g, r0, nrows, c1, gq, t, pol);
    if constexpr (!Fmt::kGroupScale) {
        for (int r = tid; r < nrows; r += kThreads)
            sc8[r] = reinterpret_cast<const float*>(scale)[r0 + r];
    }
    if (tid < kZeroRegion / 4) reinterpret_cast<uint32_t*>(smem)[tid] = 0u;

    // Without the caller's promise that x is not produced by the preceding
    // kernel, x may only be read after that kernel has completed.
    if (!g.early_x) pdl_wait_prior_grids();
    // Activations: INT4 in the permuted step order, INT8 as is.
    const int words = (int)(g.K >> 3);
    if constexpr (Fmt::kGroupScale) {
        for (int q = tid; q < words; q += kThreads) {
            const int blk = q >> 4, tt = (q >> 2) & 3, w = q & 3;
            const uint4 v = __ldg(reinterpret_cast<const uint4*>(x) + q);
            // entry (blk, w, tt): step 2w (x0, x4, x1, x5), step 2w+1 (x2, x6, x3, x7)
            uint4 e;
            e.x = prmt_i<0x5410u>(v.x, v.z);
            e.y = prmt_i<0x7632u>(v.x, v.z);
            e.z = prmt_i<0x5410u>(v.y, v.w);
            e.w = prmt_i<0x7632u>(v.y, v.w);
            reinterpret_cast<uint4*>(xs)[(blk * 4 + w) * 4 + tt] = e;
        }
    } else {
        for (int q = tid; q < words; q += kThreads)
            reinterpret_cast<uint4*>(xs)[q] = __ldg(reinterpret_cast<const uint4*>(x) + q);
    }
    __syncthreads();

    const uint4* xs4 = reinterpret_cast<const uint4*>(xs);
    const uint4* zero4 = reinterpret_cast<const uint4*>(smem);
    // Ping-pong over two register buffers: compute one while the other loads.
    while (c0.tile < n_tiles) {
        mma_item<Fmt, kAllFull>(ra, xs4, zero4, c0, g, gq, t, part);
        MmaCursor c2 = c1;
        cursor_advance(c2, kWarps, g.n_kc);
        if (c2.tile < n_tiles) mma_fetch<Fmt, kAllFull>(ra, W, scale, g, r0, nrows, c2, gq, t, pol);
        if (!(c1.tile < n_tiles)) break;
        mma_item<Fmt, kAllFull>(rb, xs4, zero4, c1, g, gq, t, part);
        MmaCursor c3 = c2;
        cursor_advance(c3, kWarps, g.n_kc);
        if (c3.tile < n_tiles) mma_fetch<Fmt, kAllFull>(rb, W, scale, g, r0, nrows, c3, gq, t, pol);
        c0 = c2;
        c1 = c3;
    }
    __syncthreads();
    // y may be read or written by the preceding kernel: store only after it.
    if (g.early_x) pdl_wait_prior_grids();
    unsigned epoch = 0;
    if constexpr (kPeer) {
        // the step number, written by the preceding step's last CTA (complete now)
        __shared__ unsigned s_epoch;
        if (tid == 0) s_epoch = *reinterpret_cast<volatile unsigned*>(po.flag[po.rank] + kStep) + 1u;
        __syncthreads();
        epoch = s_epoch;
    }
    // ---- per-row sums over chunks, in chunk order ----
    for (int r = tid; r < nrows; r += kThreads) {
        const int tile = r >> 4, rr = r & 15;
        const float* pp = part + tile * g.n_kc * 16 + rr;
        float s = 0.f;
        for (int kc = 0; kc < g.n_kc; ++kc) s += pp[kc * 16];
        if constexpr (!Fmt::kGroupScale) s *= sc8[r];
        const __half h = __float2half_rn(s);
        if constexpr (kPeer) {
            const int64_t row = po.row0 + r0 + r;
#pragma unroll
            for (int p = 0; p < kMaxPeers; ++p)
                if (p < po.world) ((epoch & 1) ? po.y[1][p] : po.y[0][p])[row] = h;
        } else {
            y[r0 + r] = h;
        }
    }
    if constexpr (kPeer) {
        __syncthreads();
        if (tid == 0) peer_arrive_and_wait(po, epoch);
    }
}

}  // namespace clb
