// Shared device helpers for the weight-only quantized GEMV kernels (sm_100a).
//
// Everything here is written for Blackwell (compute capability 10.0a):
//   * mbarrier + cp.async.bulk (the TMA bulk-copy engine) to stage weight
//     tiles into shared memory with an L2 evict-first policy,
//   * griddepcontrol (programmatic dependent launch) so that a GEMV can start
//     streaming its weights while the kernel before it drains,
//   * exact nibble/byte -> fp16 dequantisation by IEEE exponent tricks,
//   * fp32 accumulation through mixed-precision `fma.rn.f32.f16` (exact
//     fp16 x fp16 products, one rounding per term) or packed `fma.rn.f32x2`.
//
// Every spin-wait is bounded by the SM cycle counter; on expiry the kernel records
// an error code in the library's device status word that the host reads
// through the C ABI (cl_device_status) and returns without touching more
// memory.
#pragma once

#include <cuda_fp16.h>
#include <cstdint>

namespace clb {

// ---------------------------------------------------------------------------
// Tunables shared by the vectorised kernels.
// ---------------------------------------------------------------------------
constexpr int kConsumerThreads = 256;               // 8 compute warps
constexpr int kConsumerWarps = kConsumerThreads / 32;
constexpr int kChunkBytes = 16;                     // bytes of W per thread per row
constexpr int kRowsPerThread = 4;                   // rows a thread covers per tile
constexpr int kTileBytes = kConsumerThreads * kRowsPerThread * kChunkBytes;  // 16 KiB
constexpr int kMaxSliceBytes = kConsumerThreads * kChunkBytes;               // 4 KiB
constexpr int kRingBytes = 64 * 1024;               // weight staging ring per CTA
constexpr int kMaxStages = 16;
constexpr int kScaleSmemBytes = 32 * 1024;          // per-CTA cache of group scales
// Default bound of every spin-wait, in SM clock cycles (~2 s at 2 GHz).  The
// SM-local cycle counter is used because reading %globaltimer is a slow,
// long-latency operation that would dominate a short wait.  The bound a kernel
// uses is a launch parameter (GemvGeom / MmaGeom `wait_cycles`), set from the
// process-wide value of cl_set_wait_budget, so a test can make a wait expire
// after a millisecond.
constexpr long long kWaitTimeoutCycles = 4000000000ll;

// Error codes written to the device status word.
constexpr int kStatusOk = 0;
constexpr int kStatusTimeoutFull = 1;    // consumer gave up waiting for a tile
constexpr int kStatusTimeoutEmpty = 2;   // producer gave up waiting for a slot
constexpr int kStatusTimeoutScale = 3;   // consumer gave up waiting for scales
constexpr int kStatusTimeoutDrain = 4;   // producer gave up draining its copies
constexpr int kStatusTimeoutPeer = 5;    // a sharded GEMV gave up waiting for a peer rank

// Per-device status word for bounded waits, read and cleared through the C ABI
// (cl_device_status).  The first code recorded since the last clear wins.
// Exactly one translation unit defines it: the one that holds every kernel
// with a bounded wait (gemv_kernels.cu defines CLB_STATUS_OWNER before
// including this header).  Other translation units see neither the word nor
// record_status, so a kernel there cannot write a status nobody reads.
#ifdef CLB_STATUS_OWNER
__device__ int g_status;

__device__ __forceinline__ void record_status(int code) { atomicCAS(&g_status, 0, code); }
#endif

// ---------------------------------------------------------------------------
// Small PTX wrappers.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t policy_evict_first() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait on one mbarrier phase: at most `budget` SM cycles.  Returns
// false when the budget expired.
__device__ __forceinline__ bool mbar_wait_bounded(uint32_t bar, uint32_t parity,
                                                  long long budget) {
    if (mbar_try_wait(bar, parity)) return true;
    const long long t0 = clock64();
#pragma unroll 1
    while (!mbar_try_wait(bar, parity)) {
        if (clock64() - t0 > budget) return false;
    }
    return true;
}

// One bulk (TMA engine) copy global -> shared, completing on `bar`.
// Requirements (checked by the host contract): 16-byte aligned addresses,
// size a multiple of 16.
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes,
                                         uint32_t bar, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1], %2, [%3], %4;" ::"r"(dst),
        "l"(src), "r"(bytes), "r"(bar), "l"(policy)
        : "memory");
}

// Programmatic dependent launch controls. Both are no-ops for a kernel that
// was launched without the programmatic-serialization attribute.
__device__ __forceinline__ void pdl_wait_prior_grids() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
}
__device__ __forceinline__ void pdl_allow_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// System-scope release store / acquire load of a flag word that other GPUs
// read or write through peer mappings.
// Strong (relaxed) system-scope store: after a fence.sc.sys it forms a
// release pattern, without the implicit fence of st.release.
__device__ __forceinline__ void st_relaxed_sys(unsigned* p, unsigned v) {
    asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Named barrier among the consumer warps only (the producer warp never joins).
__device__ __forceinline__ void consumer_sync() {
    asm volatile("bar.sync 1, %0;" ::"n"(kConsumerThreads) : "memory");
}

// 16-byte streaming load of weights straight from global memory: bypass L1,
// mark the L2 line evict-first (the weights are read exactly once).
__device__ __forceinline__ uint4 ldg_stream16(const void* p, uint64_t policy) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.v4.u32 {%0,%1,%2,%3}, [%4], %5;"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p), "l"(policy));
    return v;
}

__device__ __forceinline__ uint4 lds16(uint32_t addr) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "r"(addr));
    return v;
}

// ---------------------------------------------------------------------------
// Exact dequantisation.
//
// lop3 with LUT 0x6A computes  b ? (a ^ c) : c  bitwise.  With b = a nibble
// (or byte) mask and c = <exponent pattern> | <sign bit of each field>, one
// instruction isolates the field, flips its sign bit (two's complement ->
// offset binary) and ORs in an IEEE exponent so that the result, read as a
// float, equals  M + (v + 8)  for a nibble v (M + v + 128 for a byte).  A
// single fused multiply-add then removes the bias exactly.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t lop3_sel_xor(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t d;
    asm("lop3.b32 %0, %1, %2, %3, 0x6A;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

// Same with the mask and the exponent pattern as instruction immediates.
template <uint32_t B, uint32_t C>
__device__ __forceinline__ uint32_t lop3_sel_xor_i(uint32_t a) {
    uint32_t d;
    asm("lop3.b32 %0, %1, %2, %3, 0x6A;" : "=r"(d) : "r"(a), "n"(B), "n"(C));
    return d;
}

template <uint32_t SEL>
__device__ __forceinline__ uint32_t prmt_i(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "n"(SEL));
    return d;
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t d;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
    return d;
}

__device__ __forceinline__ __half2 u32_as_h2(uint32_t v) {
    return *reinterpret_cast<__half2*>(&v);
}

// fp16 constants as raw bits (binary16).
constexpr unsigned short kH_one = 0x3C00;        // 1.0
constexpr unsigned short kH_1_16 = 0x2C00;       // 0.0625
constexpr unsigned short kH_m1032 = 0xE408;      // -1032
constexpr unsigned short kH_m72 = 0xD480;        // -72
constexpr unsigned short kH_m1152 = 0xE480;      // -1152

__device__ __forceinline__ __half2 h2_const(unsigned short bits) {
    return u32_as_h2((uint32_t)bits | ((uint32_t)bits << 16));
}

// 8 signed 4-bit values of one little-endian word -> 4 half2 holding exact
// integers.  Output pairs are (n0,n4) (n1,n5) (n2,n6) (n3,n7), nibble j being
// element k0+j (low nibble of byte b is element 2b).
//   binary16 with exponent field 25 (0x6400) has a unit ulp on [1024, 2048):
//   (0x6400 | u) == 1024 + u for u < 1024.  A nibble at bits 4..7 lands as
//   1024 + 16u, rescaled by 1/16 in the same FMA.
__device__ __forceinline__ void int4x8_to_h2(uint32_t w, __half2 (&q)[4]) {
    const uint32_t hi = w >> 8;
    const __half2 one = h2_const(kH_one), sixteenth = h2_const(kH_1_16);
    const __half2 b0 = h2_const(kH_m1032), b1 = h2_const(kH_m72);
    q[0] = __hfma2(u32_as_h2(lop3_sel_xor_i<0x000F000Fu, 0x64086408u>(w)), one, b0);
    q[1] = __hfma2(u32_as_h2(lop3_sel_xor_i<0x00F000F0u, 0x64806480u>(w)), sixteenth, b1);
    q[2] = __hfma2(u32_as_h2(lop3_sel_xor_i<0x000F000Fu, 0x64086408u>(hi)), one, b0);
    q[3] = __hfma2(u32_as_h2(lop3_sel_xor_i<0x00F000F0u, 0x64806480u>(hi)), sixteenth, b1);
}

// 4 signed bytes -> 2 half2 of exact integers: (b0,b1) (b2,b3).
//   bytes are flipped to offset binary (v + 128), placed under a 0x64 high
//   byte (1024 + v + 128) and un-biased by one FMA.
__device__ __forceinline__ void int8x4_to_h2(uint32_t w, __half2 (&q)[2]) {
    const uint32_t u = w ^ 0x80808080u;
    const __half2 one = h2_const(kH_one), b = h2_const(kH_m1152);
    q[0] = __hfma2(u32_as_h2(prmt_i<0x5140u>(u, 0x64646464u)), one, b);
    q[1] = __hfma2(u32_as_h2(prmt_i<0x7362u>(u, 0x64646464u)), one, b);
}

// d = a * b + c with a, b binary16 and c, d binary32: the product is exact in
// binary32 and the single rounding is the addition (PTX ISA 8.6, sm_100+).
__device__ __forceinline__ float fma_h(__half a, __half b, float c) {
    float d;
    asm("fma.rn.f32.f16 %0, %1, %2, %3;"
        : "=f"(d)
        : "h"(__half_as_ushort(a)), "h"(__half_as_ushort(b)), "f"(c));
    return d;
}

// ---------------------------------------------------------------------------
// Packed fp32 path (fma.rn.f32x2 / add.rn.f32x2, sm_100+).
// ---------------------------------------------------------------------------
__device__ __forceinline__ unsigned long long f2_pack(float lo, float hi) {
    unsigned long long r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
    return r;
}
__device__ __forceinline__ void f2_unpack(unsigned long long v, float& lo, float& hi) {
    asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ unsigned long long f2_fma(unsigned long long a, unsigned long long b,
                                                     unsigned long long c) {
    unsigned long long d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}
__device__ __forceinline__ unsigned long long f2_add(unsigned long long a, unsigned long long b) {
    unsigned long long d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}

// binary32 pattern whose value is 2^(23-4p) + u for a nibble u held in
// mantissa bits 4p..4p+3 (p = 0..5): exponent field 150 - 4p.
__host__ __device__ constexpr uint32_t f32_magic_bits(int p) {
    return static_cast<uint32_t>(150 - 4 * p) << 23;
}
__host__ __device__ constexpr float f32_pow2(int e) {
    return e >= 0 ? static_cast<float>(1ull << e) : 1.0f / static_cast<float>(1ull << (-e));
}

// Nibble at position p of `w` -> float (2^(23-4p) + v + 8) with v the signed
// value; un-biasing happens later in a packed add.
template <int P>
__device__ __forceinline__ float nib_to_biased_f32(uint32_t w) {
    return __uint_as_float(
        lop3_sel_xor(w, 0xFu << (4 * P), f32_magic_bits(P) | (0x8u << (4 * P))));
}

}  // namespace clb
