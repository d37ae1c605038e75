// Weight quantisation on the device, byte-identical to the reference's torch
// quantisers (cudalab/int4gemv_quantize.py:61-114, cudalab/qgemv_quantize.py:33-64):
//
//   INT4 (group 128 along K): s32 = max|W[n, group]| / 7 in fp32 (IEEE
//   division, round to nearest); q = clamp(round_half_even(W / s32), -7, 7);
//   an all-zero group has s32 = 0 and q = 0; scale stored as fp16(s32) (round
//   to nearest); W_packed[n, b] = (q[2b+1] & 0xF) << 4 | (q[2b] & 0xF).
//   INT8 (per row): s = max|W[n, :]| / 127 in fp32 (stored fp32);
//   q = clamp(round_half_even(W / s), -127, 127); all-zero rows give s = 0, q = 0.
//
// Every operation is exact or a single IEEE-rounded fp32 division / rint, so
// the bytes equal those of the torch path on any device.  W must be finite
// (the host wrappers check, as the reference does).  Both kernels are
// bandwidth-bound: each element is read once (INT8 reads its row a second
// time, from L1/L2) and written once.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "gemv_quantize.h"

namespace clb {
namespace {

// One warp per 128-element group: lane l holds elements 4l..4l+3 (8 bytes),
// so a warp reads the group's 256 bytes in one coalesced access and writes
// its 64 packed bytes in another.
__global__ void __launch_bounds__(256) int4_quantize_kernel(const __half* __restrict__ W,
                                                            uint8_t* __restrict__ Wp,
                                                            __half* __restrict__ scale,
                                                            int64_t groups_total) {
    const int64_t grp = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
    if (grp >= groups_total) return;
    const int lane = threadIdx.x & 31;
    const uint2 raw = reinterpret_cast<const uint2*>(W + grp * 128)[lane];
    const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&raw.x));
    const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&raw.y));
    float m = fmaxf(fmaxf(fabsf(a.x), fabsf(a.y)), fmaxf(fabsf(b.x), fabsf(b.y)));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    const float s32 = __fdiv_rn(m, 7.0f);
    const float v[4] = {a.x, a.y, b.x, b.y};
    uint32_t nib[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        float q = 0.f;
        if (s32 != 0.f) q = fminf(fmaxf(rintf(__fdiv_rn(v[i], s32)), -7.f), 7.f);
        nib[i] = (uint32_t)((int)q) & 0xFu;
    }
    const uint16_t packed = (uint16_t)(nib[0] | (nib[1] << 4) | (nib[2] << 8) | (nib[3] << 12));
    reinterpret_cast<uint16_t*>(Wp + grp * 64)[lane] = packed;
    if (lane == 0) scale[grp] = __float2half_rn(s32);
}

// One 256-thread CTA per row: block-wide max, then the quantised row.
__global__ void __launch_bounds__(256) int8_quantize_kernel(const __half* __restrict__ W,
                                                            int8_t* __restrict__ Wq,
                                                            float* __restrict__ scale, int64_t K) {
    __shared__ float red[8];
    const int64_t row = blockIdx.x;
    const __half* w = W + row * K;
    float m = 0.f;
    for (int64_t k = threadIdx.x; k < K; k += 256) m = fmaxf(m, fabsf(__half2float(w[k])));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
    __syncthreads();
    m = red[0];
#pragma unroll
    for (int i = 1; i < 8; ++i) m = fmaxf(m, red[i]);
    const float s = __fdiv_rn(m, 127.0f);
    int8_t* q = Wq + row * K;
    for (int64_t k = threadIdx.x; k < K; k += 256) {
        float v = 0.f;
        if (s != 0.f) v = fminf(fmaxf(rintf(__fdiv_rn(__half2float(w[k]), s)), -127.f), 127.f);
        q[k] = (int8_t)(int)v;
    }
    if (threadIdx.x == 0) scale[row] = s;
}

}  // namespace

cudaError_t launch_int4_quantize(const void* W, int64_t N, int64_t K, uint8_t* W_packed,
                                 void* scale, cudaStream_t stream) {
    const int64_t groups = N * (K / 128);
    const dim3 grid((unsigned)((groups + 7) / 8));
    int4_quantize_kernel<<<grid, 256, 0, stream>>>(static_cast<const __half*>(W), W_packed,
                                                   static_cast<__half*>(scale), groups);
    return cudaGetLastError();
}

cudaError_t launch_int8_quantize(const void* W, int64_t N, int64_t K, int8_t* W_q, float* scale,
                                 cudaStream_t stream) {
    int8_quantize_kernel<<<dim3((unsigned)N), 256, 0, stream>>>(static_cast<const __half*>(W),
                                                                W_q, scale, K);
    return cudaGetLastError();
}

}  // namespace clb
