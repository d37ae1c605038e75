// Internal interface between the kernel translation unit (gemv_kernels.cu)
// and the C ABI translation unit (capi.cu).  Not installed; the public ABI is
// include/cudalab_gemv.h.
#pragma once

#include <cuda_runtime.h>
#include <cstdint>

namespace clb {

// One launch: W is uint8 [N, K/2] (INT4 packed), int8 [N, K] (INT8) or the
// dense fp16 / fp32 [N, K]; scale is fp16 [N, K/128] (INT4), fp32 [N] (INT8)
// or unused (dense); x holds M activation rows of
// K halves (x_stride halves apart), y receives M rows of N halves (y_stride
// apart; in peer mode, rows of the full matrix in every rank's buffer).
// norm_w / norm_eps: RMSNorm weight (K halves, 16-byte aligned) and epsilon
// of the fused RMSNorm -> GEMV launches; unused elsewhere.
struct GemvArgs {
    const void* W;
    const void* scale;
    const void* x;
    void* y;
    int64_t N, K, M;
    int64_t x_stride, y_stride;
    const void* norm_w = nullptr;
    float norm_eps = 0.f;
};

// flags are the CL_LAUNCH_* bits of the public header.
using LaunchFn = cudaError_t (*)(const GemvArgs& args, cudaStream_t stream, unsigned flags);

struct VariantDesc {
    const char* name;
    LaunchFn fn;
    bool quarantined;  // registered but not in the normal dispatch list
};

// Row-sharded GEMV with the all-gather fused into the epilogue: pointers (in
// this process) to every rank's two y buffers (by step parity) and flag block
// (16 words), and the shard's first row.
struct PeerArgs {
    void* y[2][8];
    unsigned* flag[8];
    int64_t row0;
    int rank, world;
};

using ShardedLaunchFn = cudaError_t (*)(const GemvArgs& args, const PeerArgs& peers,
                                        cudaStream_t stream, unsigned flags);

struct ShardedVariantDesc {
    const char* name;
    ShardedLaunchFn fn;
};

const VariantDesc* int4_variants(int* count);
const VariantDesc* int8_variants(int* count);
// Fused RMSNorm -> INT4 GEMV (GemvArgs.norm_w / norm_eps set; x_stride == K).
const VariantDesc* int4_rmsnorm_variants(int* count);
// Standalone RMSNorm of M fp16 rows of H halves (H % 8 == 0, 16-byte aligned).
cudaError_t launch_rmsnorm_f16(const void* x, const void* w, float eps, void* y, int64_t M,
                               int64_t H, cudaStream_t stream, unsigned flags);
const ShardedVariantDesc* int4_sharded_variants(int* count);
const ShardedVariantDesc* int8_sharded_variants(int* count);

// Dense GEMV (gemv_dense.cu): variant table by element type (0 = fp16,
// 1 = fp32; GemvArgs.scale unused), the tensor-core fp16 launch
// (gemv_kernels.cu) and the fp16 baseline launch, which is also the fallback
// of the tensor-core path when its contract is not met.
const VariantDesc* gemv_variants(int dtype, int* count);
cudaError_t launch_gemv_f16_mma(const GemvArgs& args, cudaStream_t stream, unsigned flags);
cudaError_t launch_f16_scalar(const void* W, const void* scale, const void* x, void* y, int64_t N,
                              int64_t K, cudaStream_t stream, unsigned flags);

// Reads (optionally clears) the device-side bounded-wait status word of the
// current device.
cudaError_t read_device_status(int clear, int* status);

// Sets the bound of the device-side waits of later launches (SM cycles; <= 0
// restores the default of about two seconds) and returns the previous bound.
long long set_wait_budget(long long cycles);

}  // namespace clb
