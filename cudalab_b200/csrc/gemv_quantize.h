// Internal interface of the quantisation kernels (quantize.cu) for the C ABI
// translation unit (capi.cu).
#pragma once

#include <cuda_runtime.h>
#include <cstdint>

namespace clb {

// fp16 W [N, K] (K % 128 == 0) -> W_packed uint8 [N, K/2], scale fp16 [N, K/128].
cudaError_t launch_int4_quantize(const void* W, int64_t N, int64_t K, uint8_t* W_packed,
                                 void* scale, cudaStream_t stream);
// fp16 W [N, K] -> W_q int8 [N, K], scale fp32 [N].
cudaError_t launch_int8_quantize(const void* W, int64_t N, int64_t K, int8_t* W_q, float* scale,
                                 cudaStream_t stream);

}  // namespace clb
