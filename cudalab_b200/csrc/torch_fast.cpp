// Python binding of the operator API's success path on torch tensors (the
// role of the reference's pybind `forward` / `forward_into`,
// kernels/int4gemv/bindings.cpp:145-176 and kernels/qgemv/bindings.cpp:66-115).
//
// It makes the checks of the Python wrapper's success predicate
// (ext.py `_fast_ok`) on the tensors' metadata in C++, then calls the C ABI
// (cl_int4gemv_ex / cl_qgemv_ex) on the current stream of the tensors'
// device.  When a check fails, or the C ABI reports an error, it returns a
// nonzero code without raising, and the Python wrapper runs its ordered
// checks, which raise the reference's messages.  No computation happens here.
#include <torch/extension.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>

#include "../../include/cudalab_gemv.h"

namespace {

constexpr int kNotFast = -1000;  // a check of the success predicate failed
constexpr int kInt4 = 0, kInt8 = 1;

bool on(const at::Tensor& t, c10::DeviceIndex d) { return t.is_cuda() && t.get_device() == d; }

// W / scale / x of one GEMV: the success predicate of the Python wrapper
// (INT4: W uint8 [N, K/2] with K % 128 == 0, scale fp16 [N, K/128]; INT8: W
// int8 [N, K], scale fp32 [N]; x fp16 [K]; all contiguous, on W's device).
bool inputs_ok(int kind, const at::Tensor& W, const at::Tensor& s, const at::Tensor& x,
               int64_t& N, int64_t& K) {
    if (!W.is_cuda() || W.dim() != 2 || !W.is_contiguous()) return false;
    N = W.size(0);
    const int64_t cols = W.size(1);
    if (N <= 0 || cols <= 0) return false;
    const c10::DeviceIndex d = W.get_device();
    if (kind == kInt4) {
        if (W.scalar_type() != at::kByte || cols % 64 != 0) return false;
        K = 2 * cols;
        if (s.scalar_type() != at::kHalf || s.dim() != 2 || s.size(0) != N || s.size(1) != cols / 64)
            return false;
    } else {
        if (W.scalar_type() != at::kChar) return false;
        K = cols;
        if (s.scalar_type() != at::kFloat || s.dim() != 1 || s.size(0) != N) return false;
    }
    return s.is_contiguous() && on(s, d) && x.scalar_type() == at::kHalf && x.dim() == 1 &&
           x.size(0) == K && x.is_contiguous() && on(x, d);
}

int launch(int kind, const std::string& variant, const at::Tensor& W, const at::Tensor& s,
           const at::Tensor& x, const at::Tensor& out, int64_t N, int64_t K, uint32_t flags) {
    const c10::DeviceIndex d = W.get_device();
    c10::cuda::OptionalCUDAGuard guard;
    if (c10::cuda::current_device() != d) guard.set_index(d);
    void* st = c10::cuda::getCurrentCUDAStream(d).stream();
    if (kind == kInt4)
        return cl_int4gemv_ex(variant.c_str(), static_cast<const uint8_t*>(W.data_ptr()),
                              s.data_ptr(), x.data_ptr(), out.data_ptr(), N, K, st, flags);
    return cl_qgemv_ex(variant.c_str(), static_cast<const int8_t*>(W.data_ptr()),
                       static_cast<const float*>(s.data_ptr()), x.data_ptr(), out.data_ptr(), N, K,
                       st, flags);
}

// 0 on success; kNotFast or the C ABI's status otherwise (nothing raised).
int forward_into(int kind, const std::string& variant, const at::Tensor& W, const at::Tensor& s,
                 const at::Tensor& x, const at::Tensor& out, int64_t flags) {
    int64_t N = 0, K = 0;
    if (!inputs_ok(kind, W, s, x, N, K)) return kNotFast;
    if (out.scalar_type() != at::kHalf || out.dim() != 1 || out.size(0) != N ||
        !out.is_contiguous() || !on(out, W.get_device()))
        return kNotFast;
    return launch(kind, variant, W, s, x, out, N, K, static_cast<uint32_t>(flags));
}

// The output tensor on success; None otherwise (nothing raised).
c10::optional<at::Tensor> forward(int kind, const std::string& variant, const at::Tensor& W,
                                  const at::Tensor& s, const at::Tensor& x, int64_t flags) {
    int64_t N = 0, K = 0;
    if (!inputs_ok(kind, W, s, x, N, K)) return c10::nullopt;
    at::Tensor out = at::empty({N}, x.options());
    if (launch(kind, variant, W, s, x, out, N, K, static_cast<uint32_t>(flags)) != CL_OK)
        return c10::nullopt;
    return out;
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
    m.attr("NOT_FAST") = kNotFast;
    m.def("forward_into", &forward_into, "checked GEMV into `out` (0 on success)");
    m.def("forward", &forward, "checked GEMV into a new tensor (None when not taken)");
}
