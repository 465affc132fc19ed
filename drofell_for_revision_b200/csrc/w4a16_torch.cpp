// Torch-facing fast path of the quantized linear's forward: one C++ call that takes the
// activation tensor, allocates the output from torch's caching allocator and calls
// w4a16_gemm on torch's current stream. The same call through ctypes costs several
// microseconds of Python argument checking and conversion per projection, which at
// decode sizes is as long as the kernel itself (the reference binds its extension with
// pybind11 for the same reason, After-Revision-DROFELL/cuda_extends/exllama/entry.cpp:
// 221-251,601-623).
//
// Workspaces (act-order X gather, split-K partials) are per handle, grown on demand and
// never freed before w4a16_torch_release: a CUDA graph captured with one still writes
// into it on replay.
#include <ATen/ATen.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <torch/csrc/utils/pybind.h>

#include <mutex>
#include <string>
#include <unordered_map>
#include <vector>

#include "../../include/drofell_w4a16.h"

namespace {

struct Workspaces {
    at::Tensor current;
    std::vector<at::Tensor> retired;  // outgrown, kept alive for graphs that captured them
};

std::mutex g_mu;
std::unordered_map<uintptr_t, Workspaces> g_ws;

void check(int rc) {
    if (rc != W4A16_OK) TORCH_CHECK(false, "[w4a16 error ", rc, "] ", w4a16_last_error());
}

// Y[..., N] = X[..., K] W (+ bias): the forward of QuantLinear for any M on PATH_AUTO.
at::Tensor linear(uintptr_t handle, const at::Tensor& x, const c10::optional<at::Tensor>& bias) {
    auto* h = reinterpret_cast<w4a16_matrix*>(handle);
    TORCH_CHECK(h != nullptr, "released q4 handle");
    int info[4];
    check(w4a16_info(h, info));
    const int64_t K = info[0], N = info[1];
    TORCH_CHECK(x.is_cuda(), "x must be a CUDA tensor (no CPU path exists)");
    TORCH_CHECK(x.size(-1) == K, "x and w have incompatible shapes");
    const int dtype = x.scalar_type() == at::kHalf       ? W4A16_DTYPE_FP16
                      : x.scalar_type() == at::kBFloat16 ? W4A16_DTYPE_BF16
                                                         : -1;
    TORCH_CHECK(dtype >= 0, "x must be float16 or bfloat16");
    const at::Tensor x2 = x.reshape({-1, K}).contiguous();
    const int64_t M = x2.size(0);
    std::vector<int64_t> out_shape(x.sizes().begin(), x.sizes().end());
    out_shape.back() = N;
    at::Tensor out = at::empty(out_shape, x.options());
    if (M == 0) return out;
    const c10::cuda::CUDAGuard guard(x.device());
    void* ws_ptr = nullptr;
    size_t ws_bytes = 0;
    const size_t need = w4a16_workspace_size(h, static_cast<int>(M), dtype, W4A16_PATH_AUTO);
    if (need > 0) {
        std::lock_guard<std::mutex> lock(g_mu);
        Workspaces& w = g_ws[handle];
        if (!w.current.defined() || static_cast<size_t>(w.current.numel()) < need) {
            const int64_t size = w.current.defined() ? std::max<int64_t>(need, 2 * w.current.numel()) : need;
            if (w.current.defined()) w.retired.push_back(w.current);
            w.current = at::empty({size}, x.options().dtype(at::kByte));
        }
        ws_ptr = w.current.data_ptr();
        ws_bytes = static_cast<size_t>(w.current.numel());
    }
    const cudaStream_t stream = c10::cuda::getCurrentCUDAStream(x.device().index()).stream();
    check(w4a16_gemm(h, x2.data_ptr(), static_cast<int>(M), out.data_ptr(), dtype, ws_ptr, ws_bytes,
                     W4A16_PATH_AUTO, stream));
    if (bias.has_value() && bias->defined()) out.add_(*bias);
    return out;
}

// Drop a handle's workspaces (call before w4a16_destroy; graphs that used them must be
// released first).
void release(uintptr_t handle) {
    std::lock_guard<std::mutex> lock(g_mu);
    g_ws.erase(handle);
}

}  // namespace

PYBIND11_MODULE(_w4a16_torch, m) {
    m.doc() = "torch fast path of the W4A16 quantized linear (calls the C ABI of libdrofell_w4a16.so)";
    m.def("linear", &linear, "Y = X W (+ bias) on PATH_AUTO", pybind11::arg("handle"), pybind11::arg("x"),
          pybind11::arg("bias") = pybind11::none());
    m.def("release", &release, "free the workspaces kept for a handle");
}
