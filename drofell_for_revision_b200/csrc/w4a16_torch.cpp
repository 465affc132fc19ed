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

int dtype_of(const at::Tensor& x) {
    const int dtype = x.scalar_type() == at::kHalf       ? W4A16_DTYPE_FP16
                      : x.scalar_type() == at::kBFloat16 ? W4A16_DTYPE_BF16
                                                         : -1;
    TORCH_CHECK(dtype >= 0, "x must be float16 or bfloat16");
    return dtype;
}

// The handle's workspace of at least `need` bytes on x's device (nullptr for 0), grown
// by doubling; an outgrown one stays alive for the graphs that captured it.
void* workspace(uintptr_t handle, size_t need, const at::Tensor& x, size_t* bytes) {
    *bytes = 0;
    if (need == 0) return nullptr;
    std::lock_guard<std::mutex> lock(g_mu);
    Workspaces& w = g_ws[handle];
    if (!w.current.defined() || static_cast<size_t>(w.current.numel()) < need) {
        const int64_t size = w.current.defined() ? std::max<int64_t>(need, 2 * w.current.numel()) : need;
        if (w.current.defined()) w.retired.push_back(w.current);
        w.current = at::empty({size}, x.options().dtype(at::kByte));
    }
    *bytes = static_cast<size_t>(w.current.numel());
    return w.current.data_ptr();
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
    const int dtype = dtype_of(x);
    const at::Tensor x2 = x.reshape({-1, K}).contiguous();
    const int64_t M = x2.size(0);
    std::vector<int64_t> out_shape(x.sizes().begin(), x.sizes().end());
    out_shape.back() = N;
    at::Tensor out = at::empty(out_shape, x.options());
    if (M == 0) return out;
    const c10::cuda::CUDAGuard guard(x.device());
    size_t ws_bytes = 0;
    void* ws_ptr = workspace(handle, w4a16_workspace_size(h, static_cast<int>(M), dtype, W4A16_PATH_AUTO), x,
                             &ws_bytes);
    const cudaStream_t stream = c10::cuda::getCurrentCUDAStream(x.device().index()).stream();
    check(w4a16_gemm(h, x2.data_ptr(), static_cast<int>(M), out.data_ptr(), dtype, ws_ptr, ws_bytes,
                     W4A16_PATH_AUTO, stream));
    if (bias.has_value() && bias->defined()) out.add_(*bias);
    return out;
}

// The fused all-gather forward of a column-sharded linear: this rank's columns of
// X[M, K] W into columns [col0, col0 + N) of every rank's full Y[M, ld]
// (w4a16_gemm_gather). y_all is the address of a host array of the world's Y pointers
// that the caller keeps alive (built once per output buffer), so a call converts no
// Python objects besides x.
void gemm_gather(uintptr_t handle, uintptr_t comm, const at::Tensor& x, uintptr_t y_all, int64_t ld, int64_t col0) {
    auto* h = reinterpret_cast<w4a16_matrix*>(handle);
    TORCH_CHECK(h != nullptr, "released q4 handle");
    TORCH_CHECK(comm != 0 && y_all != 0, "the gather needs a comm and the ranks' Y pointers");
    int info[4];
    check(w4a16_info(h, info));
    TORCH_CHECK(x.is_cuda() && x.dim() == 2 && x.size(1) == info[0] && x.is_contiguous(),
                "x must be a contiguous CUDA [M, K] tensor");
    const int dtype = dtype_of(x);
    const int M = static_cast<int>(x.size(0));
    if (M == 0) return;
    const c10::cuda::CUDAGuard guard(x.device());
    size_t ws_bytes = 0;
    void* ws_ptr = workspace(handle, w4a16_workspace_size(h, M, dtype, W4A16_PATH_AUTO), x, &ws_bytes);
    const cudaStream_t stream = c10::cuda::getCurrentCUDAStream(x.device().index()).stream();
    check(w4a16_gemm_gather(h, reinterpret_cast<w4a16_comm*>(comm), x.data_ptr(), M,
                            reinterpret_cast<void* const*>(y_all), static_cast<int>(ld), static_cast<int>(col0),
                            dtype, ws_ptr, ws_bytes, stream));
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
    m.def("gemm_gather", &gemm_gather, "this rank's columns of X W into every rank's Y (w4a16_gemm_gather)",
          pybind11::arg("handle"), pybind11::arg("comm"), pybind11::arg("x"), pybind11::arg("y_all"),
          pybind11::arg("ld"), pybind11::arg("col0"));
    m.def("release", &release, "free the workspaces kept for a handle");
}
