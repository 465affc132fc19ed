// C ABI of the W4A16 library: handle construction (act-order preprocessing),
// argument validation, path dispatch and error reporting.
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/drofell_w4a16.h"
#include "w4a16_gather.cuh"
#include "w4a16_internal.h"

using namespace w4a16;

struct w4a16_matrix {
    PackedWeight pw;
    int device = 0;
    int num_sms = 148;
    int32_t* g_idx_dev = nullptr;
    int32_t* perm_dev = nullptr;      // [K] kernel row -> original row (-1 on pad rows)
    int32_t* inv_perm_dev = nullptr;  // [K_in] original row -> kernel row
    int32_t* qweight_sorted = nullptr;
    int32_t* qzeros_copy = nullptr;  // 16-byte aligned copy of a caller's qzeros that is not (bulk-copy source)
    int32_t* qw_mma = nullptr;  // weight repacked into mma.sync fragment order (GEMV)
    int gemv_mma_min_m = 3;     // smallest M the repacked-weight GEMV takes (CUDA cores below)
    int* err_dev = nullptr;
    CUtensorMap qw_map;    // box [8 rows x 128 columns] (forward GEMM)
    CUtensorMap qw_map_t;  // box [16 rows x 64 columns] (transposed GEMM)
};

namespace {

thread_local std::string g_last_error;
constexpr int kGemvMaxM = 16;  // rows the GEMV family takes under PATH_AUTO (exact-W tcgen05 GEMM above)

int fail(int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return code;
}

int cuda_fail(cudaError_t e, const char* what) {
    return fail(W4A16_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}

bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// Device whose primary context this thread has made current through cudaSetDevice.
// A thread that never called it (a worker such as autograd's backward thread) reports
// device 0 from cudaGetDevice but has no current context yet, and driver entry points
// (cuTensorMapEncodeTiled) then fail with CUDA_ERROR_INVALID_CONTEXT.
thread_local int t_bound_device = -1;

// Switches to `dev` for the scope, with its context current, and restores the caller's
// device afterwards (the reference calls cudaSetDevice and leaves it changed,
// q4_matmul.cu:248,476).
struct DeviceGuard {
    int prev = -1;
    bool ok = true;
    explicit DeviceGuard(int dev) {
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
        if (prev != dev || t_bound_device != dev) {
            ok = cudaSetDevice(dev) == cudaSuccess;
            if (ok) t_bound_device = dev;
        }
    }
    ~DeviceGuard() {
        int cur = -1;
        if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev && cudaSetDevice(prev) == cudaSuccess)
            t_bound_device = prev;
    }
};

PFN_cuTensorMapEncodeTiled_v12000 get_encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

void free_owned(w4a16_matrix* h) {
    cudaFree(h->g_idx_dev);
    cudaFree(h->perm_dev);
    cudaFree(h->inv_perm_dev);
    h->inv_perm_dev = nullptr;
    cudaFree(h->qweight_sorted);
    cudaFree(h->qzeros_copy);
    h->qzeros_copy = nullptr;
    cudaFree(h->qw_mma);
    h->qw_mma = nullptr;
    cudaFree(h->err_dev);
    h->g_idx_dev = h->perm_dev = h->qweight_sorted = nullptr;
    h->err_dev = nullptr;
}

int check_dtype(int dtype) {
    if (dtype != W4A16_DTYPE_FP16 && dtype != W4A16_DTYPE_BF16) return fail(W4A16_ERR_INVALID, "unknown dtype %d", dtype);
    return W4A16_OK;
}

// Kernel family actually launched: the CUDA-core GEMV, the exact-W tensor-core GEMM, or
// the GEMV on the handle's repacked weight (mma.sync). Family 2 (a tcgen05 decode pass)
// was retired: it never beat the GEMV on the decode sizes.
enum Kernel { kKernGemv = 1, kKernExact = 3, kKernGemvMma = 4 };

size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// What kernel selection and planning depend on: the packed shape (no device
// pointers), whether the handle holds the mma.sync repacked copy, and the SM count.
struct Shape {
    PackedWeight pw;
    bool has_repack = false;
    int gemv_mma_min_m = 3;  // smallest M the repacked-weight GEMV takes (CUDA cores below)
    int num_sms = 148;
};

Shape shape_of(const w4a16_matrix* h) {
    Shape sh;
    sh.pw = h->pw;
    sh.has_repack = h->qw_mma != nullptr;
    sh.gemv_mma_min_m = h->gemv_mma_min_m;
    sh.num_sms = h->num_sms;
    return sh;
}

int resolve_kernel(const Shape& sh, int M, int dtype, int path) {
    (void)dtype;
    // the GEMV family: mma.sync on the repacked weight from gemv_mma_min_m rows (measured:
    // it wins from M = 3; the CUDA-core kernel wins at M = 1, 2 up to K = 4096, where it
    // runs its WIDE configuration). Wide weights past that K stream faster through the
    // mma.sync kernel at every M (B200, M = 1: 8192 x 57344 53.2 vs 61.4 us, 8192 x 10240
    // 14.8 vs 15.7, 8192 x 8192 11.2 vs 11.9, 28672 x 8192 30.7 vs 30.8, 5120 x 27648
    // 19.5 vs 21.6; the other way round: 5120 x 15360 13.2 vs 13.0, 5120 x 5120 7.3 vs
    // 7.2, and every 7B shape, K = 4096 or 11008 with N <= 22016)
    const bool wide_long = (sh.pw.K >= 8192 && sh.pw.N >= 8192) || (sh.pw.K > 4096 && sh.pw.N >= 16384);
    const bool use_mma = sh.has_repack && (M >= sh.gemv_mma_min_m || wide_long || !gemv_supported(sh.pw));
    const int gemv = use_mma ? kKernGemvMma : kKernGemv;
    switch (path) {
        case W4A16_PATH_GEMV: return gemv;
        case W4A16_PATH_TC:
        case W4A16_PATH_TC_EXACT: return kKernExact;
        default: break;
    }
    static const int gemv_max_m = [] {
        const char* v = std::getenv("W4A16_GEMV_MAX_M");  // tuning override
        return v ? std::atoi(v) : kGemvMaxM;
    }();
    if (M <= gemv_max_m && (sh.has_repack || gemv_supported(sh.pw))) {
        // 9..16 rows whose staged X does not fit one pass of the mma.sync GEMV (very long K):
        // two passes over the weight cost more than one natural-orientation GEMM
        if (gemv == kKernGemvMma && M > 8 && plan_gemv_mma(sh.pw, M, sh.num_sms).mt < M) return kKernExact;
        return gemv;
    }
    return kKernExact;
}
int resolve_kernel(const w4a16_matrix* h, int M, int dtype, int path) { return resolve_kernel(shape_of(h), M, dtype, path); }

// out[0..3] as documented for w4a16_plan; out[4] bit 0: the CUDA-core GEMV runs its WIDE
// configuration, bit 1: the tcgen05 GEMM runs in the natural orientation
void plan_of(const Shape& sh, int M, int dtype, int path, int out[5]) {
    const int k = resolve_kernel(sh, M, dtype, path);
    out[0] = k;
    out[4] = 0;
    if (k == kKernGemv) {
        const GemvPlan gp = plan_gemv(sh.pw, M < 8 ? M : 8, sh.num_sms);
        out[1] = gp.bn;
        out[2] = gp.splits;
        out[3] = gp.mt;
        out[4] = gp.wide ? 1 : 0;
    } else if (k == kKernGemvMma) {
        const GemvPlan gp = plan_gemv_mma(sh.pw, M < kGemvMmaMaxTok ? M : kGemvMmaMaxTok, sh.num_sms);
        out[1] = gp.bn;
        out[2] = gp.splits;
        out[3] = gp.mt;
    } else {
        const TcPlan tp = plan_tc(sh.pw, M, sh.num_sms);
        out[1] = tp.bn;
        out[2] = tp.splits;
        out[3] = tp.cps;
        out[4] = tp.ns ? 2 : 0;
    }
}

size_t workspace_of(const Shape& sh, int M, int dtype, int path) {
    if (M <= 0) return 0;
    const int k = resolve_kernel(sh, M, dtype, path);
    const size_t gather = sh.pw.act_order ? align_up(static_cast<size_t>(M) * sh.pw.K * 2, 256) : 0;
    if (k == kKernGemv || k == kKernGemvMma) return gather;
    const TcPlan tp = plan_tc(sh.pw, M, sh.num_sms);
    return gather + tc_workspace_bytes(sh.pw, tp, M);
}


}  // namespace

namespace w4a16 {

CUresult encode_tmap_2d(CUtensorMap* map, CUtensorMapDataType dtype, const void* base, uint64_t inner,
                        uint64_t outer, uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer,
                        CUtensorMapSwizzle swizzle) {
    auto fn = get_encode_fn();
    if (!fn) return CUDA_ERROR_NOT_FOUND;
    cuuint64_t dims[2] = {inner, outer};
    cuuint64_t strides[1] = {row_stride_bytes};
    cuuint32_t box[2] = {box_inner, box_outer};
    cuuint32_t estr[2] = {1, 1};
    return fn(map, dtype, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
}

CUresult encode_tmap_3d(CUtensorMap* map, CUtensorMapDataType dtype, const void* base, const uint64_t dims[3],
                        const uint64_t strides_bytes[2], const uint32_t box[3], CUtensorMapSwizzle swizzle) {
    auto fn = get_encode_fn();
    if (!fn) return CUDA_ERROR_NOT_FOUND;
    cuuint64_t d[3] = {dims[0], dims[1], dims[2]};
    cuuint64_t st[2] = {strides_bytes[0], strides_bytes[1]};
    cuuint32_t b[3] = {box[0], box[1], box[2]};
    cuuint32_t estr[3] = {1, 1, 1};
    return fn(map, dtype, 3, const_cast<void*>(base), d, st, b, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
}

}  // namespace w4a16

extern "C" {

int w4a16_version(void) { return 101; }

const char* w4a16_last_error(void) { return g_last_error.c_str(); }

}  // extern "C"

namespace {

int create_impl(const int32_t* qweight_dev, const int32_t* qzeros_dev, const uint16_t* scales_dev,
                const int32_t* g_idx_host, int K, int N, int groups, int device, int flags, void* stream,
                w4a16_matrix** out) {
    g_last_error.clear();
    if (!out) return fail(W4A16_ERR_INVALID, "out handle pointer is null");
    *out = nullptr;
    if (!qweight_dev || !qzeros_dev || !scales_dev) return fail(W4A16_ERR_INVALID, "null qweight/qzeros/scales");
    if (K <= 0 || N <= 0 || K % 32 != 0 || N % 32 != 0)
        return fail(W4A16_ERR_INVALID, "K=%d N=%d: both must be positive multiples of 32", K, N);
    if (groups <= 0 || K % groups != 0) return fail(W4A16_ERR_INVALID, "groups=%d must divide K=%d", groups, K);
    const int gs = K / groups;
    if (gs % 8 != 0) return fail(W4A16_ERR_UNSUPPORTED, "group size %d is not a multiple of 8", gs);
    if (!aligned(qweight_dev, 16) || !aligned(scales_dev, 16) || !aligned(qzeros_dev, 4))
        return fail(W4A16_ERR_INVALID, "qweight and scales must be 16-byte aligned, qzeros 4-byte aligned");
    if (flags & ~W4A16_CREATE_NO_REPACK) return fail(W4A16_ERR_INVALID, "unknown flags %#x", flags);

    DeviceGuard guard(device);
    if (!guard.ok) return fail(W4A16_ERR_CUDA, "cudaSetDevice(%d) failed", device);
    cudaStream_t s = static_cast<cudaStream_t>(stream);

    auto* h = new w4a16_matrix();
    h->device = device;
    cudaDeviceGetAttribute(&h->num_sms, cudaDevAttrMultiProcessorCount, device);
    PackedWeight& w = h->pw;
    w.K = K;
    w.K_in = K;
    w.N = N;
    w.G = groups;
    w.group_size = gs;
    w.qweight = qweight_dev;
    w.qweight_orig = qweight_dev;
    w.qzeros = qzeros_dev;
    w.scales = scales_dev;

    cudaError_t e;
    auto bail = [&](int code) {
        free_owned(h);
        delete h;
        return code;
    };

    {
        // symmetric quantization (every zero nibble 7): the kernels skip the zero rows
        std::vector<int32_t> zh(static_cast<size_t>(groups) * (N / 8));
        if ((e = cudaMemcpyAsync(zh.data(), qzeros_dev, zh.size() * sizeof(int32_t), cudaMemcpyDeviceToHost, s)) !=
                cudaSuccess ||
            (e = cudaStreamSynchronize(s)) != cudaSuccess)
            return bail(cuda_fail(e, "qzeros read"));
        bool sym = true;
        for (int32_t z : zh) sym = sym && static_cast<uint32_t>(z) == kSymmetricZeroWord;
        w.symmetric = sym;
        // the tcgen05 GEMMs bulk-copy zero rows, which needs a 16-byte aligned source
        if (!sym && !aligned(qzeros_dev, 16)) {
            if ((e = cudaMalloc(&h->qzeros_copy, zh.size() * sizeof(int32_t))) != cudaSuccess ||
                (e = cudaMemcpyAsync(h->qzeros_copy, zh.data(), zh.size() * sizeof(int32_t), cudaMemcpyHostToDevice,
                                     s)) != cudaSuccess ||
                (e = cudaStreamSynchronize(s)) != cudaSuccess)
                return bail(cuda_fail(e, "aligned qzeros copy"));
            w.qzeros = h->qzeros_copy;
        }
    }
    if ((e = cudaMalloc(&h->err_dev, sizeof(int))) != cudaSuccess) return bail(cuda_fail(e, "cudaMalloc err"));
    if ((e = cudaMemsetAsync(h->err_dev, 0, sizeof(int), s)) != cudaSuccess)
        return bail(cuda_fail(e, "cudaMemsetAsync"));
    w.err = h->err_dev;

    if (g_idx_host) {
        // Stable counting sort of rows by group (the x_map of q4_matrix.cu:125-176). The
        // kernels find a row's group arithmetically (kernel row / group size). GPTQ gives
        // every group exactly K/groups rows; any other table gets each group padded to
        // the longest one (rounded up to 32 rows) with zero weight rows whose X is 0.
        std::vector<int> count(groups, 0);
        for (int k = 0; k < K; ++k) {
            const int g = g_idx_host[k];
            if (g < 0 || g >= groups) return bail(fail(W4A16_ERR_INVALID, "g_idx[%d]=%d outside [0, %d)", k, g, groups));
            ++count[g];
        }
        int longest = 0;
        bool equal = true;
        for (int g = 0; g < groups; ++g) {
            longest = count[g] > longest ? count[g] : longest;
            equal = equal && count[g] == gs;
        }
        const int gs_k = equal ? gs : (longest + 31) / 32 * 32;  // kernel group size
        const long long K_k = static_cast<long long>(gs_k) * groups;
        if (K_k > (1LL << 30)) return bail(fail(W4A16_ERR_UNSUPPORTED, "padded act-order K too large"));
        std::vector<int32_t> perm(static_cast<size_t>(K_k), -1);
        std::vector<int32_t> inv(K);
        std::vector<int> next(groups);
        for (int g = 0; g < groups; ++g) next[g] = g * gs_k;
        for (int k = 0; k < K; ++k) {
            const int j = next[g_idx_host[k]]++;
            perm[j] = k;
            inv[k] = j;
        }
        w.act_order = true;
        w.K = static_cast<int>(K_k);
        w.group_size = gs_k;
        if ((e = cudaMalloc(&h->g_idx_dev, K * sizeof(int32_t))) != cudaSuccess ||
            (e = cudaMalloc(&h->perm_dev, K_k * sizeof(int32_t))) != cudaSuccess ||
            (e = cudaMalloc(&h->inv_perm_dev, K * sizeof(int32_t))) != cudaSuccess ||
            (e = cudaMalloc(&h->qweight_sorted, static_cast<size_t>(K_k / 8) * N * sizeof(int32_t))) != cudaSuccess)
            return bail(cuda_fail(e, "cudaMalloc act-order buffers"));
        if ((e = cudaMemcpyAsync(h->g_idx_dev, g_idx_host, K * sizeof(int32_t), cudaMemcpyHostToDevice, s)) != cudaSuccess ||
            (e = cudaMemcpyAsync(h->perm_dev, perm.data(), K_k * sizeof(int32_t), cudaMemcpyHostToDevice, s)) != cudaSuccess ||
            (e = cudaMemcpyAsync(h->inv_perm_dev, inv.data(), K * sizeof(int32_t), cudaMemcpyHostToDevice, s)) != cudaSuccess)
            return bail(cuda_fail(e, "cudaMemcpyAsync act-order tables"));
        if ((e = launch_sort_rows(qweight_dev, h->qweight_sorted, h->perm_dev, w.K, N, s)) != cudaSuccess)
            return bail(cuda_fail(e, "sort_rows launch"));
        // The host vectors die at return: finish the copies first (one-time set-up).
        if ((e = cudaStreamSynchronize(s)) != cudaSuccess) return bail(cuda_fail(e, "cudaStreamSynchronize"));
        w.g_idx = h->g_idx_dev;
        w.perm = h->perm_dev;
        w.inv_perm = h->inv_perm_dev;
        w.qweight = h->qweight_sorted;
    } else {
        if ((e = cudaStreamSynchronize(s)) != cudaSuccess) return bail(cuda_fail(e, "cudaStreamSynchronize"));
    }

    if (encode_tmap_2d(&h->qw_map, CU_TENSOR_MAP_DATA_TYPE_INT32, w.qweight, static_cast<uint64_t>(N),
                       static_cast<uint64_t>(w.K / 8), static_cast<uint64_t>(N) * 4, 128, 8,
                       CU_TENSOR_MAP_SWIZZLE_NONE) != CUDA_SUCCESS ||
        encode_tmap_2d(&h->qw_map_t, CU_TENSOR_MAP_DATA_TYPE_INT32, w.qweight, static_cast<uint64_t>(N),
                       static_cast<uint64_t>(w.K / 8), static_cast<uint64_t>(N) * 4, 64, 16,
                       CU_TENSOR_MAP_SWIZZLE_NONE) != CUDA_SUCCESS)
        return bail(fail(W4A16_ERR_CUDA, "cuTensorMapEncodeTiled(qweight) failed"));
    // The GEMV's own copy of the weight in mma.sync fragment order (same size as
    // qweight), unless the caller opts out (W4A16_CREATE_NO_REPACK, or the environment
    // variable W4A16_NO_REPACK=1 for w4a16_create).
    if (const char* v = std::getenv("W4A16_GEMV_MMA_MIN_M")) h->gemv_mma_min_m = std::atoi(v);  // tuning override
    if (gemv_mma_supported(w) && !(flags & W4A16_CREATE_NO_REPACK)) {
        if ((e = cudaMalloc(&h->qw_mma, repack_mma_words(w) * sizeof(int32_t))) != cudaSuccess)
            return bail(cuda_fail(e, "cudaMalloc repacked weight"));
        if ((e = launch_repack_mma(w, h->qw_mma, s)) != cudaSuccess) return bail(cuda_fail(e, "repack launch"));
        if ((e = cudaStreamSynchronize(s)) != cudaSuccess) return bail(cuda_fail(e, "cudaStreamSynchronize"));
    }
    *out = h;
    return W4A16_OK;
}

int env_create_flags() {
    const char* no_repack = std::getenv("W4A16_NO_REPACK");
    return (no_repack && std::atoi(no_repack) != 0) ? W4A16_CREATE_NO_REPACK : 0;
}

}  // namespace

extern "C" {

int w4a16_create(const int32_t* qweight_dev, const int32_t* qzeros_dev, const uint16_t* scales_dev,
                 const int32_t* g_idx_host, int K, int N, int groups, int device, void* stream,
                 w4a16_matrix** out) {
    return create_impl(qweight_dev, qzeros_dev, scales_dev, g_idx_host, K, N, groups, device, env_create_flags(),
                       stream, out);
}

int w4a16_create_ex(const int32_t* qweight_dev, const int32_t* qzeros_dev, const uint16_t* scales_dev,
                    const int32_t* g_idx_host, int K, int N, int groups, int device, int flags, void* stream,
                    w4a16_matrix** out) {
    return create_impl(qweight_dev, qzeros_dev, scales_dev, g_idx_host, K, N, groups, device, flags, stream, out);
}

int w4a16_destroy(w4a16_matrix* h) {
    if (!h) return W4A16_OK;
    DeviceGuard guard(h->device);
    free_owned(h);
    delete h;
    return W4A16_OK;
}

int w4a16_info(const w4a16_matrix* h, int out[4]) {
    if (!h || !out) return fail(W4A16_ERR_INVALID, "null argument");
    out[0] = h->pw.K_in;
    out[1] = h->pw.N;
    out[2] = h->pw.G;
    out[3] = (h->pw.act_order ? 1 : 0) | (h->pw.symmetric ? 2 : 0);
    return W4A16_OK;
}

int w4a16_dequant(w4a16_matrix* h, void* w_out_dev, int dtype, void* stream) {
    g_last_error.clear();
    if (!h || !w_out_dev) return fail(W4A16_ERR_INVALID, "null argument");
    if (int rc = check_dtype(dtype)) return rc;
    if (!aligned(w_out_dev, 16)) return fail(W4A16_ERR_INVALID, "output must be 16-byte aligned");
    DeviceGuard guard(h->device);
    cudaError_t e = launch_dequant(h->pw, w_out_dev, static_cast<DType>(dtype), static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "dequant launch");
    return W4A16_OK;
}

size_t w4a16_workspace_size(const w4a16_matrix* h, int M, int dtype, int path) {
    if (!h || M <= 0) return 0;
    return workspace_of(shape_of(h), M, dtype, path);
}

int w4a16_plan(const w4a16_matrix* h, int M, int dtype, int path, int out[4]) {
    if (!h || !out || M <= 0) return fail(W4A16_ERR_INVALID, "bad argument");
    int o[5];
    plan_of(shape_of(h), M, dtype, path, o);
    for (int i = 0; i < 4; ++i) out[i] = o[i];
    return W4A16_OK;
}

int w4a16_plan_shape(int K, int N, int groups, int act_order, int M, int dtype, int path, int num_sms, int out[5],
                     size_t* workspace_bytes) {
    g_last_error.clear();
    if (!out || M <= 0 || num_sms <= 0) return fail(W4A16_ERR_INVALID, "bad argument");
    if (int rc = check_dtype(dtype)) return rc;
    if (K <= 0 || N <= 0 || K % 32 != 0 || N % 32 != 0)
        return fail(W4A16_ERR_INVALID, "K=%d N=%d: both must be positive multiples of 32", K, N);
    if (groups <= 0 || K % groups != 0) return fail(W4A16_ERR_INVALID, "groups=%d must divide K=%d", groups, K);
    if ((K / groups) % 8 != 0) return fail(W4A16_ERR_UNSUPPORTED, "group size %d is not a multiple of 8", K / groups);
    Shape sh;
    sh.pw.K = K;
    sh.pw.K_in = K;
    sh.pw.N = N;
    sh.pw.G = groups;
    sh.pw.group_size = K / groups;
    sh.pw.act_order = act_order != 0;
    // as w4a16_create decides it
    const char* no_repack = std::getenv("W4A16_NO_REPACK");
    sh.has_repack = gemv_mma_supported(sh.pw) && !(no_repack && std::atoi(no_repack) != 0);
    if (const char* v = std::getenv("W4A16_GEMV_MMA_MIN_M")) sh.gemv_mma_min_m = std::atoi(v);
    sh.num_sms = num_sms;
    plan_of(sh, M, dtype, path, out);
    if (workspace_bytes) *workspace_bytes = workspace_of(sh, M, dtype, path);
    return W4A16_OK;
}

int w4a16_gemm(w4a16_matrix* h, const void* x_dev, int M, void* y_dev, int dtype, void* workspace_dev,
               size_t workspace_bytes, int path, void* stream) {
    if (!h) return fail(W4A16_ERR_INVALID, "null handle");
    if (int rc = check_dtype(dtype)) return rc;
    if (M < 0) return fail(W4A16_ERR_INVALID, "M=%d", M);
    if (M == 0) return W4A16_OK;
    if (!x_dev || !y_dev) return fail(W4A16_ERR_INVALID, "null x or y");
    if (!aligned(x_dev, 16) || !aligned(y_dev, 16)) return fail(W4A16_ERR_INVALID, "x and y must be 16-byte aligned");
    if (path < W4A16_PATH_AUTO || path > W4A16_PATH_TC_EXACT) return fail(W4A16_ERR_INVALID, "unknown path %d", path);
    const int k = resolve_kernel(h, M, dtype, path);
    DeviceGuard guard(h->device);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    cudaError_t e = cudaSuccess;
    if (k == kKernGemv && !gemv_supported(h->pw))
        return fail(W4A16_ERR_UNSUPPORTED, "the GEMV path needs whole packed rows per group and N %% 4 == 0");
    const size_t need = w4a16_workspace_size(h, M, dtype, path);
    if (workspace_bytes < need || (need > 0 && !workspace_dev))
        return fail(W4A16_ERR_WORKSPACE, "workspace %zu bytes < %zu needed for M=%d", workspace_bytes, need, M);
    if (need > 0 && !aligned(workspace_dev, 256)) return fail(W4A16_ERR_INVALID, "workspace must be 256-byte aligned");
    if (k == kKernGemvMma) {
        const void* xin = x_dev;
        if (h->pw.act_order) {  // X columns into kernel row order
            e = launch_remap_cols(x_dev, h->pw.K_in, workspace_dev, h->pw.K, h->pw.perm, M, h->pw.K, s);
            if (e != cudaSuccess) return cuda_fail(e, "act-order gather launch");
            xin = workspace_dev;
        }
        for (int m0 = 0; m0 < M && e == cudaSuccess;) {
            const GemvPlan gp = plan_gemv_mma(h->pw, (M - m0) < kGemvMmaMaxTok ? (M - m0) : kGemvMmaMaxTok, h->num_sms);
            const int mm = gp.mt;
            e = launch_gemv_mma(h->pw, h->qw_mma, gp, static_cast<const uint16_t*>(xin) + static_cast<size_t>(m0) * h->pw.K,
                                mm, static_cast<uint16_t*>(y_dev) + static_cast<size_t>(m0) * h->pw.N,
                                static_cast<DType>(dtype), s);
            m0 += mm;
        }
        if (e != cudaSuccess) return cuda_fail(e, "gemv (repacked) launch");
        return W4A16_OK;
    }
    if (k == kKernGemv) {
        const void* xin = x_dev;
        if (h->pw.act_order) {  // X columns into kernel row order
            e = launch_remap_cols(x_dev, h->pw.K_in, workspace_dev, h->pw.K, h->pw.perm, M, h->pw.K, s);
            if (e != cudaSuccess) return cuda_fail(e, "act-order gather launch");
            xin = workspace_dev;
        }
        for (int m0 = 0; m0 < M && e == cudaSuccess;) {
            const GemvPlan gp = plan_gemv(h->pw, M - m0 < 8 ? M - m0 : 8, h->num_sms);
            const int mm = (M - m0) < gp.mt ? (M - m0) : gp.mt;
            e = launch_gemv(h->pw, gp, static_cast<const uint16_t*>(xin) + static_cast<size_t>(m0) * h->pw.K, mm,
                            static_cast<uint16_t*>(y_dev) + static_cast<size_t>(m0) * h->pw.N,
                            static_cast<DType>(dtype), s);
            m0 += mm;
        }
        if (e != cudaSuccess) return cuda_fail(e, "gemv launch");
        return W4A16_OK;
    }
    const TcPlan tp = plan_tc(h->pw, M, h->num_sms);
    const void* xin = x_dev;
    uint8_t* ws = static_cast<uint8_t*>(workspace_dev);
    size_t ws_left = workspace_bytes;
    if (h->pw.act_order) {
        e = launch_remap_cols(x_dev, h->pw.K_in, ws, h->pw.K, h->pw.perm, M, h->pw.K, s);
        if (e != cudaSuccess) return cuda_fail(e, "gather launch");
        xin = ws;
        const size_t used = align_up(static_cast<size_t>(M) * h->pw.K * 2, 256);
        ws += used;
        ws_left -= used;
    }
    e = launch_tc(h->pw, tp, &h->qw_map, xin, M, y_dev, static_cast<DType>(dtype), ws, ws_left, s);
    if (e != cudaSuccess) return cuda_fail(e, "tcgen05 gemm launch");
    return W4A16_OK;
}

size_t w4a16_workspace_size_t(const w4a16_matrix* h, int M, int dtype) {
    (void)dtype;
    if (!h || M <= 0) return 0;
    const size_t sorted = h->pw.act_order ? align_up(static_cast<size_t>(M) * h->pw.K * 2, 256) : 0;
    return sorted + tc_t_workspace_bytes(h->pw, plan_tc_t(h->pw, M, h->num_sms), M);
}

int w4a16_gemm_t(w4a16_matrix* h, const void* dy_dev, int M, void* dx_dev, int dtype, void* workspace_dev,
                 size_t workspace_bytes, void* stream) {
    if (!h) return fail(W4A16_ERR_INVALID, "null handle");
    if (int rc = check_dtype(dtype)) return rc;
    if (M < 0) return fail(W4A16_ERR_INVALID, "M=%d", M);
    if (M == 0) return W4A16_OK;
    if (!dy_dev || !dx_dev) return fail(W4A16_ERR_INVALID, "null dy or dx");
    if (!aligned(dy_dev, 16) || !aligned(dx_dev, 16)) return fail(W4A16_ERR_INVALID, "dy and dx must be 16-byte aligned");
    const size_t need = w4a16_workspace_size_t(h, M, dtype);
    if (workspace_bytes < need || (need > 0 && !workspace_dev))
        return fail(W4A16_ERR_WORKSPACE, "workspace %zu bytes < %zu needed for M=%d", workspace_bytes, need, M);
    if (need > 0 && !aligned(workspace_dev, 256)) return fail(W4A16_ERR_INVALID, "workspace must be 256-byte aligned");
    DeviceGuard guard(h->device);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const TcPlan tp = plan_tc_t(h->pw, M, h->num_sms);
    uint8_t* ws = static_cast<uint8_t*>(workspace_dev);
    size_t ws_left = workspace_bytes;
    void* out = dx_dev;
    if (h->pw.act_order) {  // dX in kernel row order first, then back to the caller's rows
        out = ws;
        const size_t used = align_up(static_cast<size_t>(M) * h->pw.K * 2, 256);
        ws += used;
        ws_left -= used;
    }
    cudaError_t e = launch_tc_t(h->pw, tp, &h->qw_map_t, dy_dev, M, out, static_cast<DType>(dtype), ws, ws_left, s);
    if (e != cudaSuccess) return cuda_fail(e, "tcgen05 transposed gemm launch");
    if (h->pw.act_order) {
        e = launch_remap_cols(out, h->pw.K, dx_dev, h->pw.K_in, h->pw.inv_perm, M, h->pw.K_in, s);
        if (e != cudaSuccess) return cuda_fail(e, "act-order row restore launch");
    }
    return W4A16_OK;
}

int w4a16_rms_norm(const void* x_dev, const void* w_dev, float eps, int M, int K, void* y_dev, int dtype, void* stream) {
    if (dtype != W4A16_DTYPE_FP16) return fail(W4A16_ERR_UNSUPPORTED, "RMSNorm is fp16 (the reference's rms_norm_cuda)");
    if (M < 0 || K <= 0 || K % 8 != 0) return fail(W4A16_ERR_INVALID, "M=%d K=%d (K a positive multiple of 8)", M, K);
    if (!x_dev || !w_dev || !y_dev || !aligned(x_dev, 16) || !aligned(w_dev, 16) || !aligned(y_dev, 16))
        return fail(W4A16_ERR_INVALID, "x, w and y must be non-null and 16-byte aligned");
    const cudaError_t e = launch_rms_norm(x_dev, w_dev, eps, M, K, y_dev, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? W4A16_OK : cuda_fail(e, "rms_norm launch");
}

int w4a16_silu_mul(const void* gate_dev, const void* up_dev, int M, int N, void* out_dev, int dtype, void* stream) {
    if (dtype != W4A16_DTYPE_FP16) return fail(W4A16_ERR_UNSUPPORTED, "silu_mul is fp16 (the reference's silu_mul_kernel)");
    if (M < 0 || N <= 0 || N % 8 != 0) return fail(W4A16_ERR_INVALID, "M=%d N=%d (N a positive multiple of 8)", M, N);
    if (!gate_dev || !up_dev || !out_dev || !aligned(gate_dev, 16) || !aligned(up_dev, 16) || !aligned(out_dev, 16))
        return fail(W4A16_ERR_INVALID, "gate, up and out must be non-null and 16-byte aligned");
    const cudaError_t e = launch_silu_mul(gate_dev, up_dev, M, N, out_dev, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? W4A16_OK : cuda_fail(e, "silu_mul launch");
}

}  // extern "C"

namespace {

size_t max3(size_t a, size_t b, size_t c) { return a > b ? (a > c ? a : c) : (b > c ? b : c); }

// The fused decode blocks take the CUDA-core GEMV with an X prologue: fp16, at most two
// rows, weights without act-order (the prologue reads X in the caller's column order),
// and the environment switch W4A16_FUSE=0 not set.
bool fusable(const w4a16_matrix* const* hs, int n, int M, int dtype) {
    if (dtype != W4A16_DTYPE_FP16 || M > 2) return false;
    const char* v = std::getenv("W4A16_FUSE");
    if (v && std::atoi(v) == 0) return false;
    for (int i = 0; i < n; ++i)
        if (hs[i]->pw.act_order || !gemv_supported(hs[i]->pw) || hs[i]->pw.K != hs[0]->pw.K ||
            hs[i]->pw.group_size != hs[0]->pw.group_size || hs[i]->device != hs[0]->device)
            return false;
    return true;
}

}  // namespace

extern "C" {

size_t w4a16_mlp_workspace_size(const w4a16_matrix* gate, const w4a16_matrix* up, const w4a16_matrix* down, int M,
                                int dtype) {
    if (!gate || !up || !down || M <= 0) return 0;
    const w4a16_matrix* hs[2] = {gate, up};
    if (fusable(hs, 2, M, dtype) && fusable(&down, 1, M, dtype)) return 0;
    return max3(w4a16_workspace_size(gate, M, dtype, W4A16_PATH_AUTO), w4a16_workspace_size(up, M, dtype, W4A16_PATH_AUTO),
                w4a16_workspace_size(down, M, dtype, W4A16_PATH_AUTO));
}

int w4a16_mlp_forward(w4a16_matrix* gate, w4a16_matrix* up, w4a16_matrix* down, const void* norm_w_dev, float eps,
                      const void* x_dev, int M, void* y_dev, void* rms_out_dev, void* gate_out_dev, void* up_out_dev,
                      int dtype, void* workspace_dev, size_t workspace_bytes, void* stream) {
    if (!gate || !up || !down) return fail(W4A16_ERR_INVALID, "null handle");
    if (up->device != gate->device || down->device != gate->device)
        return fail(W4A16_ERR_INVALID, "gate, up and down handles on different devices");
    if (dtype != W4A16_DTYPE_FP16) return fail(W4A16_ERR_UNSUPPORTED, "the fused MLP is fp16 (as mlp_forward_v2)");
    if (M < 0) return fail(W4A16_ERR_INVALID, "M=%d", M);
    if (M == 0) return W4A16_OK;
    const int K = gate->pw.K_in, I = gate->pw.N;
    if (up->pw.K_in != K || up->pw.N != I || down->pw.K_in != I)
        return fail(W4A16_ERR_INVALID, "gate [%d, %d], up [%d, %d] and down [%d, %d] do not chain", K, I, up->pw.K_in,
                    up->pw.N, down->pw.K_in, down->pw.N);
    const void* ptrs[6] = {norm_w_dev, x_dev, y_dev, rms_out_dev, gate_out_dev, up_out_dev};
    for (const void* q : ptrs)
        if (!q || !aligned(q, 16)) return fail(W4A16_ERR_INVALID, "norm_w, x, y, rms_out, gate_out and up_out must be 16-byte aligned");
    const size_t need = w4a16_mlp_workspace_size(gate, up, down, M, dtype);
    if (workspace_bytes < need || (need > 0 && !workspace_dev))
        return fail(W4A16_ERR_WORKSPACE, "workspace %zu bytes < %zu needed for M=%d", workspace_bytes, need, M);
    DeviceGuard guard(gate->device);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const w4a16_matrix* gu[2] = {gate, up};
    const w4a16_matrix* dn[1] = {down};
    if (fusable(gu, 2, M, dtype) && fusable(dn, 1, M, dtype)) {
        // two launches: RMSNorm applied while the gate + up GEMV stages X, then
        // silu(gate) * up applied while the down GEMV stages its X
        const PackedWeight* w2[2] = {&gate->pw, &up->pw};
        void* y2[2] = {gate_out_dev, up_out_dev};
        GemvPrologue pro = {};
        pro.mode = kProRmsNorm;
        pro.norm_w = static_cast<const uint16_t*>(norm_w_dev);
        pro.eps = eps;
        pro.out = static_cast<uint16_t*>(rms_out_dev);
        cudaError_t e = launch_gemv_group(w2, y2, 2, x_dev, M, kFP16, pro, gate->num_sms, s);
        if (e != cudaSuccess) return cuda_fail(e, "fused rms_norm + gate/up gemv launch");
        const PackedWeight* w1[1] = {&down->pw};
        void* y1[1] = {y_dev};
        GemvPrologue pro2 = {};
        pro2.mode = kProSiluMul;
        pro2.up = static_cast<const uint16_t*>(up_out_dev);
        e = launch_gemv_group(w1, y1, 1, gate_out_dev, M, kFP16, pro2, down->num_sms, s);
        if (e != cudaSuccess) return cuda_fail(e, "fused silu_mul + down gemv launch");
        return W4A16_OK;
    }
    // any M: RMSNorm, gate and up projections, silu(gate) * up into gate_out, down
    int rc = w4a16_rms_norm(x_dev, norm_w_dev, eps, M, K, rms_out_dev, dtype, stream);
    if (rc == W4A16_OK) rc = w4a16_gemm(gate, rms_out_dev, M, gate_out_dev, dtype, workspace_dev, workspace_bytes, W4A16_PATH_AUTO, stream);
    if (rc == W4A16_OK) rc = w4a16_gemm(up, rms_out_dev, M, up_out_dev, dtype, workspace_dev, workspace_bytes, W4A16_PATH_AUTO, stream);
    if (rc == W4A16_OK) rc = w4a16_silu_mul(gate_out_dev, up_out_dev, M, I, gate_out_dev, dtype, stream);
    if (rc == W4A16_OK) rc = w4a16_gemm(down, gate_out_dev, M, y_dev, dtype, workspace_dev, workspace_bytes, W4A16_PATH_AUTO, stream);
    return rc;
}

size_t w4a16_qkv_workspace_size(const w4a16_matrix* q, const w4a16_matrix* k, const w4a16_matrix* v, int M,
                                int dtype) {
    if (!q || !k || !v || M <= 0) return 0;
    const w4a16_matrix* hs[3] = {q, k, v};
    if (fusable(hs, 3, M, dtype)) return 0;
    return max3(w4a16_workspace_size(q, M, dtype, W4A16_PATH_AUTO), w4a16_workspace_size(k, M, dtype, W4A16_PATH_AUTO),
                w4a16_workspace_size(v, M, dtype, W4A16_PATH_AUTO));
}

int w4a16_qkv_forward(w4a16_matrix* q, w4a16_matrix* k, w4a16_matrix* v, const void* norm_w_dev, float eps,
                      const void* x_dev, int M, void* rms_out_dev, void* q_out_dev, void* k_out_dev, void* v_out_dev,
                      int dtype, void* workspace_dev, size_t workspace_bytes, void* stream) {
    if (!q || !k || !v) return fail(W4A16_ERR_INVALID, "null handle");
    if (k->device != q->device || v->device != q->device)
        return fail(W4A16_ERR_INVALID, "q, k and v handles on different devices");
    if (dtype != W4A16_DTYPE_FP16)
        return fail(W4A16_ERR_UNSUPPORTED, "the fused q/k/v stage is fp16 (as attention_forward_qkv_stage_v2)");
    if (M < 0) return fail(W4A16_ERR_INVALID, "M=%d", M);
    if (M == 0) return W4A16_OK;
    const int K = q->pw.K_in;
    if (k->pw.K_in != K || v->pw.K_in != K) return fail(W4A16_ERR_INVALID, "q, k and v must share in_features");
    const void* ptrs[6] = {norm_w_dev, x_dev, rms_out_dev, q_out_dev, k_out_dev, v_out_dev};
    for (const void* p : ptrs)
        if (!p || !aligned(p, 16)) return fail(W4A16_ERR_INVALID, "norm_w, x, rms_out, q_out, k_out and v_out must be 16-byte aligned");
    const size_t need = w4a16_qkv_workspace_size(q, k, v, M, dtype);
    if (workspace_bytes < need || (need > 0 && !workspace_dev))
        return fail(W4A16_ERR_WORKSPACE, "workspace %zu bytes < %zu needed for M=%d", workspace_bytes, need, M);
    DeviceGuard guard(q->device);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const w4a16_matrix* qkv[3] = {q, k, v};
    if (fusable(qkv, 3, M, dtype)) {  // one launch: RMSNorm applied while the q / k / v GEMV stages X
        const PackedWeight* w3[3] = {&q->pw, &k->pw, &v->pw};
        void* y3[3] = {q_out_dev, k_out_dev, v_out_dev};
        GemvPrologue pro = {};
        pro.mode = kProRmsNorm;
        pro.norm_w = static_cast<const uint16_t*>(norm_w_dev);
        pro.eps = eps;
        pro.out = static_cast<uint16_t*>(rms_out_dev);
        const cudaError_t e = launch_gemv_group(w3, y3, 3, x_dev, M, kFP16, pro, q->num_sms, s);
        return e == cudaSuccess ? W4A16_OK : cuda_fail(e, "fused rms_norm + q/k/v gemv launch");
    }
    int rc = w4a16_rms_norm(x_dev, norm_w_dev, eps, M, K, rms_out_dev, dtype, stream);
    if (rc == W4A16_OK) rc = w4a16_gemm(q, rms_out_dev, M, q_out_dev, dtype, workspace_dev, workspace_bytes, W4A16_PATH_AUTO, stream);
    if (rc == W4A16_OK) rc = w4a16_gemm(k, rms_out_dev, M, k_out_dev, dtype, workspace_dev, workspace_bytes, W4A16_PATH_AUTO, stream);
    if (rc == W4A16_OK) rc = w4a16_gemm(v, rms_out_dev, M, v_out_dev, dtype, workspace_dev, workspace_bytes, W4A16_PATH_AUTO, stream);
    return rc;
}

int w4a16_device_error(w4a16_matrix* h, void* stream, int* err_out) {
    if (!h || !err_out) return fail(W4A16_ERR_INVALID, "null argument");
    DeviceGuard guard(h->device);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    int v = 0;
    cudaError_t e = cudaMemcpyAsync(&v, h->err_dev, sizeof(int), cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaMemsetAsync(h->err_dev, 0, sizeof(int), s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) return cuda_fail(e, "device error read");
    *err_out = v;
    return W4A16_OK;
}

}  // extern "C"

// ---------------------------------------------------------------- w4a16_gemm_static
// w4a16_gemm with its workspace taken from a fixed array in device memory instead of
// the caller. It is for callers that cannot hand out device memory at call time: a
// host reaching this library through a plain C FFI with no GPU allocator of its own,
// or a serving loop whose allocator is frozen after warm-up (a cudaMalloc there would
// synchronise the device and stall every stream). It allocates nothing: the array is
// part of the library's device image, and the only set-up is looking up its address.
namespace {

constexpr size_t kStaticScratchBytes = size_t(8) << 20;  // 8 MiB per device
constexpr int kMaxScratchDevices = 64;

// Nothing in it has to start at zero: every byte w4a16_gemm reads from its workspace
// (the act-order X gather, split-K partial tiles) is written earlier in the same call.
// The array is part of the module's device image: it occupies 8 MiB on every device
// where the library is loaded, whether or not w4a16_gemm_static is ever called.
static __device__ __align__(256) unsigned char g_static_scratch[kStaticScratchBytes];

// Device address of each device's copy, looked up once. A cudaDeviceReset destroys the
// module and with it this address; after a reset the process must reload the library
// (the cached address would name freed memory).
std::mutex g_scratch_mu;
void* g_scratch_addr[kMaxScratchDevices] = {};

}  // namespace

extern "C" {

int w4a16_gemm_static(w4a16_matrix* h, const void* x_dev, int M, void* y_dev, int dtype, int path, void* stream) {
    if (!h) return fail(W4A16_ERR_INVALID, "null handle");
    if (int rc = check_dtype(dtype)) return rc;
    if (M < 0) return fail(W4A16_ERR_INVALID, "M=%d", M);
    if (M == 0) return W4A16_OK;
    // the same argument checks as w4a16_gemm, before any look-up is made
    if (!x_dev || !y_dev) return fail(W4A16_ERR_INVALID, "null x or y");
    if (!aligned(x_dev, 16) || !aligned(y_dev, 16)) return fail(W4A16_ERR_INVALID, "x and y must be 16-byte aligned");
    if (path < W4A16_PATH_AUTO || path > W4A16_PATH_TC_EXACT) return fail(W4A16_ERR_INVALID, "unknown path %d", path);
    const size_t need = w4a16_workspace_size(h, M, dtype, path);
    if (need > kStaticScratchBytes)
        return fail(W4A16_ERR_WORKSPACE,
                    "w4a16_gemm_static: M=%d needs %zu bytes of scratch, more than its fixed %zu-byte array; "
                    "call w4a16_gemm with a caller-provided workspace instead",
                    M, need, kStaticScratchBytes);
    if (h->device < 0 || h->device >= kMaxScratchDevices)
        return fail(W4A16_ERR_INVALID, "w4a16_gemm_static: device %d out of range", h->device);
    void* scratch = nullptr;
    {
        // once per device, with that device current: the address of this device's copy
        std::lock_guard<std::mutex> lock(g_scratch_mu);
        if (!g_scratch_addr[h->device]) {
            DeviceGuard guard(h->device);
            if (!guard.ok) return fail(W4A16_ERR_CUDA, "cudaSetDevice(%d) failed", h->device);
            void* p = nullptr;
            const cudaError_t e = cudaGetSymbolAddress(&p, g_static_scratch);
            if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(static scratch)");
            g_scratch_addr[h->device] = p;
        }
        scratch = g_scratch_addr[h->device];
    }
    return w4a16_gemm(h, x_dev, M, y_dev, dtype, scratch, kStaticScratchBytes, path, stream);
}

}  // extern "C"

// ---------------------------------------------------------------- peer-memory gather
// A column-sharded GEMV whose epilogue writes every rank's full output over NVLink
// (GatherArgs). The peers' buffers are mapped with CUDA IPC; the caller exchanges the
// 72-byte handles over its own channel (torch.distributed in the Python binding).
struct w4a16_comm {
    int rank = 0, world = 0, device = 0;
    uint32_t* flags = nullptr;  // [kMaxGatherRanks], written by every rank (IPC-exported)
    uint32_t* ctr = nullptr;    // [unused, epoch], this rank only
    uint32_t* peer_flags[w4a16::kMaxGatherRanks] = {};
};

namespace {

// Launched with programmatic stream serialization: it starts while the GEMV runs,
// lets the next kernel in the stream start its own prologue, and waits for the GEMV
// (griddepcontrol.wait: complete, its memory performed) before signalling.
__global__ void gather_signal_kernel(const w4a16::GatherArgs ga, int* err) {
    if (threadIdx.x == 0) w4a16::ptx::grid_dep_launch_dependents();
    w4a16::ptx::grid_dep_wait();
    w4a16::gather_signal_and_wait(ga, err);  // the whole warp
}

using PFN_getAddressRange = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);

PFN_getAddressRange get_address_range_fn() {
    static PFN_getAddressRange fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPointByVersion("cuMemGetAddressRange", &p, 12000, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_getAddressRange>(p);
    });
    return fn;
}

std::mutex g_ipc_mu;
std::vector<std::pair<void*, void*>> g_ipc_maps;  // (pointer handed out, mapping base)

}  // namespace

extern "C" {

int w4a16_comm_create(int rank, int world, int device, w4a16_comm** out) {
    if (!out) return fail(W4A16_ERR_INVALID, "null out");
    *out = nullptr;
    if (world < 1 || world > w4a16::kMaxGatherRanks || rank < 0 || rank >= world)
        return fail(W4A16_ERR_INVALID, "rank %d of world %d (1..%d ranks)", rank, world, w4a16::kMaxGatherRanks);
    DeviceGuard guard(device);
    if (!guard.ok) return fail(W4A16_ERR_CUDA, "cudaSetDevice(%d) failed", device);
    auto* c = new w4a16_comm();
    c->rank = rank;
    c->world = world;
    c->device = device;
    cudaError_t e = cudaMalloc(&c->flags, 256);
    if (e == cudaSuccess) e = cudaMalloc(&c->ctr, 256);
    if (e == cudaSuccess) e = cudaMemset(c->flags, 0, 256);
    if (e == cudaSuccess) e = cudaMemset(c->ctr, 0, 256);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
        cudaFree(c->flags);
        cudaFree(c->ctr);
        delete c;
        return cuda_fail(e, "comm buffers");
    }
    c->peer_flags[rank] = c->flags;
    *out = c;
    return W4A16_OK;
}

int w4a16_comm_destroy(w4a16_comm* c) {
    if (!c) return W4A16_OK;
    DeviceGuard guard(c->device);
    cudaFree(c->flags);
    cudaFree(c->ctr);
    delete c;
    return W4A16_OK;
}

int w4a16_comm_flags(const w4a16_comm* c, void** flags_dev) {
    if (!c || !flags_dev) return fail(W4A16_ERR_INVALID, "null argument");
    *flags_dev = c->flags;
    return W4A16_OK;
}

int w4a16_comm_set_peer_flags(w4a16_comm* c, int peer, void* flags_dev) {
    if (!c || !flags_dev || peer < 0 || peer >= c->world) return fail(W4A16_ERR_INVALID, "bad peer %d", peer);
    c->peer_flags[peer] = static_cast<uint32_t*>(flags_dev);
    return W4A16_OK;
}

int w4a16_ipc_export(const void* dev_ptr, void* handle_out) {
    if (!dev_ptr || !handle_out) return fail(W4A16_ERR_INVALID, "null argument");
    auto range = get_address_range_fn();
    if (!range) return fail(W4A16_ERR_CUDA, "cuMemGetAddressRange entry point not found");
    CUdeviceptr base = 0;
    size_t size = 0;
    if (range(&base, &size, reinterpret_cast<CUdeviceptr>(dev_ptr)) != CUDA_SUCCESS)
        return fail(W4A16_ERR_INVALID, "pointer is not device memory of this process");
    cudaIpcMemHandle_t mh;
    const cudaError_t e = cudaIpcGetMemHandle(&mh, reinterpret_cast<void*>(base));
    if (e != cudaSuccess) return cuda_fail(e, "cudaIpcGetMemHandle");
    const uint64_t offset = reinterpret_cast<CUdeviceptr>(dev_ptr) - base;
    std::memcpy(handle_out, &mh, sizeof(mh));
    std::memcpy(static_cast<char*>(handle_out) + sizeof(mh), &offset, sizeof(offset));
    return W4A16_OK;
}

int w4a16_ipc_open(const void* handle_in, int device, void** ptr_out) {
    if (!handle_in || !ptr_out) return fail(W4A16_ERR_INVALID, "null argument");
    DeviceGuard guard(device);
    if (!guard.ok) return fail(W4A16_ERR_CUDA, "cudaSetDevice(%d) failed", device);
    cudaIpcMemHandle_t mh;
    uint64_t offset = 0;
    std::memcpy(&mh, handle_in, sizeof(mh));
    std::memcpy(&offset, static_cast<const char*>(handle_in) + sizeof(mh), sizeof(offset));
    void* base = nullptr;
    const cudaError_t e = cudaIpcOpenMemHandle(&base, mh, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) return cuda_fail(e, "cudaIpcOpenMemHandle");
    void* p = static_cast<char*>(base) + offset;
    {
        std::lock_guard<std::mutex> lock(g_ipc_mu);
        g_ipc_maps.emplace_back(p, base);
    }
    *ptr_out = p;
    return W4A16_OK;
}

int w4a16_ipc_close(void* ptr) {
    void* base = nullptr;
    {
        std::lock_guard<std::mutex> lock(g_ipc_mu);
        for (size_t i = 0; i < g_ipc_maps.size(); ++i) {
            if (g_ipc_maps[i].first == ptr) {
                base = g_ipc_maps[i].second;
                g_ipc_maps.erase(g_ipc_maps.begin() + static_cast<long>(i));
                break;
            }
        }
    }
    if (!base) return fail(W4A16_ERR_INVALID, "pointer was not opened by w4a16_ipc_open");
    const cudaError_t e = cudaIpcCloseMemHandle(base);
    if (e != cudaSuccess) return cuda_fail(e, "cudaIpcCloseMemHandle");
    return W4A16_OK;
}

int w4a16_gemm_gather(w4a16_matrix* h, w4a16_comm* c, const void* x_dev, int M, void* const* y_all, int ld, int col0,
                      int dtype, void* workspace_dev, size_t workspace_bytes, void* stream) {
    if (!h || !c || !y_all) return fail(W4A16_ERR_INVALID, "null argument");
    if (int rc = check_dtype(dtype)) return rc;
    if (M < 0) return fail(W4A16_ERR_INVALID, "M=%d", M);
    if (M == 0) return W4A16_OK;
    if (!x_dev || !aligned(x_dev, 16)) return fail(W4A16_ERR_INVALID, "x must be 16-byte aligned");
    if (col0 < 0 || col0 + h->pw.N > ld) return fail(W4A16_ERR_INVALID, "columns [%d, %d) outside ld=%d", col0, col0 + h->pw.N, ld);
    if (c->device != h->device) return fail(W4A16_ERR_INVALID, "comm and handle on different devices");
    for (int r = 0; r < c->world; ++r) {
        if (!c->peer_flags[r]) return fail(W4A16_ERR_INVALID, "flags of rank %d not set", r);
        if (!y_all[r]) return fail(W4A16_ERR_INVALID, "output of rank %d is null", r);
    }
    const int k = resolve_kernel(h, M, dtype, W4A16_PATH_AUTO);
    if (k != kKernGemv && k != kKernGemvMma && k != kKernExact)
        return fail(W4A16_ERR_UNSUPPORTED,
                    "w4a16_gemm_gather covers the GEMV and exact-W GEMM kernels; use w4a16_gemm and an all-gather");
    if (k == kKernExact && (ld % 8 != 0 || col0 % 8 != 0))
        return fail(W4A16_ERR_INVALID, "ld=%d and col0=%d must be multiples of 8 for M=%d", ld, col0, M);
    // the GEMM's epilogue, and the mma.sync GEMV when ld and col0 allow it, store 16-byte
    // row pieces into every rank's Y
    const bool wide_stores = k == kKernExact || (k == kKernGemvMma && ld % 8 == 0 && col0 % 8 == 0);
    for (int r = 0; wide_stores && r < c->world; ++r)
        if (!aligned(y_all[r], 16)) return fail(W4A16_ERR_INVALID, "output of rank %d must be 16-byte aligned", r);
    const size_t need = w4a16_workspace_size(h, M, dtype, W4A16_PATH_AUTO);
    if (workspace_bytes < need || (need > 0 && !workspace_dev))
        return fail(W4A16_ERR_WORKSPACE, "workspace %zu bytes < %zu needed for M=%d", workspace_bytes, need, M);
    DeviceGuard guard(h->device);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    cudaError_t e = cudaSuccess;
    const void* xin = x_dev;
    uint8_t* ws = static_cast<uint8_t*>(workspace_dev);
    size_t ws_left = workspace_bytes;
    if (h->pw.act_order) {
        e = launch_remap_cols(x_dev, h->pw.K_in, workspace_dev, h->pw.K, h->pw.perm, M, h->pw.K, s);
        if (e != cudaSuccess) return cuda_fail(e, "act-order gather launch");
        xin = workspace_dev;
        const size_t used = align_up(static_cast<size_t>(M) * h->pw.K * 2, 256);
        ws += used;
        ws_left -= used;
    }
    w4a16::GatherArgs ga = {};
    ga.world = c->world;
    ga.rank = c->rank;
    ga.ld = ld;
    ga.col0 = col0;
    ga.my_flags = c->flags;
    ga.ctr = c->ctr;
    for (int r = 0; r < c->world; ++r) ga.flags[r] = c->peer_flags[r];
    if (k == kKernExact) {  // prefill sizes: the tcgen05 GEMM's epilogue (or split-K reduction) stores everywhere
        for (int r = 0; r < c->world; ++r) ga.y[r] = static_cast<uint16_t*>(y_all[r]);
        const TcPlan tp = plan_tc(h->pw, M, h->num_sms);
        e = launch_tc(h->pw, tp, &h->qw_map, xin, M, nullptr, static_cast<DType>(dtype), ws, ws_left, s, &ga);
    }
    for (int m0 = 0; k != kKernExact && m0 < M && e == cudaSuccess;) {
        const bool mma = k == kKernGemvMma;
        const GemvPlan gp = mma ? plan_gemv_mma(h->pw, M - m0 < kGemvMmaMaxTok ? M - m0 : kGemvMmaMaxTok, h->num_sms)
                                : plan_gemv(h->pw, M - m0 < 8 ? M - m0 : 8, h->num_sms);
        const int mm = (M - m0) < gp.mt ? (M - m0) : gp.mt;
        for (int r = 0; r < c->world; ++r)
            ga.y[r] = static_cast<uint16_t*>(y_all[r]) + static_cast<size_t>(m0) * ld;
        const void* xp = static_cast<const uint16_t*>(xin) + static_cast<size_t>(m0) * h->pw.K;
        e = mma ? launch_gemv_mma(h->pw, h->qw_mma, gp, xp, mm, nullptr, static_cast<DType>(dtype), s, &ga)
                : launch_gemv(h->pw, gp, xp, mm, nullptr, static_cast<DType>(dtype), s, &ga);
        m0 += mm;
    }
    if (e != cudaSuccess) return cuda_fail(e, "gemm + gather launch");
    // after every pass: this rank's columns are in place everywhere; raise the epoch
    // and wait for every rank's (the kernel completes when the whole Y is here)
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(1, 1, 1);
    cfg.blockDim = dim3(32, 1, 1);
    cfg.stream = s;
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr.val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    e = cudaLaunchKernelEx(&cfg, gather_signal_kernel, ga, h->err_dev);
    if (e != cudaSuccess) return cuda_fail(e, "gather signal launch");
    return W4A16_OK;
}

}  // extern "C"
