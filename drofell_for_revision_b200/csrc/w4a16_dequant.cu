// Bit-exact GPTQ dequant (packed int4 -> dense fp16/bf16 W[K, N]) and the
// act-order column gather of X.
//
// Semantics follow After-Revision-DROFELL/operators/core/linear/real_quant.py:69-90
//   W[k, n] = fp16( scales[g, n] * (q[k, n] - (z_raw[g, n] + 1)) ),  g = g_idx[k]
// and, for bf16, the reference's fp16 -> fp32 -> bf16 conversion
// (cuda_extends/exllama/q4_matrix.cu:465-467). q - z is an exact small integer,
// so one correctly rounded fp16 multiply reproduces the torch result bit for bit.
// Output rows are in the caller's original order, with or without act-order
// (the reference's v2 reconstruct scatters rows through its x_map instead,
// q4_matrix.cu:414-421; the values are the same).
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "w4a16_internal.h"

namespace w4a16 {
namespace {

constexpr int kDequantThreads = 256;

// One thread: one 8-row word x 8 consecutive columns. Reads 32 B of qweight, one
// zero word and 16 B of scales per row group, writes 8 rows x 16 B.
template <bool kBF16>
__global__ void __launch_bounds__(kDequantThreads)
    dequant_kernel(const int32_t* __restrict__ qweight, const int32_t* __restrict__ qzeros,
                   const uint16_t* __restrict__ scales, const int32_t* __restrict__ g_idx, int K, int N,
                   int group_size, uint16_t* __restrict__ out) {
    const int chunks = N >> 3;
    const long long idx = static_cast<long long>(blockIdx.x) * kDequantThreads + threadIdx.x;
    const long long total = static_cast<long long>(K >> 3) * chunks;
    if (idx >= total) return;
    const int c = static_cast<int>(idx % chunks);
    const int kw = static_cast<int>(idx / chunks);
    const int n0 = c << 3;

    const uint4* wp = reinterpret_cast<const uint4*>(qweight + static_cast<size_t>(kw) * N + n0);
    const uint4 wa = __ldg(wp);
    const uint4 wb = __ldg(wp + 1);
    const uint32_t words[8] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w};

#pragma unroll
    for (int r = 0; r < 8; ++r) {
        const int k = (kw << 3) + r;
        const int g = g_idx ? __ldg(g_idx + k) : k / group_size;
        const uint32_t zw = static_cast<uint32_t>(__ldg(qzeros + static_cast<size_t>(g) * chunks + c));
        const uint4 sv = __ldg(reinterpret_cast<const uint4*>(scales + static_cast<size_t>(g) * N + n0));
        const uint32_t s32[4] = {sv.x, sv.y, sv.z, sv.w};
        uint32_t o[4];
#pragma unroll
        for (int j2 = 0; j2 < 4; ++j2) {
            uint16_t res[2];
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int j = 2 * j2 + h;
                const int q = static_cast<int>((words[j] >> (4 * r)) & 15u);
                const int z = static_cast<int>((zw >> (4 * j)) & 15u) + 1;
                const __half s = __ushort_as_half(static_cast<unsigned short>(s32[j2] >> (16 * h)));
                const __half v = __hmul(s, __int2half_rn(q - z));
                if constexpr (kBF16) {
                    res[h] = __bfloat16_as_ushort(__float2bfloat16_rn(__half2float(v)));
                } else {
                    res[h] = __half_as_ushort(v);
                }
            }
            o[j2] = static_cast<uint32_t>(res[0]) | (static_cast<uint32_t>(res[1]) << 16);
        }
        *reinterpret_cast<uint4*>(out + static_cast<size_t>(k) * N + n0) = make_uint4(o[0], o[1], o[2], o[3]);
    }
}

// xs[m, j] = x[m, perm[j]] for 16-bit elements; one thread per 8 outputs.
__global__ void __launch_bounds__(256)
    gather_cols_kernel(const uint16_t* __restrict__ x, uint16_t* __restrict__ xs, const int32_t* __restrict__ perm,
                       int M, int K) {
    const long long idx = static_cast<long long>(blockIdx.x) * 256 + threadIdx.x;
    const int kc = K >> 3;
    if (idx >= static_cast<long long>(M) * kc) return;
    const int m = static_cast<int>(idx / kc);
    const int j0 = static_cast<int>(idx % kc) << 3;
    const int4 pa = __ldg(reinterpret_cast<const int4*>(perm + j0));
    const int4 pb = __ldg(reinterpret_cast<const int4*>(perm + j0 + 4));
    const int p[8] = {pa.x, pa.y, pa.z, pa.w, pb.x, pb.y, pb.z, pb.w};
    const uint16_t* xr = x + static_cast<size_t>(m) * K;
    uint32_t o[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        o[i] = static_cast<uint32_t>(__ldg(xr + p[2 * i])) | (static_cast<uint32_t>(__ldg(xr + p[2 * i + 1])) << 16);
    }
    *reinterpret_cast<uint4*>(xs + static_cast<size_t>(m) * K + j0) = make_uint4(o[0], o[1], o[2], o[3]);
}

// Private act-order copy of qweight with rows in group-sorted order:
// sorted row j holds original row perm[j] (the reference permutes the caller's
// qweight in place instead, q4_matrix.cu:84-123,179; this never touches it).
__global__ void __launch_bounds__(256)
    sort_rows_kernel(const int32_t* __restrict__ qweight, int32_t* __restrict__ sorted,
                     const int32_t* __restrict__ perm, int K, int N) {
    const long long idx = static_cast<long long>(blockIdx.x) * 256 + threadIdx.x;
    if (idx >= static_cast<long long>(K >> 3) * N) return;
    const int n = static_cast<int>(idx % N);
    const int kw = static_cast<int>(idx / N);
    uint32_t out = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int k = __ldg(perm + kw * 8 + i);
        const uint32_t w = static_cast<uint32_t>(__ldg(qweight + static_cast<size_t>(k >> 3) * N + n));
        out |= ((w >> (4 * (k & 7))) & 15u) << (4 * i);
    }
    sorted[static_cast<size_t>(kw) * N + n] = static_cast<int32_t>(out);
}

}  // namespace

cudaError_t launch_sort_rows(const int32_t* qweight, int32_t* sorted, const int32_t* perm, int K, int N,
                             cudaStream_t s) {
    const long long total = static_cast<long long>(K >> 3) * N;
    if (total == 0) return cudaSuccess;
    sort_rows_kernel<<<static_cast<unsigned>((total + 255) / 256), 256, 0, s>>>(qweight, sorted, perm, K, N);
    return cudaGetLastError();
}

cudaError_t launch_dequant(const PackedWeight& w, void* out, DType dt, cudaStream_t s) {
    const long long total = static_cast<long long>(w.K >> 3) * (w.N >> 3);
    const unsigned blocks = static_cast<unsigned>((total + kDequantThreads - 1) / kDequantThreads);
    if (blocks == 0) return cudaSuccess;
    const int32_t* gi = w.act_order ? w.g_idx : nullptr;
    if (dt == kBF16) {
        dequant_kernel<true><<<blocks, kDequantThreads, 0, s>>>(w.qweight_orig, w.qzeros, w.scales, gi, w.K, w.N,
                                                                w.group_size, static_cast<uint16_t*>(out));
    } else {
        dequant_kernel<false><<<blocks, kDequantThreads, 0, s>>>(w.qweight_orig, w.qzeros, w.scales, gi, w.K, w.N,
                                                                 w.group_size, static_cast<uint16_t*>(out));
    }
    return cudaGetLastError();
}

cudaError_t launch_gather_cols(const void* x, void* xs, const int32_t* perm, int M, int K, cudaStream_t s) {
    const long long total = static_cast<long long>(M) * (K >> 3);
    if (total == 0) return cudaSuccess;
    const unsigned blocks = static_cast<unsigned>((total + 255) / 256);
    gather_cols_kernel<<<blocks, 256, 0, s>>>(static_cast<const uint16_t*>(x), static_cast<uint16_t*>(xs), perm, M,
                                              K);
    return cudaGetLastError();
}

}  // namespace w4a16
