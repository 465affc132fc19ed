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
#include "w4a16_prologue.cuh"

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

// out[m, j] = map[j] >= 0 ? in[m, map[j]] : 0 for 16-bit elements, j < out_cols;
// one thread per 8 outputs. The act-order X gather into kernel row order (map = the
// padded sort, -1 on pad rows) and the return of a transposed product to the
// caller's row order (map = its inverse) are both this kernel.
__global__ void __launch_bounds__(256)
    remap_cols_kernel(const uint16_t* __restrict__ in, int in_ld, uint16_t* __restrict__ out, int out_ld,
                      const int32_t* __restrict__ map, int M, int out_cols) {
    const long long idx = static_cast<long long>(blockIdx.x) * 256 + threadIdx.x;
    const int kc = out_cols >> 3;
    if (idx >= static_cast<long long>(M) * kc) return;
    const int m = static_cast<int>(idx / kc);
    const int j0 = static_cast<int>(idx % kc) << 3;
    const int4 pa = __ldg(reinterpret_cast<const int4*>(map + j0));
    const int4 pb = __ldg(reinterpret_cast<const int4*>(map + j0 + 4));
    const int p[8] = {pa.x, pa.y, pa.z, pa.w, pb.x, pb.y, pb.z, pb.w};
    const uint16_t* row = in + static_cast<size_t>(m) * in_ld;
    uint32_t o[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const uint32_t lo = p[2 * i] >= 0 ? __ldg(row + p[2 * i]) : 0u;
        const uint32_t hi = p[2 * i + 1] >= 0 ? __ldg(row + p[2 * i + 1]) : 0u;
        o[i] = lo | (hi << 16);
    }
    *reinterpret_cast<uint4*>(out + static_cast<size_t>(m) * out_ld + j0) = make_uint4(o[0], o[1], o[2], o[3]);
}

// Private act-order copy of qweight with rows in group-sorted order:
// sorted row j holds original row perm[j], or zeros where perm[j] < 0 (pad rows of
// groups shorter than the longest one; their X is 0). The reference permutes the
// caller's qweight in place instead (q4_matrix.cu:84-123,179); this never touches it.
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
        if (k < 0) continue;
        const uint32_t w = static_cast<uint32_t>(__ldg(qweight + static_cast<size_t>(k >> 3) * N + n));
        out |= ((w >> (4 * (k & 7))) & 15u) << (4 * i);
    }
    sorted[static_cast<size_t>(kw) * N + n] = static_cast<int32_t>(out);
}

// RMSNorm, one CTA of 256 threads per row (fp16, K % 8 == 0): the same arithmetic as
// the GEMV's RMSNorm prologue (fuse_v2/rms_norm.cu:27-93 in the reference): the sum of
// squares in a fixed order, rsqrt(sum / K + eps), then fp16(x * w * rmf).
__global__ void __launch_bounds__(256)
    rms_norm_kernel(const uint16_t* __restrict__ x, const uint16_t* __restrict__ w, float eps, int K,
                    uint16_t* __restrict__ y) {
    __shared__ float wsum[8];
    __shared__ float rmf_s;
    const uint16_t* xr = x + static_cast<size_t>(blockIdx.x) * K;
    float ss = 0.f;
    for (int k8 = threadIdx.x; k8 < (K >> 3); k8 += 256) {
        const uint4 raw = __ldg(reinterpret_cast<const uint4*>(xr) + k8);
        const uint32_t r4[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const float lo = clamp_h2f(r4[e] & 0xFFFFu), hi = clamp_h2f(r4[e] >> 16);
            ss = fmaf(lo, lo, ss);
            ss = fmaf(hi, hi, ss);
        }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
    if ((threadIdx.x & 31) == 0) wsum[threadIdx.x >> 5] = ss;
    __syncthreads();
    if (threadIdx.x == 0) {
        float t = 0.f;
        for (int i = 0; i < 8; ++i) t += wsum[i];
        rmf_s = rsqrtf(t * (1.0f / static_cast<float>(K)) + eps);
    }
    __syncthreads();
    const float rmf = rmf_s;
    for (int k8 = threadIdx.x; k8 < (K >> 3); k8 += 256)
        *(reinterpret_cast<uint4*>(y + static_cast<size_t>(blockIdx.x) * K) + k8) =
            rms_apply8(__ldg(reinterpret_cast<const uint4*>(xr) + k8), __ldg(reinterpret_cast<const uint4*>(w) + k8), rmf);
}

// out = fp16(silu(gate) * up), 8 values per thread (fp16, N % 8 == 0)
__global__ void __launch_bounds__(256)
    silu_mul_kernel(const uint16_t* __restrict__ gate, const uint16_t* __restrict__ up, long long n8,
                    uint16_t* __restrict__ out) {
    const long long i = static_cast<long long>(blockIdx.x) * 256 + threadIdx.x;
    if (i >= n8) return;
    reinterpret_cast<uint4*>(out)[i] =
        silu_mul8(__ldg(reinterpret_cast<const uint4*>(gate) + i), __ldg(reinterpret_cast<const uint4*>(up) + i));
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
    // the caller's packed weight in its own row order: K_in rows, g_idx as given
    const long long total = static_cast<long long>(w.K_in >> 3) * (w.N >> 3);
    const unsigned blocks = static_cast<unsigned>((total + kDequantThreads - 1) / kDequantThreads);
    if (blocks == 0) return cudaSuccess;
    const int32_t* gi = w.act_order ? w.g_idx : nullptr;
    const int gs = w.act_order ? 1 : w.group_size;  // unused with g_idx
    if (dt == kBF16) {
        dequant_kernel<true><<<blocks, kDequantThreads, 0, s>>>(w.qweight_orig, w.qzeros, w.scales, gi, w.K_in, w.N,
                                                                gs, static_cast<uint16_t*>(out));
    } else {
        dequant_kernel<false><<<blocks, kDequantThreads, 0, s>>>(w.qweight_orig, w.qzeros, w.scales, gi, w.K_in,
                                                                 w.N, gs, static_cast<uint16_t*>(out));
    }
    return cudaGetLastError();
}

cudaError_t launch_remap_cols(const void* in, int in_ld, void* out, int out_ld, const int32_t* map, int M,
                              int out_cols, cudaStream_t s) {
    const long long total = static_cast<long long>(M) * (out_cols >> 3);
    if (total == 0) return cudaSuccess;
    const unsigned blocks = static_cast<unsigned>((total + 255) / 256);
    remap_cols_kernel<<<blocks, 256, 0, s>>>(static_cast<const uint16_t*>(in), in_ld, static_cast<uint16_t*>(out),
                                             out_ld, map, M, out_cols);
    return cudaGetLastError();
}

cudaError_t launch_rms_norm(const void* x, const void* w, float eps, int M, int K, void* y, cudaStream_t s) {
    if (M <= 0) return cudaSuccess;
    rms_norm_kernel<<<M, 256, 0, s>>>(static_cast<const uint16_t*>(x), static_cast<const uint16_t*>(w), eps, K,
                                      static_cast<uint16_t*>(y));
    return cudaGetLastError();
}

cudaError_t launch_silu_mul(const void* gate, const void* up, int M, int N, void* out, cudaStream_t s) {
    const long long n8 = static_cast<long long>(M) * N / 8;
    if (n8 == 0) return cudaSuccess;
    silu_mul_kernel<<<static_cast<unsigned>((n8 + 255) / 256), 256, 0, s>>>(
        static_cast<const uint16_t*>(gate), static_cast<const uint16_t*>(up), n8, static_cast<uint16_t*>(out));
    return cudaGetLastError();
}

}  // namespace w4a16
