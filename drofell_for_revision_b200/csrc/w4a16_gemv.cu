// Decode GEMV (M <= 8): Y[M, N] = X[M, K] * W[K, N] with W streamed from packed
// int4 straight out of HBM, on CUDA cores.
//
// Replaces the reference's v2 GEMV (After-Revision-DROFELL/cuda_extends/exllama/
// q_gemm_kernel_gptq.cuh:41-195, host q4_matmul.cu:428-456), which splits K over
// CTAs and reduces with racy fp16 atomics into an output it zeroes concurrently.
// Here the K split is a thread-block cluster: the CTAs of one cluster reduce their
// fp32 partials through distributed shared memory in a fixed order, so results
// are deterministic and no workspace or atomics are needed.
//
// Layout: CTA = 256 threads = BN/4 column quads x KL k-lanes. Each thread reads
// 16 B words (4 columns x 8 k) of qweight[kw, n..n+3] over a contiguous run of
// words, so every warp-level load is a fully used 128 B+ segment. X for the CTA's
// K range is staged in shared memory (gathered through the act-order permutation
// when needed) in the pair order the nibble unpack produces.
//
// Math per word: (q - z) is formed exactly in fp16 pairs with the 0x6400 exponent
// trick, dotted with X in fp16 over 4 terms per lane, then accumulated in fp32 and
// scaled by the fp16 group scale in fp32.
#include <cooperative_groups.h>
#include <cuda_fp16.h>

#include "w4a16_internal.h"

namespace cg = cooperative_groups;

namespace w4a16 {
namespace {

constexpr int kGemvThreads = 256;

__device__ __forceinline__ __half2 u32_as_h2(uint32_t v) {
    return *reinterpret_cast<__half2*>(&v);
}

// (q_a - z, q_b - z) for the nibble pair at bit offsets (sh, sh + 16).
__device__ __forceinline__ __half2 nib_pair_minus_z(uint32_t w, int sh, __half2 z1024) {
    const uint32_t p = ((w >> sh) & 0x000F000Fu) | 0x64006400u;  // (1024 + q_a, 1024 + q_b), exact
    return __hsub2(u32_as_h2(p), z1024);
}

template <int MT, int BN, bool ACT>
__global__ void __launch_bounds__(kGemvThreads)
    gemv_kernel(const int32_t* __restrict__ qweight, const int32_t* __restrict__ qzeros,
                const uint16_t* __restrict__ scales, const int32_t* __restrict__ word_group,
                const int32_t* __restrict__ perm, const uint16_t* __restrict__ x, uint16_t* __restrict__ y, int M,
                int K, int N, int group_size, int kw_per_cta, int cluster_size) {
    constexpr int COLQ = BN / 4;
    constexpr int KL = kGemvThreads / COLQ;
    constexpr int U = 4;  // words in flight per thread per step
    extern __shared__ __align__(16) uint8_t smem_raw[];
    uint4* xs = reinterpret_cast<uint4*>(smem_raw);

    const int KW = K >> 3;
    const int split = blockIdx.y;
    const int kw0 = split * kw_per_cta;
    const int kw1 = min(KW, kw0 + kw_per_cta);
    const int nkw = max(0, kw1 - kw0);
    const int n_base = blockIdx.x * BN;

    // ---- stage X[m, kw0*8 : kw1*8) as interleaved 8-element words
    for (int i = threadIdx.x; i < MT * nkw; i += kGemvThreads) {
        const int m = i / nkw;
        const int wl = i - m * nkw;
        const int kw = kw0 + wl;
        uint32_t v[8];
        if (m < M) {
            const uint16_t* xr = x + static_cast<size_t>(m) * K;
            if constexpr (ACT) {
#pragma unroll
                for (int j = 0; j < 8; ++j) v[j] = __ldg(xr + __ldg(perm + kw * 8 + j));
            } else {
                const uint4 raw = __ldg(reinterpret_cast<const uint4*>(xr + kw * 8));
                v[0] = raw.x & 0xFFFFu; v[1] = raw.x >> 16;
                v[2] = raw.y & 0xFFFFu; v[3] = raw.y >> 16;
                v[4] = raw.z & 0xFFFFu; v[5] = raw.z >> 16;
                v[6] = raw.w & 0xFFFFu; v[7] = raw.w >> 16;
            }
        } else {
#pragma unroll
            for (int j = 0; j < 8; ++j) v[j] = 0;
        }
        xs[m * nkw + wl] = make_uint4(v[0] | (v[4] << 16), v[1] | (v[5] << 16), v[2] | (v[6] << 16),
                                      v[3] | (v[7] << 16));
    }
    __syncthreads();

    const int cq = threadIdx.x % COLQ;
    const int kl = threadIdx.x / COLQ;
    const int n = n_base + cq * 4;
    const int per = (nkw + KL - 1) / KL;
    const int a0 = min(nkw, kl * per);
    const int a1 = min(nkw, a0 + per);

    float acc[MT][4];
#pragma unroll
    for (int m = 0; m < MT; ++m)
#pragma unroll
        for (int c = 0; c < 4; ++c) acc[m][c] = 0.f;

    int cur_g = -1;
    __half2 zz[4];
    float sf[4];
    const uint4* qp = reinterpret_cast<const uint4*>(qweight + n);
    const size_t row_u4 = static_cast<size_t>(N) >> 2;

    for (int a = a0; a < a1; a += U) {
        uint4 wv[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            if (a + u < a1) wv[u] = __ldg(qp + static_cast<size_t>(kw0 + a + u) * row_u4);
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
            if (a + u < a1) {
                const int kw = kw0 + a + u;
                const int g = ACT ? __ldg(word_group + kw) : (kw << 3) / group_size;
                if (g != cur_g) {
                    cur_g = g;
                    const uint2 sv = __ldg(reinterpret_cast<const uint2*>(scales + static_cast<size_t>(g) * N + n));
                    sf[0] = __half2float(__ushort_as_half(static_cast<unsigned short>(sv.x & 0xFFFFu)));
                    sf[1] = __half2float(__ushort_as_half(static_cast<unsigned short>(sv.x >> 16)));
                    sf[2] = __half2float(__ushort_as_half(static_cast<unsigned short>(sv.y & 0xFFFFu)));
                    sf[3] = __half2float(__ushort_as_half(static_cast<unsigned short>(sv.y >> 16)));
                    const uint32_t zw =
                        static_cast<uint32_t>(__ldg(qzeros + static_cast<size_t>(g) * (N >> 3) + (n >> 3)));
                    const int zsh = (n & 7) * 4;
#pragma unroll
                    for (int c = 0; c < 4; ++c) {
                        const uint32_t z1 = ((zw >> (zsh + 4 * c)) & 15u) + 1u;
                        const uint32_t hz = 0x6400u + z1;  // fp16 bits of 1024 + z (exact)
                        zz[c] = u32_as_h2(hz | (hz << 16));
                    }
                }
                const uint32_t w4[4] = {wv[u].x, wv[u].y, wv[u].z, wv[u].w};
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    const __half2 d0 = nib_pair_minus_z(w4[c], 0, zz[c]);   // k 0,4
                    const __half2 d1 = nib_pair_minus_z(w4[c], 4, zz[c]);   // k 1,5
                    const __half2 d2 = nib_pair_minus_z(w4[c], 8, zz[c]);   // k 2,6
                    const __half2 d3 = nib_pair_minus_z(w4[c], 12, zz[c]);  // k 3,7
#pragma unroll
                    for (int m = 0; m < MT; ++m) {
                        const uint4 xv = xs[m * nkw + a + u];
                        __half2 h = __hmul2(u32_as_h2(xv.x), d0);
                        h = __hfma2(u32_as_h2(xv.y), d1, h);
                        h = __hfma2(u32_as_h2(xv.z), d2, h);
                        h = __hfma2(u32_as_h2(xv.w), d3, h);
                        const float2 f = __half22float2(h);
                        acc[m][c] = fmaf(f.x + f.y, sf[c], acc[m][c]);
                    }
                }
            }
        }
    }

    // ---- reduce the KL k-lanes of this CTA
    __syncthreads();  // xs is dead from here on
    float* red = reinterpret_cast<float*>(smem_raw);  // [KL][MT][BN]
    float* part = red + KL * MT * BN;                 // [MT][BN]
#pragma unroll
    for (int m = 0; m < MT; ++m)
#pragma unroll
        for (int c = 0; c < 4; ++c) red[(kl * MT + m) * BN + cq * 4 + c] = acc[m][c];
    __syncthreads();
    for (int i = threadIdx.x; i < MT * BN; i += kGemvThreads) {
        const int m = i / BN;
        const int nn = i - m * BN;
        float s = 0.f;
#pragma unroll 4
        for (int l = 0; l < KL; ++l) s += red[(l * MT + m) * BN + nn];
        part[i] = s;
    }

    if (cluster_size == 1) {
        __syncthreads();
        for (int i = threadIdx.x; i < MT * BN; i += kGemvThreads) {
            const int m = i / BN;
            if (m < M) y[static_cast<size_t>(m) * N + n_base + (i - m * BN)] = __half_as_ushort(__float2half_rn(part[i]));
        }
        return;
    }

    // ---- reduce the cluster's K splits through distributed shared memory, fixed order
    cg::cluster_group cluster = cg::this_cluster();
    cluster.sync();
    const int rank = static_cast<int>(cluster.block_rank());
    const int total = MT * BN;
    const int per_rank = (total + cluster_size - 1) / cluster_size;
    const int i0 = rank * per_rank;
    const int i1 = min(total, i0 + per_rank);
    for (int i = i0 + threadIdx.x; i < i1; i += kGemvThreads) {
        const int m = i / BN;
        float s = 0.f;
        for (int r = 0; r < cluster_size; ++r) s += cluster.map_shared_rank(part, r)[i];
        if (m < M) y[static_cast<size_t>(m) * N + n_base + (i - m * BN)] = __half_as_ushort(__float2half_rn(s));
    }
    cluster.sync();  // keep this CTA's shared memory alive until every peer has read it
}

template <int MT, int BN, bool ACT>
cudaError_t launch_gemv_t(const PackedWeight& w, const GemvPlan& p, const void* x, int M, void* y, cudaStream_t s) {
    constexpr int COLQ = BN / 4;
    constexpr int KL = kGemvThreads / COLQ;
    const int KW = w.K >> 3;
    const int kw_per_cta = (KW + p.splits - 1) / p.splits;
    const size_t xs_bytes = static_cast<size_t>(MT) * kw_per_cta * 16;
    const size_t red_bytes = static_cast<size_t>(KL * MT * BN + MT * BN) * 4;
    const size_t smem = xs_bytes > red_bytes ? xs_bytes : red_bytes;
    auto kern = gemv_kernel<MT, BN, ACT>;
    // The X slice grows with K: allow the largest dynamic shared memory once per
    // instantiation (before any stream capture reuses it).
    static const cudaError_t attr_err =
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    if (attr_err != cudaSuccess) return attr_err;
    if (smem > 227 * 1024) return cudaErrorInvalidValue;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(w.N / BN, p.splits, 1);
    cfg.blockDim = dim3(kGemvThreads, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    int nattr = 0;
    if (p.splits > 1) {
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = 1;
        attr[0].val.clusterDim.y = p.splits;
        attr[0].val.clusterDim.z = 1;
        nattr = 1;
    }
    cfg.attrs = attr;
    cfg.numAttrs = nattr;
    return cudaLaunchKernelEx(&cfg, kern, w.qweight, w.qzeros, w.scales, w.word_group, w.perm,
                              static_cast<const uint16_t*>(x), static_cast<uint16_t*>(y), M, w.K, w.N, w.group_size,
                              kw_per_cta, p.splits);
}

template <int MT, bool ACT>
cudaError_t launch_gemv_bn(const PackedWeight& w, const GemvPlan& p, const void* x, int M, void* y, cudaStream_t s) {
    switch (p.bn) {
        case 128: return launch_gemv_t<MT, 128, ACT>(w, p, x, M, y, s);
        case 64: return launch_gemv_t<MT, 64, ACT>(w, p, x, M, y, s);
        case 32: return launch_gemv_t<MT, 32, ACT>(w, p, x, M, y, s);
        default: return cudaErrorInvalidValue;
    }
}

template <bool ACT>
cudaError_t launch_gemv_mt(const PackedWeight& w, const GemvPlan& p, const void* x, int M, void* y, cudaStream_t s) {
    switch (p.mt) {
        case 1: return launch_gemv_bn<1, ACT>(w, p, x, M, y, s);
        case 2: return launch_gemv_bn<2, ACT>(w, p, x, M, y, s);
        case 4: return launch_gemv_bn<4, ACT>(w, p, x, M, y, s);
        case 8: return launch_gemv_bn<8, ACT>(w, p, x, M, y, s);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace

GemvPlan plan_gemv(const PackedWeight& w, int M) {
    GemvPlan p;
    p.mt = M <= 1 ? 1 : M <= 2 ? 2 : M <= 4 ? 4 : 8;
    const int target = 2 * 148;  // >= two CTAs per SM so every SM streams weights
    int bn = (w.N % 128 == 0) ? 128 : (w.N % 64 == 0) ? 64 : 32;
    while (bn > 32 && (w.N / bn) * 8 < target && w.N % (bn / 2) == 0) bn /= 2;
    p.bn = bn;
    const int kl = kGemvThreads / (bn / 4);
    const int KW = w.K >> 3;
    int cs = 1;
    while (cs < 8 && (w.N / bn) * cs < target && (KW + 2 * cs - 1) / (2 * cs) >= kl) cs *= 2;
    p.splits = cs;
    return p;
}

cudaError_t launch_gemv(const PackedWeight& w, const GemvPlan& p, const void* x, int M, void* y, cudaStream_t s) {
    if (M <= 0) return cudaSuccess;
    if (M > p.mt) return cudaErrorInvalidValue;
    return w.act_order ? launch_gemv_mt<true>(w, p, x, M, y, s) : launch_gemv_mt<false>(w, p, x, M, y, s);
}

}  // namespace w4a16
