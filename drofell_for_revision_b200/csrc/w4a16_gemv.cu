// Decode GEMV (M <= 8): Y[M, N] = X[M, K] * W[K, N] with W streamed from packed
// int4 straight out of HBM, on CUDA cores.
//
// Replaces the reference's v2 GEMV (After-Revision-DROFELL/cuda_extends/exllama/
// q_gemm_kernel_gptq.cuh:41-195, host q4_matmul.cu:428-456), which splits K over
// CTAs and reduces with racy fp16 atomics into an output it zeroes concurrently.
//
// Structure (128 threads = 4 warps, 128 output columns per CTA):
//   * The CTA's K range is cut into blocks of 8 packed rows (64 k). Each warp owns a
//     contiguous run of blocks and streams them through its own 4-deep ring: lane 0
//     issues a TMA copy of the block's [8 rows x 128 columns] qweight tile (4 KB) and
//     bulk copies of its groups' zero and scale rows, all completing on the slot's
//     mbarrier. Up to 16 blocks (64 KB) per CTA, two CTAs per SM, are in flight.
//   * The weight copies of the first ring slots are issued before
//     griddepcontrol.wait, so they overlap the previous kernel in the stream; X (the
//     only input another kernel writes) is staged after it, gathered through the
//     act-order permutation when needed, in the pair order the unpack produces.
//   * Lane l owns columns n0 + 4l .. 4l + 3: one 16-byte shared load per row gives
//     its four words. (q - z) is formed exactly in fp16 pairs with the 0x6400
//     exponent trick, dotted with X in fp16 over 4 terms, accumulated in fp32 and
//     scaled by the fp16 group scale in fp32.
//   * The K split across CTAs is a thread-block cluster: partials are reduced in a
//     fixed order through distributed shared memory, so results are deterministic
//     and need neither workspace nor atomics.
#include <cooperative_groups.h>
#include <cuda_fp16.h>

#include <cmath>
#include <cstdlib>

#include "w4a16_internal.h"
#include "w4a16_ptx.cuh"

namespace cg = cooperative_groups;

namespace w4a16 {
namespace {

constexpr int kGemvThreads = 128;
constexpr int kGemvWarps = kGemvThreads / 32;
constexpr int kRing = 4;                      // slots per warp
constexpr int kBlockRows = 8;                 // packed rows per block (64 k)
constexpr int kTileCols = 128;
constexpr int kRawBytes = kBlockRows * kTileCols * 4;  // 4 KB
constexpr int kMaxGroups = 2;                 // groups per block: group size >= 32
constexpr int kScOff = kRawBytes;
constexpr int kZrOff = kScOff + kMaxGroups * kTileCols * 2;
constexpr int kSlotBytes = 5120;              // 4096 + 512 + 128, rounded
constexpr uint32_t kWaitLimit = 1u << 26;
constexpr int kErrGemvTimeout = 16;

__device__ __forceinline__ __half2 u32_as_h2(uint32_t v) { return *reinterpret_cast<__half2*>(&v); }

// (q_a - z, q_b - z) for the nibble pair at bit offsets (sh, sh + 16), exact.
__device__ __forceinline__ __half2 nib_pair_minus_z(uint32_t w, int sh, __half2 z1024) {
    const uint32_t p = ((w >> sh) & 0x000F000Fu) | 0x64006400u;  // (1024 + q_a, 1024 + q_b)
    return __hsub2(u32_as_h2(p), z1024);
}

struct GemvSmem {
    static size_t bytes(int mt, int nkw) {
        const size_t ring = static_cast<size_t>(kGemvWarps) * kRing * kSlotBytes;
        const size_t xs = static_cast<size_t>(mt) * nkw * 16;
        return ring + ((xs + 127) / 128) * 128 + 256 /*barriers*/ + 128 /*align*/;
    }
};

template <int MT, bool ACT>
__global__ void __launch_bounds__(kGemvThreads)
    gemv_kernel(const __grid_constant__ CUtensorMap tm_qw, const int32_t* __restrict__ qzeros,
                const uint16_t* __restrict__ scales, const int32_t* __restrict__ perm,
                const uint16_t* __restrict__ x, uint16_t* __restrict__ y, int M, int K, int N, int G,
                int group_size, int kw_per_cta, int cluster_size, int* __restrict__ err) {
    extern __shared__ __align__(128) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~uintptr_t(127));
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    const int KW = K >> 3;
    const int kw0 = blockIdx.y * kw_per_cta;
    const int kw1 = min(KW, kw0 + kw_per_cta);
    const int nkw = max(0, kw1 - kw0);
    const int n0 = blockIdx.x * kTileCols;
    const int wpg = group_size >> 3;

    uint8_t* ring = smem + static_cast<size_t>(warp) * kRing * kSlotBytes;
    uint4* xs = reinterpret_cast<uint4*>(smem + static_cast<size_t>(kGemvWarps) * kRing * kSlotBytes);
    uint64_t* bars = reinterpret_cast<uint64_t*>(reinterpret_cast<uint8_t*>(xs) + ((MT * nkw * 16 + 127) / 128) * 128);
    uint64_t* my_bars = bars + warp * kRing;

    // this warp's blocks of 8 packed rows: [b0, b1)
    const int nblk = (nkw + kBlockRows - 1) / kBlockRows;
    const int bpw = (nblk + kGemvWarps - 1) / kGemvWarps;
    const int b0 = min(nblk, warp * bpw);
    const int b1 = min(nblk, b0 + bpw);
    const int my_blocks = b1 - b0;

    const int ncols = min(kTileCols, N - n0);
    const uint32_t sbytes = static_cast<uint32_t>(ncols) * 2;
    const uint32_t zbytes = static_cast<uint32_t>(ncols) / 2;

    if (lane == 0) {
        for (int s = 0; s < kRing; ++s) ptx::mbar_init(&my_bars[s], 1);
        ptx::fence_mbar_init();
    }
    __syncwarp();

    auto issue = [&](int j) {  // block b0 + j into slot j % kRing (lane 0 only)
        const int s = j % kRing;
        uint8_t* slot = ring + s * kSlotBytes;
        const int kwb = kw0 + (b0 + j) * kBlockRows;
        const int g_first = kwb / wpg;
        const int g_last = min(G - 1, (kwb + kBlockRows - 1) / wpg);
        const int cnt = g_last - g_first + 1;
        ptx::mbar_arrive_expect_tx(&my_bars[s], kRawBytes + cnt * (sbytes + zbytes));
        ptx::tma_load_2d(slot, &tm_qw, &my_bars[s], n0, kwb);
        for (int c = 0; c < cnt; ++c) {
            const int g = g_first + c;
            ptx::bulk_load(slot + kScOff + c * kTileCols * 2, scales + static_cast<size_t>(g) * N + n0, sbytes,
                           &my_bars[s]);
            ptx::bulk_load(slot + kZrOff + c * (kTileCols / 2), qzeros + static_cast<size_t>(g) * (N >> 3) + (n0 >> 3),
                           zbytes, &my_bars[s]);
        }
    };

    if (lane == 0) {
        for (int j = 0; j < min(kRing, my_blocks); ++j) issue(j);
    }
    if (threadIdx.x == 0) ptx::grid_dep_launch_dependents();
    ptx::grid_dep_wait();  // X and Y belong to the previous kernel in the stream

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

    float acc[MT][4];
#pragma unroll
    for (int m = 0; m < MT; ++m)
#pragma unroll
        for (int c = 0; c < 4; ++c) acc[m][c] = 0.f;

    const int cq = lane;  // columns n0 + 4 cq .. + 3
    const bool col_ok = n0 + cq * 4 < N;
    bool ok = true;
    for (int j = 0; j < my_blocks; ++j) {
        const int s = j % kRing;
        if (!ptx::mbar_wait_bounded(&my_bars[s], (j / kRing) & 1, kWaitLimit, err, kErrGemvTimeout)) {
            ok = false;
            break;
        }
        const uint8_t* slot = ring + s * kSlotBytes;
        const int kwb = kw0 + (b0 + j) * kBlockRows;
        const int g_first = kwb / wpg;
        int cur = -1;
        float sf[4] = {0.f, 0.f, 0.f, 0.f};
        __half2 zz[4];
#pragma unroll
        for (int c = 0; c < 4; ++c) zz[c] = __float2half2_rn(0.f);
        if (col_ok) {
#pragma unroll 2
            for (int r = 0; r < kBlockRows; ++r) {
                const int kw = kwb + r;
                if (kw >= kw1) break;
                const int local = kw / wpg - g_first;
                if (local != cur) {
                    cur = local;
                    const uint2 sv = *reinterpret_cast<const uint2*>(slot + kScOff + local * kTileCols * 2 + cq * 8);
                    sf[0] = __half2float(__ushort_as_half(static_cast<unsigned short>(sv.x & 0xFFFFu)));
                    sf[1] = __half2float(__ushort_as_half(static_cast<unsigned short>(sv.x >> 16)));
                    sf[2] = __half2float(__ushort_as_half(static_cast<unsigned short>(sv.y & 0xFFFFu)));
                    sf[3] = __half2float(__ushort_as_half(static_cast<unsigned short>(sv.y >> 16)));
                    const uint32_t zw = *reinterpret_cast<const uint32_t*>(slot + kZrOff + local * (kTileCols / 2) +
                                                                           (cq >> 1) * 4);
                    const int zsh = (cq & 1) * 16;
#pragma unroll
                    for (int c = 0; c < 4; ++c) {
                        const uint32_t hz = 0x6400u + ((zw >> (zsh + 4 * c)) & 15u) + 1u;  // 1024 + z, exact
                        zz[c] = u32_as_h2(hz | (hz << 16));
                    }
                }
                const uint4 wv = *reinterpret_cast<const uint4*>(slot + r * (kTileCols * 4) + cq * 16);
                const uint32_t w4[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    const __half2 d0 = nib_pair_minus_z(w4[c], 0, zz[c]);   // k 0,4
                    const __half2 d1 = nib_pair_minus_z(w4[c], 4, zz[c]);   // k 1,5
                    const __half2 d2 = nib_pair_minus_z(w4[c], 8, zz[c]);   // k 2,6
                    const __half2 d3 = nib_pair_minus_z(w4[c], 12, zz[c]);  // k 3,7
#pragma unroll
                    for (int m = 0; m < MT; ++m) {
                        const uint4 xv = xs[m * nkw + (kw - kw0)];
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
        __syncwarp();
        if (lane == 0 && j + kRing < my_blocks) {
            ptx::fence_proxy_async_smem();  // our reads of the slot before the async overwrite
            issue(j + kRing);
        }
    }
    if (!ok && lane == 0) {
        // give every copy this warp may still have in flight a bounded chance to land
        for (int s = 0; s < kRing; ++s) ptx::mbar_wait_bounded(&my_bars[s], 0, kWaitLimit, nullptr, 0);
        for (int s = 0; s < kRing; ++s) ptx::mbar_wait_bounded(&my_bars[s], 1, kWaitLimit, nullptr, 0);
    }

    // ---- reduce the 4 warps (all ring traffic has landed: every slot was waited on)
    __syncthreads();
    float* red = reinterpret_cast<float*>(smem);      // [warps][MT][128]
    float* part = red + kGemvWarps * MT * kTileCols;  // [MT][128]
#pragma unroll
    for (int m = 0; m < MT; ++m)
#pragma unroll
        for (int c = 0; c < 4; ++c) red[(warp * MT + m) * kTileCols + cq * 4 + c] = acc[m][c];
    __syncthreads();
    for (int i = threadIdx.x; i < MT * kTileCols; i += kGemvThreads) {
        const int m = i / kTileCols;
        const int nn = i - m * kTileCols;
        float sum = 0.f;
#pragma unroll
        for (int w = 0; w < kGemvWarps; ++w) sum += red[(w * MT + m) * kTileCols + nn];
        part[i] = sum;
    }

    if (cluster_size == 1) {
        __syncthreads();
        for (int i = threadIdx.x; i < MT * kTileCols; i += kGemvThreads) {
            const int m = i / kTileCols;
            const int nn = n0 + (i - m * kTileCols);
            if (m < M && nn < N) y[static_cast<size_t>(m) * N + nn] = __half_as_ushort(__float2half_rn(part[i]));
        }
        return;
    }

    // ---- reduce the cluster's K splits through distributed shared memory, fixed order
    cg::cluster_group cluster = cg::this_cluster();
    cluster.sync();
    const int rank = static_cast<int>(cluster.block_rank());
    const int total = MT * kTileCols;
    const int per_rank = (total + cluster_size - 1) / cluster_size;
    const int i0 = rank * per_rank;
    const int i1 = min(total, i0 + per_rank);
    for (int i = i0 + threadIdx.x; i < i1; i += kGemvThreads) {
        const int m = i / kTileCols;
        const int nn = n0 + (i - m * kTileCols);
        float sum = 0.f;
        for (int r = 0; r < cluster_size; ++r) sum += cluster.map_shared_rank(part, r)[i];
        if (m < M && nn < N) y[static_cast<size_t>(m) * N + nn] = __half_as_ushort(__float2half_rn(sum));
    }
    cluster.sync();  // keep this CTA's shared memory alive until every peer has read it
}

template <int MT, bool ACT>
cudaError_t launch_gemv_t(const PackedWeight& w, const GemvPlan& p, const CUtensorMap* qw_map, const void* x, int M,
                          void* y, cudaStream_t s) {
    const int KW = w.K >> 3;
    const int kw_per_cta = (KW + p.splits - 1) / p.splits;
    const size_t smem = GemvSmem::bytes(MT, kw_per_cta);
    // the reduction scratch reuses the ring
    const size_t red = static_cast<size_t>(kGemvWarps * MT * kTileCols + MT * kTileCols) * 4;
    if (smem > 227 * 1024 || red > static_cast<size_t>(kGemvWarps) * kRing * kSlotBytes) return cudaErrorInvalidValue;
    auto kern = gemv_kernel<MT, ACT>;
    // Once per instantiation (and so before any stream capture that reuses it).
    static const cudaError_t attr_err = [&] {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
        if (e == cudaSuccess) e = cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
        return e;
    }();
    if (attr_err != cudaSuccess) return attr_err;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((w.N + kTileCols - 1) / kTileCols, p.splits, 1);
    cfg.blockDim = dim3(kGemvThreads, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    int nattr = 0;
    attr[nattr].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[nattr].val.programmaticStreamSerializationAllowed = 1;
    ++nattr;
    if (p.splits > 1) {
        attr[nattr].id = cudaLaunchAttributeClusterDimension;
        attr[nattr].val.clusterDim.x = 1;
        attr[nattr].val.clusterDim.y = p.splits;
        attr[nattr].val.clusterDim.z = 1;
        ++nattr;
    }
    cfg.attrs = attr;
    cfg.numAttrs = nattr;
    return cudaLaunchKernelEx(&cfg, kern, *qw_map, w.qzeros, w.scales, w.perm, static_cast<const uint16_t*>(x),
                              static_cast<uint16_t*>(y), M, w.K, w.N, w.G, w.group_size, kw_per_cta, p.splits, w.err);
}

template <bool ACT>
cudaError_t launch_gemv_mt(const PackedWeight& w, const GemvPlan& p, const CUtensorMap* qw_map, const void* x, int M,
                           void* y, cudaStream_t s) {
    switch (p.mt) {
        case 1: return launch_gemv_t<1, ACT>(w, p, qw_map, x, M, y, s);
        case 2: return launch_gemv_t<2, ACT>(w, p, qw_map, x, M, y, s);
        case 4: return launch_gemv_t<4, ACT>(w, p, qw_map, x, M, y, s);
        case 8: return launch_gemv_t<8, ACT>(w, p, qw_map, x, M, y, s);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace

bool gemv_supported(const PackedWeight& w) { return w.group_size >= 32; }

GemvPlan plan_gemv(const PackedWeight& w, int M, int num_sms) {
    GemvPlan p;
    p.mt = M <= 1 ? 1 : M <= 2 ? 2 : M <= 4 ? 4 : 8;
    p.bn = kTileCols;
    const int tiles = (w.N + kTileCols - 1) / kTileCols;
    const int KW = w.K >> 3;
    const int slots = 2 * num_sms;  // two CTAs per SM
    // cluster size along K: the most splits that still fit one wave of CTA slots,
    // keeping at least one 8-row block per warp and the staged X slice small
    int best = 0;
    for (int cs = 1; cs <= 16; cs *= 2) {
        const int kw_per = (KW + cs - 1) / cs;
        if (cs > 1 && kw_per < kGemvWarps * kBlockRows) break;
        if (GemvSmem::bytes(p.mt, kw_per) > 110 * 1024) continue;  // two CTAs per SM
        if (best > 0 && tiles * cs > slots) break;
        best = cs;
    }
    static const int env_cs = [] {
        const char* v = std::getenv("W4A16_GEMV_SPLITS");  // tuning override
        return v ? std::atoi(v) : 0;
    }();
    if (env_cs > 0) best = env_cs;
    p.splits = best > 0 ? best : 16;
    return p;
}

cudaError_t launch_gemv(const PackedWeight& w, const GemvPlan& p, const CUtensorMap* qw_map, const void* x, int M,
                        void* y, cudaStream_t s) {
    if (M <= 0) return cudaSuccess;
    if (M > p.mt || !gemv_supported(w)) return cudaErrorInvalidValue;
    return w.act_order ? launch_gemv_mt<true>(w, p, qw_map, x, M, y, s)
                       : launch_gemv_mt<false>(w, p, qw_map, x, M, y, s);
}

}  // namespace w4a16
