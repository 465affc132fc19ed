// Decode GEMV (M <= 8): Y[M, N] = X[M, K] * W[K, N] with W streamed from packed
// int4 straight out of HBM, on CUDA cores.
//
// Replaces the reference's v2 GEMV (After-Revision-DROFELL/cuda_extends/exllama/
// q_gemm_kernel_gptq.cuh:41-195, host q4_matmul.cu:428-456), which splits K over
// CTAs and reduces with racy fp16 atomics into an output it zeroes concurrently.
//
// At M = 1 the job is reading K*N/2 bytes once; the kernel keeps HBM busy with few
// instructions per packed word:
//   * 256 threads = 8 warps on one 128-column tile; lane l owns columns 4l .. 4l+3, so
//     one 16-byte load per lane reads a warp-wide 512-byte row segment. Each warp
//     streams a contiguous run of packed rows in batches of up to 8 rows, double
//     buffered in registers (the next batch is in flight while this one is consumed).
//     Batches never cross a quantization group. The first batch, and the CTA's scale
//     and zero rows (staged in shared memory), are requested before
//     griddepcontrol.wait, overlapping the previous kernel in the stream.
//   * fp16: (q - z) is formed exactly as fp16 pairs (k_i, k_{i+4}) with the 0x6400
//     exponent trick (one shift, four lop3, two sub.f16x2, two fma.f16x2 per word),
//     dotted with X in f16x2 over 4 terms per half, and once per load batch (8 rows,
//     or 4 in the WIDE configuration) the f16x2 partial is scaled by the group scale
//     into an fp32 accumulator.
//     bf16: the same pairs built on 0x4300 (128 + q), bf16x2 products, scaled into
//     fp32 every row.
//   * Warps reduce through shared memory in a fixed order; a K split across CTAs is a
//     thread-block cluster reduced through distributed shared memory in rank order.
//     Results are deterministic and need neither workspace nor atomics.
//   * Two compiled configurations at M = 1: 2 CTAs per SM with 8-row batches (128
//     registers), and WIDE, 3 CTAs per SM with 4-row batches (85 registers), which
//     hides the weight-load latency better on wide, short-K shapes (plan_gemv).
//   * The planner never picks a single wave over 90 % of the CTA slots: the next
//     kernel in the stream needs room to start early under PDL.
#include <cooperative_groups.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <cmath>
#include <cstdlib>
#include <type_traits>

#include "w4a16_gather.cuh"
#include "w4a16_internal.h"
#include "w4a16_prologue.cuh"
#include "w4a16_ptx.cuh"

namespace cg = cooperative_groups;

namespace w4a16 {
namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kTileCols = 128;                // 32 lanes x 4 columns
constexpr int kMaxSplits = 8;                 // cluster size along K (portable)
constexpr size_t kMaxStageBytes = 64 * 1024;  // X, scale and zero rows staged per CTA
constexpr int kMinBlocks = 2;                 // resident CTAs per SM the register budget is sized for
constexpr int kMinBlocksWide = 3;             // the same for the WIDE configuration (M = 1 only)

// packed rows per load batch: two batches of weights live in registers at once
template <int MT>
constexpr int batch_rows() { return MT == 1 ? 8 : MT == 2 ? 4 : MT == 4 ? 4 : 2; }
// WIDE (M = 1): 3 CTAs per SM (<= 85 registers), so batches of 4 rows
template <int MT, bool WIDE>
constexpr int batch_rows_cfg() { return WIDE ? 4 : batch_rows<MT>(); }

// ---------------------------------------------------------------- one-instruction helpers
__device__ __forceinline__ uint4 ld_stream(const int32_t* p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}
__device__ __forceinline__ uint32_t and_or(uint32_t a, uint32_t mask, uint32_t bits) {  // (a & mask) | bits
    uint32_t r;
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(r) : "r"(a), "r"(mask), "r"(bits));
    return r;
}
template <int DT>
__device__ __forceinline__ uint32_t sub2(uint32_t a, uint32_t b) {
    uint32_t r;
    if constexpr (DT == kFP16)
        asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
    else
        asm("sub.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
    return r;
}
template <int DT>
__device__ __forceinline__ uint32_t mul2(uint32_t a, uint32_t b) {
    uint32_t r;
    if constexpr (DT == kFP16)
        asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
    else
        asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
    return r;
}
template <int DT>
__device__ __forceinline__ uint32_t fma2(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t r;
    if constexpr (DT == kFP16)
        asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(c));
    else
        asm("fma.rn.bf16x2 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(c));
    return r;
}
// sum of the two halves in fp32
template <int DT>
__device__ __forceinline__ float hsum(uint32_t p) {
    if constexpr (DT == kFP16) {
        float lo, hi;
        asm("{\n\t.reg .f16 l, h;\n\tmov.b32 {l, h}, %2;\n\tcvt.f32.f16 %0, l;\n\tcvt.f32.f16 %1, h;\n\t}"
            : "=f"(lo), "=f"(hi)
            : "r"(p));
        return lo + hi;
    } else {
        return __uint_as_float(p << 16) + __uint_as_float(p & 0xFFFF0000u);
    }
}

// exact (q - z) pairs (k_i, k_{i+4}), i = 0..3, of one packed word.
// fp16: z0 = (1024 + z) pairs, z1 = -(64 + z) pairs; bf16: z0 = (128 + z) pairs.
template <int DT>
__device__ __forceinline__ void dq(uint32_t w, uint32_t z0, uint32_t z1, uint32_t (&d)[4]) {
    if constexpr (DT == kFP16) {
        constexpr uint32_t kSixteenth = 0x2C002C00u;  // (1/16, 1/16)
        const uint32_t hi = w >> 8;
        d[0] = sub2<DT>(and_or(w, 0x000F000Fu, 0x64006400u), z0);             // 1024 + q - (1024 + z)
        d[1] = fma2<DT>(and_or(w, 0x00F000F0u, 0x64006400u), kSixteenth, z1);  // (1024 + 16 q) / 16 - (64 + z)
        d[2] = sub2<DT>(and_or(hi, 0x000F000Fu, 0x64006400u), z0);
        d[3] = fma2<DT>(and_or(hi, 0x00F000F0u, 0x64006400u), kSixteenth, z1);
    } else {
        d[0] = sub2<DT>(and_or(w, 0x000F000Fu, 0x43004300u), z0);
        d[1] = sub2<DT>(and_or(w >> 4, 0x000F000Fu, 0x43004300u), z0);
        d[2] = sub2<DT>(and_or(w >> 8, 0x000F000Fu, 0x43004300u), z0);
        d[3] = sub2<DT>(and_or(w >> 12, 0x000F000Fu, 0x43004300u), z0);
    }
}

// zero constants of one stored zero nibble (z = nibble + 1), all exact
template <int DT>
__device__ __forceinline__ void zero_consts(uint32_t nib, uint32_t& z0, uint32_t& z1) {
    const uint32_t zp = (nib & 15u) + 1u;
    if constexpr (DT == kFP16) {
        z0 = (0x6400u | zp) * 0x10001u;         // 1024 + z
        z1 = (0xD400u | (zp << 4)) * 0x10001u;  // -(64 + z)
    } else {
        z0 = (0x4300u | zp) * 0x10001u;  // 128 + z
        z1 = 0;
    }
}

// f16x2 / bf16x2 dot of 4 pairs, continuing the partial p (or starting it)
template <int DT>
__device__ __forceinline__ uint32_t dot(const uint32_t (&d)[4], const uint4& xq, uint32_t p, bool start) {
    uint32_t h = start ? mul2<DT>(d[0], xq.x) : fma2<DT>(d[0], xq.x, p);
    h = fma2<DT>(d[1], xq.y, h);
    h = fma2<DT>(d[2], xq.z, h);
    return fma2<DT>(d[3], xq.w, h);
}

template <int B>
struct Batch {
    uint4 w[B];    // 4 words (this lane's columns) per packed row
    int row, n;    // first packed row, rows (0: none)
    int g;         // group of every row of the batch
};

struct Cursor {
    int row, g, rem;  // next packed row, its group, rows left in that group
};

// groups a run of kw_per_cta packed rows can touch (not aligned to groups: one more)
__host__ __device__ __forceinline__ int groups_bound(int kw_per_cta, int rpg) { return (kw_per_cta + rpg - 1) / rpg + 1; }

template <int MT, int DT, bool WIDE, int PRO, int SEGS>
__global__ void __launch_bounds__(kThreads, WIDE ? kMinBlocksWide : kMinBlocks)
    gemv_kernel(const GemvSegs segs, const uint16_t* __restrict__ x, int M, int K, int rpg, int kw_per_warp,
                int* __restrict__ err, const GatherArgs ga, const GemvPrologue pro) {
    constexpr int B = batch_rows_cfg<MT, WIDE>();
    // fp16 f16x2 partials span this many rows (up to 32 products per half) before they
    // are scaled into fp32: relative error ~1e-3 at K = 4096, against 6e-4 at 2 rows
    constexpr int kSpan = (MT == 1 && DT == kFP16) ? B : 1;
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    // this CTA's weight segment (one launch covers up to kMaxSegs projections that read
    // the same X, e.g. q / k / v): constant-index selects keep the parameters in place
    // (SEGS = 1: the single weight of a plain call, read at fixed indices)
    int seg = 0;
#pragma unroll
    for (int i = 1; i < SEGS; ++i)
        if (i < segs.count && static_cast<int>(blockIdx.x) >= segs.tile0[i]) seg = i;
    // a field of this CTA's segment, read from the parameters where it is used (only the
    // index stays live across the main loop)
    auto pick = [&](auto const (&arr)[kMaxSegs]) {
        auto v = arr[0];
#pragma unroll
        for (int i = 1; i < SEGS; ++i)
            if (seg == i) v = arr[i];
        return v;
    };
    const int N = pick(segs.N);
    int tile_base = 0;
#pragma unroll
    for (int i = 1; i < SEGS; ++i)
        if (seg == i) tile_base = segs.tile0[i];
    const int n0 = (static_cast<int>(blockIdx.x) - tile_base) * kTileCols;
    const int KW = K >> 3;
    const int kw_per_cta = kw_per_warp * kWarps;
    const int c_r0 = blockIdx.y * kw_per_cta;
    const int c_r1 = min(KW, c_r0 + kw_per_cta);
    const int r0 = min(c_r1, c_r0 + warp * kw_per_warp);
    const int r1 = min(c_r1, r0 + kw_per_warp);
    const int g_lo = c_r0 / rpg;
    const int ng = c_r1 > c_r0 ? (c_r1 - 1) / rpg - g_lo + 1 : 0;
    // lanes past N read the last valid columns; their sums are never stored
    const int colc = min(n0 + lane * 4, N - 4);
    const int zsh = (colc & 7) * 4;

    // shared memory: X rows in pair order [rows][MT] (uint4), scale rows [ng][128]
    // fp16, zero words [ng][16], then warp partials [kWarps][MT][128] and the CTA tile
    // [MT][128] (fp32). Offsets come from the group bound every CTA shares, so the
    // tile sits at the same address in each CTA of a cluster (peers read it by offset).
    const int ng_max = groups_bound(kw_per_cta, rpg);
    extern __shared__ __align__(16) uint4 smem[];
    uint4* xs = smem;
    uint2* sc_s = reinterpret_cast<uint2*>(xs + static_cast<size_t>(kw_per_cta) * MT);
    uint32_t* zr_s = reinterpret_cast<uint32_t*>(sc_s + static_cast<size_t>(ng_max) * 32);
    float* red = reinterpret_cast<float*>(zr_s + ((static_cast<size_t>(ng_max) * 16 + 3) & ~static_cast<size_t>(3)));

    const int32_t* qw = pick(segs.qweight) + colc;
    auto load = [&](Batch<B>& b, Cursor& cur) {
        b.row = cur.row;
        b.g = cur.g;
        b.n = min(B, min(cur.rem, r1 - cur.row));
        if (b.n <= 0) {
            b.n = 0;
            return;
        }
        const int32_t* p = qw + static_cast<size_t>(cur.row) * N;
#pragma unroll
        for (int j = 0; j < B; ++j)
            if (j < b.n) b.w[j] = ld_stream(p + static_cast<size_t>(j) * N);
        cur.row += b.n;
        cur.rem -= b.n;
        if (cur.rem == 0) {
            ++cur.g;
            cur.rem = rpg;
        }
    };

    float acc[MT][4];
#pragma unroll
    for (int m = 0; m < MT; ++m)
#pragma unroll
        for (int c = 0; c < 4; ++c) acc[m][c] = 0.f;

    Cursor cur;
    cur.row = r0;
    cur.g = r0 / rpg;
    cur.rem = rpg - (r0 - cur.g * rpg);
    Batch<B> a, b;
    load(a, cur);  // weights: requested before the previous kernel has finished
    // the CTA's scale and zero rows (weights too)
    const uint16_t* __restrict__ scales = pick(segs.scales);
    const int32_t* __restrict__ qzeros = pick(segs.qzeros);
    for (int i = threadIdx.x; i < ng * 32; i += kThreads) {
        const int gl = i >> 5;
        const int c = min(n0 + (i & 31) * 4, N - 4);
        sc_s[i] = __ldg(reinterpret_cast<const uint2*>(scales + static_cast<size_t>(g_lo + gl) * N + c));
    }
    for (int i = threadIdx.x; i < ng * 16; i += kThreads) {
        const int gl = i >> 4;
        const int wc = min((n0 >> 3) + (i & 15), (N >> 3) - 1);
        zr_s[i] = qzeros ? static_cast<uint32_t>(__ldg(qzeros + static_cast<size_t>(g_lo + gl) * (N >> 3) + wc))
                         : kSymmetricZeroWord;
    }
    if (threadIdx.x == 0) ptx::grid_dep_launch_dependents();
    ptx::grid_dep_wait();  // X (and Y) belong to the previous kernel in the stream
    [[maybe_unused]] __shared__ float rmf_s[MT];
    if constexpr (PRO == kProRmsNorm) {
        // RMSNorm factor of each row over all of K, in one fixed order in every CTA:
        // rsqrt(sum(x^2) / K + eps) (fuse_v2/rms_norm.cu:48-78)
        __shared__ float wsum[kWarps][MT];
        float ss[MT];
#pragma unroll
        for (int m = 0; m < MT; ++m) ss[m] = 0.f;
        for (int k8 = threadIdx.x; k8 < (K >> 3); k8 += kThreads) {
#pragma unroll
            for (int m = 0; m < MT; ++m) {
                if (m < M) {
                    const uint4 raw = __ldg(reinterpret_cast<const uint4*>(x + static_cast<size_t>(m) * K) + k8);
                    const uint32_t r4[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const float lo = clamp_h2f(r4[e] & 0xFFFFu), hi = clamp_h2f(r4[e] >> 16);
                        ss[m] = fmaf(lo, lo, ss[m]);
                        ss[m] = fmaf(hi, hi, ss[m]);
                    }
                }
            }
        }
#pragma unroll
        for (int m = 0; m < MT; ++m) {
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) ss[m] += __shfl_xor_sync(0xffffffffu, ss[m], off);
            if (lane == 0) wsum[warp][m] = ss[m];
        }
        __syncthreads();
        if (threadIdx.x < MT) {
            float t = 0.f;
            for (int w = 0; w < kWarps; ++w) t += wsum[w][threadIdx.x];
            rmf_s[threadIdx.x] = rsqrtf(t * (1.0f / static_cast<float>(K)) + pro.eps);
        }
        __syncthreads();
    }
    // stage X[:, c_r0*8 : c_r1*8) as pairs (k_i, k_{i+4}) per packed row, after the
    // prologue: RMSNorm of X (its result also written to pro.out by the CTAs of the first
    // column tile, which together cover all of K), or silu(X) * pro.up
    for (int i = threadIdx.x; i < (c_r1 - c_r0) * MT; i += kThreads) {
        const int r = i / MT;
        const int m = i - r * MT;
        uint4 v = make_uint4(0, 0, 0, 0);
        if (m < M) {
            uint4 raw = __ldg(reinterpret_cast<const uint4*>(x + static_cast<size_t>(m) * K) + (c_r0 + r));
            if constexpr (PRO == kProRmsNorm) {
                raw = rms_apply8(raw, __ldg(reinterpret_cast<const uint4*>(pro.norm_w) + (c_r0 + r)), rmf_s[m]);
                if (pro.out && blockIdx.x == 0)
                    *(reinterpret_cast<uint4*>(pro.out + static_cast<size_t>(m) * K) + (c_r0 + r)) = raw;
            } else if constexpr (PRO == kProSiluMul) {
                raw = silu_mul8(raw, __ldg(reinterpret_cast<const uint4*>(pro.up + static_cast<size_t>(m) * K) + (c_r0 + r)));
            }
            v.x = __byte_perm(raw.x, raw.z, 0x5410);
            v.y = __byte_perm(raw.x, raw.z, 0x7632);
            v.z = __byte_perm(raw.y, raw.w, 0x5410);
            v.w = __byte_perm(raw.y, raw.w, 0x7632);
        }
        xs[i] = v;
    }
    __syncthreads();

    // FULL: b.n == B, so every guard and flush point is a compile-time constant
    auto consume = [&](const Batch<B>& b, auto full_tag) {
        constexpr bool FULL = decltype(full_tag)::value;
        const int gl = b.g - g_lo;
        const uint2 s2 = sc_s[gl * 32 + lane];
        const uint32_t zw = zr_s[gl * 16 + ((colc - n0) >> 3)] >> zsh;
        float s[4];
        s[0] = __half2float(__ushort_as_half(static_cast<uint16_t>(s2.x & 0xFFFFu)));
        s[1] = __half2float(__ushort_as_half(static_cast<uint16_t>(s2.x >> 16)));
        s[2] = __half2float(__ushort_as_half(static_cast<uint16_t>(s2.y & 0xFFFFu)));
        s[3] = __half2float(__ushort_as_half(static_cast<uint16_t>(s2.y >> 16)));
        uint32_t z0[4], z1[4];
#pragma unroll
        for (int c = 0; c < 4; ++c) zero_consts<DT>(zw >> (4 * c), z0[c], z1[c]);
        const uint4* xb = xs + (b.row - c_r0) * MT;
        [[maybe_unused]] uint32_t part[MT][4];  // MT < 4: f16x2 partials carried across kSpan rows
#pragma unroll
        for (int j = 0; j < B; ++j) {
            if (FULL || j < b.n) {
                if constexpr (MT >= 4) {
                    // several rows of X: dequantize the row's four words once, then stream X
                    uint32_t d[4][4];
#pragma unroll
                    for (int c = 0; c < 4; ++c) dq<DT>((&b.w[j].x)[c], z0[c], z1[c], d[c]);
#pragma unroll
                    for (int m = 0; m < MT; ++m) {
                        if (m < M) {
                            const uint4 xq = xb[j * MT + m];
#pragma unroll
                            for (int c = 0; c < 4; ++c)
                                acc[m][c] = fmaf(s[c], hsum<DT>(dot<DT>(d[c], xq, 0u, true)), acc[m][c]);
                        }
                    }
                } else {
                    // MT = 1 and 2 mean exactly that many rows of X
                    uint4 xq[MT];
#pragma unroll
                    for (int m = 0; m < MT; ++m) xq[m] = xb[j * MT + m];
                    const bool start = j % kSpan == 0;
                    const bool flush = j % kSpan == kSpan - 1 || (FULL ? j + 1 == B : j + 1 == b.n);
#pragma unroll
                    for (int c = 0; c < 4; ++c) {
                        uint32_t d[4];
                        dq<DT>((&b.w[j].x)[c], z0[c], z1[c], d);
#pragma unroll
                        for (int m = 0; m < MT; ++m) {
                            part[m][c] = dot<DT>(d, xq[m], part[m][c], start);
                            if (flush) acc[m][c] = fmaf(s[c], hsum<DT>(part[m][c]), acc[m][c]);
                        }
                    }
                }
            }
        }
    };
    auto consume_any = [&](const Batch<B>& b) {
        if (b.n == B)
            consume(b, std::true_type{});
        else
            consume(b, std::false_type{});
    };

    // two batches per warp: the next one is in flight while this one is consumed
    while (a.n > 0) {
        load(b, cur);
        consume_any(a);
        if (b.n == 0) break;
        load(a, cur);
        consume_any(b);
    }

    // ---- fixed-order reduction: warps, then the cluster's CTAs
    float* mine = red + (warp * MT) * kTileCols + lane * 4;
#pragma unroll
    for (int m = 0; m < MT; ++m)
        *reinterpret_cast<float4*>(mine + m * kTileCols) = make_float4(acc[m][0], acc[m][1], acc[m][2], acc[m][3]);
    __syncthreads();
    float* tile = red + kWarps * MT * kTileCols;
    const int splits = gridDim.y;
    for (int i = threadIdx.x; i < MT * kTileCols; i += kThreads) {
        float sum = 0.f;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) sum += red[w * MT * kTileCols + i];
        if (splits == 1) {
            const int m = i / kTileCols;
            const int n = n0 + (i - m * kTileCols);
            if (m < M && n < N) {
                out_store(ga, pick(segs.y), N, m, n,
                                                                          DT == kFP16 ? __half_as_ushort(__float2half_rn(sum)) : __bfloat16_as_ushort(__float2bfloat16_rn(sum)));
            }
        } else {
            tile[i] = sum;
        }
    }
    if (splits == 1) return;
    cg::cluster_group cluster = cg::this_cluster();
    cluster.sync();
    const int rank = static_cast<int>(cluster.block_rank());
    const int total = min(M, MT) * kTileCols;
    const int per = (total + splits - 1) / splits;
    const int i0 = rank * per;
    const int i1 = min(total, i0 + per);
    for (int i = i0 + static_cast<int>(threadIdx.x); i < i1; i += kThreads) {
        float sum = 0.f;
#pragma unroll
        for (int r = 0; r < kMaxSplits; ++r)  // independent remote loads, summed in rank order
            if (r < splits) sum += cluster.map_shared_rank(tile, r)[i];
        const int m = i / kTileCols;
        const int n = n0 + (i - m * kTileCols);
        if (n < N) {
            out_store(ga, pick(segs.y), N, m, n,
                                                                      DT == kFP16 ? __half_as_ushort(__float2half_rn(sum)) : __bfloat16_as_ushort(__float2bfloat16_rn(sum)));
        }
    }
    cluster.sync();  // keep this CTA's shared memory alive until every peer has read it
}

size_t stage_bytes(int mt, int kw_per_cta, int rpg) {
    const size_t ng = static_cast<size_t>(groups_bound(kw_per_cta, rpg));
    return static_cast<size_t>(kw_per_cta) * mt * 16 + ng * kTileCols * 2 + ((ng * 16 + 3) & ~size_t(3)) * 4;
}

size_t smem_bytes(int mt, int kw_per_cta, int rpg) {
    return stage_bytes(mt, kw_per_cta, rpg) + static_cast<size_t>(kWarps + 1) * mt * kTileCols * 4;
}

template <int MT, int DT, bool WIDE, int PRO, int SEGS = 1>
cudaError_t launch_t(const PackedWeight& w, const GemvSegs& segs, const GemvPlan& p, const void* x, int M,
                     cudaStream_t s, const GatherArgs& ga, const GemvPrologue& pro) {
    const int rpg = w.group_size >> 3;
    const int kw_per_cta = p.kpw * kWarps;
    if (segs.count > SEGS) return cudaErrorInvalidValue;
    auto kern = gemv_kernel<MT, DT, WIDE, PRO, SEGS>;
    // Once per instantiation (and so before any stream capture that reuses it).
    static const cudaError_t attr_err = [&] {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(kMaxStageBytes + (kWarps + 1) * MT * kTileCols * 4));
        if (e == cudaSuccess) e = cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
        return e;
    }();
    if (attr_err != cudaSuccess) return attr_err;
    if (stage_bytes(MT, kw_per_cta, rpg) > kMaxStageBytes || p.splits > kMaxSplits || p.kpw <= 0)
        return cudaErrorInvalidValue;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(segs.tile0[segs.count], p.splits, 1);
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = smem_bytes(MT, kw_per_cta, rpg);
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
    return cudaLaunchKernelEx(&cfg, kern, segs, static_cast<const uint16_t*>(x), M, w.K, rpg, p.kpw, w.err, ga, pro);
}

template <int DT>
cudaError_t launch_mt(const PackedWeight& w, const GemvSegs& segs, const GemvPlan& p, const void* x, int M,
                      cudaStream_t s, const GatherArgs& ga, const GemvPrologue& pro) {
    if (pro.mode != kProNone) {  // prologues: fp16, M <= 2
        if constexpr (DT == kFP16) {
            // the RMSNorm prologue serves grouped launches (q / k / v, gate + up), silu * mul
            // the single down projection
            if (p.mt == 1) {
                if (pro.mode == kProRmsNorm)
                    return p.wide ? launch_t<1, DT, true, kProRmsNorm, kMaxSegs>(w, segs, p, x, M, s, ga, pro)
                                  : launch_t<1, DT, false, kProRmsNorm, kMaxSegs>(w, segs, p, x, M, s, ga, pro);
                return p.wide ? launch_t<1, DT, true, kProSiluMul>(w, segs, p, x, M, s, ga, pro)
                              : launch_t<1, DT, false, kProSiluMul>(w, segs, p, x, M, s, ga, pro);
            }
            if (p.mt == 2)
                return pro.mode == kProRmsNorm
                           ? launch_t<2, DT, false, kProRmsNorm, kMaxSegs>(w, segs, p, x, M, s, ga, pro)
                           : launch_t<2, DT, false, kProSiluMul>(w, segs, p, x, M, s, ga, pro);
        }
        return cudaErrorInvalidValue;
    }
    switch (p.mt) {
        case 1:
            return p.wide ? launch_t<1, DT, true, kProNone>(w, segs, p, x, M, s, ga, pro)
                          : launch_t<1, DT, false, kProNone>(w, segs, p, x, M, s, ga, pro);
        case 2: return launch_t<2, DT, false, kProNone>(w, segs, p, x, M, s, ga, pro);
        case 4: return launch_t<4, DT, false, kProNone>(w, segs, p, x, M, s, ga, pro);
        case 8: return launch_t<8, DT, false, kProNone>(w, segs, p, x, M, s, ga, pro);
        default: return cudaErrorInvalidValue;
    }
}

int batch_rows_rt(int mt, bool wide) {
    if (wide) return batch_rows_cfg<1, true>();
    return mt == 1 ? batch_rows<1>() : mt == 2 ? batch_rows<2>() : mt == 4 ? batch_rows<4>() : batch_rows<8>();
}

}  // namespace

bool gemv_supported(const PackedWeight& w) {
    // whole packed rows per group; 16-byte row segments for every lane; the staged
    // slice of the widest split fits
    if (w.group_size % 8 != 0 || w.N % 4 != 0 || w.N < 4) return false;
    const int KW = w.K >> 3;
    const int b = batch_rows<1>();
    const int kpw = ((KW + kMaxSplits * kWarps - 1) / (kMaxSplits * kWarps) + b - 1) / b * b;
    return stage_bytes(1, kpw * kWarps, w.group_size >> 3) <= kMaxStageBytes;
}

GemvPlan plan_gemv(const PackedWeight& w, int M, int num_sms) {
    GemvPlan p;
    p.mt = M <= 1 ? 1 : M <= 2 ? 2 : M <= 4 ? 4 : 8;
    p.bn = kTileCols;
    const int tiles = (w.N + kTileCols - 1) / kTileCols;
    const int KW = w.K >> 3;
    const int rpg = w.group_size >> 3;
    // WIDE configuration (M = 1): 3 CTAs per SM of 4-row batches. Measured faster on
    // wide, short-K shapes (4096 x 22016: 15.3 vs 16.4 us; 4096 x 12288: 9.7 vs 10.4 us)
    // and slower elsewhere (4096 x 11008, 8192 x 28672, 11008 x 4096).
    static const int env_wide = [] {
        const char* v = std::getenv("W4A16_GEMV_WIDE");  // tuning override (0 or 1)
        return v ? std::atoi(v) : -1;
    }();
    p.wide = p.mt == 1 && tiles >= 96 && KW <= 512;
    if (p.mt == 1 && (env_wide == 0 || env_wide == 1)) p.wide = env_wide == 1;
    const int slots = (p.wide ? kMinBlocksWide : kMinBlocks) * num_sms;
    // rows per warp for a given split: whole batches, so warps start on batch boundaries
    auto kpw_of = [&](int cs) {
        const int b = batch_rows_rt(p.mt, p.wide);
        const int kpw = (KW + cs * kWarps - 1) / (cs * kWarps);
        return (kpw + b - 1) / b * b;
    };
    auto fits = [&](int cs) { return stage_bytes(p.mt, kpw_of(cs) * kWarps, rpg) <= kMaxStageBytes; };
    // the staged slice must fit: fewer rows of X per pass for very long K
    while (p.mt > 1 && !fits(kMaxSplits)) p.mt >>= 1;
    // Cluster size along K. A CTA pays a fixed ramp (launch, staging, first load
    // latency: about as long as streaming kRampRows rows per warp), so the estimate is
    // waves x (rows per warp + ramp): one wave of long per-warp streams wins. A single
    // wave that fills more than 90 % of the CTA slots is skipped: it leaves the next
    // kernel in the stream no room to start early (PDL) and measured up to 27 % slower
    // (4096 x 12288 at M = 1, B200).
    constexpr int kRampRows = 10;
    int best = 0;
    long long best_cost = 0;
    for (int cs = 1; cs <= kMaxSplits; ++cs) {
        if (!fits(cs)) continue;
        const int kpw = kpw_of(cs);
        const int eff = (KW + kpw * kWarps - 1) / (kpw * kWarps);  // CTAs that get rows
        if (eff != cs) continue;
        const long long ctas = static_cast<long long>(tiles) * cs;
        const long long waves = (ctas + slots - 1) / slots;
        if (waves == 1 && ctas * 10 > static_cast<long long>(slots) * 9) continue;
        const long long cost = waves * (kpw + kRampRows);
        if (best == 0 || cost < best_cost) {
            best = cs;
            best_cost = cost;
        }
    }
    static const int env_cs = [] {
        const char* v = std::getenv("W4A16_GEMV_SPLITS");  // tuning override
        return v ? std::atoi(v) : 0;
    }();
    if (env_cs >= 1 && env_cs <= kMaxSplits && fits(env_cs)) best = env_cs;
    if (best == 0) best = kMaxSplits;
    p.kpw = kpw_of(best);
    p.splits = (KW + p.kpw * kWarps - 1) / (p.kpw * kWarps);
    return p;
}

cudaError_t launch_gemv(const PackedWeight& w, const GemvPlan& p, const void* x, int M, void* y, DType dt,
                        cudaStream_t s, const GatherArgs* gather) {
    if (M <= 0) return cudaSuccess;
    if (M > p.mt || !gemv_supported(w)) return cudaErrorInvalidValue;
    GatherArgs ga = {};
    if (gather) ga = *gather;
    GemvSegs segs = {};
    segs.count = 1;
    segs.qweight[0] = w.qweight;
    segs.qzeros[0] = w.kernel_qzeros();
    segs.scales[0] = w.scales;
    segs.y[0] = static_cast<uint16_t*>(y);
    segs.N[0] = w.N;
    segs.tile0[1] = (w.N + kTileCols - 1) / kTileCols;
    const GemvPrologue pro = {};
    return dt == kFP16 ? launch_mt<kFP16>(w, segs, p, x, M, s, ga, pro) : launch_mt<kBF16>(w, segs, p, x, M, s, ga, pro);
}

cudaError_t launch_gemv_group(const PackedWeight* const* ws, void* const* ys, int count, const void* x, int M,
                              DType dt, const GemvPrologue& pro, int num_sms, cudaStream_t s) {
    if (M <= 0) return cudaSuccess;
    if (count < 1 || count > kMaxSegs) return cudaErrorInvalidValue;
    GemvSegs segs = {};
    segs.count = count;
    int tiles = 0;
    for (int i = 0; i < count; ++i) {
        const PackedWeight& w = *ws[i];
        if (!gemv_supported(w) || w.K != ws[0]->K || w.group_size != ws[0]->group_size || w.act_order)
            return cudaErrorInvalidValue;
        segs.qweight[i] = w.qweight;
        segs.qzeros[i] = w.kernel_qzeros();
        segs.scales[i] = w.scales;
        segs.y[i] = static_cast<uint16_t*>(ys[i]);
        segs.N[i] = w.N;
        segs.tile0[i] = tiles;
        tiles += (w.N + kTileCols - 1) / kTileCols;
    }
    segs.tile0[count] = tiles;
    PackedWeight all = *ws[0];  // planned as one weight of every segment's columns
    all.N = tiles * kTileCols;
    const GemvPlan p = plan_gemv(all, M, num_sms);
    if (M > p.mt) return cudaErrorInvalidValue;
    const GatherArgs ga = {};
    return dt == kFP16 ? launch_mt<kFP16>(all, segs, p, x, M, s, ga, pro) : launch_mt<kBF16>(all, segs, p, x, M, s, ga, pro);
}

}  // namespace w4a16
