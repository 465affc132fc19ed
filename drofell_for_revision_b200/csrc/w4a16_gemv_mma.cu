// Decode GEMV on a repacked weight (M <= 8 per pass): the dot products run on the
// tensor cores with warp-level mma.sync m16n8k16 (fp32 accumulate), so each packed
// word costs its dequantization (one shift, four lop3, four f16x2 ops) and 1/32 of an
// MMA instead of ~15 more CUDA-core instructions.
//
// Why a repack: the MMA's A fragment gives lane l = 4g + t the elements
// (row g | g+8) x (k 2t, 2t+1 | 2t+8, 2t+9) of a 16 x 16 tile, where a GPTQ word holds
// 8 consecutive k of one column. repack_mma_kernel (run once, at handle creation)
// writes, for every 16-column x 16-k tile, lane l's eight nibbles into one word whose
// lop3 extraction yields the fragment registers directly:
//   nibble 0,4 -> (col g,   k 2t, 2t+1)   register 0 (E0 = w & 0x000F000F)
//   nibble 2,6 -> (col g+8, k 2t, 2t+1)   register 1 (E2 = (w >> 8) & 0x000F000F)
//   nibble 1,5 -> (col g,   k 2t+8, 2t+9) register 2 (E1 = w & 0x00F000F0, x16)
//   nibble 3,7 -> (col g+8, k 2t+8, 2t+9) register 3 (E3 = (w >> 8) & 0x00F000F0, x16)
// Words are stored [64-column stripe][16-k block][lane][4 tiles of the stripe], so a
// warp streaming one stripe along K reads 512 contiguous bytes per k block.
//
// The caller's qweight is untouched (the reference shuffles it in place,
// q4_matrix.cu:16-30,179); the repacked copy is the handle's own.
//
// Kernel: a CTA owns one 64-column stripe; its 4 warps split the CTA's K range in
// batches of up to 4 k blocks that never cross a quantization group, double buffered
// in registers. The A fragments are the magic-biased nibbles straight out of lop3
// (fp16: 1024 + q, and 1024 + 16 q for k % 16 >= 8 with those X values pre-scaled by
// 1/16; bf16: 128 + q). The tensor core multiplies them exactly and accumulates in
// fp32, so the bias and the zero point come off afterwards: two more MMAs per k block
// with constant A fragments give, per token, C = sum of bias * X and S = sum of X over
// the same k, and at each group end
//     Y += s * (D - C - z * S)            (bf16: D - (128 + z) * S)
// in fp32. Per packed word that is one shift and four lop3 (bf16: three shifts) plus
// 1/32 of the tile MMA. Warps reduce through shared memory in a fixed order, a K split
// across CTAs through distributed shared memory of a cluster in rank order:
// deterministic, no workspace, no atomics.
#include <cooperative_groups.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <cstdlib>
#include <type_traits>

#include "w4a16_gather.cuh"
#include "w4a16_internal.h"
#include "w4a16_ptx.cuh"

namespace cg = cooperative_groups;

namespace w4a16 {
namespace {

constexpr int kThreads = 128;
constexpr int kWarps = 4;
constexpr int kStripe = 64;   // columns per CTA: 4 MMA tiles of 16
constexpr int kMaxTok = 8;    // MMA N
constexpr int kBatch = 8;     // k blocks (16 k) per ring slot: 4 KB
constexpr int kSlots = 2;     // ring slots per warp: up to 8 KB in flight per warp
constexpr int kMaxSplits = 8;
constexpr int kMinBlocks = 3;
constexpr size_t kSmemBudget = 75 * 1024;  // three CTAs per SM
constexpr size_t kRingBytes = static_cast<size_t>(kWarps) * kSlots * kBatch * 512;
constexpr uint32_t kWaitLimit = 1u << 26;
constexpr int kErrGemvMmaTimeout = 64;

__device__ __forceinline__ uint32_t and_or(uint32_t a, uint32_t mask, uint32_t bits) {  // (a & mask) | bits
    uint32_t r;
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(r) : "r"(a), "r"(mask), "r"(bits));
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
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    if constexpr (DT == kFP16)
        asm volatile(
            "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
            "{%0, %1, %2, %3};"
            : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
            : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
    else
        asm volatile(
            "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
            "{%0, %1, %2, %3};"
            : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
            : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// A fragment of one repacked word, magic-biased: fp16 (1024 + q) for k % 16 < 8 and
// (1024 + 16 q) for k % 16 >= 8; bf16 (128 + q). Exact values; the bias comes off later.
template <int DT>
__device__ __forceinline__ void biased_frag(uint32_t w, uint32_t (&a)[4]) {
    if constexpr (DT == kFP16) {
        const uint32_t hi = w >> 8;
        a[0] = and_or(w, 0x000F000Fu, 0x64006400u);
        a[1] = and_or(hi, 0x000F000Fu, 0x64006400u);
        a[2] = and_or(w, 0x00F000F0u, 0x64006400u);
        a[3] = and_or(hi, 0x00F000F0u, 0x64006400u);
    } else {
        a[0] = and_or(w, 0x000F000Fu, 0x43004300u);
        a[1] = and_or(w >> 8, 0x000F000Fu, 0x43004300u);
        a[2] = and_or(w >> 4, 0x000F000Fu, 0x43004300u);
        a[3] = and_or(w >> 12, 0x000F000Fu, 0x43004300u);
    }
}

// ------------------------------------------------------------------ repack
// One thread per output word. src: qweight in kernel row order [K/8, N].
__global__ void repack_mma_kernel(const int32_t* __restrict__ src, int32_t* __restrict__ dst, int K, int N,
                                  int stripes) {
    const long long o = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
    const int kb_count = K >> 4;
    const long long total = static_cast<long long>(stripes) * kb_count * 128;
    if (o >= total) return;
    const int w = static_cast<int>(o & 3);
    const int lane = static_cast<int>((o >> 2) & 31);
    const long long rest = o >> 7;
    const int kb = static_cast<int>(rest % kb_count);
    const int stripe = static_cast<int>(rest / kb_count);
    const int n0 = (stripe * 4 + w) * 16;
    const int g = lane >> 2, t = lane & 3;
    auto q = [&](int n, int k) -> uint32_t {
        if (n >= N) return 0u;
        return (static_cast<uint32_t>(__ldg(src + static_cast<size_t>(k >> 3) * N + n)) >> ((k & 7) * 4)) & 15u;
    };
    const int k0 = kb * 16;
    uint32_t v = 0;
    v |= q(n0 + g, k0 + 2 * t) << 0;
    v |= q(n0 + g, k0 + 2 * t + 8) << 4;
    v |= q(n0 + g + 8, k0 + 2 * t) << 8;
    v |= q(n0 + g + 8, k0 + 2 * t + 8) << 12;
    v |= q(n0 + g, k0 + 2 * t + 1) << 16;
    v |= q(n0 + g, k0 + 2 * t + 9) << 20;
    v |= q(n0 + g + 8, k0 + 2 * t + 1) << 24;
    v |= q(n0 + g + 8, k0 + 2 * t + 9) << 28;
    dst[o] = static_cast<int32_t>(v);
}

struct Cursor {
    int kb, g, rem;  // next k block, its group, k blocks left in that group
};
struct Batch {
    int kb, n, g;  // first k block, k blocks (0: none), group of all of them
    bool flush;    // the batch ends its group or this warp's range
};

// ------------------------------------------------------------------ GEMV
template <int DT>
__global__ void __launch_bounds__(kThreads, kMinBlocks)
    gemv_mma_kernel(const int32_t* __restrict__ qw_mma, const int32_t* __restrict__ qzeros,
                    const uint16_t* __restrict__ scales, const uint16_t* __restrict__ x, uint16_t* __restrict__ y,
                    int M, int K, int N, int bpg, int kb_per_warp, int* __restrict__ err, const GatherArgs ga) {
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int g8 = lane >> 2, t = lane & 3;
    const int stripe = blockIdx.x;
    const int n0 = stripe * kStripe;
    const int KB = K >> 4;
    const int kb_per_cta = kb_per_warp * kWarps;
    const int c_b0 = blockIdx.y * kb_per_cta;
    const int c_b1 = min(KB, c_b0 + kb_per_cta);
    const int b0 = min(c_b1, c_b0 + warp * kb_per_warp);
    const int b1 = min(c_b1, b0 + kb_per_warp);
    const int grp_lo = c_b0 / bpg;
    const int ng = c_b1 > c_b0 ? (c_b1 - 1) / bpg - grp_lo + 1 : 0;
    const int ng_max = (kb_per_cta + bpg - 1) / bpg + 1;  // the same in every CTA (peers read by offset)
    const int xstride = kb_per_cta * 16 + 8;                 // halves per staged X row (+16 B: banks)

    // shared memory: the weight ring [kWarps][kSlots][kBatch][32 lanes] uint4, its
    // mbarriers [kWarps][kSlots], X rows [M][xstride] fp16/bf16 (fp16: k % 16 >= 8
    // pre-scaled by 1/16), scales [ng_max][64] and zero offsets [ng_max][64] fp32.
    // After the stream the ring holds the warp partials [kWarps][M][64] and the CTA
    // tile [M][64] fp32 (at the same offset in every CTA: cluster peers read it).
    extern __shared__ __align__(128) uint8_t smem[];
    uint4* ring = reinterpret_cast<uint4*>(smem) + static_cast<size_t>(warp) * kSlots * kBatch * 32;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kRingBytes) + warp * kSlots;
    uint16_t* xs = reinterpret_cast<uint16_t*>(smem + kRingBytes + kWarps * kSlots * 8);
    float* sf_s = reinterpret_cast<float*>(xs + static_cast<size_t>(M) * xstride);
    float* zf_s = sf_s + static_cast<size_t>(ng_max) * kStripe;
    float* red = reinterpret_cast<float*>(smem);  // the ring, once every warp has drained its copies

    const int32_t* wp = qw_mma + (static_cast<size_t>(stripe) * KB) * 128;
    auto next = [&](Cursor& c) {
        Batch b;
        b.kb = c.kb;
        b.g = c.g;
        b.n = max(0, min(kBatch, min(c.rem, b1 - c.kb)));
        c.kb += b.n;
        c.rem -= b.n;
        b.flush = c.rem == 0 || c.kb == b1;
        if (c.rem == 0) {
            ++c.g;
            c.rem = bpg;
        }
        return b;
    };
    // one bulk copy per batch: this warp's k blocks of the stripe are contiguous
    auto issue = [&](const Batch& bt, int slot) {  // lane 0
        ptx::mbar_arrive_expect_tx(&bars[slot], static_cast<uint32_t>(bt.n) * 512u);
        ptx::bulk_load(ring + slot * kBatch * 32, wp + static_cast<size_t>(bt.kb) * 128,
                       static_cast<uint32_t>(bt.n) * 512u, &bars[slot]);
    };

    if (lane == 0) {
        for (int sl = 0; sl < kSlots; ++sl) ptx::mbar_init(&bars[sl], 1);
        ptx::fence_mbar_init();
    }
    __syncwarp();
    Cursor ic;  // issue cursor, kSlots batches ahead of the consume cursor
    ic.kb = b0;
    ic.g = b0 / bpg;
    ic.rem = bpg - (b0 - ic.g * bpg);
    Cursor cc = ic;
    int issued = 0;
    // weights: requested before the previous kernel has finished
    for (int sl = 0; sl < kSlots; ++sl) {
        const Batch bt = next(ic);
        if (bt.n == 0) break;
        if (lane == 0) issue(bt, sl);
        ++issued;
    }
    // the CTA's scale and zero rows of the stripe (weights too)
    for (int i = threadIdx.x; i < ng * kStripe; i += kThreads) {
        const int gl = i / kStripe;
        const int c = n0 + (i - gl * kStripe);
        float sv = 0.f, zv = 0.f;
        if (c < N) {
            const size_t g = static_cast<size_t>(grp_lo + gl);
            sv = __half2float(__ushort_as_half(__ldg(scales + g * N + c)));
            const uint32_t zw = qzeros ? static_cast<uint32_t>(__ldg(qzeros + g * (N >> 3) + (c >> 3))) : kSymmetricZeroWord;
            zv = static_cast<float>(((zw >> ((c & 7) * 4)) & 15u) + 1u) + (DT == kFP16 ? 0.f : 128.f);
        }
        sf_s[i] = sv;
        zf_s[i] = zv;  // z, or 128 + z for bf16 (its bias rides on S)
    }
    if (threadIdx.x == 0) ptx::grid_dep_launch_dependents();
    ptx::grid_dep_wait();  // X (and Y) belong to the previous kernel in the stream
    // stage X[m, c_b0*16 : c_b1*16) (8-byte chunks)
    {
        const int kc = (c_b1 - c_b0) * 4;  // chunks of 4 halves per token row
        for (int i = threadIdx.x; i < M * kc; i += kThreads) {
            const int m = i / kc;
            const int c = i - m * kc;
            uint2 v = __ldg(reinterpret_cast<const uint2*>(x + static_cast<size_t>(m) * K + c_b0 * 16) + c);
            if (DT == kFP16 && (c & 3) >= 2) {  // k % 16 >= 8: meets the x16 nibbles
                v.x = mul2<kFP16>(v.x, 0x2C002C00u);
                v.y = mul2<kFP16>(v.y, 0x2C002C00u);
            }
            *reinterpret_cast<uint2*>(xs + static_cast<size_t>(m) * xstride + c * 4) = v;
        }
    }
    __syncthreads();

    float tot[4][4];  // fp32 totals: tile j, fragment element i
    float acc[4][4];  // the current group's MMA accumulators
    float acc_c[4] = {0.f, 0.f, 0.f, 0.f};  // fp16: sum of bias * X per token (elements 0, 1)
    float acc_s[4] = {0.f, 0.f, 0.f, 0.f};  // sum of X per token (elements 0, 1)
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int i = 0; i < 4; ++i) tot[j][i] = acc[j][i] = 0.f;
    // constant A fragments (every row the same): bias per k, and the factor that turns
    // a staged X value back into X
    const uint32_t a_bias[4] = {0x64006400u, 0x64006400u, 0x64006400u, 0x64006400u};  // 1024
    // fp16: 1 for k % 16 < 8, 16 for the pre-scaled k % 16 >= 8; bf16: 1
    const uint32_t a_one[4] = {DT == kFP16 ? 0x3C003C00u : 0x3F803F80u, DT == kFP16 ? 0x3C003C00u : 0x3F803F80u,
                               DT == kFP16 ? 0x4C004C00u : 0x3F803F80u, DT == kFP16 ? 0x4C004C00u : 0x3F803F80u};
    const bool tok_ok = g8 < M;  // this lane's B column (token g8) is real
    const uint16_t* xrow = xs + static_cast<size_t>(tok_ok ? g8 : 0) * xstride + 2 * t;

    auto consume = [&](const Batch& bt, const uint4* wslot, auto full_tag) {
        constexpr bool FULL = decltype(full_tag)::value;
        const int gl = bt.g - grp_lo;
#pragma unroll
        for (int jb = 0; jb < kBatch; ++jb) {
            if (FULL || jb < bt.n) {
                const int kl = (bt.kb + jb - c_b0) * 16;
                uint32_t bx0 = 0, bx1 = 0;
                if (tok_ok) {
                    bx0 = *reinterpret_cast<const uint32_t*>(xrow + kl);
                    bx1 = *reinterpret_cast<const uint32_t*>(xrow + kl + 8);
                }
                const uint4 wv = wslot[jb * 32];
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    uint32_t af[4];
                    biased_frag<DT>((&wv.x)[j], af);
                    mma16816<DT>(acc[j], af, bx0, bx1);
                }
                if constexpr (DT == kFP16) mma16816<DT>(acc_c, a_bias, bx0, bx1);
                mma16816<DT>(acc_s, a_one, bx0, bx1);
            }
        }
        // group finished (or this warp's range ends inside it): remove bias and zero,
        // scale into the totals
        if (bt.flush) {
            const float* srow = sf_s + gl * kStripe;
            const float* zrow = zf_s + gl * kStripe;
            const float c0 = DT == kFP16 ? acc_c[0] : 0.f, c1 = DT == kFP16 ? acc_c[1] : 0.f;
            const float s0 = acc_s[0], s1 = acc_s[1];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int ca = j * 16 + g8;
                const float sa = srow[ca], sb = srow[ca + 8];
                const float za = zrow[ca], zb = zrow[ca + 8];
                tot[j][0] = fmaf(sa, fmaf(-za, s0, acc[j][0] - c0), tot[j][0]);
                tot[j][1] = fmaf(sa, fmaf(-za, s1, acc[j][1] - c1), tot[j][1]);
                tot[j][2] = fmaf(sb, fmaf(-zb, s0, acc[j][2] - c0), tot[j][2]);
                tot[j][3] = fmaf(sb, fmaf(-zb, s1, acc[j][3] - c1), tot[j][3]);
#pragma unroll
                for (int i = 0; i < 4; ++i) acc[j][i] = 0.f;
            }
#pragma unroll
            for (int i = 0; i < 4; ++i) acc_c[i] = acc_s[i] = 0.f;
        }
    };

    // batch i sits in slot i % kSlots (its (i / kSlots)-th use of the slot)
    int done = 0;
    for (int slot = 0;; slot = slot + 1 == kSlots ? 0 : slot + 1) {
        const Batch bt = next(cc);
        if (bt.n == 0) break;
        if (!ptx::mbar_wait_bounded(&bars[slot], (done / kSlots) & 1, kWaitLimit, err, kErrGemvMmaTimeout)) break;
        const uint4* wslot = ring + slot * kBatch * 32 + lane;
        if (bt.n == kBatch)
            consume(bt, wslot, std::true_type{});
        else
            consume(bt, wslot, std::false_type{});
        ++done;
        __syncwarp();  // every lane has read the slot before it is refilled
        const Batch nb = next(ic);
        if (nb.n > 0) {
            if (lane == 0) {
                ptx::fence_proxy_async_smem();  // generic reads before the async-proxy overwrite
                issue(nb, slot);
            }
            ++issued;
        }
    }
    // after a timeout: let the copies still in flight land before the CTA exits
    for (int i = done; i < issued; ++i)
        ptx::mbar_wait_bounded(&bars[i % kSlots], (i / kSlots) & 1, kWaitLimit, err, kErrGemvMmaTimeout);

    // ---- fixed-order reduction: warps (shared memory), then the cluster's CTAs
    __syncthreads();  // every warp is out of its ring before the ring holds the partials
    float* mine = red + static_cast<size_t>(warp) * M * kStripe;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const int ca = j * 16 + g8;
        if (2 * t < M) {
            mine[(2 * t) * kStripe + ca] = tot[j][0];
            mine[(2 * t) * kStripe + ca + 8] = tot[j][2];
        }
        if (2 * t + 1 < M) {
            mine[(2 * t + 1) * kStripe + ca] = tot[j][1];
            mine[(2 * t + 1) * kStripe + ca + 8] = tot[j][3];
        }
    }
    __syncthreads();
    float* tile = red + static_cast<size_t>(kWarps) * M * kStripe;
    const int splits = gridDim.y;
    for (int i = threadIdx.x; i < M * kStripe; i += kThreads) {
        float sum = 0.f;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) sum += red[static_cast<size_t>(w) * M * kStripe + i];
        if (splits == 1) {
            const int m = i / kStripe;
            const int n = n0 + (i - m * kStripe);
            if (n < N)
                out_store(ga, y, N, m, n,
                                                                          DT == kFP16 ? __half_as_ushort(__float2half_rn(sum)) : __bfloat16_as_ushort(__float2bfloat16_rn(sum)));
        } else {
            tile[i] = sum;
        }
    }
    if (splits == 1) return;
    cg::cluster_group cluster = cg::this_cluster();
    cluster.sync();
    const int rank = static_cast<int>(cluster.block_rank());
    const int total = M * kStripe;
    const int per = (total + splits - 1) / splits;
    const int i0 = rank * per;
    const int i1 = min(total, i0 + per);
    for (int i = i0 + static_cast<int>(threadIdx.x); i < i1; i += kThreads) {
        float sum = 0.f;
#pragma unroll
        for (int r = 0; r < kMaxSplits; ++r)  // independent remote loads, summed in rank order
            if (r < splits) sum += cluster.map_shared_rank(tile, r)[i];
        const int m = i / kStripe;
        const int n = n0 + (i - m * kStripe);
        if (n < N)
            out_store(ga, y, N, m, n,
                                                                      DT == kFP16 ? __half_as_ushort(__float2half_rn(sum)) : __bfloat16_as_ushort(__float2bfloat16_rn(sum)));
    }
    cluster.sync();  // keep this CTA's shared memory alive until every peer has read it
}

size_t smem_bytes(int kb_per_cta, int bpg, int M) {
    const size_t ng_max = static_cast<size_t>((kb_per_cta + bpg - 1) / bpg + 1);
    const size_t xs = (static_cast<size_t>(M) * (kb_per_cta * 16 + 8) * 2 + 15) / 16 * 16;
    return kRingBytes + kWarps * kSlots * 8 + xs + ng_max * kStripe * 8;  // partials reuse the ring
}

int stripes_of(int N) { return (N + kStripe - 1) / kStripe; }

template <int DT>
cudaError_t launch_t(const PackedWeight& w, const int32_t* qw_mma, const GemvPlan& p, const void* x, int M, void* y,
                     cudaStream_t s, const GatherArgs& ga) {
    const int bpg = w.group_size >> 4;
    auto kern = gemv_mma_kernel<DT>;
    static const cudaError_t attr_err = [&] {
        cudaError_t e =
            cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(kSmemBudget));
        if (e == cudaSuccess) e = cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
        return e;
    }();
    if (attr_err != cudaSuccess) return attr_err;
    const size_t smem = smem_bytes(p.kpw * kWarps, bpg, M);
    if (smem > kSmemBudget || p.splits > kMaxSplits || p.kpw <= 0) return cudaErrorInvalidValue;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(stripes_of(w.N), p.splits, 1);
    cfg.blockDim = dim3(kThreads, 1, 1);
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
    return cudaLaunchKernelEx(&cfg, kern, qw_mma, w.kernel_qzeros(), w.scales, static_cast<const uint16_t*>(x),
                              static_cast<uint16_t*>(y), M, w.K, w.N, bpg, p.kpw, w.err, ga);
}

}  // namespace

bool gemv_mma_supported(const PackedWeight& w) {
    // k blocks of 16 never straddle groups; the widest split's staged slice fits
    if (w.group_size % 16 != 0 || w.K % 16 != 0) return false;
    const int KB = w.K >> 4;
    const int kpw = (KB + kMaxSplits * kWarps - 1) / (kMaxSplits * kWarps);
    return smem_bytes(kpw * kWarps, w.group_size >> 4, 1) <= kSmemBudget;
}

size_t repack_mma_words(const PackedWeight& w) {
    return static_cast<size_t>(stripes_of(w.N)) * (w.K >> 4) * 128;
}

cudaError_t launch_repack_mma(const PackedWeight& w, int32_t* dst, cudaStream_t s) {
    const long long total = static_cast<long long>(repack_mma_words(w));
    if (total == 0) return cudaSuccess;
    const unsigned blocks = static_cast<unsigned>((total + 255) / 256);
    repack_mma_kernel<<<blocks, 256, 0, s>>>(w.qweight, dst, w.K, w.N, stripes_of(w.N));
    return cudaGetLastError();
}

GemvPlan plan_gemv_mma(const PackedWeight& w, int M, int num_sms) {
    GemvPlan p;
    p.bn = kStripe;
    const int tiles = stripes_of(w.N);
    const int KB = w.K >> 4;
    const int bpg = w.group_size >> 4;
    const int slots = kMinBlocks * num_sms;
    auto kpw_of = [&](int cs) { return (KB + cs * kWarps - 1) / (cs * kWarps); };
    // rows of X per pass: as many as fit at the widest split
    int m = M < 1 ? 1 : (M > kMaxTok ? kMaxTok : M);
    while (m > 1 && smem_bytes(kpw_of(kMaxSplits) * kWarps, bpg, m) > kSmemBudget) --m;
    p.mt = m;
    auto fits = [&](int cs) { return smem_bytes(kpw_of(cs) * kWarps, bpg, m) <= kSmemBudget; };
    // one wave of long per-warp streams: cost = waves x (k blocks per warp + ramp); a
    // single wave over 90 % of the slots leaves the next kernel no room to start early
    // (as in plan_gemv)
    constexpr int kRampBlocks = 12;
    int best = 0;
    long long best_cost = 0;
    for (int cs = 1; cs <= kMaxSplits; ++cs) {
        if (!fits(cs)) continue;
        const int kpw = kpw_of(cs);
        if ((KB + kpw * kWarps - 1) / (kpw * kWarps) != cs) continue;
        const long long ctas = static_cast<long long>(tiles) * cs;
        const long long waves = (ctas + slots - 1) / slots;
        if (waves == 1 && ctas * 10 > static_cast<long long>(slots) * 9) continue;
        const long long cost = waves * (kpw + kRampBlocks);
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
    p.splits = (KB + p.kpw * kWarps - 1) / (p.kpw * kWarps);
    return p;
}

cudaError_t launch_gemv_mma(const PackedWeight& w, const int32_t* qw_mma, const GemvPlan& p, const void* x, int M,
                            void* y, DType dt, cudaStream_t s, const GatherArgs* gather) {
    if (M <= 0) return cudaSuccess;
    if (M > kMaxTok || !gemv_mma_supported(w) || !qw_mma) return cudaErrorInvalidValue;
    GatherArgs ga = {};
    if (gather) ga = *gather;
    return dt == kFP16 ? launch_t<kFP16>(w, qw_mma, p, x, M, y, s, ga) : launch_t<kBF16>(w, qw_mma, p, x, M, y, s, ga);
}

}  // namespace w4a16
