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
// Kernel: a CTA owns one 64-column stripe; its 4 warps split the CTA's K range and
// stream it through per-warp rings of 4 KB bulk copies (8 k blocks, never crossing a
// quantization group). The A fragments are the magic-biased nibbles straight out of
// lop3 (fp16: 1024 + q, and 1024 + 16 q for k % 16 >= 8 with those X values pre-scaled
// by 1/16; bf16: 128 + q). The tensor core multiplies them exactly and accumulates in
// fp32, so the bias and the zero point come off afterwards: each lane also sums, in
// fp32 on the CUDA cores, the X values of its own B fragment, which after a reduction
// over the lane quad gives per token C = 1024 * sum(staged X) and S = sum(X), and at
// each group end
//     Y += s * (D - C - z * S)            (bf16: D - (128 + z) * S)
// in fp32. Per packed word that is one shift and four lop3 (bf16: three shifts) plus
// 1/32 of the tile MMA. The prologue issues every global read as one round trip: the
// first ring slots and the CTA's scale / zero rows before the grid-dependency wait, X as
// one bulk copy per token row after it. Warps reduce through shared memory in a fixed
// order, a K split across CTAs through distributed shared memory of a cluster in rank
// order: deterministic, no workspace, no atomics.
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
constexpr int kMaxTok = kGemvMmaMaxTok;  // two MMA N tiles of 8
constexpr int kBatch = 8;     // k blocks (16 k) per ring slot: 4 KB
constexpr int kSlots = 2;     // ring slots per warp: up to 8 KB in flight per warp
constexpr int kMaxSplits = 16;  // CTAs along K: one cluster (non-portable above 8)
constexpr int kMinBlocks = 3;
constexpr size_t kSmemBudget = 75 * 1024;  // three CTAs per SM
constexpr size_t kRingBytes = static_cast<size_t>(kWarps) * kSlots * kBatch * 512;
constexpr size_t kBarBytes = (static_cast<size_t>(kWarps) * kSlots + 1) * 8 + 8;  // ring and X mbarriers, 16-B rounded
static_assert(kBarBytes % 16 == 0, "X rows are bulk-copy destinations");
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

template <int DT>
__device__ __forceinline__ float2 to_float2(uint32_t v) {  // two packed fp16 / bf16 values
    if constexpr (DT == kFP16)
        return __half22float2(*reinterpret_cast<const __half2*>(&v));
    else
        return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&v));
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
// Shared-memory carve-up, the same in every CTA of a launch (cluster peers read the
// tile by offset): weight ring, mbarriers, X rows, scale rows (fp16), zero words.
struct MmaSmem {
    int xstride;   // halves per staged X row: 32 B per k block, padded to 32 mod 128 B (banks)
    int ng_max;    // scale / zero rows (groups a CTA's K range can touch)
    size_t x_off, sc_off, zw_off, total;
};
__host__ __device__ inline MmaSmem mma_smem(int kb_per_cta, int bpg, int M, int wc) {
    MmaSmem m;
    m.xstride = (32 * kb_per_cta + ((32 - 32 * kb_per_cta) % 128 + 128) % 128) / 2;
    m.ng_max = (kb_per_cta + bpg - 1) / bpg + 1;
    m.x_off = kRingBytes + kBarBytes;
    m.sc_off = m.x_off + (static_cast<size_t>(M) * m.xstride * 2 + 15) / 16 * 16;
    m.zw_off = m.sc_off + (static_cast<size_t>(m.ng_max) * wc * kStripe * 2 + 15) / 16 * 16;
    m.total = m.zw_off + static_cast<size_t>(m.ng_max) * wc * (kStripe / 8) * 4;
    return m;
}

// NT: token tiles of 8 (M <= 8 * NT). The CTA's 4 warps form a grid of wc column
// stripes x (4 / wc) K slices; every warp streams its own stripe over its own slice.
template <int DT, int NT>
__global__ void __launch_bounds__(kThreads, kMinBlocks)
    gemv_mma_kernel(const int32_t* __restrict__ qw_mma, const int32_t* __restrict__ qzeros,
                    const uint16_t* __restrict__ scales, const uint16_t* __restrict__ x, uint16_t* __restrict__ y,
                    int M, int K, int N, int bpg, int kb_per_warp, int wc, int* __restrict__ err,
                    const GatherArgs ga) {
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int g8 = lane >> 2, t = lane & 3;
    const int wk = kWarps / wc;          // K slices per CTA
    const int wcol = warp % wc, wrow = warp / wc;
    const int cta_cols = wc * kStripe;
    const int stripes = (N + kStripe - 1) / kStripe;
    const int stripe = blockIdx.x * wc + wcol;
    const int n0c = blockIdx.x * cta_cols;  // the CTA's first column
    const int KB = K >> 4;
    const int kb_per_cta = kb_per_warp * wk;
    const int c_b0 = blockIdx.y * kb_per_cta;
    const int c_b1 = min(KB, c_b0 + kb_per_cta);
    const int b0 = min(c_b1, c_b0 + wrow * kb_per_warp);
    const int b1 = stripe < stripes ? min(c_b1, b0 + kb_per_warp) : b0;  // a stripe past N: no work
    const int grp_lo = c_b0 / bpg;
    const int ng = c_b1 > c_b0 ? (c_b1 - 1) / bpg - grp_lo + 1 : 0;
    const MmaSmem lay = mma_smem(kb_per_cta, bpg, M, wc);
    const int xstride = lay.xstride;

    // shared memory: the weight ring [kWarps][kSlots][kBatch][32 lanes] uint4, its
    // mbarriers [kWarps][kSlots] and X's, X rows [M][xstride] fp16/bf16 (fp16: k % 16 >= 8
    // pre-scaled by 1/16), scale rows [ng_max][cta_cols] fp16 and zero words
    // [ng_max][cta_cols / 8]. After the stream the ring holds the warp partials
    // [wk][M][cta_cols] and the CTA tile [M][cta_cols] fp32.
    extern __shared__ __align__(128) uint8_t smem[];
    uint4* ring = reinterpret_cast<uint4*>(smem) + static_cast<size_t>(warp) * kSlots * kBatch * 32;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kRingBytes) + warp * kSlots;
    uint64_t* xbar = reinterpret_cast<uint64_t*>(smem + kRingBytes) + kWarps * kSlots;
    uint16_t* xs = reinterpret_cast<uint16_t*>(smem + lay.x_off);
    uint16_t* sc_s = reinterpret_cast<uint16_t*>(smem + lay.sc_off);
    uint32_t* zw_s = reinterpret_cast<uint32_t*>(smem + lay.zw_off);
    float* red = reinterpret_cast<float*>(smem);  // the ring, once every warp has drained its copies

    const int32_t* wp = qw_mma + (static_cast<size_t>(min(stripe, stripes - 1)) * KB) * 128;
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
        if (warp == 0) ptx::mbar_init(xbar, 1);
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
    // the CTA's scale and zero rows (weights too): per group and 8-column chunk one
    // 16-byte scale load and one zero word, all of a thread's loads issued before any
    // is used (one memory round trip, not one per item)
    {
        const int chunks = cta_cols / 8;
        const int items = ng * chunks;
        for (int base = 0; base < items; base += 4 * kThreads) {
            uint4 sv[4];
            uint32_t zw[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int i = base + u * kThreads + static_cast<int>(threadIdx.x);
                const int gl = i / chunks;
                const int c = n0c + (i - gl * chunks) * 8;
                sv[u] = make_uint4(0, 0, 0, 0);
                zw[u] = kSymmetricZeroWord;
                if (i < items && c < N) {
                    const size_t g = static_cast<size_t>(grp_lo + gl);
                    sv[u] = __ldg(reinterpret_cast<const uint4*>(scales + g * N + c));
                    if (qzeros) zw[u] = static_cast<uint32_t>(__ldg(qzeros + g * (N >> 3) + (c >> 3)));
                }
            }
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int i = base + u * kThreads + static_cast<int>(threadIdx.x);
                if (i < items) {
                    reinterpret_cast<uint4*>(sc_s)[i] = sv[u];
                    zw_s[i] = zw[u];
                }
            }
        }
    }
    if (threadIdx.x == 0) ptx::grid_dep_launch_dependents();
    __syncthreads();  // X's mbarrier is initialised
    ptx::grid_dep_wait();  // X (and Y) belong to the previous kernel in the stream
    // stage X[m, c_b0*16 : c_b1*16): one bulk copy per token row
    const int nkb = c_b1 - c_b0;
    if (threadIdx.x == 0 && nkb > 0) {
        ptx::mbar_arrive_expect_tx(xbar, static_cast<uint32_t>(M) * nkb * 32u);
        for (int m = 0; m < M; ++m)
            ptx::bulk_load(xs + static_cast<size_t>(m) * xstride, x + static_cast<size_t>(m) * K + c_b0 * 16,
                           static_cast<uint32_t>(nkb) * 32u, xbar);
    }
    const bool x_ok = nkb == 0 || ptx::mbar_wait_bounded(xbar, 0, kWaitLimit, err, kErrGemvMmaTimeout);
    // each k block of a staged row into B-fragment order: lane t's four values (k 2t,
    // 2t+1, 2t+8, 2t+9) side by side, one 8-byte load per k block; fp16: the values at
    // k % 16 >= 8 meet the x16 nibbles, so they are scaled by 1/16
    for (int i = threadIdx.x; i < M * nkb; i += kThreads) {
        const int m = i / nkb;
        uint4* p = reinterpret_cast<uint4*>(xs + static_cast<size_t>(m) * xstride + (i - m * nkb) * 16);
        const uint4 lo = p[0];
        uint4 hi = p[1];
        if constexpr (DT == kFP16) {
            hi.x = mul2<kFP16>(hi.x, 0x2C002C00u);
            hi.y = mul2<kFP16>(hi.y, 0x2C002C00u);
            hi.z = mul2<kFP16>(hi.z, 0x2C002C00u);
            hi.w = mul2<kFP16>(hi.w, 0x2C002C00u);
        }
        p[0] = make_uint4(lo.x, hi.x, lo.y, hi.y);
        p[1] = make_uint4(lo.z, hi.z, lo.w, hi.w);
    }
    __syncthreads();

    float tot[4][NT][4];  // fp32 totals: tile j, token tile, fragment element i
    float acc[4][NT][4];  // the current group's MMA accumulators
    // one more MMA per k block and token tile with constant A: rows 0-7 the bias
    // (fp16: 1024 for every k, giving C = 1024 * sum of staged X), rows 8-15 the factor
    // back to X (1 for k % 16 < 8, 16 for the pre-scaled k % 16 >= 8; bf16: 1), giving
    // S = sum of X. D elements 0/1 are then C and 2/3 S of this lane's tokens 2t, 2t+1.
    float bs[NT][4];
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int u = 0; u < NT; ++u)
#pragma unroll
            for (int i = 0; i < 4; ++i) tot[j][u][i] = acc[j][u][i] = 0.f;
#pragma unroll
    for (int u = 0; u < NT; ++u)
#pragma unroll
        for (int i = 0; i < 4; ++i) bs[u][i] = 0.f;
    const uint32_t a_bs[4] = {DT == kFP16 ? 0x64006400u : 0u, DT == kFP16 ? 0x3C003C00u : 0x3F803F80u,
                              DT == kFP16 ? 0x64006400u : 0u, DT == kFP16 ? 0x4C004C00u : 0x3F803F80u};
    // shared addresses: this lane's word of k block 0 in slot 0, and its B fragment of
    // k block c_b0 for token 8u + g8 (a token past M reads token 0: its column of D is
    // never stored)
    const uint32_t ring_s = ptx::smem_u32(ring) + lane * 16;
    uint32_t xrow_s[NT];
#pragma unroll
    for (int u = 0; u < NT; ++u)
        xrow_s[u] = ptx::smem_u32(xs) + static_cast<uint32_t>((8 * u + g8 < M ? 8 * u + g8 : 0) * xstride * 2 + t * 8);
    // this lane's zero nibble: columns j*16 + g8 (+8) share the shift g8 * 4
    const int zsh = g8 * 4;
    const int ccol = wcol * kStripe + g8;  // the lane's first column within the CTA

    auto consume = [&](const Batch& bt, int slot, auto full_tag) {
        constexpr bool FULL = decltype(full_tag)::value;
        const int gl = bt.g - grp_lo;
        const uint32_t wb = ring_s + static_cast<uint32_t>(slot * kBatch * 512);
        const uint32_t xo = static_cast<uint32_t>((bt.kb - c_b0) * 32);
        uint4 wv[2];
        uint2 xv[2][NT];
        auto load = [&](int jb, int buf) {  // k block jb of the batch: the next one is loaded while this one computes
            wv[buf] = ptx::ld_shared_v4(wb + jb * 512);
#pragma unroll
            for (int u = 0; u < NT; ++u) xv[buf][u] = ptx::ld_shared_v2(xrow_s[u] + xo + jb * 32);
        };
        load(0, 0);
#pragma unroll
        for (int jb = 0; jb < kBatch; ++jb) {
            if (FULL || jb < bt.n) {
                const int c = jb & 1;
                if (jb + 1 < kBatch && (FULL || jb + 1 < bt.n)) load(jb + 1, c ^ 1);
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    uint32_t af[4];
                    biased_frag<DT>((&wv[c].x)[j], af);
#pragma unroll
                    for (int u = 0; u < NT; ++u) mma16816<DT>(acc[j][u], af, xv[c][u].x, xv[c][u].y);
                }
#pragma unroll
                for (int u = 0; u < NT; ++u) mma16816<DT>(bs[u], a_bs, xv[c][u].x, xv[c][u].y);
            }
        }
        // group finished (or this warp's range ends inside it): remove bias and zero,
        // scale into the totals. The MMA gave, per column and token,
        //   D = sum (bias + q) * xs,   bias 1024 (fp16, xs = X or X/16) or 128 (bf16)
        // so q.X = D - C; bf16 folds its bias into the zero offset (128 + z):
        //   Y += s * (D - C - z * S)
        if (bt.flush) {
            float sa[4], sb[4], za[4], zb[4];
            const uint16_t* srow = sc_s + static_cast<size_t>(gl) * cta_cols + ccol;
            const uint32_t* zrow = zw_s + static_cast<size_t>(gl) * (cta_cols / 8) + (ccol >> 3);
            constexpr float kZBias = DT == kFP16 ? 1.f : 129.f;  // z = nibble + 1 (bf16: + 128)
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                sa[j] = __half2float(__ushort_as_half(srow[j * 16]));
                sb[j] = __half2float(__ushort_as_half(srow[j * 16 + 8]));
                za[j] = static_cast<float>((zrow[2 * j] >> zsh) & 15u) + kZBias;
                zb[j] = static_cast<float>((zrow[2 * j + 1] >> zsh) & 15u) + kZBias;
            }
#pragma unroll
            for (int u = 0; u < NT; ++u) {
                const float c0 = DT == kFP16 ? bs[u][0] : 0.f, c1 = DT == kFP16 ? bs[u][1] : 0.f;
                const float s0 = bs[u][2], s1 = bs[u][3];
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    tot[j][u][0] = fmaf(sa[j], fmaf(-za[j], s0, acc[j][u][0] - c0), tot[j][u][0]);
                    tot[j][u][1] = fmaf(sa[j], fmaf(-za[j], s1, acc[j][u][1] - c1), tot[j][u][1]);
                    tot[j][u][2] = fmaf(sb[j], fmaf(-zb[j], s0, acc[j][u][2] - c0), tot[j][u][2]);
                    tot[j][u][3] = fmaf(sb[j], fmaf(-zb[j], s1, acc[j][u][3] - c1), tot[j][u][3]);
#pragma unroll
                    for (int i = 0; i < 4; ++i) acc[j][u][i] = 0.f;
                }
#pragma unroll
                for (int i = 0; i < 4; ++i) bs[u][i] = 0.f;
            }
        }
    };

    // batch i sits in slot i % kSlots (its (i / kSlots)-th use of the slot)
    int done = 0;
    for (int slot = 0;; slot = slot + 1 == kSlots ? 0 : slot + 1) {
        const Batch bt = next(cc);
        if (bt.n == 0) break;
        if (!ptx::mbar_wait_bounded(&bars[slot], (done / kSlots) & 1, kWaitLimit, err, kErrGemvMmaTimeout)) break;
        if (bt.n == kBatch)
            consume(bt, slot, std::true_type{});
        else
            consume(bt, slot, std::false_type{});
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
    __syncwarp();
    if (lane == 0) {  // the partials below may cover the mbarriers
        for (int sl = 0; sl < kSlots; ++sl) ptx::mbar_inval(&bars[sl]);
        if (warp == 0) {
            if (!x_ok) ptx::mbar_wait_bounded(xbar, 0, kWaitLimit, err, kErrGemvMmaTimeout);  // X copy after a timeout
            ptx::mbar_inval(xbar);
        }
    }

    // ---- fixed-order reduction: the K slices of a stripe (shared memory), then the
    // cluster's CTAs
    __syncthreads();  // every warp is out of its ring before the ring holds the partials
    if (gridDim.y > 1) ptx::cluster_arrive_relaxed();  // this CTA's ring is free for its peers' stores
    const int tile_elems = M * cta_cols;
    float* mine = red + static_cast<size_t>(wrow) * tile_elems;
#pragma unroll
    for (int u = 0; u < NT; ++u) {
        const int m0 = 8 * u + 2 * t;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int ca = wcol * kStripe + j * 16 + g8;
            if (m0 < M) {
                mine[m0 * cta_cols + ca] = tot[j][u][0];
                mine[m0 * cta_cols + ca + 8] = tot[j][u][2];
            }
            if (m0 + 1 < M) {
                mine[(m0 + 1) * cta_cols + ca] = tot[j][u][1];
                mine[(m0 + 1) * cta_cols + ca + 8] = tot[j][u][3];
            }
        }
    }
    __syncthreads();
    // 8 consecutive columns per step: the K slices summed in order, then stored as
    // 16 bytes (one CTA along K) or kept as this CTA's tile for the cluster
    // this CTA's sums (with a K split), then the receive rows its peers store into
    float* tile = red + static_cast<size_t>(wk) * tile_elems;
    float* recv = tile + tile_elems;
    const int splits = gridDim.y;
    const int row_chunks = cta_cols / 8;
    const int chunks = M * row_chunks;
    const bool wide_store = ga.world == 0 || (ga.ld % 8 == 0 && ga.col0 % 8 == 0);
    auto store8 = [&](int ci, const float (&v)[8]) {
        const int m = ci / row_chunks;
        const int n = n0c + (ci - m * row_chunks) * 8;
        if (n >= N) return;
        uint16_t h[8];
#pragma unroll
        for (int e = 0; e < 8; ++e)
            h[e] = DT == kFP16 ? __half_as_ushort(__float2half_rn(v[e])) : __bfloat16_as_ushort(__float2bfloat16_rn(v[e]));
        if (wide_store) {
            out_store16(ga, y, N, m, n,
                        make_uint4(h[0] | (static_cast<uint32_t>(h[1]) << 16), h[2] | (static_cast<uint32_t>(h[3]) << 16),
                                   h[4] | (static_cast<uint32_t>(h[5]) << 16), h[6] | (static_cast<uint32_t>(h[7]) << 16)));
        } else {
#pragma unroll
            for (int e = 0; e < 8; ++e) out_store(ga, y, N, m, n + e, h[e]);
        }
    };
    for (int ci = threadIdx.x; ci < chunks; ci += kThreads) {
        float v[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        for (int w = 0; w < wk; ++w) {
            const float4* src = reinterpret_cast<const float4*>(red + static_cast<size_t>(w) * tile_elems) + 2 * ci;
            const float4 a = src[0], b = src[1];
            v[0] += a.x; v[1] += a.y; v[2] += a.z; v[3] += a.w;
            v[4] += b.x; v[5] += b.y; v[6] += b.z; v[7] += b.w;
        }
        if (splits == 1) {
            store8(ci, v);
        } else {
            float4* dst = reinterpret_cast<float4*>(tile) + 2 * ci;
            dst[0] = make_float4(v[0], v[1], v[2], v[3]);
            dst[1] = make_float4(v[4], v[5], v[6], v[7]);
        }
    }
    if (splits == 1) return;
    // The cluster: this CTA's sums of every chunk go to the chunk's owner rank (remote
    // shared-memory stores into its receive rows [splits][per]), one cluster barrier,
    // then each owner adds its rows in rank order and stores.
    cg::cluster_group cluster = cg::this_cluster();
    const int rank = static_cast<int>(cluster.block_rank());
    const int per = (chunks + splits - 1) / splits;
    ptx::cluster_wait();  // every CTA of the cluster is out of its ring: receive rows are free
    for (int ci = threadIdx.x; ci < chunks; ci += kThreads) {
        const float4* src = reinterpret_cast<const float4*>(tile) + 2 * ci;
        const int o = ci / per;
        float4* dst = reinterpret_cast<float4*>(cluster.map_shared_rank(recv, o)) + 2 * (rank * per + ci - o * per);
        dst[0] = src[0];
        dst[1] = src[1];
    }
    cluster.sync();  // every CTA's stores have landed
    const int my = min(per, chunks - rank * per);
    for (int i = threadIdx.x; i < my; i += kThreads) {
        float v[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        for (int r = 0; r < splits; ++r) {  // summed in rank order
            const float4* src = reinterpret_cast<const float4*>(recv) + 2 * (r * per + i);
            const float4 a = src[0], b = src[1];
            v[0] += a.x; v[1] += a.y; v[2] += a.z; v[3] += a.w;
            v[4] += b.x; v[5] += b.y; v[6] += b.z; v[7] += b.w;
        }
        store8(rank * per + i, v);
    }
}

size_t smem_bytes(int kb_per_cta, int bpg, int M, int wc) {
    const MmaSmem m = mma_smem(kb_per_cta, bpg, M, wc);
    // the partials and the CTA tile reuse the ring
    // partials [wk][tile], the CTA's sums [tile] and the receive rows [splits][per] of
    // 8-column chunks (at most kMaxSplits - 1 chunks past a tile)
    const size_t red = (static_cast<size_t>(kWarps / wc + 2) * M * wc * kStripe + (kMaxSplits - 1) * 8) * 4;
    return red > m.total ? red : m.total;
}

int stripes_of(int N) { return (N + kStripe - 1) / kStripe; }

template <int DT, int NT>
cudaError_t launch_t(const PackedWeight& w, const int32_t* qw_mma, const GemvPlan& p, const void* x, int M, void* y,
                     cudaStream_t s, const GatherArgs& ga) {
    const int bpg = w.group_size >> 4;
    auto kern = gemv_mma_kernel<DT, NT>;
    static const cudaError_t attr_err = [&] {
        cudaError_t e =
            cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(kSmemBudget));
        if (e == cudaSuccess) e = cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
        return e;
    }();
    if (attr_err != cudaSuccess) return attr_err;
    const int wc = p.bn / kStripe;
    if (wc != 1 && wc != 2 && wc != 4) return cudaErrorInvalidValue;
    const size_t smem = smem_bytes(p.kpw * (kWarps / wc), bpg, M, wc);
    if (smem > kSmemBudget || p.splits > kMaxSplits || p.kpw <= 0) return cudaErrorInvalidValue;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((stripes_of(w.N) + wc - 1) / wc, p.splits, 1);
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
                              static_cast<uint16_t*>(y), M, w.K, w.N, bpg, p.kpw, wc, w.err, ga);
}

}  // namespace

bool gemv_mma_supported(const PackedWeight& w) {
    // k blocks of 16 never straddle groups; the widest split's staged slice fits
    if (w.group_size % 16 != 0 || w.K % 16 != 0) return false;
    const int KB = w.K >> 4;
    const int kpw = (KB + kMaxSplits * kWarps - 1) / (kMaxSplits * kWarps);
    return smem_bytes(kpw * kWarps, w.group_size >> 4, 1, 1) <= kSmemBudget;
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
    const int stripes = stripes_of(w.N);
    const int KB = w.K >> 4;
    const int bpg = w.group_size >> 4;
    // rows of X per pass: as many as fit at the widest split
    int m = M < 1 ? 1 : (M > kMaxTok ? kMaxTok : M);
    while (m > 1 && smem_bytes((KB + kMaxSplits * kWarps - 1) / (kMaxSplits * kWarps) * kWarps, bpg, m, 1) >
                        kSmemBudget)
        --m;
    p.mt = m;
    // two token tiles cost the same for any 9..16 rows: plan them as 16 when that fits
    const int mp = m > 8 && smem_bytes((KB + kMaxSplits * kWarps - 1) / (kMaxSplits * kWarps) * kWarps, bpg, 16, 1) <=
                                kSmemBudget ? 16 : m;
    // CTAs resident per SM: shared memory (228 KB per SM, 1 KB reserved per CTA) and
    // registers (96 per thread with one token tile, 148 with two: 5 and 3 CTAs of 128)
    const int reg_ctas = m <= 8 ? 5 : 3;
    auto resident = [&](size_t smem) {
        const int by_smem = static_cast<int>((228u * 1024u) / (smem + 1024u));
        return by_smem < reg_ctas ? by_smem : reg_ctas;
    };
    // Measured on B200 over the Llama-2 7B/13B/70B projections at M = 8 and 16: the
    // fastest launches fill 55-100 % of the resident CTA slots in one wave with as few
    // CTAs along K (cluster size) as that allows. So: among the configurations in that
    // window take the fewest splits (then the narrowest CTA); when none falls in it
    // (large weights), the least (waves of CTAs x k blocks per warp), waves counted
    // fractionally (under PDL the next kernel fills a partial last wave).
    constexpr int kRampBlocks = 12;
    int best_wc = 0, best_kpw = 0;
    bool best_in_window = false;
    double best_cost = 0;
    for (int wc = 1; wc <= 4; wc <<= 1) {
        const int wk = kWarps / wc;
        const long long col_ctas = (stripes + wc - 1) / wc;
        for (int cs = 1; cs <= kMaxSplits; ++cs) {
            const int kpw = (KB + cs * wk - 1) / (cs * wk);
            if ((KB + kpw * wk - 1) / (kpw * wk) != cs) continue;
            const size_t smem = smem_bytes(kpw * wk, bpg, mp, wc);
            if (smem > kSmemBudget) continue;
            const long long slots = static_cast<long long>(resident(smem)) * num_sms;
            const long long ctas = col_ctas * cs;
            const bool in_window = ctas * 100 >= slots * 55 && ctas <= slots;
            const double rounds = ctas > slots ? static_cast<double>(ctas) / slots : 1.0;
            const double cost = in_window ? static_cast<double>(cs) : rounds * (kpw + kRampBlocks) + 4.0 * cs;
            const bool better = best_wc == 0 || (in_window && !best_in_window) ||
                                (in_window == best_in_window && cost < best_cost);
            if (better) {
                best_wc = wc;
                best_kpw = kpw;
                best_cost = cost;
                best_in_window = in_window;
            }
        }
    }
    // tuning overrides: stripes per CTA (1, 2, 4) and CTAs along K
    static const int env_wc = [] {
        const char* v = std::getenv("W4A16_GEMV_MMA_WC");
        return v ? std::atoi(v) : 0;
    }();
    static const int env_cs = [] {
        const char* v = std::getenv("W4A16_GEMV_SPLITS");
        return v ? std::atoi(v) : 0;
    }();
    if (env_cs >= 1 && env_cs <= kMaxSplits) {
        const int wc = env_wc == 2 || env_wc == 4 ? env_wc : 1;
        const int wk = kWarps / wc;
        const int kpw = (KB + env_cs * wk - 1) / (env_cs * wk);
        if (smem_bytes(kpw * wk, bpg, m, wc) <= kSmemBudget) {
            best_wc = wc;
            best_kpw = kpw;
        }
    }
    if (best_wc == 0) {  // the widest split of one-stripe CTAs (fits: gemv_mma_supported)
        best_wc = 1;
        best_kpw = (KB + kMaxSplits * kWarps - 1) / (kMaxSplits * kWarps);
    }
    const int wk = kWarps / best_wc;
    p.bn = best_wc * kStripe;
    p.kpw = best_kpw;
    p.splits = (KB + p.kpw * wk - 1) / (p.kpw * wk);
    return p;
}

cudaError_t launch_gemv_mma(const PackedWeight& w, const int32_t* qw_mma, const GemvPlan& p, const void* x, int M,
                            void* y, DType dt, cudaStream_t s, const GatherArgs* gather) {
    if (M <= 0) return cudaSuccess;
    if (M > kMaxTok || !gemv_mma_supported(w) || !qw_mma) return cudaErrorInvalidValue;
    GatherArgs ga = {};
    if (gather) ga = *gather;
    if (M > p.mt) return cudaErrorInvalidValue;
    if (M <= 8)
        return dt == kFP16 ? launch_t<kFP16, 1>(w, qw_mma, p, x, M, y, s, ga)
                           : launch_t<kBF16, 1>(w, qw_mma, p, x, M, y, s, ga);
    return dt == kFP16 ? launch_t<kFP16, 2>(w, qw_mma, p, x, M, y, s, ga)
                       : launch_t<kBF16, 2>(w, qw_mma, p, x, M, y, s, ga);
}

}  // namespace w4a16
