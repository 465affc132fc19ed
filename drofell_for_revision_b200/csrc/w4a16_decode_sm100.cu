// Decode W4A16 (M <= 16, fp16) on the sm_100a tensor cores, shaped for HBM speed.
//
// At M = 1 the tensor cores are nearly idle; a decode projection is bounded by HBM
// bandwidth and by how fast one SM can issue and land copies. This kernel keeps the
// copies few and large and the dequantized operand out of shared memory:
//
//   * weights arrive in TMA boxes of [32 packed rows x 128 columns] (16 KB = four
//     64-wide K chunks); X arrives in 3-D TMA boxes of four [16 tokens x 64 k]
//     tiles (8 KB, 128-byte swizzled as the MMA reads them); the CTA's scale and
//     zero rows arrive once, as one 2-D box each;
//   * eight "A" warps turn each packed word into the exact integers (q - z) as fp16
//     pairs in natural k order (prmt + lop3 + hfma2 per pair) and write them into a
//     tensor-memory ring with tcgen05.st; the MMA reads A from tensor memory
//     (tcgen05.mma kind::f16, A in TMEM, B = X tile in shared memory);
//   * every quantization group accumulates into its own 16-column TMEM block, in a
//     ring of 4 blocks; four "flush" warps drain a finished block, scale it by the
//     fp16 group scale in fp32 and keep the running sum in registers, then free the
//     block for the group four ahead. A CTA therefore spans any number of groups.
//
// Y[m, n] = sum_g s[g, n] * sum_{k in g} (q[k, n] - z[g, n]) x[m, k], fp32 throughout
// (the reference's dequant-then-matmul up to the rounding of the fp16 weights).
//
// Warp roles (448 threads): warp 0 producer (TMA), warp 1 TMEM owner + MMA issuer,
// warps 2-9 A warps, warps 10-13 flush warps. A K split is a cluster along z:
// partial tiles are summed in a fixed order through distributed shared memory
// (deterministic, no workspace, no atomics).
#include <cooperative_groups.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <cmath>
#include <cstdlib>

#include "w4a16_internal.h"
#include "w4a16_ptx.cuh"

namespace cg = cooperative_groups;

namespace w4a16 {
namespace {

constexpr int kThreads = 448;
constexpr int kAWarps = 8;                      // warps 2-9
constexpr int kFlushWarp0 = 10;                 // warps 10-13
constexpr int kChunkK = 64;
constexpr int kTileN = 128;
constexpr int kTok = 16;                        // MMA N: token rows of a tile
constexpr int kBlk = 4;                         // chunks per copy
constexpr int kRawChunk = kTileN * 8 * 4;       // 4 KB of packed words per chunk
constexpr int kWBlock = kBlk * kRawChunk;       // 16 KB weight box
constexpr int kXChunk = kTok * kChunkK * 2;     // 2 KB X tile (SW128)
constexpr int kXBlock = kBlk * kXChunk;         // 8 KB X box
constexpr int kLS = 4;                          // weight ring (16 KB slots)
constexpr int kXS = 4;                          // X ring (8 KB slots)
constexpr int kAS = 4;                          // TMEM A ring (32 columns each)
constexpr int kGS = 4;                          // TMEM group-accumulator ring (16 columns each)
constexpr int kACol0 = kGS * kTok;              // A ring starts after the accumulators
constexpr int kTmemCols = 256;                  // 64 + 4 x 32 = 192, rounded up
constexpr int kMaxGB = 32;                      // scale / zero rows per CTA
constexpr int kMaxSteps = 1024;                 // 16-k MMA steps per CTA (K range <= 16384)
constexpr uint32_t kWaitLimit = 1u << 26;
enum : int { kErrDecTimeout = 32 };

struct DecSmem {
    static constexpr int kXOff = 0;                            // X ring (1024-aligned)
    static constexpr int kWOff = kXOff + kXS * kXBlock;        // weight ring
    static constexpr int kScOff = kWOff + kLS * kWBlock;       // [kMaxGB][128] fp16
    static constexpr int kZrOff = kScOff + kMaxGB * kTileN * 2;  // [kMaxGB][16] int32
    static constexpr int kStepOff = kZrOff + kMaxGB * kTileN / 2;  // [kMaxSteps] uint16
    static constexpr int kBarOff = kStepOff + kMaxSteps * 2;
    static constexpr int kBytes = kBarOff + 512 + 1024;        // barriers + alignment slack
    static_assert(kTok * kTileN * 4 <= kLS * kWBlock, "fp32 output tile reuses the weight ring");
    static_assert(kBytes <= 113 * 1024, "two CTAs per SM");
};

__device__ __forceinline__ uint32_t h2u(__half2 v) { return *reinterpret_cast<uint32_t*>(&v); }

__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1, int c2) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(
            ptx::smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(ptx::smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
        : "memory");
}

// Two CTAs per SM: TMEM (2 x 256 columns), shared memory and registers all fit.
__global__ void __launch_bounds__(kThreads, 2)
    dec_kernel(const __grid_constant__ CUtensorMap tm_qw, const __grid_constant__ CUtensorMap tm_x,
               const __grid_constant__ CUtensorMap tm_sc, const __grid_constant__ CUtensorMap tm_zr,
               uint16_t* __restrict__ y, int M, int K, int N, int group_size, int chunks_per_split, int num_chunks,
               int gb, int* __restrict__ err) {
    extern __shared__ __align__(1024) uint8_t smem_dyn[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_dyn) + 1023) & ~uintptr_t(1023));
    uint8_t* xring = smem + DecSmem::kXOff;
    uint8_t* wring = smem + DecSmem::kWOff;
    const uint16_t* sc_s = reinterpret_cast<const uint16_t*>(smem + DecSmem::kScOff);
    const uint32_t* zr_s = reinterpret_cast<const uint32_t*>(smem + DecSmem::kZrOff);
    // step table: bits 0-11 local group, 12 first step of the group, 13 last step, 14 valid
    uint16_t* steps = reinterpret_cast<uint16_t*>(smem + DecSmem::kStepOff);
    uint64_t* lfull = reinterpret_cast<uint64_t*>(smem + DecSmem::kBarOff);
    uint64_t* lempty = lfull + kLS;
    uint64_t* xfull = lempty + kLS;
    uint64_t* xempty = xfull + kXS;
    uint64_t* afull = xempty + kXS;
    uint64_t* aempty = afull + kAS;
    uint64_t* gdone = aempty + kAS;
    uint64_t* gfree = gdone + kGS;
    uint64_t* gpar = gfree + kGS;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(gpar + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int n0 = blockIdx.x * kTileN;
    const int z = blockIdx.z;
    const int splits = gridDim.z;
    const int c0 = z * chunks_per_split;
    const int c1 = min(num_chunks, c0 + chunks_per_split);
    const int nc = max(0, c1 - c0);
    const int nb = (nc + kBlk - 1) / kBlk;                 // copies per ring
    const int KW = K >> 3;
    const int kend = min(K, c1 * kChunkK);                 // this CTA's K range: [c0*64, kend)
    const int g0 = (c0 * kChunkK) / group_size;
    const int ng = nc > 0 ? (kend - 1) / group_size - g0 + 1 : 0;

    // one division per step, here, instead of several per step in the hot loops
    for (int st = threadIdx.x; st < nc * 4; st += kThreads) {
        const int kabs = c0 * kChunkK + st * 16;
        uint16_t e = 0;
        if (kabs < kend) {
            const int g = kabs / group_size;
            const bool first = (kabs % group_size == 0) || st == 0;
            const bool last = (kabs + 16 >= kend) || ((kabs + 16) / group_size != g);
            e = static_cast<uint16_t>((g - g0) | (first ? 1 << 12 : 0) | (last ? 1 << 13 : 0) | (1 << 14));
        }
        steps[st] = e;
    }
    if (threadIdx.x == 0) {
        for (int s = 0; s < kLS; ++s) {
            ptx::mbar_init(&lfull[s], 1);
            ptx::mbar_init(&lempty[s], kAWarps);
        }
        for (int s = 0; s < kXS; ++s) {
            ptx::mbar_init(&xfull[s], 1);
            ptx::mbar_init(&xempty[s], 1);
        }
        for (int s = 0; s < kAS; ++s) {
            ptx::mbar_init(&afull[s], kAWarps);
            ptx::mbar_init(&aempty[s], 1);
        }
        for (int s = 0; s < kGS; ++s) {
            ptx::mbar_init(&gdone[s], 1);
            ptx::mbar_init(&gfree[s], 4);
        }
        ptx::mbar_init(gpar, 1);
        ptx::fence_mbar_init();
        ptx::prefetch_tmap(&tm_qw);
        ptx::prefetch_tmap(&tm_x);
    }
    if (warp == 1) {
        ptx::tmem_alloc(tmem_slot, kTmemCols);
        ptx::tmem_relinquish();
    }
    ptx::tc_fence_before();
    __syncthreads();
    ptx::tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    if (threadIdx.x == 0) ptx::grid_dep_launch_dependents();

    if (warp == 0) {
        // ------------------------------------------------ producer
        if (lane == 0) {
            // the CTA's scale and zero rows: one box each
            ptx::mbar_arrive_expect_tx(gpar, gb * (kTileN * 2 + kTileN / 2));
            ptx::tma_load_2d(smem + DecSmem::kScOff, &tm_sc, gpar, n0, g0);
            ptx::tma_load_2d(smem + DecSmem::kZrOff, &tm_zr, gpar, n0 >> 3, g0);
            auto issue_w = [&](int b) {
                const int s = b % kLS;
                ptx::mbar_arrive_expect_tx(&lfull[s], kWBlock);
                ptx::tma_load_2d(wring + s * kWBlock, &tm_qw, &lfull[s], n0, (c0 + b * kBlk) * 8);
            };
            auto issue_x = [&](int b) {
                const int s = b % kXS;
                ptx::mbar_arrive_expect_tx(&xfull[s], kXBlock);
                tma_load_3d(xring + s * kXBlock, &tm_x, &xfull[s], 0, 0, c0 + b * kBlk);
            };
            const int pre_w = min(nb, kLS);
            const int pre_x = min(nb, kXS);
            for (int b = 0; b < pre_w; ++b) issue_w(b);
            ptx::grid_dep_wait();  // X belongs to the previous kernel in the stream
            for (int b = 0; b < pre_x; ++b) issue_x(b);
            int iw = pre_w, ix = pre_x;
            // Refill both rings as their slots free up, never blocking on one while the
            // other could proceed (the MMA needs X tiles to release weight slots).
            uint32_t idle = 0;
            while ((iw < nb || ix < nb) && idle < kWaitLimit) {
                bool progressed = false;
                if (iw < nb && ptx::mbar_try_wait(&lempty[iw % kLS], ((iw / kLS) - 1) & 1)) {
                    issue_w(iw++);
                    progressed = true;
                }
                if (ix < nb && ptx::mbar_try_wait(&xempty[ix % kXS], ((ix / kXS) - 1) & 1)) {
                    issue_x(ix++);
                    progressed = true;
                }
                idle = progressed ? 0u : idle + 1u;
            }
            if (iw < nb || ix < nb) atomicCAS(err, 0, kErrDecTimeout);
            // drain: no copy may still be landing when the CTA exits
            for (int b = max(0, iw - kLS); b < iw; ++b)
                ptx::mbar_wait_bounded(&lfull[b % kLS], (b / kLS) & 1, kWaitLimit, err, kErrDecTimeout);
            for (int b = max(0, ix - kXS); b < ix; ++b)
                ptx::mbar_wait_bounded(&xfull[b % kXS], (b / kXS) & 1, kWaitLimit, err, kErrDecTimeout);
            ptx::mbar_wait_bounded(gpar, 0, kWaitLimit, err, kErrDecTimeout);
        }
    } else if (warp == 1) {
        // ------------------------------------------------ MMA issuer
        if (lane == 0) {
            constexpr uint32_t idesc = ptx::umma_idesc_f16(128, kTok, false);
            bool ok = true;
            for (int i = 0; i < nc && ok; ++i) {
                const int a = i % kAS;
                const int b = i / kBlk;
                const int sub = i % kBlk;
                const int xs = b % kXS;
                if (sub == 0) ok = ptx::mbar_wait_bounded(&xfull[xs], (b / kXS) & 1, kWaitLimit, err, kErrDecTimeout);
                ok = ok && ptx::mbar_wait_bounded(&afull[a], (i / kAS) & 1, kWaitLimit, err, kErrDecTimeout);
                if (!ok) break;
                ptx::tc_fence_after();
                const uint32_t b_base = ptx::smem_u32(xring + xs * kXBlock + sub * kXChunk);
#pragma unroll
                for (int kk = 0; kk < kChunkK / 16; ++kk) {
                    const uint32_t e = steps[i * 4 + kk];
                    if (!(e & (1u << 14))) break;  // past the end of K
                    const int gl = static_cast<int>(e & 0xFFFu);
                    const int gs = gl & (kGS - 1);
                    const bool first = (e >> 12) & 1u;
                    if (first && gl >= kGS) {
                        // the block's previous group must have been drained
                        ok = ptx::mbar_wait_bounded(&gfree[gs], ((gl / kGS) - 1) & 1, kWaitLimit, err, kErrDecTimeout);
                        if (!ok) break;
                        ptx::tc_fence_after();
                    }
                    ptx::umma_f16_ts(tmem + static_cast<uint32_t>(gs * kTok),
                                     tmem + static_cast<uint32_t>(kACol0 + a * (kChunkK / 2) + kk * 8),
                                     ptx::umma_desc_sw128(b_base + kk * 32), idesc, first ? 0u : 1u);
                    if ((e >> 13) & 1u) ptx::umma_commit(&gdone[gs]);
                }
                ptx::umma_commit(&aempty[a]);
                if (sub == kBlk - 1 || i == nc - 1) ptx::umma_commit(&xempty[xs]);
            }
        }
    } else if (warp < kFlushWarp0) {
        // ------------------------------------------------ A warps: (q - z) pairs into TMEM
        const int q = warp & 3;               // TMEM lane quadrant this warp may access
        const int half = (warp - 2) >> 2;     // words 4*half .. 4*half+3 of each chunk
        const int nl = q * 32 + lane;         // column within the tile = TMEM lane
        const bool col_ok = n0 + nl < N;
        const int zsh = (nl & 7) * 4;
        const __half2 mul = __halves2half2(__float2half_rn(1.0f), __float2half_rn(0.0625f));
        const uint32_t lane_base = static_cast<uint32_t>(q * 32) << 16;
        bool ok = ptx::mbar_wait_bounded(gpar, 0, kWaitLimit, err, kErrDecTimeout);  // zero rows
        for (int i = 0; i < nc && ok; ++i) {
            const int b = i / kBlk;
            const int sub = i % kBlk;
            const int s = b % kLS;
            const int a = i % kAS;
            if (sub == 0 && !ptx::mbar_wait_bounded(&lfull[s], (b / kLS) & 1, kWaitLimit, err, kErrDecTimeout)) break;
            const uint32_t* raw = reinterpret_cast<const uint32_t*>(wring + s * kWBlock + sub * kRawChunk);
            uint32_t wv[4], zw[4];
#pragma unroll
            for (int rr = 0; rr < 4; ++rr) {
                const int r = half * 4 + rr;
                wv[rr] = raw[r * kTileN + nl];
                // group of word r: its 16-k step is r / 2
                const int gl = static_cast<int>(steps[i * 4 + (r >> 1)] & 0xFFFu);
                zw[rr] = zr_s[gl * (kTileN / 8) + (nl >> 3)];
            }
            if (sub == kBlk - 1 || i == nc - 1) {
                __syncwarp();
                if (lane == 0) ptx::mbar_arrive(&lempty[s]);  // the weight box can refill now
            }
            if (i >= kAS &&
                !ptx::mbar_wait_bounded(&aempty[a], ((i / kAS) - 1) & 1, kWaitLimit, err, kErrDecTimeout))
                break;
            ptx::tc_fence_after();
            uint32_t o[16];
            const int kw0 = (c0 + i) * 8 + half * 4;
#pragma unroll
            for (int rr = 0; rr < 4; ++rr) {
                const float zf = static_cast<float>(((zw[rr] >> zsh) & 15u) + 1u);
                const __half2 zoff = __floats2half2_rn(-(1024.0f + zf), -(64.0f + zf));
                const bool live = kw0 + rr < KW && col_ok;
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const uint32_t bsel = __byte_perm(wv[rr], 0u, static_cast<uint32_t>(j | (j << 8)));
                    const uint32_t p = (bsel & 0x00F0000Fu) | 0x64006400u;  // (1024 + q0, 1024 + 16 q1)
                    const __half2 d = __hfma2(*reinterpret_cast<const __half2*>(&p), mul, zoff);  // exact q - z
                    o[rr * 4 + j] = live ? h2u(d) : 0u;
                }
            }
            ptx::tmem_st_32x32b_x16(tmem + lane_base + static_cast<uint32_t>(kACol0 + a * (kChunkK / 2) + half * 16), o);
            ptx::tmem_st_wait();
            ptx::tc_fence_before();
            __syncwarp();
            if (lane == 0) ptx::mbar_arrive(&afull[a]);
        }
    } else {
        // ------------------------------------------------ flush warps: scaled group sums
        const int q = warp & 3;
        const int nl = q * 32 + lane;
        const uint32_t lane_base = static_cast<uint32_t>(q * 32) << 16;
        float acc[kTok];
#pragma unroll
        for (int m = 0; m < kTok; ++m) acc[m] = 0.f;
        bool ok = ptx::mbar_wait_bounded(gpar, 0, kWaitLimit, err, kErrDecTimeout);  // scale rows
        for (int gl = 0; gl < ng && ok; ++gl) {
            const int gs = gl % kGS;
            const float sv = __half2float(__ushort_as_half(sc_s[gl * kTileN + nl]));
            ok = ptx::mbar_wait_bounded(&gdone[gs], (gl / kGS) & 1, kWaitLimit, err, kErrDecTimeout);
            if (!ok) break;
            ptx::tc_fence_after();
            uint32_t v[16];
            ptx::tmem_ld_32x32b_x16(tmem + lane_base + static_cast<uint32_t>(gs * kTok), v);
            ptx::tmem_ld_wait();
            ptx::tc_fence_before();
            __syncwarp();
            if (lane == 0) ptx::mbar_arrive(&gfree[gs]);
#pragma unroll
            for (int m = 0; m < kTok; ++m) acc[m] = fmaf(sv, __uint_as_float(v[m]), acc[m]);
        }
        // every copy has landed and been consumed once the last group is drained
        float* tile = reinterpret_cast<float*>(wring);  // [16 tokens][128 columns]
        const int rows = min(M, kTok);
#pragma unroll
        for (int m = 0; m < kTok; ++m)
            if (m < rows) tile[m * kTileN + nl] = ok ? acc[m] : 0.f;  // constant index: acc stays in registers
    }

    // ---- K splits: fixed-order sum over the cluster through distributed shared memory
    __syncthreads();
    float* tile = reinterpret_cast<float*>(wring);
    const int rows = min(M, kTok);
    ptx::grid_dep_wait();  // every thread that writes Y orders itself after the previous kernel
    if (splits > 1) {
        cg::cluster_group cluster = cg::this_cluster();
        cluster.sync();
        const int rank = static_cast<int>(cluster.block_rank());
        const int total = rows * kTileN;
        const int per = (total + splits - 1) / splits;
        const int i0 = rank * per;
        const int i1 = min(total, i0 + per);
        for (int idx = i0 + static_cast<int>(threadIdx.x); idx < i1; idx += kThreads) {
            const int m = idx / kTileN;
            const int nn = n0 + (idx - m * kTileN);
            float sum = 0.f;
            for (int r = 0; r < splits; ++r) sum += cluster.map_shared_rank(tile, r)[idx];
            if (nn < N) y[static_cast<size_t>(m) * N + nn] = __half_as_ushort(__float2half_rn(sum));
        }
        cluster.sync();
    } else {
        for (int idx = threadIdx.x; idx < rows * (kTileN / 8); idx += kThreads) {
            const int m = idx / (kTileN / 8);
            const int ch = idx - m * (kTileN / 8);
            const int nn = n0 + ch * 8;
            if (nn < N) {
                const float* src = tile + m * kTileN + ch * 8;
                uint32_t o[4];
#pragma unroll
                for (int e = 0; e < 4; ++e)
                    o[e] = static_cast<uint32_t>(__half_as_ushort(__float2half_rn(src[2 * e]))) |
                           (static_cast<uint32_t>(__half_as_ushort(__float2half_rn(src[2 * e + 1]))) << 16);
                *reinterpret_cast<uint4*>(y + static_cast<size_t>(m) * N + nn) = make_uint4(o[0], o[1], o[2], o[3]);
            }
        }
    }

    ptx::tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        ptx::tc_fence_after();
        ptx::tmem_dealloc(tmem, kTmemCols);
    }
}

int groups_touched(int cps, int group_size) {
    // a range of cps chunks not aligned to groups touches at most this many groups
    return (cps * kChunkK + group_size - 1) / group_size + 1;
}

// chunks per split: a whole number of weight boxes, so no box straddles two splits
int cps_for(int chunks, int splits) { return ((chunks + splits - 1) / splits + kBlk - 1) / kBlk * kBlk; }

// a split's steps fit the step table and its groups fit the scale / zero boxes
bool split_fits(const PackedWeight& w, int splits) {
    const int cps = cps_for((w.K + kChunkK - 1) / kChunkK, splits);
    return cps * 4 <= kMaxSteps && groups_touched(cps, w.group_size) <= kMaxGB;
}

}  // namespace

bool dec_supported(const PackedWeight& w, int M, int dtype) {
    // 16-k MMA steps must not straddle groups
    // K % 64: X is read through a [K/64][M][64] view; N % 32: zero rows are 16-byte multiples
    return dtype == kFP16 && M >= 1 && M <= kTok && w.group_size % 16 == 0 && w.K % kChunkK == 0 && w.N % 32 == 0 &&
           split_fits(w, 8);
}

DecPlan plan_dec(const PackedWeight& w, int num_sms) {
    DecPlan p;
    p.chunks = (w.K + kChunkK - 1) / kChunkK;
    const int tiles = (w.N + kTileN - 1) / kTileN;
    const int slots = num_sms * 2;  // two CTAs per SM
    auto cps_of = [&](int splits) { return cps_for(p.chunks, splits); };
    auto fits = [&](int splits) { return split_fits(w, splits); };
    // K splits (a cluster, at most 8): as many CTAs as fill the slots in one wave,
    // with at least 8 chunks of streaming per CTA
    int best = 0;
    double best_score = -1e9;
    for (int splits = 1; splits <= 8; ++splits) {
        const int cps = cps_of(splits);
        if (!fits(splits) || (p.chunks + cps - 1) / cps != splits) continue;
        if (best > 0 && cps < 8) break;
        const double ctas = static_cast<double>(tiles) * splits;
        const double waves = std::ceil(ctas / slots);
        const double score = ctas / (waves * slots) - 0.3 * (waves - 1) - 0.01 * splits;
        if (score > best_score) {
            best_score = score;
            best = splits;
        }
    }
    static const int env_splits = [] {
        const char* v = std::getenv("W4A16_DEC_SPLITS");  // tuning override
        return v ? std::atoi(v) : 0;
    }();
    if (env_splits > 0 && env_splits <= 8 && fits(env_splits)) best = env_splits;
    if (best == 0) best = 8;  // dec_supported guarantees that 8 splits fit
    p.cps = cps_of(best);
    p.splits = (p.chunks + p.cps - 1) / p.cps;
    p.gb = std::min(w.G, groups_touched(p.cps, w.group_size));
    return p;
}

size_t dec_workspace_bytes(const PackedWeight& w, int M) {
    // act-order: X gathered into kernel row order
    return w.act_order ? (static_cast<size_t>(M) * w.K * 2 + 255) / 256 * 256 : 0;
}

cudaError_t launch_dec(const PackedWeight& w, const DecPlan& p, const CUtensorMap* qw_map32, const void* x, int M,
                       void* y, void* ws, size_t ws_bytes, cudaStream_t s) {
    if (M <= 0) return cudaSuccess;
    if (ws_bytes < dec_workspace_bytes(w, M) || p.splits > 8 || p.cps % kBlk != 0 || p.cps * 4 > kMaxSteps ||
        p.gb > kMaxGB || p.gb < std::min(w.G, groups_touched(p.cps, w.group_size)))
        return cudaErrorInvalidValue;
    const void* xin = x;
    if (w.act_order) {
        cudaError_t e = launch_gather_cols(x, ws, w.perm, M, w.K, s);
        if (e != cudaSuccess) return e;
        xin = ws;
    }
    // X viewed as [K/64 chunks][M rows][64 k]: one box = four 128-byte-swizzled [16 x 64] tiles
    CUtensorMap x_map, sc_map, zr_map;
    const uint64_t xd[3] = {static_cast<uint64_t>(kChunkK), static_cast<uint64_t>(M),
                            static_cast<uint64_t>((w.K + kChunkK - 1) / kChunkK)};
    const uint64_t xs[2] = {static_cast<uint64_t>(w.K) * 2, static_cast<uint64_t>(kChunkK) * 2};
    const uint32_t xb[3] = {kChunkK, kTok, kBlk};
    if (encode_tmap_3d(&x_map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, xin, xd, xs, xb, CU_TENSOR_MAP_SWIZZLE_128B) !=
            CUDA_SUCCESS ||
        encode_tmap_2d(&sc_map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, w.scales, static_cast<uint64_t>(w.N),
                       static_cast<uint64_t>(w.G), static_cast<uint64_t>(w.N) * 2, kTileN, static_cast<uint32_t>(p.gb),
                       CU_TENSOR_MAP_SWIZZLE_NONE) != CUDA_SUCCESS ||
        encode_tmap_2d(&zr_map, CU_TENSOR_MAP_DATA_TYPE_INT32, w.qzeros, static_cast<uint64_t>(w.N / 8),
                       static_cast<uint64_t>(w.G), static_cast<uint64_t>(w.N / 8) * 4, kTileN / 8,
                       static_cast<uint32_t>(p.gb), CU_TENSOR_MAP_SWIZZLE_NONE) != CUDA_SUCCESS)
        return cudaErrorInvalidValue;
    static const cudaError_t attr_err = [] {
        cudaError_t e = cudaFuncSetAttribute(dec_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, DecSmem::kBytes);
        if (e == cudaSuccess) e = cudaFuncSetAttribute(dec_kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
        return e;
    }();
    if (attr_err != cudaSuccess) return attr_err;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((w.N + kTileN - 1) / kTileN, 1, p.splits);
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = DecSmem::kBytes;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    int na = 0;
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
    if (p.splits > 1) {
        attr[na].id = cudaLaunchAttributeClusterDimension;
        attr[na].val.clusterDim.x = 1;
        attr[na].val.clusterDim.y = 1;
        attr[na].val.clusterDim.z = p.splits;
        ++na;
    }
    cfg.attrs = attr;
    cfg.numAttrs = na;
    return cudaLaunchKernelEx(&cfg, dec_kernel, *qw_map32, x_map, sc_map, zr_map, static_cast<uint16_t*>(y), M, w.K,
                              w.N, w.group_size, p.cps, p.chunks, p.gb, w.err);
}

}  // namespace w4a16
