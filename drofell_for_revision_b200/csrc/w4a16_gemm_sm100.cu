// W4A16 GEMM on the sm_100a tensor cores: Y[M, N] = X[M, K] * W[K, N], W packed
// GPTQ int4, dequantized into shared memory and fed to tcgen05.mma with the
// accumulator in tensor memory.
//
// Replaces the reference's prefill path (After-Revision-DROFELL/cuda_extends/
// exllama/q4_matmul.cu:459-510: reconstruct the whole fp16 W into a scratch
// buffer, then cublasHgemm), and covers the batched-decode range its GEMV and
// Marlin's mma.sync kernel serve (marlin.cu:548-903).
//
// Orientation ("swap AB"): the MMA's M side (128 rows) is 128 output columns n
// of W^T; its N side is a tile of BN tokens of X. A = W^T tile [128 n x 64 k],
// B = X tile [BN tokens x 64 k], both K-major with the 128-byte swizzle, so
// D[n, m] = sum_k W[k, n] X[m, k] lands in TMEM lane n, column m.
//
// The A tile holds W = fp16(s * (q - z)), the same bits the dequant kernel writes
// (bf16 of them for bf16 inputs), so the product is the reference's dense GEMM on
// the reference's weights with fp32 accumulation.
//
// Warp roles (320 threads):
//   warp 0  producer: per 64-wide K chunk, TMA of the packed qweight tile
//           [8 words x 128 n] (4 KB) and of the X tile [BN x 64] (SW128), plus
//           bulk copies of the zero and scale rows of the chunk's
//           groups, into an LS-deep "load" ring. The weight part of the first LS
//           chunks is issued before griddepcontrol.wait, so it overlaps the
//           previous kernel in the stream.
//   warp 1  TMEM allocation; one elected thread issues 4 x tcgen05.mma
//           (K = 16 each) per chunk, then commits to the A slot's and the load
//           slot's "empty" barriers.
//   warps 2-9  dequant: thread t owns column n0 + (t % 128) and half of the 8
//           words of a chunk; each packed word (8 k of one column) becomes one
//           16-byte swizzled chunk of the A tile in an AS-deep operand ring.
//           Afterwards the same warps run the epilogue: tcgen05.ld of their TMEM
//           lane quadrant -> fp16/bf16 staged in shared memory -> coalesced
//           16-byte stores; or, with split-K, fp32 partials that
//           tc_splitk_reduce_kernel (launched next in the stream, on every SM) sums
//           in split order (deterministic). For a column-sharded layer
//           (w4a16_gemm_gather) the same 16-byte stores go to every rank's full Y
//           over NVLink peer memory (out_store16): the all-gather is the epilogue.
//
// Two 256-token tiles per CTA (NT = 2) share each dequantized A tile; their two
// accumulators fill the SM's 512 TMEM columns. plan_tc picks the token tile, NT and
// the K split from measured per-chunk costs.
//
// CTA pairs (PAIR, forward, 256-token tiles; W4A16_TC_PAIR=1): a cluster of two CTAs on
// adjacent column tiles runs M = 256 MMAs (cta_group::2) issued by rank 0: each CTA
// dequantizes its own 128 columns into its A ring and loads half of each token tile's X
// (its TMA completes on rank 0's barrier); rank 0's commits arrive on both CTAs'
// barriers, and each CTA drains its own tensor memory. No multicast load is used.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <cmath>
#include <cstdlib>

#include "w4a16_gather.cuh"
#include "w4a16_internal.h"
#include "w4a16_ptx.cuh"
#include "w4a16_tc_common.cuh"

namespace w4a16 {
namespace {

constexpr int kChunkK = 64;
constexpr int kTileN = 128;
constexpr int kATileBytes = kTileN * kChunkK * 2;  // 16 KB
constexpr int kRawTileBytes = kTileN * 8 * 4;      // 4 KB
constexpr int kMaxGroupsPerChunk = 8;              // group size >= 8
constexpr int kScaleRowBytes = kTileN * 2;         // 256 B
constexpr int kZeroRowBytes = kTileN / 2;          // 64 B
constexpr uint32_t kSleepLimit = 1u << 18;  // x ~10 us sleeps: a few seconds

enum : int { kErrTimeoutProducer = 1, kErrTimeoutMma = 2, kErrTimeoutDequant = 3, kErrTimeoutEpilogue = 4 };

// Epilogue shared by the forward and transposed GEMMs, run by the 256 dequant threads
// (warps 2-9) once the last MMA has committed: TMEM lane quadrant -> fp32 tile
// [BN tokens][128 columns] staged in the load ring -> 16-byte row pieces of
// Y[m, col0 + c] (row stride ld, columns < ncols), or fp32 partials of split z.
template <int BN, int NT, bool BF16, int EPI>
__device__ __forceinline__ void tc_epilogue(bool ok, int nc, uint64_t* accf, int* err, int warp, int lane, int t,
                                            uint32_t tmem, uint8_t* load_ring, int nt_live, int m0, int col0,
                                            int M, int ncols, int ld, int splits, int z, float* ws_part,
                                            uint16_t* y, const GatherArgs& ga) {
    // EPI threads (warps 2 .. 2 + EPI / 32 - 1) take part; warps 2-9 drain TMEM
    if (ok && nc > 0) ok = ptx::mbar_wait_sleep_bounded(accf, 0, kSleepLimit, err, kErrTimeoutEpilogue);
    ptx::tc_fence_after();
    ptx::grid_dep_wait();  // Y may still be read or written by the previous kernel
    const int q = warp & 3;                // TMEM lane quadrant this warp may access
    const int col_half = (warp - 2) >> 2;  // which half of the token columns (drain warps)
    const int tl = q * 32 + lane;          // local column (TMEM lane)
    const bool live = ok && nc > 0;
    float* fstage = reinterpret_cast<float*>(load_ring);  // [BN][128] fp32 tile
    for (int tt = 0; tt < nt_live; ++tt) {
        const int mt0 = m0 + tt * BN;  // first token of this tile
        const uint32_t trow = tmem + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(tt * BN);
        {
            constexpr int kHalfCols = BN / 2;
            if (warp < 10) {
#pragma unroll 1
                for (int c = col_half * kHalfCols; c < (col_half + 1) * kHalfCols; c += 8) {
                    uint32_t v[8];
                    ptx::tmem_ld_32x32b_x8(trow + c, v);
                    ptx::tmem_ld_wait();
#pragma unroll
                    for (int j = 0; j < 8; ++j) fstage[(c + j) * kTileN + tl] = live ? __uint_as_float(v[j]) : 0.f;
                }
            }
            ptx::named_bar_sync(1, EPI);
        }
        // fstage now holds the CTA's fp32 tile [BN tokens][128 columns]
        if (splits == 1) {
            if (ok) {
                // coalesced copy-out: 16 x 16 B per token row
                for (int idx = t; idx < BN * 16; idx += EPI) {
                    const int ml = idx >> 4;
                    const int ch = idx & 15;
                    const int m = mt0 + ml;
                    const int nn = col0 + ch * 8;
                    if (m < M && nn < ncols) {
                        const float* src = fstage + ml * kTileN + ch * 8;
                        uint32_t o[4];
#pragma unroll
                        for (int e = 0; e < 4; ++e)
                            o[e] = static_cast<uint32_t>(to_out<BF16>(src[2 * e])) |
                                   (static_cast<uint32_t>(to_out<BF16>(src[2 * e + 1])) << 16);
                        out_store16(ga, y, ld, m, nn, make_uint4(o[0], o[1], o[2], o[3]));
                    }
                }
            }
        } else if (ok) {
            // fp32 partial of split z (summed by tc_splitk_reduce_kernel)
            for (int idx = t; idx < BN * 32; idx += EPI) {
                const int ml = idx >> 5;
                const int ch = idx & 31;
                const int m = mt0 + ml;
                const int nn = col0 + ch * 4;
                if (m < M && nn < ncols)
                    *reinterpret_cast<float4*>(ws_part + (static_cast<size_t>(z) * M + m) * ld + nn) =
                        *reinterpret_cast<const float4*>(fstage + ml * kTileN + ch * 4);
            }
        }
        ptx::named_bar_sync(1, EPI);  // fstage is rewritten by the next token tile
    }
}

// ---------------------------------------------------------------- the GEMM kernel
// One kernel computes both products of the packed weight (TRANS selects):
//   forward     Y[M, N] = X[M, K] W: the MMA's M side is 128 output columns n of W^T
//               (A = [128 n x 64 k], K-major), its N side BN tokens of X (B, K-major).
//   transposed  dX[M, K] = dY[M, N] W^T, the input gradient. Replaces the reference's
//               backward (After-Revision-DROFELL/cuda_extends/exllama/
//               q4_transpose_matmul.cu:115-167: reconstruct W, then cublasHgemm with
//               OP_T, fp16 accumulate). The MMA's M side is 128 weight rows k, its N side
//               BN tokens, the reduction runs along the weight's columns n in chunks of 64:
//               A = W tile [128 k x 64 n], MN-major, so a packed word (8 consecutive k of
//               one column n) dequantizes to exactly one 16-byte chunk of it (one swizzled
//               st.shared.v4, nothing transposed in registers); B = dY tile [BN x 64 n],
//               K-major. The 128 k rows of a CTA touch a fixed set of groups, whose scale
//               and zero rows are bulk-copied per 64-column chunk.
// D lands in TMEM lane (column n, or row k), column m; the shared epilogue writes rows.
//
// Warp roles (608 threads):
//   warp 0       weight producer: per 64-wide chunk of the reduction, TMA of a 4 KB packed
//                qweight tile ([8 words x 128 n] forward, [16 words x 64 n] transposed)
//                and bulk copies of its zero and scale rows into a WS-deep ring, refilled as soon as the dequant warps have read a slot. The
//                weights do not depend on the previous kernel, so this warp never waits for
//                it (griddepcontrol): they stream from the CTA's start.
//   warp 18      X producer: after griddepcontrol.wait, the X tiles [BN tokens x 64 k]
//                (SW128) of each chunk into an XS-deep ring, refilled when the MMAs that
//                read a slot have completed. X is shared by every column tile and served
//                from L2, so its round trip is short; keeping it apart from the HBM-bound
//                weights keeps that round trip off the tensor pipe's critical path.
//   warp 1       TMEM allocation; one elected thread issues 4 x tcgen05.mma (K = 16 each)
//                per chunk and commits to the A slot's and the X slot's "empty" barriers.
//   warps 2-17   dequant, two groups of 8 warps taking alternate chunks (a chunk's dequant
//                is a dependent chain of smem reads and f16x2 math: one group alone leaves
//                the tensor pipe waiting). Thread t of a group owns column n0 + (t % 128)
//                and half of the 8 words of its chunks; each packed word (8 k of one column)
//                becomes one 16-byte swizzled chunk of the A tile in an AS-deep ring.
//                Afterwards all 16 warps run the epilogue (warps 2-9 drain TMEM).
// transposed tiles: 128 weight rows = 16 packed rows x 64 columns (4 KB), up to 16 groups
constexpr int kTRows = 16;
constexpr int kTMaxGroups = 16;          // group size >= 8
constexpr int kTScaleRowBytes = 64 * 2;  // 128 B
constexpr int kTZeroRowBytes = 64 / 2;   // 32 B
// MN-major SW128 A tile of the transposed product: 64-row blocks b (LBO apart) of
// 8-column atoms j (SBO apart), atom (b, j) at (b * 8 + j) * 1024 bytes.
constexpr uint32_t kTLbo = 8 * 1024;
constexpr uint32_t kTSbo = 1024;

constexpr int kFwdThreads = 19 * 32;
constexpr int kFwdDqThreads = 512;
constexpr int kFwdXWarp = 18;
constexpr int kWSlotBytes = 7 * 1024;  // raw tile 4 KB | 8 scale rows 2 KB | 8 zero rows 512 B
constexpr int kWScOff = kRawTileBytes;
constexpr int kWZrOff = kWScOff + kMaxGroupsPerChunk * kScaleRowBytes;

template <int BN, int NT, bool PAIR = false>
struct FwdCfg {
    // one token tile's X chunk (SW128) in this CTA: a CTA pair splits the tile's tokens
    static constexpr int kXBytes = (PAIR ? BN / 2 : BN) * kChunkK * 2;
    static constexpr int kXStage = NT * kXBytes;
    static constexpr int XS = PAIR ? (NT == 2 ? 4 : 8) : NT == 2 ? 2 : BN == 256 ? 4 : BN == 128 ? 6 : 8;
    static constexpr int WS = BN >= 256 ? 6 : 8;
    static constexpr int AS = BN >= 256 ? 3 : 4;
    static constexpr int kWOff = XS * kXStage;
    static constexpr int kAOff = kWOff + WS * kWSlotBytes;
    static constexpr int kBarOff = kAOff + AS * kATileBytes;
    static constexpr int kTmemCols = (BN < 32 ? 32 : BN) * NT;
    static constexpr int kSmemBytes = kBarOff + 1024 /*barriers*/ + 1024 /*align*/;
    static_assert(kSmemBytes <= 227 * 1024, "shared memory budget");
    static_assert(BN * kTileN * 4 <= XS * kXStage, "epilogue staging must fit in the X ring");
    static_assert(kWZrOff + kMaxGroupsPerChunk * kZeroRowBytes <= kWSlotBytes, "weight slot layout");
    static_assert(kWScOff + kTMaxGroups * kTScaleRowBytes <= kWZrOff &&
                      kWZrOff + kTMaxGroups * kTZeroRowBytes <= kWSlotBytes,
                  "transposed weight slot layout");
};

template <int BN, int NT, bool BF16, bool TRANS, bool PAIR = false>
__global__ void __launch_bounds__(kFwdThreads, 1)
    tc_gemm_kernel(const __grid_constant__ CUtensorMap tm_qw, const __grid_constant__ CUtensorMap tm_x,
                   const int32_t* __restrict__ qzeros, const uint16_t* __restrict__ scales,
                   uint16_t* __restrict__ y, float* __restrict__ ws_part, int M, int K,
                   int N, int G, int group_size, int chunks_per_split, int num_chunks, int splits,
                   int* __restrict__ err, const GatherArgs ga) {
    static_assert(!PAIR || (BN == 256 && !TRANS), "CTA pairs: forward product, 256-token tiles");
    using C = FwdCfg<BN, NT, PAIR>;
    constexpr int XS = C::XS;
    constexpr int WS = C::WS;
    constexpr int AS = C::AS;
    extern __shared__ __align__(1024) uint8_t smem_dyn[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_dyn) + 1023) & ~uintptr_t(1023));
    uint8_t* x_ring = smem;
    uint8_t* w_ring = smem + C::kWOff;
    uint8_t* a_ring = smem + C::kAOff;
    uint64_t* xfull = reinterpret_cast<uint64_t*>(smem + C::kBarOff);
    uint64_t* xempty = xfull + XS;
    uint64_t* wfull = xempty + XS;
    uint64_t* wempty = wfull + WS;
    uint64_t* afull = wempty + WS;
    uint64_t* aempty = afull + AS;
    uint64_t* accf = aempty + AS;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accf + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    // CTA pairs: rank 0 issues the MMAs for both; barriers it waits on live in its memory
    const uint32_t rank = PAIR ? ptx::cluster_ctarank() : 0u;
    const bool leader = rank == 0;
    const int n0 = blockIdx.x * kTileN;  // first output column: n (forward) or k (transposed)
    const int m0 = blockIdx.y * BN * NT;
    const int nt_live = min(NT, (M - m0 + BN - 1) / BN);  // token tiles of this CTA inside M
    const int z = blockIdx.z;
    const int c0 = z * chunks_per_split;
    const int c1 = min(num_chunks, c0 + chunks_per_split);
    const int nc = max(0, c1 - c0);
    const int KW = K >> 3;
    const int wpg = group_size >> 3;  // packed words per group

    if (threadIdx.x == 0) {
        for (int s = 0; s < XS; ++s) {
            ptx::mbar_init(&xfull[s], 1);
            ptx::mbar_init(&xempty[s], 1);
        }
        for (int s = 0; s < WS; ++s) {
            ptx::mbar_init(&wfull[s], 1);
            ptx::mbar_init(&wempty[s], 8);  // the 8 warps of the group that read the slot
        }
        for (int s = 0; s < AS; ++s) {
            ptx::mbar_init(&afull[s], PAIR ? 16 : 8);  // the dequant group's 8 warps (of both CTAs)
            ptx::mbar_init(&aempty[s], 1);
        }
        ptx::mbar_init(accf, 1);
        ptx::fence_mbar_init();
        ptx::prefetch_tmap(&tm_qw);
        ptx::prefetch_tmap(&tm_x);
    }
    if (warp == 1) {
        if constexpr (PAIR) {  // both CTAs, same warp, same slot offset
            ptx::tmem_alloc_pair(tmem_slot, C::kTmemCols);
            ptx::tmem_relinquish_pair();
        } else {
            ptx::tmem_alloc(tmem_slot, C::kTmemCols);
            ptx::tmem_relinquish();
        }
    }
    ptx::tc_fence_before();
    __syncthreads();
    if constexpr (PAIR) ptx::cluster_sync_all();  // the peer's barriers and tensor memory are ready
    ptx::tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    if (threadIdx.x == 0) ptx::grid_dep_launch_dependents();

    if (warp == 0) {
        // ------------------------------------------------ weight producer
        if (lane == 0) {
            int issued = 0;
            for (int i = 0; i < nc; ++i) {
                const int s = i % WS;
                if (i >= WS && !ptx::mbar_wait_sleep_bounded(&wempty[s], ((i / WS) - 1) & 1, kSleepLimit, err,
                                                       kErrTimeoutProducer))
                    break;
                uint8_t* slot = w_ring + s * kWSlotBytes;
                const int cg = c0 + i;
                // the chunk's tile origin (column, packed row), its groups and row widths
                int tx, ty, g_first, g_last, wcols, sc_row, zr_row;
                if constexpr (TRANS) {
                    tx = cg * 64;                      // columns n of this chunk
                    ty = blockIdx.x * kTRows;          // the CTA's 16 packed rows
                    g_first = n0 / group_size;
                    g_last = min(G - 1, (min(K, n0 + kTileN) - 1) / group_size);
                    wcols = min(64, N - tx);
                    sc_row = kTScaleRowBytes;
                    zr_row = kTZeroRowBytes;
                } else {
                    tx = n0;
                    ty = cg * 8;
                    g_first = (cg * kChunkK) / group_size;
                    g_last = min(G - 1, (cg * kChunkK + kChunkK - 1) / group_size);
                    wcols = min(kTileN, N - n0);
                    sc_row = kScaleRowBytes;
                    zr_row = kZeroRowBytes;
                }
                const int cnt = wcols > 0 ? g_last - g_first + 1 : 0;  // no columns (a pair's CTA past N)
                const uint32_t sbytes = static_cast<uint32_t>(max(wcols, 0)) * 2;
                const uint32_t zbytes = qzeros ? static_cast<uint32_t>(max(wcols, 0)) / 2 : 0u;  // none when symmetric
                ptx::mbar_arrive_expect_tx(&wfull[s], kRawTileBytes + cnt * (sbytes + zbytes));
                ptx::tma_load_2d(slot, &tm_qw, &wfull[s], tx, ty);
                for (int j = 0; j < cnt; ++j) {
                    const int g = g_first + j;
                    ptx::bulk_load(slot + kWScOff + j * sc_row, scales + static_cast<size_t>(g) * N + tx, sbytes,
                                   &wfull[s]);
                    if (qzeros)
                        ptx::bulk_load(slot + kWZrOff + j * zr_row, qzeros + static_cast<size_t>(g) * (N >> 3) + (tx >> 3),
                                       zbytes, &wfull[s]);
                }
                ++issued;
            }
            // Drain: do not leave the CTA while a copy issued above may still land.
            for (int i = max(0, issued - WS); i < issued; ++i)
                ptx::mbar_wait_sleep_bounded(&wfull[i % WS], (i / WS) & 1, kSleepLimit, err, kErrTimeoutProducer);
        }
    } else if (warp == kFwdXWarp) {
        // ------------------------------------------------ X producer
        if (lane == 0) {
            ptx::grid_dep_wait();  // X (and Y) belong to the previous kernel in the stream
            int issued = 0;
            for (int i = 0; i < nc; ++i) {
                const int s = i % XS;
                if (i >= XS && !ptx::mbar_wait_sleep_bounded(&xempty[s], ((i / XS) - 1) & 1, kSleepLimit, err,
                                                       kErrTimeoutProducer))
                    break;
                if constexpr (PAIR) {
                    // each CTA loads its half of every token tile; rank 0's barrier counts both
                    if (leader) ptx::mbar_arrive_expect_tx(&xfull[s], 2 * nt_live * C::kXBytes);
                    const uint32_t bar0 = ptx::mapa_shared(ptx::smem_u32(&xfull[s]), 0);
                    for (int tt = 0; tt < nt_live; ++tt)
                        ptx::tma_load_2d_pair(x_ring + s * C::kXStage + tt * C::kXBytes, &tm_x, bar0,
                                              (c0 + i) * kChunkK, m0 + tt * BN + static_cast<int>(rank) * (BN / 2));
                } else {
                    ptx::mbar_arrive_expect_tx(&xfull[s], nt_live * C::kXBytes);
                    for (int tt = 0; tt < nt_live; ++tt)
                        ptx::tma_load_2d(x_ring + s * C::kXStage + tt * C::kXBytes, &tm_x, &xfull[s],
                                         (c0 + i) * kChunkK, m0 + tt * BN);
                }
                ++issued;
            }
            // (a pair's rank 1 has no barrier to drain: its loads complete on rank 0's, before
            // the MMAs that precede the final cluster barrier)
            if (leader)
                for (int i = max(0, issued - XS); i < issued; ++i)
                    ptx::mbar_wait_sleep_bounded(&xfull[i % XS], (i / XS) & 1, kSleepLimit, err, kErrTimeoutProducer);
        }
    } else if (warp == 1) {
        // ------------------------------------------------ MMA issuer
        if (lane == 0 && leader) {
            constexpr uint32_t idesc =
                ptx::umma_idesc_f16(PAIR ? 256 : 128, BN, BF16) | (TRANS ? (1u << 15) : 0u);  // A MN-major
            for (int i = 0; i < nc; ++i) {
                const int a = i % AS;
                const int x = i % XS;
                if (!ptx::mbar_wait_sleep_bounded(&afull[a], (i / AS) & 1, kSleepLimit, err, kErrTimeoutMma)) break;
                if (!ptx::mbar_wait_sleep_bounded(&xfull[x], (i / XS) & 1, kSleepLimit, err, kErrTimeoutMma)) break;
                ptx::tc_fence_after();
                const uint32_t a_base = ptx::smem_u32(a_ring + a * kATileBytes);
                const uint32_t b_base = ptx::smem_u32(x_ring + x * C::kXStage);
#pragma unroll
                for (int kk = 0; kk < kChunkK / 16; ++kk) {
                    const uint64_t da = TRANS ? ptx::umma_desc_sw128_mn(a_base + kk * 2 * kTSbo, kTLbo, kTSbo)
                                              : ptx::umma_desc_sw128(a_base + kk * 32);
#pragma unroll
                    for (int tt = 0; tt < NT; ++tt) {
                        if (tt < nt_live) {
                            const uint64_t db = ptx::umma_desc_sw128(b_base + tt * C::kXBytes + kk * 32);
                            if constexpr (PAIR)
                                ptx::umma_f16_pair(tmem + static_cast<uint32_t>(tt * BN), da, db, idesc,
                                                   (i > 0 || kk > 0) ? 1u : 0u);
                            else
                                ptx::umma_f16(tmem + static_cast<uint32_t>(tt * BN), da, db, idesc,
                                              (i > 0 || kk > 0) ? 1u : 0u);
                        }
                    }
                }
                if constexpr (PAIR) {
                    ptx::umma_commit_pair(&aempty[a], 0x3);
                    ptx::umma_commit_pair(&xempty[x], 0x3);
                } else {
                    ptx::umma_commit(&aempty[a]);
                    ptx::umma_commit(&xempty[x]);
                }
            }
            if constexpr (PAIR)
                ptx::umma_commit_pair(accf, 0x3);
            else
                ptx::umma_commit(accf);
        }
    } else {
        // ------------------------------------------------ dequant warps (two groups)
        const int dq = threadIdx.x - 64;  // 0..511
        const int grp = dq >> 8;          // this group takes chunks i with i % 2 == grp
        const int t = dq & 255;
        bool ok = true;
        if constexpr (TRANS) {
            const int nl = t & 63;  // column within the 64-wide chunk (the MMA's K index)
            const int rq = t >> 6;  // packed rows rq, rq + 4, rq + 8, rq + 12 of the tile
            const int kw0 = blockIdx.x * kTRows;
            const int zsh = (nl & 7) * 4;
            const uint32_t row_off = static_cast<uint32_t>((nl >> 3) * 1024 + (nl & 7) * 128);
            // this thread's 4 packed rows are the same in every chunk: their slot group rows once
            const int g_first = n0 / group_size;
            int glr[4];
#pragma unroll
            for (int jj = 0; jj < 4; ++jj) glr[jj] = ((kw0 + rq + 4 * jj) * 8) / group_size - g_first;
            for (int i = grp; i < nc; i += 2) {
                const int s = i % WS;
                const int a = i % AS;
                if (!ptx::mbar_wait_sleep_bounded(&wfull[s], (i / WS) & 1, kSleepLimit, err, kErrTimeoutDequant)) {
                    ok = false;
                    break;
                }
                if (i >= AS &&
                    !ptx::mbar_wait_sleep_bounded(&aempty[a], ((i / AS) - 1) & 1, kSleepLimit, err, kErrTimeoutDequant)) {
                    ok = false;
                    break;
                }
                const uint8_t* slot = w_ring + s * kWSlotBytes;
                const uint32_t* raw = reinterpret_cast<const uint32_t*>(slot);
                const uint16_t* sc = reinterpret_cast<const uint16_t*>(slot + kWScOff);
                const uint32_t* zr = reinterpret_cast<const uint32_t*>(slot + kWZrOff);
                const uint32_t a_tile = ptx::smem_u32(a_ring + a * kATileBytes) + row_off;
                const bool col_ok = (c0 + i) * 64 + nl < N;
#pragma unroll
                for (int jj = 0; jj < 4; ++jj) {
                    const int r = rq + 4 * jj;  // packed row within the tile: weight rows 8r .. 8r + 7
                    uint4 o = make_uint4(0u, 0u, 0u, 0u);
                    if (kw0 + r < KW && col_ok) {
                        const int gl = glr[jj];
                        const uint32_t zw = qzeros ? zr[gl * 8 + (nl >> 3)] : kSymmetricZeroWord;
                        const uint32_t zp = ((zw >> zsh) & 15u) + 1u;
                        const uint32_t zb = (0xE400u + zp) | ((0xD400u + (zp << 4)) << 16);  // -(1024 + z), -(64 + z)
                        const __half2 zoff = *reinterpret_cast<const __half2*>(&zb);
                        const __half2 s2 = __half2half2(__ushort_as_half(sc[gl * 64 + nl]));
                        o = dequant_word<BF16>(raw[r * 64 + nl], s2, zoff);
                    }
                    // rows 8r .. 8r + 7: 64-row block r / 8, 16-byte chunk r % 8 of the swizzled 128-byte line
                    ptx::st_shared_v4(a_tile + (r >> 3) * kTLbo + ((((r & 7) ^ (nl & 7))) << 4), o);
                }
                ptx::fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) {
                    ptx::mbar_arrive(&afull[a]);
                    ptx::mbar_arrive(&wempty[s]);
                }
            }
        } else {
            const int nl = t & (kTileN - 1);  // column within the tile
            const int half = t >> 7;          // words 4*half .. 4*half+3 of each chunk
            const int n = n0 + nl;
            const bool col_ok = n < N;
            const int zsh = (nl & 7) * 4;
            // Group bookkeeping without a division per word: (gh, oh) = group of this thread's
            // first row of its chunk and the offset inside it, (gf, of) the same for the chunk's
            // first row (the slot's first scale / zero row); both advance 16 packed rows (two
            // chunks) a step.
            int gh, oh, gf, of;
            {
                const int kw_h = (c0 + grp) * 8 + half * 4;
                gh = kw_h / wpg;
                oh = kw_h - gh * wpg;
                gf = ((c0 + grp) * 8) / wpg;
                of = (c0 + grp) * 8 - gf * wpg;
            }
            // A group boundary inside this thread's 4 rows of a chunk needs group sizes that
            // are not a multiple of 32 (4 packed rows); otherwise the 4 words share one scale
            // and zero and dequantize as independent straight-line work.
            const bool whole = (wpg & 3) == 0;
            for (int i = grp; i < nc; i += 2) {
                const int s = i % WS;
                const int a = i % AS;
                if (!ptx::mbar_wait_sleep_bounded(&wfull[s], (i / WS) & 1, kSleepLimit, err, kErrTimeoutDequant)) {
                    ok = false;
                    break;
                }
                const uint8_t* slot = w_ring + s * kWSlotBytes;
                const uint32_t* raw = reinterpret_cast<const uint32_t*>(slot);
                const uint16_t* sc = reinterpret_cast<const uint16_t*>(slot + kWScOff);
                const uint32_t* zr = reinterpret_cast<const uint32_t*>(slot + kWZrOff);
                const int kw_h = (c0 + i) * 8 + half * 4;
                // this thread's 4 packed words, read before waiting for the A slot
                uint32_t wv[4];
#pragma unroll
                for (int rr = 0; rr < 4; ++rr)
                    wv[rr] = (kw_h + rr < KW && col_ok) ? raw[(half * 4 + rr) * kTileN + nl] : 0u;
                int gl = gh - gf;     // slot row of the current group
                int left = wpg - oh;  // rows of it from kw_h on
                __half2 s2, zoff;
                auto fetch = [&](int g) {
                    const uint32_t zw = qzeros ? zr[g * (kTileN / 8) + (nl >> 3)] : kSymmetricZeroWord;
                    const uint32_t zp = ((zw >> zsh) & 15u) + 1u;
                    // (-(1024 + z), -(64 + z)) as exact fp16 bits: 1024 and 64 carry unit and 1/16 steps
                    const uint32_t zb = (0xE400u + zp) | ((0xD400u + (zp << 4)) << 16);
                    zoff = *reinterpret_cast<const __half2*>(&zb);
                    s2 = __half2half2(__ushort_as_half(sc[g * kTileN + nl]));
                };
                fetch(gl);
                if (whole) {  // everything this thread needs from the slot is in registers: free it now
                    __syncwarp();
                    if (lane == 0) ptx::mbar_arrive(&wempty[s]);
                }
                if (i >= AS &&
                    !ptx::mbar_wait_sleep_bounded(&aempty[a], ((i / AS) - 1) & 1, kSleepLimit, err, kErrTimeoutDequant)) {
                    ok = false;
                    break;
                }
                const uint32_t a_row = ptx::smem_u32(a_ring + a * kATileBytes) + nl * 128;
                if (whole) {
                    uint4 o[4];
#pragma unroll
                    for (int rr = 0; rr < 4; ++rr)
                        o[rr] = (kw_h + rr < KW && col_ok) ? dequant_word<BF16>(wv[rr], s2, zoff)
                                                           : make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
                    for (int rr = 0; rr < 4; ++rr) {
                        const int r = half * 4 + rr;
                        ptx::st_shared_v4(a_row + ((r ^ (nl & 7)) << 4), o[rr]);
                    }
                } else {
#pragma unroll
                    for (int rr = 0; rr < 4; ++rr) {
                        if (rr == left) {  // the next row starts a new group (group size < 32 rows)
                            ++gl;
                            left += wpg;
                            fetch(gl);
                        }
                        const int r = half * 4 + rr;
                        uint4 o = make_uint4(0u, 0u, 0u, 0u);
                        if (kw_h + rr < KW && col_ok) o = dequant_word<BF16>(wv[rr], s2, zoff);
                        ptx::st_shared_v4(a_row + ((r ^ (nl & 7)) << 4), o);
                    }
                }
                ptx::fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) {
                    if constexpr (PAIR)  // the MMA that reads this A half is issued by rank 0
                        ptx::mbar_arrive_cluster(ptx::mapa_shared(ptx::smem_u32(&afull[a]), 0));
                    else
                        ptx::mbar_arrive(&afull[a]);
                    if (!whole) ptx::mbar_arrive(&wempty[s]);  // the slot's words, scales and zeros have been read
                }
                oh += 16;
                while (oh >= wpg) {
                    oh -= wpg;
                    ++gh;
                }
                of += 16;
                while (of >= wpg) {
                    of -= wpg;
                    ++gf;
                }
            }
        }

        // ------------------------------------------------ epilogue
        const int ncols_out = TRANS ? K : N;  // dX rows are K long, Y rows N
        tc_epilogue<BN, NT, BF16, kFwdDqThreads>(ok, nc, accf, err, warp, lane, dq, tmem, x_ring, nt_live, m0, n0, M,
                                                 ncols_out, ncols_out, splits, z, ws_part, y, ga);
    }

    ptx::tc_fence_before();
    __syncthreads();
    if constexpr (PAIR) ptx::cluster_sync_all();  // both CTAs are done with the pair's tensor memory
    if (warp == 1) {
        ptx::tc_fence_after();
        if constexpr (PAIR)
            ptx::tmem_dealloc_pair(tmem, C::kTmemCols);
        else
            ptx::tmem_dealloc(tmem, C::kTmemCols);
    }
}

// Split-K: Y[m, n] = the fp32 partials of splits 0, 1, ... summed in that order.
// 8 outputs per thread (two 16-byte loads per split, one 16-byte store); N % 8 == 0.
template <bool BF16>
__global__ void __launch_bounds__(256) tc_splitk_reduce_kernel(const float* __restrict__ ws, uint16_t* __restrict__ y,
                                                               int M, int N, int splits, const GatherArgs ga) {
    ptx::grid_dep_wait();  // the partials come from the GEMM before it in the stream
    const size_t total8 = static_cast<size_t>(M) * N / 8;
    const size_t plane = static_cast<size_t>(M) * N;
    for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total8;
         i += static_cast<size_t>(gridDim.x) * blockDim.x) {
        float a[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        for (int z = 0; z < splits; ++z) {
            const float4* src = reinterpret_cast<const float4*>(ws + z * plane) + 2 * i;
            const float4 u = __ldcs(src), v = __ldcs(src + 1);  // read once
            a[0] += u.x;
            a[1] += u.y;
            a[2] += u.z;
            a[3] += u.w;
            a[4] += v.x;
            a[5] += v.y;
            a[6] += v.z;
            a[7] += v.w;
        }
        uint32_t o[4];
#pragma unroll
        for (int e = 0; e < 4; ++e)
            o[e] = static_cast<uint32_t>(to_out<BF16>(a[2 * e])) | (static_cast<uint32_t>(to_out<BF16>(a[2 * e + 1])) << 16);
        const int m = static_cast<int>(8 * i / N);
        out_store16(ga, y, N, m, static_cast<int>(8 * i - static_cast<size_t>(m) * N), make_uint4(o[0], o[1], o[2], o[3]));
    }
}

template <bool BF16>
cudaError_t launch_splitk_reduce(const float* ws, void* y, int M, int N, int splits, int num_sms, cudaStream_t s,
                                 const GatherArgs& ga) {
    const size_t total8 = static_cast<size_t>(M) * N / 8;
    const size_t want = (total8 + 255) / 256;
    const unsigned blocks = static_cast<unsigned>(std::min<size_t>(want, static_cast<size_t>(num_sms) * 8));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(blocks, 1, 1);
    cfg.blockDim = dim3(256, 1, 1);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, tc_splitk_reduce_kernel<BF16>, ws, static_cast<uint16_t*>(y), M, N, splits, ga);
}

template <int BN, int NT, bool BF16, bool PAIR = false>
cudaError_t launch_tc_t(const PackedWeight& w, const TcPlan& p, const CUtensorMap* qw_map, const CUtensorMap& x_map,
                        int M, void* y, float* ws_part, cudaStream_t s, const GatherArgs& ga) {
    using C = FwdCfg<BN, NT, PAIR>;
    auto kern = tc_gemm_kernel<BN, NT, BF16, false, PAIR>;
    // Once per instantiation (and so before any stream capture that reuses it).
    static const cudaError_t attr_err =
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmemBytes);
    if (attr_err != cudaSuccess) return attr_err;
    int n_tiles = (w.N + kTileN - 1) / kTileN;
    if (PAIR) n_tiles += n_tiles & 1;  // whole pairs (a CTA past N computes zeros and stores nothing)
    const int m_tiles = (M + BN - 1) / BN;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(n_tiles, (m_tiles + NT - 1) / NT, p.splits);
    cfg.blockDim = dim3(kFwdThreads, 1, 1);
    cfg.dynamicSmemBytes = C::kSmemBytes;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = 2;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = PAIR ? 2 : 1;
    cudaError_t e = cudaLaunchKernelEx(&cfg, kern, *qw_map, x_map, w.kernel_qzeros(), w.scales, static_cast<uint16_t*>(y),
                                       ws_part, M, w.K, w.N, w.G, w.group_size, p.cps, p.chunks, p.splits, w.err, ga);
    if (e == cudaSuccess && p.splits > 1)
        e = launch_splitk_reduce<BF16>(ws_part, y, M, w.N, p.splits, p.num_sms, s, ga);
    return e;
}

template <bool BF16>
cudaError_t launch_tc_bn(const PackedWeight& w, const TcPlan& p, const CUtensorMap* qw_map, const CUtensorMap& x_map,
                         int M, void* y, float* ws_part, cudaStream_t s, const GatherArgs& ga) {
    switch (p.bn) {
        case 16: return launch_tc_t<16, 1, BF16>(w, p, qw_map, x_map, M, y, ws_part, s, ga);
        case 32: return launch_tc_t<32, 1, BF16>(w, p, qw_map, x_map, M, y, ws_part, s, ga);
        case 64: return launch_tc_t<64, 1, BF16>(w, p, qw_map, x_map, M, y, ws_part, s, ga);
        case 128: return launch_tc_t<128, 1, BF16>(w, p, qw_map, x_map, M, y, ws_part, s, ga);
        case 256:
            if (p.pair)
                return p.nt == 2 ? launch_tc_t<256, 2, BF16, true>(w, p, qw_map, x_map, M, y, ws_part, s, ga)
                                 : launch_tc_t<256, 1, BF16, true>(w, p, qw_map, x_map, M, y, ws_part, s, ga);
            return p.nt == 2 ? launch_tc_t<256, 2, BF16>(w, p, qw_map, x_map, M, y, ws_part, s, ga)
                             : launch_tc_t<256, 1, BF16>(w, p, qw_map, x_map, M, y, ws_part, s, ga);
        default: return cudaErrorInvalidValue;
    }
}


template <int BN, int NT, bool BF16>
cudaError_t launch_tc_t_t(const PackedWeight& w, const TcPlan& p, const CUtensorMap* qwt_map,
                          const CUtensorMap& dy_map, int M, void* dx, float* ws_part, cudaStream_t s) {
    using C = FwdCfg<BN, NT>;
    auto kern = tc_gemm_kernel<BN, NT, BF16, true>;
    static const cudaError_t attr_err =
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmemBytes);
    if (attr_err != cudaSuccess) return attr_err;
    const int k_tiles = (w.K + kTileN - 1) / kTileN;
    const int m_tiles = (M + BN - 1) / BN;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(k_tiles, (m_tiles + NT - 1) / NT, p.splits);
    cfg.blockDim = dim3(kFwdThreads, 1, 1);
    cfg.dynamicSmemBytes = C::kSmemBytes;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e = cudaLaunchKernelEx(&cfg, kern, *qwt_map, dy_map, w.kernel_qzeros(), w.scales, static_cast<uint16_t*>(dx),
                                       ws_part, M, w.K, w.N, w.G, w.group_size, p.cps, p.chunks, p.splits, w.err,
                                       GatherArgs{});
    if (e == cudaSuccess && p.splits > 1)
        e = launch_splitk_reduce<BF16>(ws_part, dx, M, w.K, p.splits, p.num_sms, s, GatherArgs{});
    return e;
}

template <bool BF16>
cudaError_t launch_tc_t_bn(const PackedWeight& w, const TcPlan& p, const CUtensorMap* qwt_map,
                           const CUtensorMap& dy_map, int M, void* dx, float* ws_part, cudaStream_t s) {
    switch (p.bn) {
        case 16: return launch_tc_t_t<16, 1, BF16>(w, p, qwt_map, dy_map, M, dx, ws_part, s);
        case 32: return launch_tc_t_t<32, 1, BF16>(w, p, qwt_map, dy_map, M, dx, ws_part, s);
        case 64: return launch_tc_t_t<64, 1, BF16>(w, p, qwt_map, dy_map, M, dx, ws_part, s);
        case 128: return launch_tc_t_t<128, 1, BF16>(w, p, qwt_map, dy_map, M, dx, ws_part, s);
        case 256:
            return p.nt == 2 ? launch_tc_t_t<256, 2, BF16>(w, p, qwt_map, dy_map, M, dx, ws_part, s)
                             : launch_tc_t_t<256, 1, BF16>(w, p, qwt_map, dy_map, M, dx, ws_part, s);
        default: return cudaErrorInvalidValue;
    }
}

template <int BN, int NT>
int ctas_per_sm_t() {  // the forward GEMM's residency (one CTA per SM at every tile width)
    const int by_smem = (228 * 1024) / (FwdCfg<BN, NT>::kSmemBytes + 1024);
    const int by_tmem = 512 / FwdCfg<BN, NT>::kTmemCols;
    return std::max(1, std::min(by_smem, by_tmem));
}

int ctas_per_sm(int bn, int nt) {
    switch (bn) {
        case 16: return ctas_per_sm_t<16, 1>();
        case 32: return ctas_per_sm_t<32, 1>();
        case 64: return ctas_per_sm_t<64, 1>();
        case 128: return ctas_per_sm_t<128, 1>();
        default: return nt == 2 ? ctas_per_sm_t<256, 2>() : ctas_per_sm_t<256, 1>();
    }
}

}  // namespace

TcPlan plan_tc(const PackedWeight& w, int M, int num_sms) {
    TcPlan p;
    p.num_sms = num_sms;
    p.chunks = (w.K + kChunkK - 1) / kChunkK;
    const int n_tiles = (w.N + kTileN - 1) / kTileN;
    static const int env_nt = [] {
        const char* v = std::getenv("W4A16_TC_NT");  // tuning override (1 or 2)
        return v ? std::atoi(v) : 0;
    }();
    static const int env_cps = [] {
        const char* v = std::getenv("W4A16_TC_CPS");  // tuning override
        return v ? std::atoi(v) : 0;
    }();
    // Candidates: token tile BN (and for M > 128, one or two 256-token tiles per CTA),
    // each with a K split. Estimated time: waves x chunks per CTA x the per-chunk cost
    // measured on B200 (1.06 us for two 256-token tiles and 0.75 for one, at M = 2048;
    // 0.88 for 128 tokens at M = 128; 0.89 for 16 at M = 16), plus the split-K partial
    // round trip (fp32 partials written, then read and summed by tc_splitk_reduce_kernel).
    // The natural-orientation kernel (w4a16_gemm_ns.cu: 128 tokens x 256 weight columns per
    // MMA) for 9 <= M <= 256: 0.81 us per chunk of a CTA with one 128-token tile, 1.0 with
    // two (B200, 70B and 7B projections).
    static const int env_ns = [] {
        const char* v = std::getenv("W4A16_TC_NS");  // tuning override: 0 never, 1 always (9..256)
        return v ? std::atoi(v) : -1;
    }();
    struct Cand {
        int bn, nt;
        double us_per_chunk;  // one 64-wide K chunk of one CTA (B200)
        bool ns;
    };
    Cand cands[3];
    int nc = 0;
    const int bn = M <= 16 ? 16 : M <= 32 ? 32 : M <= 64 ? 64 : M <= 128 ? 128 : 256;
    if (env_ns != 1 || M <= 8 || M > 256) {
        if (bn == 256) {
            if ((M + 255) / 256 >= 2) cands[nc++] = {256, 2, 1.06, false};
            cands[nc++] = {256, 1, 0.75, false};
            if (env_nt == 1 || env_nt == 2) {
                nc = 1;
                cands[0] = env_nt == 2 && (M + 255) / 256 >= 2 ? Cand{256, 2, 1.06, false} : Cand{256, 1, 0.75, false};
            }
        } else {
            cands[nc++] = {bn, 1, bn == 128 ? 0.88 : 0.89, false};
        }
    }
    if (env_ns != 0 && M > 8 && M <= 256) cands[nc++] = {128, M > 128 ? 2 : 1, M > 128 ? 1.0 : 0.81, true};
    double best = 0.0;
    for (int ci = 0; ci < nc; ++ci) {
        const Cand& cd = cands[ci];
        const int tiles = cd.ns ? ((w.N + 255) / 256) * ((M + 128 * cd.nt - 1) / (128 * cd.nt))
                                : n_tiles * (((M + cd.bn - 1) / cd.bn + cd.nt - 1) / cd.nt);
        const int slots = cd.ns ? num_sms : num_sms * ctas_per_sm(cd.bn, cd.nt);
        // split K only while the tiles leave at least a quarter of one wave idle
        int max_splits = 1;
        if (4 * tiles <= 3 * slots) max_splits = std::min(16, std::max(1, p.chunks / 4));
        for (int sp = 1; sp <= max_splits; ++sp) {
            const int cps = (p.chunks + sp - 1) / sp;
            const int splits = (p.chunks + cps - 1) / cps;
            const long long ctas = static_cast<long long>(tiles) * splits;
            const long long waves = (ctas + slots - 1) / slots;
            double us = static_cast<double>(waves) * cps * cd.us_per_chunk;
            if (splits > 1)  // partials out and back at ~5 TB/s, plus a launch
                us += (static_cast<double>(splits) * M * w.N * 8.0 + 2.0 * M * w.N) / 5.0e6 + 2.0;
            if (best == 0.0 || us < best * 0.97) {  // a split must win clearly
                best = us;
                p.bn = cd.bn;
                p.nt = cd.nt;
                p.cps = cps;
                p.ns = cd.ns;
            }
        }
    }
    static const int env_pair = [] {
        const char* v = std::getenv("W4A16_TC_PAIR");
        return v ? std::atoi(v) : 0;
    }();
    p.pair = !p.ns && p.bn == 256 && n_tiles >= 2 && env_pair == 1;
    if (env_cps > 0) p.cps = std::min(p.chunks, env_cps);
    p.splits = (p.chunks + p.cps - 1) / p.cps;  // no empty split
    if (w.N % 8 != 0) {  // the split-K reduction stores 8 outputs at a time
        p.cps = p.chunks;
        p.splits = 1;
    }
    return p;
}

size_t tc_workspace_bytes(const PackedWeight& w, const TcPlan& p, int M) {
    if (p.splits <= 1) return 0;
    return static_cast<size_t>(p.splits) * M * w.N * sizeof(float);
}

cudaError_t launch_tc(const PackedWeight& w, const TcPlan& p, const CUtensorMap* qw_map, const void* x, int M,
                      void* y, DType dt, void* ws, size_t ws_bytes, cudaStream_t s, const GatherArgs* gather) {
    if (M <= 0) return cudaSuccess;
    if (p.splits > 1 && (ws_bytes < tc_workspace_bytes(w, p, M) || w.N % 8 != 0)) return cudaErrorInvalidValue;
    CUtensorMap x_map;
    const CUtensorMapDataType xdt = dt == kBF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    // a CTA pair loads half of each token tile per CTA; the natural orientation 128 tokens
    const uint32_t box_rows = p.ns ? 128u : static_cast<uint32_t>(p.pair ? p.bn / 2 : p.bn);
    if (encode_tmap_2d(&x_map, xdt, x, static_cast<uint64_t>(w.K), static_cast<uint64_t>(M),
                       static_cast<uint64_t>(w.K) * 2, kChunkK, box_rows, CU_TENSOR_MAP_SWIZZLE_128B) != CUDA_SUCCESS)
        return cudaErrorInvalidValue;
    float* ws_part = static_cast<float*>(ws);
    GatherArgs ga = {};
    if (gather) ga = *gather;
    if (p.ns) {
        cudaError_t e = launch_tc_ns(w, p, qw_map, x_map, M, y, dt, ws_part, s, ga);
        if (e == cudaSuccess && p.splits > 1)
            e = dt == kBF16 ? launch_splitk_reduce<true>(ws_part, y, M, w.N, p.splits, p.num_sms, s, ga)
                            : launch_splitk_reduce<false>(ws_part, y, M, w.N, p.splits, p.num_sms, s, ga);
        return e;
    }
    if (dt == kBF16) return launch_tc_bn<true>(w, p, qw_map, x_map, M, y, ws_part, s, ga);
    return launch_tc_bn<false>(w, p, qw_map, x_map, M, y, ws_part, s, ga);
}

// The transposed product is planned as a forward GEMM whose reduction runs over the
// weight's N columns and whose output columns are its K rows.
TcPlan plan_tc_t(const PackedWeight& w, int M, int num_sms) {
    PackedWeight t = w;
    t.K = w.N;
    t.N = w.K;
    return plan_tc(t, M, num_sms);
}

size_t tc_t_workspace_bytes(const PackedWeight& w, const TcPlan& p, int M) {
    if (p.splits <= 1) return 0;
    return static_cast<size_t>(p.splits) * M * w.K * sizeof(float);
}

cudaError_t launch_tc_t(const PackedWeight& w, const TcPlan& p, const CUtensorMap* qwt_map, const void* dy, int M,
                        void* dx, DType dt, void* ws, size_t ws_bytes, cudaStream_t s) {
    if (M <= 0) return cudaSuccess;
    if (w.group_size < 8 || (p.splits > 1 && ws_bytes < tc_t_workspace_bytes(w, p, M))) return cudaErrorInvalidValue;
    CUtensorMap dy_map;
    const CUtensorMapDataType ddt = dt == kBF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    if (encode_tmap_2d(&dy_map, ddt, dy, static_cast<uint64_t>(w.N), static_cast<uint64_t>(M),
                       static_cast<uint64_t>(w.N) * 2, 64, static_cast<uint32_t>(p.bn),
                       CU_TENSOR_MAP_SWIZZLE_128B) != CUDA_SUCCESS)
        return cudaErrorInvalidValue;
    float* ws_part = static_cast<float*>(ws);
    if (dt == kBF16) return launch_tc_t_bn<true>(w, p, qwt_map, dy_map, M, dx, ws_part, s);
    return launch_tc_t_bn<false>(w, p, qwt_map, dy_map, M, dx, ws_part, s);
}

}  // namespace w4a16
