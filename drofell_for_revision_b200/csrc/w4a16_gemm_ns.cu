// W4A16 GEMM on the sm_100a tensor cores for 17 <= M <= 256 tokens, in the natural
// orientation: the MMA's M side is 128 tokens of X, its N side 256 output columns of W.
//
// Why a second orientation: a tcgen05.mma of M = 128, K = 16 takes about the same time on
// B200 for every N from 32 to 256 (measured ~137 cycles per instruction). The swap-AB
// kernel (w4a16_gemm_sm100.cu) puts 128 weight columns on M and the tokens on N, so at
// M <= 128 tokens it runs the tensor pipe at N = M and streams 128 weight columns per
// instruction. Here the weight is the N = 256 operand: 256 columns per instruction, half
// the instructions per weight byte, whatever M is up to 128 (two 128-token tiles share each
// dequantized weight tile up to M = 256).
//
// Operands, both K-major with the 128-byte swizzle:
//   A = X tile [128 tokens x 64 k] by TMA (rows past M read as zeros);
//   B = W^T tile [256 n x 64 k] written by the dequant warps: the same fp16(s (q - z))
//       bits as the dequant kernel (bf16 of them for bf16 inputs), two 128-column halves
//       stacked (each exactly the swap-AB kernel's A tile).
// D[token, n] lands in TMEM lane = token, column = n; the epilogue turns each lane's 256
// columns into 16-byte row pieces of Y (or fp32 split-K partials, or every rank's Y for
// a column-sharded layer).
//
// Warp roles (608 threads), as in the swap-AB kernel:
//   warp 0      weight producer: two TMA loads of [8 packed rows x 128 n] and the chunk's
//               scale / zero rows of 256 columns into a WS-deep ring, never waiting for the
//               previous kernel;
//   warp 18     X producer (after griddepcontrol.wait) into an XS-deep ring;
//   warp 1      TMEM allocation and the MMA issuer (one thread);
//   warps 2-17  dequant, two groups of 8 warps on alternate chunks: thread t owns column t
//               of the 256 and the chunk's 8 packed words of it; then warps 2-9 drain TMEM.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <cstdlib>

#include "w4a16_gather.cuh"
#include "w4a16_internal.h"
#include "w4a16_ptx.cuh"
#include "w4a16_tc_common.cuh"

namespace w4a16 {
namespace {

constexpr int kChunkK = 64;
constexpr int kTileTok = 128;                       // tokens per MMA (M)
constexpr int kTileCols = 256;                      // weight columns per CTA (MMA N)
constexpr int kHalfCols = 128;                      // columns of one qweight TMA box
constexpr int kBTileBytes = kTileCols * kChunkK * 2;  // 32 KB dequantized W^T tile
constexpr int kXTileBytes = kTileTok * kChunkK * 2;   // 16 KB X tile
constexpr int kRawBytes = kTileCols * 8 * 4;          // 8 KB: 8 packed rows x 256 columns
constexpr int kMaxGroupsPerChunk = 8;                 // group size >= 8
constexpr int kScOff = kRawBytes;
constexpr int kZrOff = kScOff + kMaxGroupsPerChunk * kTileCols * 2;
constexpr int kWSlotBytes = kZrOff + kMaxGroupsPerChunk * kTileCols / 2;  // 13 KB
constexpr int kThreads = 19 * 32;
constexpr int kXWarp = 18;
constexpr uint32_t kSleepLimit = 1u << 18;  // x ~10 us sleeps: a few seconds

enum : int { kErrNsProducer = 5, kErrNsMma = 6, kErrNsDequant = 7, kErrNsEpilogue = 8 };

template <int NT>
struct NsCfg {
    // X comes from L2 (short round trip); the weights from HBM, held by a dequant group for
    // ~1.6 us per chunk: the weight ring is the deep one
    static constexpr int XS = 2;                // X chunks in flight (NT token tiles each)
    static constexpr int WS = NT == 2 ? 7 : 8;  // weight slots
    static constexpr int AS = 2;                // dequantized W^T tiles
    static constexpr int kXStage = NT * kXTileBytes;
    static constexpr int kWOff = XS * kXStage;
    static constexpr int kBOff = kWOff + WS * kWSlotBytes;
    static constexpr int kBarOff = kBOff + AS * kBTileBytes;
    static constexpr int kTmemCols = NT * kTileCols;
    static constexpr int kSmemBytes = kBarOff + 1024 /*barriers*/ + 1024 /*align*/;
    static_assert(kSmemBytes <= 227 * 1024, "shared memory budget");
};

template <int NT, bool BF16>
__global__ void __launch_bounds__(kThreads, 1)
    tc_ns_kernel(const __grid_constant__ CUtensorMap tm_qw, const __grid_constant__ CUtensorMap tm_x,
                 const int32_t* __restrict__ qzeros, const uint16_t* __restrict__ scales, uint16_t* __restrict__ y,
                 float* __restrict__ ws_part, int M, int K, int N, int G, int group_size, int chunks_per_split,
                 int num_chunks, int splits, int* __restrict__ err, const GatherArgs ga) {
    using C = NsCfg<NT>;
    constexpr int XS = C::XS, WS = C::WS, AS = C::AS;
    extern __shared__ __align__(1024) uint8_t smem_dyn[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_dyn) + 1023) & ~uintptr_t(1023));
    uint8_t* x_ring = smem;
    uint8_t* w_ring = smem + C::kWOff;
    uint8_t* b_ring = smem + C::kBOff;
    uint64_t* xfull = reinterpret_cast<uint64_t*>(smem + C::kBarOff);
    uint64_t* xempty = xfull + XS;
    uint64_t* wfull = xempty + XS;
    uint64_t* wempty = wfull + WS;
    uint64_t* bfull = wempty + WS;
    uint64_t* bempty = bfull + AS;
    uint64_t* accf = bempty + AS;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accf + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int n0 = blockIdx.x * kTileCols;
    const int m0 = blockIdx.y * kTileTok * NT;
    const int nt_live = min(NT, (M - m0 + kTileTok - 1) / kTileTok);
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
            ptx::mbar_init(&bfull[s], 8);
            ptx::mbar_init(&bempty[s], 1);
        }
        ptx::mbar_init(accf, 1);
        ptx::fence_mbar_init();
        ptx::prefetch_tmap(&tm_qw);
        ptx::prefetch_tmap(&tm_x);
    }
    if (warp == 1) {
        ptx::tmem_alloc(tmem_slot, C::kTmemCols);
        ptx::tmem_relinquish();
    }
    ptx::tc_fence_before();
    __syncthreads();
    ptx::tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    if (threadIdx.x == 0) ptx::grid_dep_launch_dependents();

    if (warp == 0) {
        // ------------------------------------------------ weight producer
        if (lane == 0) {
            int issued = 0;
            const int wcols = min(kTileCols, N - n0);
            const uint32_t sbytes = static_cast<uint32_t>(wcols) * 2;
            const uint32_t zbytes = qzeros ? static_cast<uint32_t>(wcols) / 2 : 0u;  // none when symmetric
            for (int i = 0; i < nc; ++i) {
                const int s = i % WS;
                if (i >= WS && !ptx::mbar_wait_sleep_bounded(&wempty[s], ((i / WS) - 1) & 1, kSleepLimit, err, kErrNsProducer))
                    break;
                uint8_t* slot = w_ring + s * kWSlotBytes;
                const int cg = c0 + i;
                const int g_first = (cg * kChunkK) / group_size;
                const int g_last = min(G - 1, (cg * kChunkK + kChunkK - 1) / group_size);
                const int cnt = g_last - g_first + 1;
                const int halves = wcols > kHalfCols ? 2 : 1;
                ptx::mbar_arrive_expect_tx(&wfull[s], halves * (kRawBytes / 2) + cnt * (sbytes + zbytes));
                for (int hh = 0; hh < halves; ++hh)
                    ptx::tma_load_2d(slot + hh * (kRawBytes / 2), &tm_qw, &wfull[s], n0 + hh * kHalfCols, cg * 8);
                for (int j = 0; j < cnt; ++j) {
                    const int g = g_first + j;
                    ptx::bulk_load(slot + kScOff + j * kTileCols * 2, scales + static_cast<size_t>(g) * N + n0, sbytes,
                                   &wfull[s]);
                    if (qzeros)
                        ptx::bulk_load(slot + kZrOff + j * (kTileCols / 2), qzeros + static_cast<size_t>(g) * (N >> 3) + (n0 >> 3),
                                       zbytes, &wfull[s]);
                }
                ++issued;
            }
            for (int i = max(0, issued - WS); i < issued; ++i)
                ptx::mbar_wait_sleep_bounded(&wfull[i % WS], (i / WS) & 1, kSleepLimit, err, kErrNsProducer);
        }
    } else if (warp == kXWarp) {
        // ------------------------------------------------ X producer
        if (lane == 0) {
            ptx::grid_dep_wait();  // X (and Y) belong to the previous kernel in the stream
            int issued = 0;
            for (int i = 0; i < nc; ++i) {
                const int s = i % XS;
                if (i >= XS && !ptx::mbar_wait_sleep_bounded(&xempty[s], ((i / XS) - 1) & 1, kSleepLimit, err, kErrNsProducer))
                    break;
                ptx::mbar_arrive_expect_tx(&xfull[s], nt_live * kXTileBytes);
                for (int tt = 0; tt < nt_live; ++tt)
                    ptx::tma_load_2d(x_ring + s * C::kXStage + tt * kXTileBytes, &tm_x, &xfull[s], (c0 + i) * kChunkK,
                                     m0 + tt * kTileTok);
                ++issued;
            }
            for (int i = max(0, issued - XS); i < issued; ++i)
                ptx::mbar_wait_sleep_bounded(&xfull[i % XS], (i / XS) & 1, kSleepLimit, err, kErrNsProducer);
        }
    } else if (warp == 1) {
        // ------------------------------------------------ MMA issuer
        if (lane == 0) {
            constexpr uint32_t idesc = ptx::umma_idesc_f16(kTileTok, kTileCols, BF16);
            for (int i = 0; i < nc; ++i) {
                const int a = i % AS;
                const int x = i % XS;
                if (!ptx::mbar_wait_sleep_bounded(&bfull[a], (i / AS) & 1, kSleepLimit, err, kErrNsMma)) break;
                if (!ptx::mbar_wait_sleep_bounded(&xfull[x], (i / XS) & 1, kSleepLimit, err, kErrNsMma)) break;
                ptx::tc_fence_after();
                const uint32_t b_base = ptx::smem_u32(b_ring + a * kBTileBytes);
                const uint32_t x_base = ptx::smem_u32(x_ring + x * C::kXStage);
#pragma unroll
                for (int kk = 0; kk < kChunkK / 16; ++kk) {
                    const uint64_t db = ptx::umma_desc_sw128(b_base + kk * 32);
#pragma unroll
                    for (int tt = 0; tt < NT; ++tt) {
                        if (tt < nt_live) {
                            const uint64_t da = ptx::umma_desc_sw128(x_base + tt * kXTileBytes + kk * 32);
                            ptx::umma_f16(tmem + static_cast<uint32_t>(tt * kTileCols), da, db, idesc,
                                          (i > 0 || kk > 0) ? 1u : 0u);
                        }
                    }
                }
                ptx::umma_commit(&bempty[a]);
                ptx::umma_commit(&xempty[x]);
            }
            ptx::umma_commit(accf);
        }
    } else {
        // ------------------------------------------------ dequant warps (two groups)
        const int dq = threadIdx.x - 64;  // 0..511
        const int grp = dq >> 8;          // this group takes chunks i with i % 2 == grp
        const int t = dq & 255;           // column within the 256
        const int n = n0 + t;
        const bool col_ok = n < N;
        const int zsh = (t & 7) * 4;
        const int raw_col = (t >> 7) * (kRawBytes / 8) + (t & (kHalfCols - 1));  // word offset of row 0
        bool ok = true;
        // the chunk's 8 packed rows share one group when the group holds a multiple of 64 k
        const bool whole = (wpg & 7) == 0;
        for (int i = grp; i < nc; i += 2) {
            const int s = i % WS;
            const int a = i % AS;
            if (!ptx::mbar_wait_sleep_bounded(&wfull[s], (i / WS) & 1, kSleepLimit, err, kErrNsDequant)) {
                ok = false;
                break;
            }
            const uint8_t* slot = w_ring + s * kWSlotBytes;
            const uint32_t* raw = reinterpret_cast<const uint32_t*>(slot);
            const uint16_t* sc = reinterpret_cast<const uint16_t*>(slot + kScOff);
            const uint32_t* zr = reinterpret_cast<const uint32_t*>(slot + kZrOff);
            const int cg = c0 + i;
            const int kw0 = cg * 8;
            uint32_t wv[8];
#pragma unroll
            for (int r = 0; r < 8; ++r) wv[r] = (kw0 + r < KW && col_ok) ? raw[r * kHalfCols + raw_col] : 0u;
            const int g_first = (cg * kChunkK) / group_size;
            auto fetch = [&](int gl, __half2& s2, __half2& zoff) {
                const uint32_t zw = qzeros ? zr[gl * (kTileCols / 8) + (t >> 3)] : kSymmetricZeroWord;
                const uint32_t zp = ((zw >> zsh) & 15u) + 1u;
                // (-(1024 + z), -(64 + z)) as exact fp16 bits: 1024 and 64 carry unit and 1/16 steps
                const uint32_t zb = (0xE400u + zp) | ((0xD400u + (zp << 4)) << 16);
                zoff = *reinterpret_cast<const __half2*>(&zb);
                s2 = __half2half2(__ushort_as_half(sc[gl * kTileCols + t]));
            };
            __half2 s2, zoff;
            fetch(kw0 / wpg - g_first, s2, zoff);
            if (whole) {  // everything this thread needs from the slot is in registers: free it now
                __syncwarp();
                if (lane == 0) ptx::mbar_arrive(&wempty[s]);
            }
            if (i >= AS && !ptx::mbar_wait_sleep_bounded(&bempty[a], ((i / AS) - 1) & 1, kSleepLimit, err, kErrNsDequant)) {
                ok = false;
                break;
            }
            const uint32_t b_row = ptx::smem_u32(b_ring + a * kBTileBytes) + t * 128;
            if (whole) {
#pragma unroll
                for (int r = 0; r < 8; ++r) {
                    const uint4 o = (kw0 + r < KW && col_ok) ? dequant_word<BF16>(wv[r], s2, zoff)
                                                             : make_uint4(0u, 0u, 0u, 0u);
                    ptx::st_shared_v4(b_row + ((r ^ (t & 7)) << 4), o);
                }
            } else {
                int gcur = kw0 / wpg;
                int left = (gcur + 1) * wpg - kw0;  // rows of the current group from kw0 on
#pragma unroll
                for (int r = 0; r < 8; ++r) {
                    if (r == left) {  // the next row starts a new group
                        ++gcur;
                        left += wpg;
                        fetch(gcur - g_first, s2, zoff);
                    }
                    uint4 o = make_uint4(0u, 0u, 0u, 0u);
                    if (kw0 + r < KW && col_ok) o = dequant_word<BF16>(wv[r], s2, zoff);
                    ptx::st_shared_v4(b_row + ((r ^ (t & 7)) << 4), o);
                }
            }
            ptx::fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
                ptx::mbar_arrive(&bfull[a]);
                if (!whole) ptx::mbar_arrive(&wempty[s]);  // the slot's words, scales and zeros have been read
            }
        }

        // ------------------------------------------------ epilogue (warps 2-9)
        if (ok && nc > 0) ok = ptx::mbar_wait_sleep_bounded(accf, 0, kSleepLimit, err, kErrNsEpilogue);
        ptx::tc_fence_after();
        ptx::grid_dep_wait();  // Y may still be read or written by the previous kernel
        if (warp < 10) {
            const int q = warp & 3;                 // TMEM lane quadrant: tokens q*32 .. q*32+31
            const int ch = (warp - 2) >> 2;         // columns ch*128 .. ch*128+127
            for (int tt = 0; tt < nt_live; ++tt) {
                const int m = m0 + tt * kTileTok + q * 32 + lane;
                const uint32_t trow = tmem + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(tt * kTileCols);
#pragma unroll 1
                for (int c = ch * 128; c < ch * 128 + 128; c += 8) {
                    uint32_t v[8];
                    ptx::tmem_ld_32x32b_x8(trow + c, v);
                    ptx::tmem_ld_wait();
                    const int nn = n0 + c;
                    if (!ok || nc == 0 || m >= M || nn >= N) continue;
                    if (splits == 1) {
                        uint32_t o[4];
#pragma unroll
                        for (int e = 0; e < 4; ++e)
                            o[e] = static_cast<uint32_t>(to_out<BF16>(__uint_as_float(v[2 * e]))) |
                                   (static_cast<uint32_t>(to_out<BF16>(__uint_as_float(v[2 * e + 1]))) << 16);
                        out_store16(ga, y, N, m, nn, make_uint4(o[0], o[1], o[2], o[3]));
                    } else {
                        float4* dst = reinterpret_cast<float4*>(ws_part + (static_cast<size_t>(z) * M + m) * N + nn);
                        dst[0] = make_float4(__uint_as_float(v[0]), __uint_as_float(v[1]), __uint_as_float(v[2]),
                                             __uint_as_float(v[3]));
                        dst[1] = make_float4(__uint_as_float(v[4]), __uint_as_float(v[5]), __uint_as_float(v[6]),
                                             __uint_as_float(v[7]));
                    }
                }
            }
        }
    }

    ptx::tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        ptx::tc_fence_after();
        ptx::tmem_dealloc(tmem, C::kTmemCols);
    }
}

template <int NT, bool BF16>
cudaError_t launch_ns_t(const PackedWeight& w, const TcPlan& p, const CUtensorMap* qw_map, const CUtensorMap& x_map,
                        int M, void* y, float* ws_part, cudaStream_t s, const GatherArgs& ga) {
    using C = NsCfg<NT>;
    auto kern = tc_ns_kernel<NT, BF16>;
    static const cudaError_t attr_err =
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmemBytes);
    if (attr_err != cudaSuccess) return attr_err;
    const int n_tiles = (w.N + kTileCols - 1) / kTileCols;
    const int m_tiles = (M + kTileTok * NT - 1) / (kTileTok * NT);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(n_tiles, m_tiles, p.splits);
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = C::kSmemBytes;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, *qw_map, x_map, w.kernel_qzeros(), w.scales, static_cast<uint16_t*>(y),
                              ws_part, M, w.K, w.N, w.G, w.group_size, p.cps, p.chunks, p.splits, w.err, ga);
}

}  // namespace

cudaError_t launch_tc_ns(const PackedWeight& w, const TcPlan& p, const CUtensorMap* qw_map, const CUtensorMap& x_map,
                         int M, void* y, DType dt, float* ws_part, cudaStream_t s, const GatherArgs& ga) {
    if (p.nt == 2)
        return dt == kBF16 ? launch_ns_t<2, true>(w, p, qw_map, x_map, M, y, ws_part, s, ga)
                           : launch_ns_t<2, false>(w, p, qw_map, x_map, M, y, ws_part, s, ga);
    return dt == kBF16 ? launch_ns_t<1, true>(w, p, qw_map, x_map, M, y, ws_part, s, ga)
                       : launch_ns_t<1, false>(w, p, qw_map, x_map, M, y, ws_part, s, ga);
}

}  // namespace w4a16
