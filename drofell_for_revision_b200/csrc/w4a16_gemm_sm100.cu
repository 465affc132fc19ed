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
// Warp roles (192 threads):
//   warp 0  TMA producer: packed qweight tile [8 words x 128 n] (4 KB) and the X
//           tile [BN x 64] (SW128) per 64-wide K chunk, into a STAGES-deep ring.
//   warp 1  TMEM allocation; one elected thread issues 4 x tcgen05.mma
//           (K = 16 each) per chunk and commits to the stage's "empty" barrier.
//   warps 2-5  dequant: thread t owns column n0 + t; each packed word (8 k of
//           one column) becomes one 16-byte swizzled chunk of the A tile, with
//           W = fp16(s * (q - z)) computed exactly (the same bits the dequant
//           kernel writes). Afterwards the same warps run the epilogue:
//           tcgen05.ld of their TMEM lane quadrant -> fp16/bf16 -> global, or
//           fp32 partials for split-K, reduced in split order by the last CTA of
//           the tile (deterministic).
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "w4a16_internal.h"
#include "w4a16_ptx.cuh"

namespace w4a16 {
namespace {

constexpr int kTcThreads = 192;
constexpr int kChunkK = 64;
constexpr int kTileN = 128;
constexpr int kATileBytes = kTileN * kChunkK * 2;  // 16 KB
constexpr int kRawTileBytes = kTileN * 8 * 4;      // 4 KB
constexpr uint32_t kWaitLimit = 1u << 26;

enum : int { kErrTimeoutProducer = 1, kErrTimeoutMma = 2, kErrTimeoutDequant = 3, kErrTimeoutEpilogue = 4 };

template <int BN>
struct TcLayout {
    static constexpr int kXTileBytes = BN * kChunkK * 2;
    static constexpr int kStageBytes = kATileBytes + kXTileBytes + kRawTileBytes;
    static constexpr int kTmemCols = BN < 32 ? 32 : BN;
    static_assert(kStageBytes % 1024 == 0, "stage must keep 1024-byte alignment for SW128 tiles");
};

__device__ __forceinline__ uint32_t h2_bits(__half2 v) { return *reinterpret_cast<uint32_t*>(&v); }
__device__ __forceinline__ __half2 bits_h2(uint32_t v) { return *reinterpret_cast<__half2*>(&v); }

// 8 dequantized weights of one packed word, natural k order, as 16 bytes.
template <bool BF16>
__device__ __forceinline__ uint4 dequant_word(uint32_t w, __half2 s2, __half2 zoff) {
    const __half2 mul = __halves2half2(__float2half_rn(1.0f), __float2half_rn(0.0625f));
    uint32_t o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        // byte j holds k = 2j (low nibble) and k = 2j + 1 (high nibble)
        const uint32_t b = __byte_perm(w, 0u, static_cast<uint32_t>(j | (j << 8)));
        const uint32_t p = (b & 0x00F0000Fu) | 0x64006400u;     // (1024 + q0, 1024 + 16 q1)
        const __half2 d = __hfma2(bits_h2(p), mul, zoff);         // (q0 - z, q1 - z), exact
        const __half2 v = __hmul2(d, s2);                         // one rounding: fp16(s (q - z))
        if constexpr (BF16) {
            const __nv_bfloat162 bv = __float22bfloat162_rn(__half22float2(v));
            o[j] = *reinterpret_cast<const uint32_t*>(&bv);
        } else {
            o[j] = h2_bits(v);
        }
    }
    return make_uint4(o[0], o[1], o[2], o[3]);
}

template <int BN, int STAGES, bool BF16, bool ACT>
__global__ void __launch_bounds__(kTcThreads, 1)
    tc_gemm_kernel(const __grid_constant__ CUtensorMap tm_qw, const __grid_constant__ CUtensorMap tm_x,
                   const int32_t* __restrict__ qzeros, const uint16_t* __restrict__ scales,
                   const int32_t* __restrict__ word_group, uint16_t* __restrict__ y, float* __restrict__ ws_part,
                   int* __restrict__ counters, int M, int K, int N, int group_size, int chunks_per_split,
                   int num_chunks, int splits, int* __restrict__ err) {
    using L = TcLayout<BN>;
    extern __shared__ __align__(1024) uint8_t smem_dyn[];
    // 1024-byte alignment for the swizzled tiles
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_dyn) + 1023) & ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * L::kStageBytes);
    uint64_t* afull = full + STAGES;
    uint64_t* empty = afull + STAGES;
    uint64_t* accf = empty + STAGES;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accf + 1);
    int* ticket_slot = reinterpret_cast<int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int n0 = blockIdx.x * kTileN;
    const int m0 = blockIdx.y * BN;
    const int z = blockIdx.z;
    const int c0 = z * chunks_per_split;
    const int c1 = min(num_chunks, c0 + chunks_per_split);
    const int nc = max(0, c1 - c0);
    const int KW = K >> 3;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            ptx::mbar_init(&full[s], 1);
            ptx::mbar_init(&afull[s], 4);
            ptx::mbar_init(&empty[s], 1);
        }
        ptx::mbar_init(accf, 1);
        ptx::fence_mbar_init();
        ptx::prefetch_tmap(&tm_qw);
        ptx::prefetch_tmap(&tm_x);
    }
    if (warp == 1) {
        ptx::tmem_alloc(tmem_slot, L::kTmemCols);
        ptx::tmem_relinquish();
    }
    ptx::tc_fence_before();
    __syncthreads();
    ptx::tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            int issued = 0;
            for (int i = 0; i < nc; ++i) {
                const int s = i % STAGES;
                if (i >= STAGES &&
                    !ptx::mbar_wait_bounded(&empty[s], ((i / STAGES) - 1) & 1, kWaitLimit, err, kErrTimeoutProducer))
                    break;
                uint8_t* st = smem + s * L::kStageBytes;
                ptx::mbar_arrive_expect_tx(&full[s], kRawTileBytes + L::kXTileBytes);
                ptx::tma_load_2d(st + kATileBytes + L::kXTileBytes, &tm_qw, &full[s], n0, (c0 + i) * 8);
                ptx::tma_load_2d(st + kATileBytes, &tm_x, &full[s], (c0 + i) * kChunkK, m0);
                ++issued;
            }
            // Drain: do not leave the CTA while a copy issued above may still land.
            for (int i = max(0, issued - STAGES); i < issued; ++i) {
                ptx::mbar_wait_bounded(&full[i % STAGES], (i / STAGES) & 1, kWaitLimit, err, kErrTimeoutProducer);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc = ptx::umma_idesc_f16(128, BN, BF16);
            for (int i = 0; i < nc; ++i) {
                const int s = i % STAGES;
                if (!ptx::mbar_wait_bounded(&afull[s], (i / STAGES) & 1, kWaitLimit, err, kErrTimeoutMma)) break;
                ptx::tc_fence_after();
                const uint32_t a_base = ptx::smem_u32(smem + s * L::kStageBytes);
                const uint32_t b_base = a_base + kATileBytes;
#pragma unroll
                for (int kk = 0; kk < kChunkK / 16; ++kk) {
                    const uint64_t da = ptx::umma_desc_sw128(a_base + kk * 32);
                    const uint64_t db = ptx::umma_desc_sw128(b_base + kk * 32);
                    ptx::umma_f16(tmem, da, db, idesc, (i > 0 || kk > 0) ? 1u : 0u);
                }
                ptx::umma_commit(&empty[s]);
            }
            ptx::umma_commit(accf);
        }
    } else {
        // ------------------------------------------------ dequant warps
        const int t = threadIdx.x - 64;  // 0..127
        const int n = n0 + t;
        const bool col_ok = n < N;
        int cur_g = -1;
        int g_end_kw = 0;
        __half2 s2 = __float2half2_rn(0.f);
        __half2 zoff = __float2half2_rn(0.f);
        const int wpg = group_size >> 3;  // words per group (group_size % 8 == 0)
        bool ok = true;
        for (int i = 0; i < nc; ++i) {
            const int s = i % STAGES;
            if (!ptx::mbar_wait_bounded(&full[s], (i / STAGES) & 1, kWaitLimit, err, kErrTimeoutDequant)) {
                ok = false;
                break;
            }
            uint8_t* st = smem + s * L::kStageBytes;
            const uint32_t* raw = reinterpret_cast<const uint32_t*>(st + kATileBytes + L::kXTileBytes);
            const uint32_t a_row = ptx::smem_u32(st) + t * 128;
#pragma unroll
            for (int r = 0; r < 8; ++r) {
                const int kw = (c0 + i) * 8 + r;
                uint4 o = make_uint4(0u, 0u, 0u, 0u);
                if (kw < KW && col_ok) {
                    int g;
                    if constexpr (ACT) {
                        g = __ldg(word_group + kw);
                    } else {
                        if (kw >= g_end_kw || cur_g < 0) {
                            g = kw / wpg;
                        } else {
                            g = cur_g;
                        }
                    }
                    if (g != cur_g) {
                        cur_g = g;
                        g_end_kw = (g + 1) * wpg;
                        const __half sv = __ushort_as_half(__ldg(scales + static_cast<size_t>(g) * N + n));
                        const uint32_t zw =
                            static_cast<uint32_t>(__ldg(qzeros + static_cast<size_t>(g) * (N >> 3) + (n >> 3)));
                        const float zf = static_cast<float>(((zw >> ((n & 7) * 4)) & 15u) + 1u);
                        s2 = __half2half2(sv);
                        zoff = __floats2half2_rn(-(1024.0f + zf), -(64.0f + zf));
                    }
                    o = dequant_word<BF16>(raw[r * kTileN + t], s2, zoff);
                }
                ptx::st_shared_v4(a_row + ((r ^ (t & 7)) << 4), o);
            }
            ptx::fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) ptx::mbar_arrive(&afull[s]);
        }

        // ------------------------------------------------ epilogue
        if (ok && nc > 0) ok = ptx::mbar_wait_bounded(accf, 0, kWaitLimit, err, kErrTimeoutEpilogue);
        ptx::tc_fence_after();
        const int q = warp & 3;  // TMEM lane quadrant this warp may access
        const int nl = q * 32 + lane;
        const int ncol = n0 + nl;
        const bool write_ok = ok && ncol < N;
#pragma unroll 1
        for (int c = 0; c < BN; c += 16) {
            uint32_t v[16];
            ptx::tmem_ld_32x32b_x16(tmem + (static_cast<uint32_t>(q * 32) << 16) + c, v);
            ptx::tmem_ld_wait();
            if (!write_ok) continue;
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                const int m = m0 + c + j;
                if (m < M) {
                    const float f = nc > 0 ? __uint_as_float(v[j]) : 0.f;
                    if (splits == 1) {
                        uint16_t b;
                        if constexpr (BF16) {
                            b = __bfloat16_as_ushort(__float2bfloat16_rn(f));
                        } else {
                            b = __half_as_ushort(__float2half_rn(f));
                        }
                        y[static_cast<size_t>(m) * N + ncol] = b;
                    } else {
                        ws_part[(static_cast<size_t>(z) * M + m) * N + ncol] = f;
                    }
                }
            }
        }
        if (splits > 1) {
            __threadfence();
            ptx::named_bar_sync(1, 128);
            const int tile_id = blockIdx.y * gridDim.x + blockIdx.x;
            if (t == 0) *ticket_slot = atomicAdd(&counters[tile_id], 1);
            ptx::named_bar_sync(1, 128);
            if (*ticket_slot == splits - 1) {
                __threadfence();
                if (ncol < N) {
                    for (int j = 0; j < BN; ++j) {
                        const int m = m0 + j;
                        if (m >= M) break;
                        float acc = 0.f;
                        for (int zz = 0; zz < splits; ++zz)
                            acc += __ldcg(ws_part + (static_cast<size_t>(zz) * M + m) * N + ncol);
                        uint16_t b;
                        if constexpr (BF16) {
                            b = __bfloat16_as_ushort(__float2bfloat16_rn(acc));
                        } else {
                            b = __half_as_ushort(__float2half_rn(acc));
                        }
                        y[static_cast<size_t>(m) * N + ncol] = b;
                    }
                }
                if (t == 0) counters[tile_id] = 0;  // self-reset for the next call
            }
        }
    }

    ptx::tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        ptx::tc_fence_after();
        ptx::tmem_dealloc(tmem, L::kTmemCols);
    }
}

template <int BN, int STAGES, bool BF16, bool ACT>
cudaError_t launch_tc_t(const PackedWeight& w, const TcPlan& p, const CUtensorMap* qw_map, const CUtensorMap& x_map,
                        int M, void* y, float* ws_part, int* counters, cudaStream_t s) {
    using L = TcLayout<BN>;
    const size_t smem = static_cast<size_t>(STAGES) * L::kStageBytes + 1024 /*barriers*/ + 1024 /*align*/;
    auto kern = tc_gemm_kernel<BN, STAGES, BF16, ACT>;
    // Once per instantiation (and so before any stream capture that reuses it).
    static const cudaError_t attr_err =
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (attr_err != cudaSuccess) return attr_err;
    const int n_tiles = (w.N + kTileN - 1) / kTileN;
    const int m_tiles = (M + BN - 1) / BN;
    const int cps = (p.chunks + p.splits - 1) / p.splits;
    dim3 grid(n_tiles, m_tiles, p.splits);
    kern<<<grid, kTcThreads, smem, s>>>(*qw_map, x_map, w.qzeros, w.scales, w.word_group, static_cast<uint16_t*>(y),
                                        ws_part, counters, M, w.K, w.N, w.group_size, cps, p.chunks, p.splits, w.err);
    return cudaGetLastError();
}

template <int BN, bool BF16, bool ACT>
cudaError_t launch_tc_stages(const PackedWeight& w, const TcPlan& p, const CUtensorMap* qw_map,
                             const CUtensorMap& x_map, int M, void* y, float* ws_part, int* counters,
                             cudaStream_t s) {
    // Largest ring that fits in 227 KB of shared memory.
    constexpr int kStage = TcLayout<BN>::kStageBytes;
    constexpr int kMax = (227 * 1024 - 2048) / kStage;
    constexpr int kStages = kMax > 8 ? 8 : kMax;
    static_assert(kStages >= 2, "pipeline needs at least two stages");
    return launch_tc_t<BN, kStages, BF16, ACT>(w, p, qw_map, x_map, M, y, ws_part, counters, s);
}

template <bool BF16, bool ACT>
cudaError_t launch_tc_bn(const PackedWeight& w, const TcPlan& p, const CUtensorMap* qw_map, const CUtensorMap& x_map,
                         int M, void* y, float* ws_part, int* counters, cudaStream_t s) {
    switch (p.bn) {
        case 16: return launch_tc_stages<16, BF16, ACT>(w, p, qw_map, x_map, M, y, ws_part, counters, s);
        case 32: return launch_tc_stages<32, BF16, ACT>(w, p, qw_map, x_map, M, y, ws_part, counters, s);
        case 64: return launch_tc_stages<64, BF16, ACT>(w, p, qw_map, x_map, M, y, ws_part, counters, s);
        case 128: return launch_tc_stages<128, BF16, ACT>(w, p, qw_map, x_map, M, y, ws_part, counters, s);
        case 256: return launch_tc_stages<256, BF16, ACT>(w, p, qw_map, x_map, M, y, ws_part, counters, s);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace

TcPlan plan_tc(const PackedWeight& w, int M, int num_sms) {
    TcPlan p;
    p.bn = M <= 16 ? 16 : M <= 32 ? 32 : M <= 64 ? 64 : M <= 128 ? 128 : 256;
    p.chunks = (w.K + kChunkK - 1) / kChunkK;
    const int n_tiles = (w.N + kTileN - 1) / kTileN;
    const int m_tiles = (M + p.bn - 1) / p.bn;
    const int tiles = n_tiles * m_tiles;
    int splits = 1;
    if (tiles < num_sms) {
        splits = (num_sms + tiles - 1) / tiles;
        const int max_splits = p.chunks / 4 > 1 ? p.chunks / 4 : 1;
        if (splits > max_splits) splits = max_splits;
        if (splits > 16) splits = 16;
    }
    const int cps = (p.chunks + splits - 1) / splits;
    p.splits = (p.chunks + cps - 1) / cps;  // no empty split
    return p;
}

size_t tc_workspace_bytes(const PackedWeight& w, const TcPlan& p, int M) {
    if (p.splits <= 1) return 0;
    return static_cast<size_t>(p.splits) * M * w.N * sizeof(float);
}

cudaError_t launch_tc(const PackedWeight& w, const TcPlan& p, const CUtensorMap* qw_map, const void* x, int M,
                      void* y, DType dt, void* ws, size_t ws_bytes, int* counters, int max_counters,
                      cudaStream_t s) {
    if (M <= 0) return cudaSuccess;
    const int n_tiles = (w.N + kTileN - 1) / kTileN;
    const int m_tiles = (M + p.bn - 1) / p.bn;
    if (p.splits > 1 && (ws_bytes < tc_workspace_bytes(w, p, M) || n_tiles * m_tiles > max_counters))
        return cudaErrorInvalidValue;
    CUtensorMap x_map;
    const CUtensorMapDataType xdt = dt == kBF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    if (encode_tmap_2d(&x_map, xdt, x, static_cast<uint64_t>(w.K), static_cast<uint64_t>(M),
                       static_cast<uint64_t>(w.K) * 2, kChunkK, static_cast<uint32_t>(p.bn),
                       CU_TENSOR_MAP_SWIZZLE_128B) != CUDA_SUCCESS)
        return cudaErrorInvalidValue;
    float* ws_part = static_cast<float*>(ws);
    if (dt == kBF16) {
        return w.act_order ? launch_tc_bn<true, true>(w, p, qw_map, x_map, M, y, ws_part, counters, s)
                           : launch_tc_bn<true, false>(w, p, qw_map, x_map, M, y, ws_part, counters, s);
    }
    return w.act_order ? launch_tc_bn<false, true>(w, p, qw_map, x_map, M, y, ws_part, counters, s)
                       : launch_tc_bn<false, false>(w, p, qw_map, x_map, M, y, ws_part, counters, s);
}

}  // namespace w4a16
