// Internal declarations shared by the W4A16 translation units (not part of the C ABI).
#pragma once
#include <cstddef>
#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

namespace w4a16 {

enum DType : int { kFP16 = 0, kBF16 = 1 };

// Packed GPTQ weight as the kernels see it. Pointers are device pointers.
// K is the row count the kernels see. Without act-order it is the caller's K_in. With
// act-order the rows are sorted by group into a private copy; when the groups differ in
// size every group is padded to the same length (a multiple of 32 rows) with zero rows
// whose X is 0, so K = G * group_size >= K_in and group(row) = row / group_size always.
struct PackedWeight {
    int K = 0, N = 0, G = 0;
    int K_in = 0;            // the caller's in_features (columns of X, rows of its qweight)
    int group_size = 0;      // K / G
    bool act_order = false;  // rows sorted by group into a private copy: group(row) = row / group_size
    const int32_t* qweight = nullptr;     // [K/8, N] in kernel row order (sorted when act_order)
    const int32_t* qweight_orig = nullptr;  // caller's qweight, original row order [K_in/8, N]
    const int32_t* qzeros = nullptr;      // [G, N/8]
    const uint16_t* scales = nullptr;     // [G, N] fp16 bits
    const int32_t* g_idx = nullptr;       // [K_in] original group table (act_order) or nullptr
    const int32_t* perm = nullptr;        // [K] kernel row -> original row, -1 on pad rows (act_order)
    const int32_t* inv_perm = nullptr;    // [K_in] original row -> kernel row (act_order)
    int* err = nullptr;                   // device error word (bounded waits)
    // every zero nibble is 7 (z = 8, GPTQ's symmetric quantization, the only kind Marlin
    // takes): the kernels get a null qzeros and use the constant instead of loading zeros
    bool symmetric = false;
    const int32_t* kernel_qzeros() const { return symmetric ? nullptr : qzeros; }
};
constexpr uint32_t kSymmetricZeroWord = 0x77777777u;

// ---------------- launchers (return cudaError_t of the launch) ----------------
cudaError_t launch_dequant(const PackedWeight& w, void* out, DType dt, cudaStream_t s);
cudaError_t launch_sort_rows(const int32_t* qweight, int32_t* sorted, const int32_t* perm, int K, int N,
                             cudaStream_t s);
// out[m, j] = map[j] >= 0 ? in[m, map[j]] : 0 for j < out_cols (a multiple of 8)
cudaError_t launch_remap_cols(const void* in, int in_ld, void* out, int out_ld, const int32_t* map, int M,
                              int out_cols, cudaStream_t s);

// All-gather fused into a column-sharded GEMV (w4a16_gemm_gather): the GEMV stores
// every output element into each rank's full Y (peer memory mapped over NVLink); a
// one-warp kernel after it raises this rank's epoch flag in every rank's flags and
// waits (bounded) until every rank's flag has reached the same epoch.
constexpr int kMaxGatherRanks = 8;
struct GatherArgs {
    uint16_t* y[kMaxGatherRanks];          // full Y [M, ld] of each rank, in this process
    uint32_t* flags[kMaxGatherRanks];      // flags [world] of each rank, in this process
    uint32_t* my_flags;                    // this rank's flags (written by every rank)
    uint32_t* ctr;                         // this rank's [unused, epoch] (local)
    int world, rank, ld, col0;
};

struct GemvPlan {
    int mt = 1;      // rows of X per pass (1, 2, 4, 8)
    int bn = 128;    // columns per CTA
    int splits = 1;  // CTAs along K in one cluster (1..8)
    int kpw = 0;     // packed rows per warp (a whole number of load batches)
    bool wide = false;  // CUDA-core GEMV, M = 1: 3 CTAs per SM of 4-row batches
};
// One launch of the CUDA-core GEMV over up to kMaxSegs weights that read the same X
// (same K and group size): segment i owns column tiles [tile0[i], tile0[i + 1]).
constexpr int kMaxSegs = 3;
struct GemvSegs {
    const int32_t* qweight[kMaxSegs];
    const int32_t* qzeros[kMaxSegs];
    const uint16_t* scales[kMaxSegs];
    uint16_t* y[kMaxSegs];
    int N[kMaxSegs];
    int tile0[kMaxSegs + 1];
    int count;
};
// Transform applied to X while the GEMV stages it (fp16, M <= 2):
//   kProRmsNorm: X = fp16(x * norm_w * rsqrt(mean(x^2) + eps)); `out` (when set) gets it;
//   kProSiluMul: X = fp16(silu(x) * up).
enum : int { kProNone = 0, kProRmsNorm = 1, kProSiluMul = 2 };
struct GemvPrologue {
    int mode;
    const uint16_t* norm_w;  // [K]
    float eps;
    const uint16_t* up;      // [M, K]
    uint16_t* out;           // [M, K] or nullptr
};
bool gemv_supported(const PackedWeight& w);  // whole packed rows per group, N % 4 == 0
GemvPlan plan_gemv(const PackedWeight& w, int M, int num_sms);
// x in kernel row order (gathered through perm for act-order), M <= p.mt
cudaError_t launch_gemv(const PackedWeight& w, const GemvPlan& p, const void* x, int M, void* y, DType dt,
                        cudaStream_t s, const GatherArgs* gather = nullptr);
// One launch over `count` weights without act-order, Y_i = prologue(X) * W_i.
cudaError_t launch_gemv_group(const PackedWeight* const* ws, void* const* ys, int count, const void* x, int M,
                              DType dt, const GemvPrologue& pro, int num_sms, cudaStream_t s);
// Standalone RMSNorm (fp16, any M) and silu(gate) * up (fp16), same arithmetic as the
// GEMV prologues.
cudaError_t launch_rms_norm(const void* x, const void* w, float eps, int M, int K, void* y, cudaStream_t s);
cudaError_t launch_silu_mul(const void* gate, const void* up, int M, int N, void* out, cudaStream_t s);

// GEMV on the handle's repacked weight (mma.sync m16n8k16, M <= 16 per pass). Its
// GemvPlan: bn = columns per CTA (64, 128 or 256: 1, 2 or 4 warp stripes), kpw = k blocks
// of 16 per warp, splits = CTAs along K (one cluster), mt = rows of X per pass.
constexpr int kGemvMmaMaxTok = 16;
bool gemv_mma_supported(const PackedWeight& w);  // group size % 16 == 0
size_t repack_mma_words(const PackedWeight& w);  // int32 words of the repacked copy
cudaError_t launch_repack_mma(const PackedWeight& w, int32_t* dst, cudaStream_t s);
GemvPlan plan_gemv_mma(const PackedWeight& w, int M, int num_sms);
cudaError_t launch_gemv_mma(const PackedWeight& w, const int32_t* qw_mma, const GemvPlan& p, const void* x, int M,
                            void* y, DType dt, cudaStream_t s, const GatherArgs* gather = nullptr);

struct TcPlan {
    int bn = 128;        // tokens per tile (16, 32, 64, 128, 256)
    int splits = 1;      // CTAs along K (deterministic reduction through workspace)
    int cps = 0;         // 64-wide K chunks per split
    int chunks = 0;      // 64-wide K chunks
    int nt = 1;          // token tiles per CTA (2: two BN = 256 tiles share each dequantized weight tile)
    int num_sms = 148;   // SMs (grid of the split-K reduction)
    bool pair = false;   // forward, BN = 256: CTA pairs (cta_group::2), each CTA loading half of the X tile
    bool ns = false;     // forward, M <= 256: natural orientation (128 tokens x 256 weight columns per MMA)
};
TcPlan plan_tc(const PackedWeight& w, int M, int num_sms);
// The natural-orientation kernel (w4a16_gemm_ns.cu); x_map boxes [64 k x 128 tokens].
cudaError_t launch_tc_ns(const PackedWeight& w, const TcPlan& p, const CUtensorMap* qw_map, const CUtensorMap& x_map,
                         int M, void* y, DType dt, float* ws_part, cudaStream_t s, const GatherArgs& ga);
size_t tc_workspace_bytes(const PackedWeight& w, const TcPlan& p, int M);
// gather: store Y into every rank's full output instead of y (ld, col0 multiples of 8)
cudaError_t launch_tc(const PackedWeight& w, const TcPlan& p, const CUtensorMap* qw_map, const void* x, int M,
                      void* y, DType dt, void* ws, size_t ws_bytes, cudaStream_t s,
                      const GatherArgs* gather = nullptr);

// Transposed GEMM dX[M, K] = dY[M, N] * W^T (input gradient). qwt_map: qweight in
// kernel row order, box [64 columns x 16 packed rows]. dX is written in kernel row order
// (the caller remaps act-order rows); the split-K partials are [splits, M, K] fp32.
TcPlan plan_tc_t(const PackedWeight& w, int M, int num_sms);
size_t tc_t_workspace_bytes(const PackedWeight& w, const TcPlan& p, int M);
cudaError_t launch_tc_t(const PackedWeight& w, const TcPlan& p, const CUtensorMap* qwt_map, const void* dy, int M,
                        void* dx, DType dt, void* ws, size_t ws_bytes, cudaStream_t s);

// cuTensorMapEncodeTiled through the runtime's driver entry point (no -lcuda).
CUresult encode_tmap_2d(CUtensorMap* map, CUtensorMapDataType dtype, const void* base, uint64_t inner,
                        uint64_t outer, uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer,
                        CUtensorMapSwizzle swizzle);
CUresult encode_tmap_3d(CUtensorMap* map, CUtensorMapDataType dtype, const void* base, const uint64_t dims[3],
                        const uint64_t strides_bytes[2], const uint32_t box[3], CUtensorMapSwizzle swizzle);

}  // namespace w4a16
