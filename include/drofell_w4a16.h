/*
 * drofell_w4a16.h - C ABI of the B200 (sm_100a) GPTQ W4A16 quantized-linear library.
 *
 * Plain pointers and sizes only. Every pointer argument named *_dev is a device
 * pointer on the handle's device; g_idx_host is a host pointer. `stream` is a
 * cudaStream_t passed as void* (NULL = legacy default stream). Every function
 * returns W4A16_OK or an error code; w4a16_last_error() gives the message of the
 * last failure on the calling thread.
 *
 * Packed layout (unchanged GPTQ layout of the reference,
 * After-Revision-DROFELL/operators/core/linear/real_quant.py:25-49):
 *   qweight int32 [K/8, N]  nibble i of qweight[r, n] is q[8r + i, n]
 *   qzeros  int32 [G, N/8]  nibble j of qzeros[g, c] is z[g, 8c + j] - 1
 *   scales  fp16  [G, N]
 *   g_idx   int32 [K]       (act-order only)
 *   W[k, n] = fp16(scales[g, n] * (q[k, n] - z[g, n])), g = g_idx[k] or k / (K / G)
 * The library never writes to qweight / qzeros / scales (the reference permutes
 * and shuffles qweight in place, q4_matrix.cu:67-75,179).
 */
#ifndef DROFELL_W4A16_H_
#define DROFELL_W4A16_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define W4A16_API __attribute__((visibility("default")))
#else
#define W4A16_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define W4A16_OK 0
#define W4A16_ERR_INVALID 1      /* bad argument: shape, alignment, null pointer */
#define W4A16_ERR_CUDA 2         /* a CUDA runtime / launch error */
#define W4A16_ERR_UNSUPPORTED 3  /* valid input this kernel family does not handle */
#define W4A16_ERR_WORKSPACE 4    /* workspace too small (see w4a16_workspace_size) */

#define W4A16_DTYPE_FP16 0
#define W4A16_DTYPE_BF16 1

#define W4A16_PATH_AUTO 0     /* the GEMV family for M <= 16 (one pass of the mma.sync GEMV; 9..16 rows of a
                                 very long K that would need two passes go to the tcgen05 GEMM), else the
                                 tcgen05 exact-W GEMM: natural orientation or swap-AB, chosen by cost */
#define W4A16_PATH_GEMV 1     /* decode GEMV (fp16 / bf16): CUDA cores for M <= 2 (passes of <= 8 rows),
                                 mma.sync on the handle's repacked weight (group size % 16 == 0) above
                                 (passes of <= 16 rows), and at every M for K >= 8192 and N >= 8192 or
                                 K > 4096 and N >= 16384 */
#define W4A16_PATH_TC 2       /* tcgen05 exact-W dequant-in-smem GEMM, any M (same as PATH_TC_EXACT) */
#define W4A16_PATH_TC_EXACT 3 /* tcgen05 exact-W dequant-in-smem GEMM, any M */

typedef struct w4a16_matrix w4a16_matrix;

/* Build a handle over a packed GPTQ weight. Replaces make_q4
 * (After-Revision-DROFELL/cuda_extends/exllama/entry.cpp:18-62, Q4Matrix ctor
 * q4_matrix.cu:33-76). The handle keeps non-owning pointers to qweight, qzeros and
 * scales (the caller keeps them alive and unchanged) and owns the act-order
 * buffers it allocates. qweight and scales must be 16-byte aligned; qzeros 4-byte
 * aligned (a qzeros that is not 16-byte aligned is copied once into the handle). g_idx_host != NULL selects act-order (use_act = true in the
 * reference); its groups are sorted into a private row order (any table: groups of
 * unequal sizes are padded to the longest with zero rows). When the group size
 * is a multiple of 16 the handle also keeps its own copy of the weight repacked for
 * the decode GEMV (the same size as qweight; environment W4A16_NO_REPACK=1 at
 * creation skips it). K % 32 == 0,
 * N % 32 == 0, K % groups == 0 and (K / groups) % 8 == 0. Synchronises `stream`. */
W4A16_API int w4a16_create(const int32_t* qweight_dev, const int32_t* qzeros_dev, const uint16_t* scales_dev,
                 const int32_t* g_idx_host, int K, int N, int groups, int device, void* stream,
                 w4a16_matrix** out);

/* w4a16_create with creation flags. W4A16_CREATE_NO_REPACK: keep no mma.sync-ordered
 * copy of the weight (the decode GEMV then runs on CUDA cores for every M <= 16; the
 * copy is the same size as qweight, so this halves the handle's weight bytes). No
 * counterpart in the reference (its make_q4 has no options of this kind). */
#define W4A16_CREATE_NO_REPACK 1
W4A16_API int w4a16_create_ex(const int32_t* qweight_dev, const int32_t* qzeros_dev, const uint16_t* scales_dev,
                              const int32_t* g_idx_host, int K, int N, int groups, int device, int flags,
                              void* stream, w4a16_matrix** out);

/* Free the handle and the buffers it owns (the reference never frees its
 * Q4Matrix, q4_matrix.cu:78-80). */
W4A16_API int w4a16_destroy(w4a16_matrix* h);

/* Dense W[K, N] in original row order, fp16 or bf16 (bf16 = bf16(fp32(fp16 W))).
 * Bit-exact with the reference's torch dequant. Replaces q4_to_half_matrix_v2 /
 * q4_to_bfloat16_matrix_v2 (entry.cpp:75-122, q4_matrix.cu:319-614). */
W4A16_API int w4a16_dequant(w4a16_matrix* h, void* w_out_dev, int dtype, void* stream);

/* Bytes of workspace w4a16_gemm needs for M rows on `path` (0 when none). */
W4A16_API size_t w4a16_workspace_size(const w4a16_matrix* h, int M, int dtype, int path);

/* Y[M, N] = X[M, K] * W (fp32 accumulate), X and Y of `dtype`, row-major and
 * 16-byte aligned. Replaces q4_matmul_cuda_v2 (entry.cpp:221-251 ->
 * q4_matmul.cu:428-456) and q4_matmul_blas_v2 without a cached weight
 * (entry.cpp -> q4_matmul.cu:459-510). No host synchronisation and no allocation:
 * capturable in a CUDA graph. Calls on one handle may overlap on different streams
 * when each has its own workspace: the handle is only read during a call (a call
 * whose bounded wait gives up sets the handle's device error word). */
W4A16_API int w4a16_gemm(w4a16_matrix* h, const void* x_dev, int M, void* y_dev, int dtype, void* workspace_dev,
               size_t workspace_bytes, int path, void* stream);

/* dX[M, K] = dY[M, N] * W^T (fp32 accumulate), dY and dX of `dtype`, row-major and
 * 16-byte aligned, dX in the caller's original row order: the input gradient of the
 * quantized linear, on the tcgen05 tensor cores straight from the packed weight.
 * Replaces q4_transpose_matmul_blas_v2 (entry.cpp:392-430 ->
 * q4_transpose_matmul.cu:115-167: reconstruct + cublasHgemm OP_T). Workspace as
 * w4a16_workspace_size_t (act-order: the product in kernel row order; split-K
 * partials). No host synchronisation and no allocation. */
W4A16_API int w4a16_gemm_t(w4a16_matrix* h, const void* dy_dev, int M, void* dx_dev, int dtype, void* workspace_dev,
                           size_t workspace_bytes, void* stream);

/* Bytes of workspace w4a16_gemm_t needs for M rows (0 when none). */
W4A16_API size_t w4a16_workspace_size_t(const w4a16_matrix* h, int M, int dtype);

/* The launch plan w4a16_gemm would use: out[0] = kernel family (1 CUDA-core GEMV,
 * 3 tcgen05 exact-W GEMM, 4 GEMV on the handle's repacked weight with mma.sync), out[1] = tile (GEMV: columns per CTA, tcgen05: tokens per
 * tile), out[2] = K splits, out[3] = GEMV rows per pass or tcgen05 K chunks (64
 * wide) per split. w4a16_plan_shape's out[4] tells the tcgen05 orientations apart. */
W4A16_API int w4a16_plan(const w4a16_matrix* h, int M, int dtype, int path, int out[4]);

/* The plan and workspace w4a16_create + w4a16_plan / w4a16_workspace_size would give
 * for a weight of this shape on a GPU with `num_sms` SMs, without a GPU or a handle.
 * The weight is assumed repacked for the mma.sync GEMV when its group size allows it,
 * as w4a16_create does by default. out[0..3] as w4a16_plan; out[4] bit 0 = the
 * CUDA-core GEMV runs its WIDE configuration (3 CTAs per SM, 4-row batches), bit 1 =
 * the tcgen05 GEMM runs in the natural orientation (128 tokens x 256 weight columns
 * per MMA). No counterpart in the reference. */
W4A16_API int w4a16_plan_shape(int K, int N, int groups, int act_order, int M, int dtype, int path, int num_sms,
                               int out[5], size_t* workspace_bytes);

/* Shape of the handle: out[0] = K, out[1] = N, out[2] = groups, out[3] = bit 0:
 * act-order, bit 1: symmetric (every stored zero nibble is 7, z = 8; found at creation,
 * the kernels then skip the zero-point loads). */
W4A16_API int w4a16_info(const w4a16_matrix* h, int out[4]);

/* ---- Decoder-layer blocks around the projections (fp16) ----------------------------
 * RMSNorm of each row of x [M, K]: y = fp16(x * w * rsqrt(mean(x^2) + eps)), x clamped
 * to the fp16 range. Replaces rms_norm_cuda (fuse_v2/rms_norm.cu:27-93,109-131). */
W4A16_API int w4a16_rms_norm(const void* x_dev, const void* w_dev, float eps, int M, int K, void* y_dev, int dtype,
                             void* stream);
/* out [M, N] = fp16(silu(gate) * up), silu(g) = g / (1 + e^-g) in fp32; out may alias
 * gate. Replaces silu_mul_kernel (fuse_v2/q_mlp.cu:12-33,43-85). */
W4A16_API int w4a16_silu_mul(const void* gate_dev, const void* up_dev, int M, int N, void* out_dev, int dtype,
                             void* stream);

/* The MLP block of a decoder layer: y = down(silu(gate(r)) * up(r)), r = RMSNorm(x;
 * norm_w, eps); x [M, K], y [M, K_down_out]. Replaces mlp_forward_v2 (entry.cpp:431-481
 * -> fuse_v2/q_mlp.cu:96-133: five launches). rms_out [M, K] receives r; gate_out and
 * up_out [M, I] are scratch of the block (the reference's temp buffers), their contents
 * afterwards unspecified. For M <= 2 without act-order it is two launches: the RMSNorm
 * is applied while the gate + up GEMV stages X, and silu * mul while the down GEMV
 * stages its X (no workspace). Otherwise RMSNorm, the three projections on their usual
 * kernels and silu * mul; workspace as w4a16_mlp_workspace_size. */
W4A16_API int w4a16_mlp_forward(w4a16_matrix* gate, w4a16_matrix* up, w4a16_matrix* down, const void* norm_w_dev,
                                float eps, const void* x_dev, int M, void* y_dev, void* rms_out_dev,
                                void* gate_out_dev, void* up_out_dev, int dtype, void* workspace_dev,
                                size_t workspace_bytes, void* stream);
W4A16_API size_t w4a16_mlp_workspace_size(const w4a16_matrix* gate, const w4a16_matrix* up,
                                          const w4a16_matrix* down, int M, int dtype);

/* The q / k / v stage of attention: r = RMSNorm(x), q_out = r Wq, k_out = r Wk, v_out =
 * r Wv, rms_out = r. Replaces attention_forward_qkv_stage_v2 (entry.cpp:483-532 ->
 * fuse_v2/q_attn.cu:23-54: four launches). For M <= 2 without act-order it is one
 * launch over the three weights with the RMSNorm applied while X is staged. */
W4A16_API int w4a16_qkv_forward(w4a16_matrix* q, w4a16_matrix* k, w4a16_matrix* v, const void* norm_w_dev,
                                float eps, const void* x_dev, int M, void* rms_out_dev, void* q_out_dev,
                                void* k_out_dev, void* v_out_dev, int dtype, void* workspace_dev,
                                size_t workspace_bytes, void* stream);
W4A16_API size_t w4a16_qkv_workspace_size(const w4a16_matrix* q, const w4a16_matrix* k, const w4a16_matrix* v,
                                          int M, int dtype);

/* Read (and clear) the handle's device error word: nonzero means a bounded wait
 * inside a kernel gave up. Synchronises `stream`. Diagnostic only. */
W4A16_API int w4a16_device_error(w4a16_matrix* h, void* stream, int* err_out);

/* w4a16_gemm without a caller workspace. No counterpart in the reference (its
 * GEMV needs no workspace; its prefill path takes a caller scratch weight,
 * exllama.py:358-378). For callers that cannot allocate device memory at call time
 * (a plain C FFI host with no GPU allocator, a serving loop whose allocator is
 * frozen after warm-up). It allocates nothing: the workspace is a fixed 8 MiB array
 * in the library's device image, one per device. The first call on a device looks
 * up that array's address (cudaGetSymbolAddress with the device current), so make
 * it before any stream capture. Calls needing more than 8 MiB of workspace
 * (w4a16_workspace_size) fail with W4A16_ERR_WORKSPACE. All calls on a device share
 * the array: calls that overlap on the GPU, from any handle or stream, race. The
 * array is resident (8 MiB) on every device where the library is loaded, whether or
 * not this entry point is called; after a cudaDeviceReset the library must be
 * reloaded before this entry point is used again. */
W4A16_API int w4a16_gemm_static(w4a16_matrix* h, const void* x_dev, int M, void* y_dev, int dtype, int path,
                      void* stream);

/* ---- Column-sharded GEMV with its all-gather fused in, over peer memory ----
 * No counterpart in the reference (its multi-GPU mode is a layer pipeline over TCP);
 * this replaces "GEMV on this rank's columns, then ncclAllGather" for the decode
 * sizes. Rank r holds the handle of columns [col0, col0 + N) of a [K, ld] weight;
 * every rank's full output Y [M, ld] is written by every rank's kernel over NVLink,
 * and the kernel completes only when every rank's columns have arrived (a bounded
 * wait on per-rank epoch flags; a timeout sets the handle's device error word).
 * Buffers of other processes are mapped with CUDA IPC: the caller moves the
 * W4A16_IPC_HANDLE_BYTES-byte handles between ranks over its own channel. */
#define W4A16_IPC_HANDLE_BYTES 72

typedef struct w4a16_comm w4a16_comm;

/* Flags and counters of one rank of a gather group of `world` ranks (<= 8). */
W4A16_API int w4a16_comm_create(int rank, int world, int device, w4a16_comm** out);
W4A16_API int w4a16_comm_destroy(w4a16_comm* c);
/* This rank's flags buffer (to export with w4a16_ipc_export). */
W4A16_API int w4a16_comm_flags(const w4a16_comm* c, void** flags_dev);
/* Rank `peer`'s flags as mapped in this process (w4a16_ipc_open of its export). */
W4A16_API int w4a16_comm_set_peer_flags(w4a16_comm* c, int peer, void* flags_dev);

/* Export a device pointer of this process (any cudaMalloc-backed memory, at any
 * offset inside its allocation) / map another process's export on `device` / unmap. */
W4A16_API int w4a16_ipc_export(const void* dev_ptr, void* handle_out);
W4A16_API int w4a16_ipc_open(const void* handle_in, int device, void** ptr_out);
W4A16_API int w4a16_ipc_close(void* ptr);

/* Y_r[M, ld] (row-major, every rank r) gets this rank's X[M, K] * W in columns
 * [col0, col0 + N); y_all[r] = rank r's Y as addressable here. Decode sizes run the
 * GEMV, which stores each output into every rank's Y; larger M runs the tcgen05 GEMM,
 * whose epilogue (or split-K reduction) stores 16-byte row pieces the same way (ld
 * and col0 multiples of 8, every y_all[r] 16-byte aligned; the mma.sync GEMV does the
 * same when ld and col0 are multiples of 8). W4A16_ERR_UNSUPPORTED where W4A16_PATH_AUTO would pick
 * the tcgen05 decode pass. All ranks must make the same sequence of calls; a Y buffer
 * must not be rewritten by a later call before every rank has consumed it. Workspace
 * as w4a16_workspace_size(h, M, dtype, W4A16_PATH_AUTO). */
W4A16_API int w4a16_gemm_gather(w4a16_matrix* h, w4a16_comm* c, const void* x_dev, int M, void* const* y_all, int ld,
                      int col0, int dtype, void* workspace_dev, size_t workspace_bytes, void* stream);

/* Message of the last failure on this thread ("" if none). */
W4A16_API const char* w4a16_last_error(void);

/* ABI version (major * 100 + minor). */
W4A16_API int w4a16_version(void);

#ifdef __cplusplus
}
#endif

#endif /* DROFELL_W4A16_H_ */
