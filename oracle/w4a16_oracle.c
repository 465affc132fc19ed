/*
 * Plain-C restatement of the reference's GPTQ W4A16 dequantize-then-matmul.
 *
 * TEST INFRASTRUCTURE ONLY: used by tests/ as a checker and by bench.py as the
 * timed CPU baseline. The product library never links it.
 *
 * Dequant follows After-Revision-DROFELL/operators/core/linear/real_quant.py:69-90:
 *   q[k,n] = (qweight[k/8, n] >> 4*(k%8)) & 15
 *   z[g,n] = ((qzeros[g, n/8] >> 4*(n%8)) & 15) + 1
 *   W[k,n] = fp16( scales[g_idx[k], n] * (q[k,n] - z[g_idx[k], n]) )
 * computed as one round-to-nearest-even of the exact fp32 product.
 * bf16 weights: bf16(fp32(fp16 W)), as q4_matrix.cu:465-467 converts them.
 * Matmul: Y = X.float() @ W.float() with fp32 accumulation.
 */
#include <stdint.h>
#include <stddef.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

typedef _Float16 f16;

static inline uint16_t f32_to_f16_bits(float v) {
    f16 h = (f16)v; /* IEEE round-to-nearest-even */
    uint16_t b;
    memcpy(&b, &h, 2);
    return b;
}

static inline float f16_bits_to_f32(uint16_t b) {
    f16 h;
    memcpy(&h, &b, 2);
    return (float)h;
}

static inline uint16_t f32_to_bf16_bits(float v) {
    uint32_t u;
    memcpy(&u, &v, 4);
    uint32_t rounding = ((u >> 16) & 1u) + 0x7FFFu;
    return (uint16_t)((u + rounding) >> 16);
}

static inline float bf16_bits_to_f32(uint16_t b) {
    uint32_t u = ((uint32_t)b) << 16;
    float v;
    memcpy(&v, &u, 4);
    return v;
}

static int check_args(int K, int N, int group_size) {
    if (K <= 0 || N <= 0 || (K % 8) || (N % 8)) return 1;
    if (group_size <= 0 || (K % group_size)) return 2;
    return 0;
}

/* One dequantized fp16 weight, as a float (exactly representable). */
static inline uint16_t dq_one(const int32_t* qweight, const int32_t* qzeros, const uint16_t* scales,
                              int k, int n, int g, int N) {
    uint32_t w = (uint32_t)qweight[(size_t)(k >> 3) * N + n];
    int q = (int)((w >> (4 * (k & 7))) & 15u);
    uint32_t zw = (uint32_t)qzeros[(size_t)g * (N >> 3) + (n >> 3)];
    int z = (int)((zw >> (4 * (n & 7))) & 15u) + 1;
    float s = f16_bits_to_f32(scales[(size_t)g * N + n]);
    return f32_to_f16_bits(s * (float)(q - z));
}

int oracle_dequant_fp16(const int32_t* qweight, const int32_t* qzeros, const uint16_t* scales,
                        const int32_t* g_idx, int K, int N, int group_size, uint16_t* out, int threads) {
    int rc = check_args(K, N, group_size);
    if (rc) return rc;
#ifdef _OPENMP
    if (threads > 0) omp_set_num_threads(threads);
#pragma omp parallel for schedule(static)
#endif
    for (int k = 0; k < K; ++k) {
        int g = g_idx ? g_idx[k] : k / group_size;
        for (int n = 0; n < N; ++n) out[(size_t)k * N + n] = dq_one(qweight, qzeros, scales, k, n, g, N);
    }
    (void)threads;
    return 0;
}

int oracle_dequant_bf16(const int32_t* qweight, const int32_t* qzeros, const uint16_t* scales,
                        const int32_t* g_idx, int K, int N, int group_size, uint16_t* out, int threads) {
    int rc = check_args(K, N, group_size);
    if (rc) return rc;
#ifdef _OPENMP
    if (threads > 0) omp_set_num_threads(threads);
#pragma omp parallel for schedule(static)
#endif
    for (int k = 0; k < K; ++k) {
        int g = g_idx ? g_idx[k] : k / group_size;
        for (int n = 0; n < N; ++n) {
            uint16_t h = dq_one(qweight, qzeros, scales, k, n, g, N);
            out[(size_t)k * N + n] = f32_to_bf16_bits(f16_bits_to_f32(h));
        }
    }
    (void)threads;
    return 0;
}

/* Y[M,N] (fp32) = X[M,K] @ W[K,N]; X and W are fp16 bits (is_bf16 = 0) or bf16 bits. */
int oracle_matmul_f16w(const uint16_t* x, int M, const uint16_t* w, int K, int N, float* y,
                       int is_bf16, int threads) {
    if (M < 0 || K <= 0 || N <= 0) return 1;
    const int NB = 256;
    int nblocks = (N + NB - 1) / NB;
#ifdef _OPENMP
    if (threads > 0) omp_set_num_threads(threads);
#pragma omp parallel for collapse(2) schedule(static)
#endif
    for (int m = 0; m < M; ++m) {
        for (int nb = 0; nb < nblocks; ++nb) {
            float acc[256];
            int n0 = nb * NB;
            int n1 = n0 + NB < N ? n0 + NB : N;
            for (int n = n0; n < n1; ++n) acc[n - n0] = 0.0f;
            for (int k = 0; k < K; ++k) {
                uint16_t xb = x[(size_t)m * K + k];
                float xv = is_bf16 ? bf16_bits_to_f32(xb) : f16_bits_to_f32(xb);
                const uint16_t* wr = w + (size_t)k * N;
                if (is_bf16) {
                    for (int n = n0; n < n1; ++n) acc[n - n0] += xv * bf16_bits_to_f32(wr[n]);
                } else {
                    for (int n = n0; n < n1; ++n) acc[n - n0] += xv * f16_bits_to_f32(wr[n]);
                }
            }
            for (int n = n0; n < n1; ++n) y[(size_t)m * N + n] = acc[n - n0];
        }
    }
    (void)threads;
    return 0;
}

/* Whole reference forward: dequant into w_scratch (K*N uint16), then fp32 matmul. */
int oracle_linear(const uint16_t* x, int M, const int32_t* qweight, const int32_t* qzeros,
                  const uint16_t* scales, const int32_t* g_idx, int K, int N, int group_size,
                  uint16_t* w_scratch, float* y, int is_bf16, int threads) {
    int rc = is_bf16 ? oracle_dequant_bf16(qweight, qzeros, scales, g_idx, K, N, group_size, w_scratch, threads)
                     : oracle_dequant_fp16(qweight, qzeros, scales, g_idx, K, N, group_size, w_scratch, threads);
    if (rc) return rc;
    return oracle_matmul_f16w(x, M, w_scratch, K, N, y, is_bf16, threads);
}
