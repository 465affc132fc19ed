// Device helpers shared by the tcgen05 GEMM kernels: one packed GPTQ word to 16 bytes
// of dequantized weights, and the fp32 -> output conversion.
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <cstdint>

namespace w4a16 {

__device__ __forceinline__ uint32_t h2_bits(__half2 v) { return *reinterpret_cast<uint32_t*>(&v); }
__device__ __forceinline__ __half2 bits_h2(uint32_t v) { return *reinterpret_cast<__half2*>(&v); }

// 8 weights of one packed word, natural k order, as 16 bytes: fp16(s (q - z))
// (bf16 of it for bf16 inputs).
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

template <bool BF16>
__device__ __forceinline__ uint16_t to_out(float f) {
    if constexpr (BF16) {
        return __bfloat16_as_ushort(__float2bfloat16_rn(f));
    } else {
        return __half_as_ushort(__float2half_rn(f));
    }
}

}  // namespace w4a16
