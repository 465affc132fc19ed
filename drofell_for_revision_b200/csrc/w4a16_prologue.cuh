// Element transforms of the decoder-layer blocks that sit before a W4A16 projection,
// shared by the GEMV prologues and the standalone kernels so both give the same bits.
#pragma once
#include <cuda_fp16.h>

#include <cstdint>

namespace w4a16 {

// fp16 of x clamped to the fp16 range, as the reference's RMSNorm reads it
// (fuse_v2/rms_norm.cu:57-58)
__device__ __forceinline__ float clamp_h2f(uint32_t bits16) {
    const float f = __half2float(__ushort_as_half(static_cast<uint16_t>(bits16)));
    return fmaxf(-65504.0f, fminf(f, 65504.0f));
}

// 8 values of RMSNorm output: fp16(x * w * rmf) (fuse_v2/rms_norm.cu:88-91)
__device__ __forceinline__ uint4 rms_apply8(uint4 xr, uint4 wr, float rmf) {
    const uint32_t xs[4] = {xr.x, xr.y, xr.z, xr.w}, ws[4] = {wr.x, wr.y, wr.z, wr.w};
    uint32_t o[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float a = clamp_h2f(xs[i] & 0xFFFFu) * __half2float(__ushort_as_half(static_cast<uint16_t>(ws[i]))) * rmf;
        const float b = clamp_h2f(xs[i] >> 16) * __half2float(__ushort_as_half(static_cast<uint16_t>(ws[i] >> 16))) * rmf;
        o[i] = static_cast<uint32_t>(__half_as_ushort(__float2half_rn(a))) |
               (static_cast<uint32_t>(__half_as_ushort(__float2half_rn(b))) << 16);
    }
    return make_uint4(o[0], o[1], o[2], o[3]);
}

// 8 values of fp16(silu(g) * u), silu(g) = g / (1 + e^-g), in fp32 (the reference's
// silu_mul_kernel computes the same in fp16 half2 arithmetic, fuse_v2/q_mlp.cu:12-80)
__device__ __forceinline__ uint4 silu_mul8(uint4 gr, uint4 ur) {
    const uint32_t gs[4] = {gr.x, gr.y, gr.z, gr.w}, us[4] = {ur.x, ur.y, ur.z, ur.w};
    uint32_t o[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        uint32_t r = 0;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const float g = __half2float(__ushort_as_half(static_cast<uint16_t>(gs[i] >> (16 * h))));
            const float u = __half2float(__ushort_as_half(static_cast<uint16_t>(us[i] >> (16 * h))));
            const float v = g / (1.0f + __expf(-g)) * u;
            r |= static_cast<uint32_t>(__half_as_ushort(__float2half_rn(v))) << (16 * h);
        }
        o[i] = r;
    }
    return make_uint4(o[0], o[1], o[2], o[3]);
}

}  // namespace w4a16
