// int8 KV quantisation shared by the append kernel and the cache row kernels.
#pragma once

#include "common.cuh"

namespace brk {

// quantize_kv (shaders.ts:1673-1705) of one head row by one warp, in the shader's f32 arithmetic:
// amax = max |x|, scale = amax / 127 (1e-8 for an all-zero row), inv = 1 / scale,
// code = clamp(round_half_even(x * inv), -127, 127).  Codes are stored biased by +128 (the
// decode kernel turns a biased byte into an exact fp16 with one permute and one subtraction);
// lane 0 stores the scale.  D is a multiple of 4; `dst` is 4-byte aligned.
__device__ __forceinline__ void quantize_row_warp(const float *x, int D, uint8_t *dst, float *sdst, int lane) {
    float amax = 0.f;
    for (int d = lane; d < D; d += 32) amax = fmaxf(amax, fabsf(x[d]));
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
    const float scale = amax == 0.f ? 1e-8f : __fdiv_rn(amax, 127.f);
    const float inv = __frcp_rn(scale);  // the correctly rounded 1/scale
    if (lane == 0) *sdst = scale;
    for (int d4 = lane; d4 < D / 4; d4 += 32) {
        uint32_t w = 0;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            int c = __float2int_rn(__fmul_rn(x[4 * d4 + e], inv));
            c = min(127, max(-127, c));
            w |= (uint32_t)(c + 128) << (8 * e);
        }
        *reinterpret_cast<uint32_t *>(dst + 4 * d4) = w;
    }
}

}  // namespace brk
