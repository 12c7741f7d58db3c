// Staging kernels of non-causal attention (brk_attn_full; attention_full / attention_full_wg,
// shaders.ts:1530-1667): token-major f32 K/V become the head-major fp16 rows the attention
// kernels read through TMA, with the head dim zero-padded to a kernel size; q is zero-padded the
// same way when needed.  Zero lanes add nothing to q.k and produce output lanes that are dropped.
#include "internal.h"

namespace brk {

namespace {

// One thread per 8 padded head-dim lanes of one (sequence, kv head, key) row.
__global__ void stage_kv_kernel(const float *k, const float *v, __half *ks, __half *vs, int B, int L, int H, int D,
                                int Dp) {
    const int c8s = Dp / 8;
    const long long n = (long long)B * H * L * c8s;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
        const int c8 = (int)(i % c8s);
        const long long r = i / c8s;
        const int j = (int)(r % L);
        const long long bh = r / L;
        const int h = (int)(bh % H), b = (int)(bh / H);
        const size_t src = (((size_t)b * L + j) * H + h) * D;
        const size_t dst = (((size_t)b * H + h) * L + j) * Dp + 8 * c8;
        __align__(16) __half hk[8], hv[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            const int d = 8 * c8 + e;
            hk[e] = __float2half_rn(d < D ? k[src + d] : 0.f);
            hv[e] = __float2half_rn(d < D ? v[src + d] : 0.f);
        }
        *reinterpret_cast<uint4 *>(ks + dst) = *reinterpret_cast<const uint4 *>(hk);
        *reinterpret_cast<uint4 *>(vs + dst) = *reinterpret_cast<const uint4 *>(hv);
    }
}

__global__ void pad_rows_kernel(const float *src, float *dst, long long rows, int D, int Dp) {
    const long long n = rows * Dp;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
        const int d = (int)(i % Dp);
        dst[i] = d < D ? src[(i / Dp) * D + d] : 0.f;
    }
}

unsigned grid_for(long long n, int threads) {
    const long long g = (n + threads - 1) / threads;
    return (unsigned)(g < 8192 ? (g > 0 ? g : 1) : 8192);
}

}  // namespace

cudaError_t launch_stage_kv(const float *k, const float *v, __half *ks, __half *vs, int B, int L, int H, int D, int Dp,
                            cudaStream_t s) {
    const long long n = (long long)B * H * L * (Dp / 8);
    if (n == 0) return cudaSuccess;
    stage_kv_kernel<<<grid_for(n, 256), 256, 0, s>>>(k, v, ks, vs, B, L, H, D, Dp);
    return cudaGetLastError();
}

cudaError_t launch_pad_rows(const float *src, float *dst, long long rows, int D, int Dp, cudaStream_t s) {
    if (rows == 0) return cudaSuccess;
    pad_rows_kernel<<<grid_for(rows * Dp, 256), 256, 0, s>>>(src, dst, rows, D, Dp);
    return cudaGetLastError();
}

}  // namespace brk
