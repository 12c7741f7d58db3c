// Row kernels of the int8 KV cache: quantised row store (the quantize_kv pass of
// recQuantizeKv, kernels.ts:1644-1648, for rows that need no norm or rotation), direct store of
// given codes and scales (the inputs of attentionQ8Kv, kernels.ts:681), read-back in the
// reference's token-major layout (quantizeKvReadback, kernels.ts:664), and dequantisation of one
// layer into fp16 staging for the tensor-core prefill kernel.
#include "internal.h"
#include "kv_q8.cuh"

namespace brk {

namespace {

constexpr int kWarps = 4;

// One warp per (row, kv head) of the f32 input [n_rows][Hkv][D].
__global__ void __launch_bounds__(kWarps * 32)
    kv_write_q8_kernel(uint8_t *kc, uint8_t *vc, float *sc, const float *k, const float *v, int n_rows, int Hkv,
                       int D, int cap, int pitch) {
    const int lane = threadIdx.x & 31;
    const long long item = (long long)blockIdx.x * kWarps + (threadIdx.x >> 5);
    if (item >= 2LL * n_rows * Hkv) return;
    const bool is_v = item >= (long long)n_rows * Hkv;
    const int rh = (int)(is_v ? item - (long long)n_rows * Hkv : item);
    const int r = rh / Hkv, h = rh % Hkv;
    const float *src = (is_v ? v : k);
    if (!src) return;
    src += (size_t)rh * D;
    uint8_t *dst = (is_v ? vc : kc) + ((size_t)h * cap + r) * D;
    float *sdst = sc + ((size_t)h * 2 + (is_v ? 1 : 0)) * pitch + r;
    quantize_row_warp(src, D, dst, sdst, lane);
}

__global__ void kv_store_codes_kernel(uint8_t *kc, uint8_t *vc, float *sc, const int8_t *k, const float *ks,
                                      const int8_t *v, const float *vs, int n_rows, int Hkv, int D, int cap,
                                      int pitch) {
    const long long n = (long long)n_rows * Hkv * D;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
        const int d = (int)(i % D);
        const int h = (int)((i / D) % Hkv);
        const int r = (int)(i / ((long long)D * Hkv));
        const size_t dst = ((size_t)h * cap + r) * D + d;
        if (k) kc[dst] = (uint8_t)(k[i] + 128);
        if (v) vc[dst] = (uint8_t)(v[i] + 128);
        if (d == 0) {
            if (ks) sc[((size_t)h * 2) * pitch + r] = ks[(size_t)r * Hkv + h];
            if (vs) sc[((size_t)h * 2 + 1) * pitch + r] = vs[(size_t)r * Hkv + h];
        }
    }
}

__global__ void kv_read_q8_kernel(const uint8_t *kc, const uint8_t *vc, const float *sc, int8_t *k, float *ks,
                                  int8_t *v, float *vs, int n_rows, int Hkv, int D, int cap, int pitch) {
    const long long n = (long long)n_rows * Hkv * D;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
        const int d = (int)(i % D);
        const int h = (int)((i / D) % Hkv);
        const int r = (int)(i / ((long long)D * Hkv));
        const size_t src = ((size_t)h * cap + r) * D + d;
        if (k) k[i] = (int8_t)((int)kc[src] - 128);
        if (v) v[i] = (int8_t)((int)vc[src] - 128);
        if (d == 0) {
            if (ks) ks[(size_t)r * Hkv + h] = sc[((size_t)h * 2) * pitch + r];
            if (vs) vs[(size_t)r * Hkv + h] = sc[((size_t)h * 2 + 1) * pitch + r];
        }
    }
}

// Rows [0, rows) of every (sequence, kv head) segment of `layer`, 8 codes per thread:
// fp16(f32(code * scale)), i.e. the fp16 rounding of the dequantised value of kernels.ts:2577-2588.
__global__ void kv_dequant_kernel(const uint8_t *kc, const uint8_t *vc, const float *sc, __half *k, __half *v,
                                  int layer, int B, int Hkv, int D, int cap, int pitch, int rows) {
    const int c8s = D / 8;
    const long long n = (long long)B * Hkv * rows * c8s;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
        const int c8 = (int)(i % c8s);
        const long long rr = i / c8s;
        const int r = (int)(rr % rows);
        const int segl = (int)(rr / rows);
        const size_t seg = (size_t)layer * B * Hkv + segl;
        const size_t src = (seg * cap + r) * D + 8 * c8;
        const size_t dst = ((size_t)segl * rows + r) * D + 8 * c8;
        const float sk = sc[(seg * 2) * pitch + r], sv = sc[(seg * 2 + 1) * pitch + r];
        const uint2 wk = *reinterpret_cast<const uint2 *>(kc + src);
        const uint2 wv = *reinterpret_cast<const uint2 *>(vc + src);
        uint32_t hk[4], hv[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const uint32_t ck = e < 2 ? wk.x : wk.y, cv = e < 2 ? wv.x : wv.y;
            const int sh = (e & 1) * 16;
            const float k0 = (float)((int)((ck >> sh) & 0xffu) - 128), k1 = (float)((int)((ck >> (sh + 8)) & 0xffu) - 128);
            const float v0 = (float)((int)((cv >> sh) & 0xffu) - 128), v1 = (float)((int)((cv >> (sh + 8)) & 0xffu) - 128);
            hk[e] = pack_half2(__fmul_rn(k0, sk), __fmul_rn(k1, sk));
            hv[e] = pack_half2(__fmul_rn(v0, sv), __fmul_rn(v1, sv));
        }
        *reinterpret_cast<uint4 *>(k + dst) = make_uint4(hk[0], hk[1], hk[2], hk[3]);
        *reinterpret_cast<uint4 *>(v + dst) = make_uint4(hv[0], hv[1], hv[2], hv[3]);
    }
}

unsigned grid_for(long long n, int threads) {
    const long long g = (n + threads - 1) / threads;
    return (unsigned)(g < 8192 ? (g > 0 ? g : 1) : 8192);
}

}  // namespace

cudaError_t launch_kv_write_q8(uint8_t *kc, uint8_t *vc, float *sc, const float *k, const float *v, int n_rows,
                               int Hkv, int D, int cap, int pitch, cudaStream_t s) {
    const long long items = 2LL * n_rows * Hkv;
    if (items == 0) return cudaSuccess;
    kv_write_q8_kernel<<<(unsigned)((items + kWarps - 1) / kWarps), kWarps * 32, 0, s>>>(kc, vc, sc, k, v, n_rows,
                                                                                         Hkv, D, cap, pitch);
    return cudaGetLastError();
}

cudaError_t launch_kv_store_codes(uint8_t *kc, uint8_t *vc, float *sc, const int8_t *k, const float *ks,
                                  const int8_t *v, const float *vs, int n_rows, int Hkv, int D, int cap, int pitch,
                                  cudaStream_t s) {
    const long long n = (long long)n_rows * Hkv * D;
    if (n == 0) return cudaSuccess;
    kv_store_codes_kernel<<<grid_for(n, 256), 256, 0, s>>>(kc, vc, sc, k, ks, v, vs, n_rows, Hkv, D, cap, pitch);
    return cudaGetLastError();
}

cudaError_t launch_kv_read_q8(const uint8_t *kc, const uint8_t *vc, const float *sc, int8_t *k, float *ks, int8_t *v,
                              float *vs, int n_rows, int Hkv, int D, int cap, int pitch, cudaStream_t s) {
    const long long n = (long long)n_rows * Hkv * D;
    if (n == 0) return cudaSuccess;
    kv_read_q8_kernel<<<grid_for(n, 256), 256, 0, s>>>(kc, vc, sc, k, ks, v, vs, n_rows, Hkv, D, cap, pitch);
    return cudaGetLastError();
}

cudaError_t launch_kv_dequant(const uint8_t *kc, const uint8_t *vc, const float *sc, __half *k, __half *v, int layer,
                              int B, int Hkv, int D, int cap, int pitch, int rows, cudaStream_t s) {
    const long long n = (long long)B * Hkv * rows * (D / 8);
    if (n == 0) return cudaSuccess;
    kv_dequant_kernel<<<grid_for(n, 256), 256, 0, s>>>(kc, vc, sc, k, v, layer, B, Hkv, D, cap, pitch, rows);
    return cudaGetLastError();
}

}  // namespace brk
