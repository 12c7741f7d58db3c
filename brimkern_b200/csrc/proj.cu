// The projections either side of the attention operator: the recordLayerKV slice
// (kernels.ts:1700-1736; layerForwardCpu kernels.ts:3501-3522) -- RMSNorm of the layer input, the
// q / k / v projections (+ biases) that feed the append, and the output projection with the
// residual add (and Gemma-2's post-attention RMSNorm) that consumes the attention output.
//
// The reference multiplies f32 activations by f16 weight matrices [n][k] (matmul_t_f16w,
// C = A W^T).  Here the activations are cast to fp16 once (the RMSNorm fused into that cast) and
// both products run as weight-streaming GEMMs on the 5th-generation tensor cores:
//   - one CTA per (NT output columns, 128 rows); warp 4 streams [128 rows][64 k] activation boxes
//     and [NT][64 k] weight boxes through a TMA ring (128-byte swizzle, CTA-local loads);
//   - warp 5 issues tcgen05.mma (M 128, N NT, K 16; fp16 in, fp32 accumulators in TMEM) and
//     commits each stage back to the producer;
//   - warps 0-3 (thread r <-> row r <-> TMEM lane r) read the accumulators with tcgen05.ld and
//     write f32 outputs plus bias and residual.
// At decode (M = B rows) the GEMM is bound by streaming the weights from HBM; prefill-sized M
// makes it tensor-bound.
#include "common.cuh"
#include "internal.h"
#include "tcgen05.cuh"

namespace brk {

namespace {

constexpr int kPM = 128;       // rows per tile (MMA M; rows past the end are zero-filled by TMA)
constexpr int kPK = 64;        // k per stage (one 128-byte swizzled box column)
constexpr int kPThreads = 192;
constexpr int kPProducer = 4, kPMma = 5;

template <int NT>
struct ProjLayout {
    static constexpr uint32_t kABytes = kPM * 128;   // [128][64] fp16
    static constexpr uint32_t kWBytes = NT * 128;    // [NT][64] fp16
    static constexpr uint32_t kStageBytes = kABytes + kWBytes;
    // NT 32 (decode): two CTAs per SM stream different weight columns; NT 128: one deep ring.
    static constexpr int kStages = NT <= 32 ? 5 : 6;
    static constexpr uint32_t kBarOff = kStages * kStageBytes;
    static constexpr uint32_t kSmemBytes = 1024 + kBarOff + (2 * kStages + 1) * 8 + 16;
};

// One warp per row: out = fp16(x * inv * g) with inv = 1/sqrt(mean(x^2) + eps) (rmsnorm shader,
// shaders.ts:580-598), or a plain fp16 cast when gain is null.
__global__ void norm_cast_kernel(const float *x, const float *gain, float eps, int one_plus, __half *out, int rows,
                                 int K) {
    const int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (row >= rows) return;
    const float4 *src = reinterpret_cast<const float4 *>(x + (size_t)row * K);
    float inv = 1.f;
    if (gain) {
        float ss = 0.f;
        for (int c = lane; c < K / 4; c += 32) {
            const float4 v = src[c];
            ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
        inv = 1.f / sqrtf(ss / (float)K + eps);
    }
    uint2 *dst = reinterpret_cast<uint2 *>(out + (size_t)row * K);
    for (int c = lane; c < K / 4; c += 32) {
        float4 v = src[c];
        if (gain) {
            const float4 g = reinterpret_cast<const float4 *>(gain)[c];
            v.x *= inv * (one_plus ? 1.f + g.x : g.x);
            v.y *= inv * (one_plus ? 1.f + g.y : g.y);
            v.z *= inv * (one_plus ? 1.f + g.z : g.z);
            v.w *= inv * (one_plus ? 1.f + g.w : g.w);
        }
        dst[c] = make_uint2(pack_half2(v.x, v.y), pack_half2(v.z, v.w));
    }
}

// h = x + rmsnorm(h) in place, one warp per row (Gemma-2's post-attention norm before the
// residual, kernels.ts:1733-1734).
__global__ void post_norm_residual_kernel(float *h, const float *x, const float *gain, float eps, int one_plus,
                                          int rows, int n) {
    const int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (row >= rows) return;
    float4 *p = reinterpret_cast<float4 *>(h + (size_t)row * n);
    const float4 *xr = reinterpret_cast<const float4 *>(x + (size_t)row * n);
    float ss = 0.f;
    for (int c = lane; c < n / 4; c += 32) {
        const float4 v = p[c];
        ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
    const float inv = 1.f / sqrtf(ss / (float)n + eps);
    for (int c = lane; c < n / 4; c += 32) {
        const float4 v = p[c], r = xr[c], g = reinterpret_cast<const float4 *>(gain)[c];
        p[c] = make_float4(r.x + v.x * inv * (one_plus ? 1.f + g.x : g.x), r.y + v.y * inv * (one_plus ? 1.f + g.y : g.y),
                           r.z + v.z * inv * (one_plus ? 1.f + g.z : g.z), r.w + v.w * inv * (one_plus ? 1.f + g.w : g.w));
    }
}

template <int NT>
__global__ void __launch_bounds__(kPThreads, 1)
    proj_gemm_kernel(const __grid_constant__ CUtensorMap ta, const __grid_constant__ CUtensorMap tw0,
                     const __grid_constant__ CUtensorMap tw1, const __grid_constant__ CUtensorMap tw2,
                     const __grid_constant__ ProjArgs a) {
    using L = ProjLayout<NT>;
    constexpr int S = L::kStages;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + L::kBarOff);
    uint64_t *empty = full + S;
    uint64_t *done = empty + S;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(done + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n0 = blockIdx.x * NT;
    const int m0 = blockIdx.y * kPM;
    int mi = 0;
    while (mi + 1 < a.nmat && n0 >= a.n_end[mi]) ++mi;
    const int col0 = n0 - (mi ? a.n_end[mi - 1] : 0);   // first column inside matrix mi
    const int ncols = a.n_end[mi] - (mi ? a.n_end[mi - 1] : 0);
    const CUtensorMap *tw = mi == 0 ? &tw0 : mi == 1 ? &tw1 : &tw2;
    const int nk = (a.K + kPK - 1) / kPK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(done, 1);
        fence_barrier_init();
    }
    if (warp == kPMma) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(tmem_slot)),
                     "r"((uint32_t)NT)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == kPProducer) {
        if (lane == 0) {
            tma_prefetch_desc(&ta);
            tma_prefetch_desc(tw);
            int issued = 0;
            for (int j = 0; j < nk; ++j) {
                const int s = j % S;
                if (j >= S && !mbar_wait(&empty[s], ((j / S) - 1) & 1, a.err, kErrSlotTimeout)) break;
                uint8_t *st = smem + s * L::kStageBytes;
                mbar_arrive_expect_tx(&full[s], L::kStageBytes);
                tma_load_2d(st, &ta, j * kPK, m0, &full[s]);
                tma_load_2d(st + L::kABytes, tw, j * kPK, col0, &full[s]);
                issued = j + 1;
            }
            for (int j = issued > S ? issued - S : 0; j < issued; ++j)
                mbar_wait(&full[j % S], (j / S) & 1, a.err, kErrTmaTimeout);
        }
        __syncwarp();
    } else if (warp == kPMma) {
        if (lane == 0) {
            constexpr uint32_t idesc = f16_idesc(kPM, NT, 0, 0);
            bool ok = true;
            for (int j = 0; j < nk && ok; ++j) {
                const int s = j % S;
                if (!mbar_wait(&full[s], (j / S) & 1, a.err, kErrTmaTimeout)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t a_base = smem_addr(smem + s * L::kStageBytes), w_base = a_base + L::kABytes;
#pragma unroll
                for (int ks = 0; ks < kPK / 16; ++ks)
                    tc_mma(tmem, sw128_desc(a_base + ks * 32, 16, 1024), sw128_desc(w_base + ks * 32, 16, 1024), idesc,
                           j > 0 || ks > 0);
                tc_commit(&empty[s]);  // the stage is free once these MMAs have read it
            }
            tc_commit(done);
            mbar_wait(done, 0, a.err, kErrMmaTimeout);
        }
        __syncwarp();
    } else {
        // Epilogue: thread r owns row m0 + r (TMEM lane r).
        const int r = warp * 32 + lane;
        const int row = m0 + r;
        const bool ok = mbar_wait(done, 0, a.err, kErrMmaTimeout);
        tc_fence_after();
        if (ok) {
            const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
            float *dst = a.out[mi] + (size_t)row * ncols + col0;
            const float *bias = a.bias[mi] ? a.bias[mi] + col0 : nullptr;
            const float *res = a.residual && mi == 0 ? a.residual + (size_t)row * ncols + col0 : nullptr;
#pragma unroll 1
            for (int c = 0; c < NT / 32; ++c) {
                uint32_t v[32];
                tc_ld32_nowait(tmem + lane_base + c * 32, v);
                tc_wait_ld();
                if (row < a.M) {
#pragma unroll
                    for (int e = 0; e < 32; e += 4) {
                        float4 o = make_float4(__uint_as_float(v[e]), __uint_as_float(v[e + 1]),
                                               __uint_as_float(v[e + 2]), __uint_as_float(v[e + 3]));
                        if (bias) {
                            const float4 b = *reinterpret_cast<const float4 *>(bias + c * 32 + e);
                            o.x += b.x, o.y += b.y, o.z += b.z, o.w += b.w;
                        }
                        if (res) {
                            const float4 x = *reinterpret_cast<const float4 *>(res + c * 32 + e);
                            o.x += x.x, o.y += x.y, o.z += x.z, o.w += x.w;
                        }
                        *reinterpret_cast<float4 *>(dst + c * 32 + e) = o;
                    }
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == kPMma)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"((uint32_t)NT) : "memory");
}

template <int NT>
cudaError_t launch_gemm_t(const CUtensorMap &ta, const CUtensorMap *tw, const ProjArgs &a, cudaStream_t s) {
    static unsigned long long configured = 0;
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 64 || !(configured & (1ull << dev))) {
        cudaError_t e = cudaFuncSetAttribute(proj_gemm_kernel<NT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             ProjLayout<NT>::kSmemBytes);
        if (e != cudaSuccess) return e;
        if (dev < 64) configured |= 1ull << dev;
    }
    const dim3 grid(a.n_end[a.nmat - 1] / NT, (a.M + kPM - 1) / kPM);
    proj_gemm_kernel<NT><<<grid, kPThreads, ProjLayout<NT>::kSmemBytes, s>>>(ta, tw[0], tw[1], tw[2], a);
    return cudaGetLastError();
}

}  // namespace

int proj_tile_cols(int rows) { return rows <= kPM ? 32 : 128; }

cudaError_t launch_norm_cast(const float *x, const float *gain, float eps, int one_plus, __half *out, int rows, int K,
                             cudaStream_t s) {
    if (rows == 0) return cudaSuccess;
    const long long threads = (long long)rows * 32;
    norm_cast_kernel<<<(unsigned)((threads + 255) / 256), 256, 0, s>>>(x, gain, eps, one_plus, out, rows, K);
    return cudaGetLastError();
}

cudaError_t launch_post_norm_residual(float *h, const float *x, const float *gain, float eps, int one_plus, int rows,
                                      int n, cudaStream_t s) {
    if (rows == 0) return cudaSuccess;
    const long long threads = (long long)rows * 32;
    post_norm_residual_kernel<<<(unsigned)((threads + 255) / 256), 256, 0, s>>>(h, x, gain, eps, one_plus, rows, n);
    return cudaGetLastError();
}

cudaError_t launch_proj_gemm(int nt, const CUtensorMap &ta, const CUtensorMap *tw, const ProjArgs &a, cudaStream_t s) {
    switch (nt) {
        case 32: return launch_gemm_t<32>(ta, tw, a, s);
        case 128: return launch_gemm_t<128>(ta, tw, a, s);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace brk
