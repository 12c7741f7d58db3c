// The projections either side of the attention operator: the recordLayerKV slice
// (kernels.ts:1700-1736; layerForwardCpu kernels.ts:3501-3522) -- RMSNorm of the layer input, the
// q / k / v projections (+ biases) that feed the append, and the output projection with the
// residual add (and Gemma-2's post-attention RMSNorm) that consumes the attention output.
//
// The reference multiplies f32 activations by f16 weight matrices [n][k] (matmul_t_f16w,
// C = A W^T).  Here the activations are cast to fp16 once (the RMSNorm fused into that cast) and
// the products run on the 5th-generation tensor cores with the operands swapped, D^T = W X^T:
//   - the weight rows are the MMA's M (128 output features per CTA, TMEM lane = feature) and the
//     tokens its N (32..256 per CTA, TMEM column = token), so a decode step with a few dozen tokens
//     wastes no MMA rows and every CTA streams 16 KB of weights per 64-wide k step;
//   - when the output tiles cannot fill the SMs (decode), K is split over up to 8 CTAs along z;
//     the activation-cast kernel first fills the outputs with the bias (or the residual), and every
//     split adds its partial with a TMA reduce-add (cp.reduce.async.bulk.tensor ... .add, f32 in
//     L2).  The order of those adds is not fixed, so split-K results may differ in the last bit
//     from run to run; with one split the epilogue stores with a plain TMA store;
//   - warp 4 streams [128 features][64 k] weight boxes and [tokens][64 k] activation boxes
//     through a TMA ring (128-byte swizzle, CTA-local loads); the weight loads of the first ring
//     are issued before griddepcontrol.wait, so they overlap the kernel that produced the
//     activations (programmatic dependent launch);
//   - warp 5 issues tcgen05.mma (M 128, N tokens, K 16; fp16 in, fp32 in TMEM) and commits each
//     stage back to the producer; warps 0-3 (thread r <-> feature r) drain TMEM with tcgen05.ld
//     32 tokens at a time into a [32 tokens][128 features] f32 staging tile (double-buffered in the
//     idle ring) that one thread hands to the TMA engine.
#include <algorithm>

#include "common.cuh"
#include "internal.h"
#include "tcgen05.cuh"

namespace brk {

namespace {

constexpr int kFM = 128;      // output features per CTA (MMA M, TMEM lanes)
constexpr int kBoxK = 64;     // k per TMA box (one 128-byte swizzled row)
constexpr int kPThreads = 192;
constexpr int kPProducer = 4, kPMma = 5;

template <int NTOK>
struct ProjLayout {
    static constexpr int kKB = 1;                        // boxes along k per stage
    static constexpr int kStepK = kKB * kBoxK;           // k per stage
    static constexpr uint32_t kWBox = kFM * 128;         // [128][64] fp16 weights
    static constexpr uint32_t kXBox = NTOK * 128;        // [NTOK][64] fp16 activations
    static constexpr uint32_t kWBytes = kKB * kWBox;
    static constexpr uint32_t kStageBytes = kKB * (kWBox + kXBox);
    // Decode-sized token tiles keep two CTAs per SM (more clusters resident for split-K).
    static constexpr int kStages = (NTOK <= 64 ? 4 : NTOK == 128 ? 6 : 4) / kKB;
    static constexpr int kCtasPerSm = NTOK <= 64 ? 2 : 1;  // resident CTAs per SM the ring allows
    static constexpr uint32_t kBarOff = kStages * kStageBytes;
    static constexpr uint32_t kSmemBytes = 1024 + kBarOff + (2 * kStages + 1) * 8 + 16;
    // Two [32 tokens][128 features] f32 staging tiles reuse the ring once the MMAs are done.
    static constexpr uint32_t kOutTile = 32 * kFM * 4;
    static_assert(2 * kOutTile <= kBarOff, "staging tiles do not fit the ring");
};

// TMA store / reduce-add of a shared-memory box into the tensor at (x, y), in this thread's bulk
// group.  x * 4 bytes must be a multiple of 16.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap *map, const void *src, int x, int y) {
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.tile.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                     reinterpret_cast<uint64_t>(map)),
                 "r"(smem_addr(src)), "r"(x), "r"(y)
                 : "memory");
}
__device__ __forceinline__ void tma_reduce_add_2d(const CUtensorMap *map, const void *src, int x, int y) {
    asm volatile("cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.tile.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                     reinterpret_cast<uint64_t>(map)),
                 "r"(smem_addr(src)), "r"(x), "r"(y)
                 : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// Wait until at most one of this thread's bulk groups still reads shared memory.
__device__ __forceinline__ void bulk_wait_read_1() { asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

constexpr int kRowThreads = 128;  // threads per row of the norm kernels

// Sum of v over the block's kRowThreads threads (red: kRowThreads / 32 floats of shared memory).
__device__ __forceinline__ float block_row_sum(float v, float *red) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    float t = 0.f;
#pragma unroll
    for (int w = 0; w < kRowThreads / 32; ++w) t += red[w];
    return t;
}

// One block per row: out = fp16(x * inv * g) with inv = 1/sqrt(mean(x^2) + eps) (rmsnorm shader,
// shaders.ts:580-598), or a plain fp16 cast when gain is null.  The loads of a pass are unrolled
// so that they are in flight together.  With split-K the block also fills the row of every output
// with its bias (or the residual row, or zero) for the GEMM's reduce-adds.
__global__ void __launch_bounds__(kRowThreads) norm_cast_kernel(const float *__restrict__ x,
                                                                const float *__restrict__ gain, float eps,
                                                                int one_plus, __half *__restrict__ out, int K,
                                                                const __grid_constant__ ProjArgs pa, int fill) {
    griddep_launch_dependents();  // the GEMM may start streaming weights meanwhile
    __shared__ float red[kRowThreads / 32];
    const int row = blockIdx.x;
    const float4 *src = reinterpret_cast<const float4 *>(x + (size_t)row * K);
    const int n4 = K / 4;
    float inv = 1.f;
    if (gain) {
        float ss = 0.f;
#pragma unroll 4
        for (int c = threadIdx.x; c < n4; c += kRowThreads) {
            const float4 v = src[c];
            ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
        }
        inv = 1.f / sqrtf(block_row_sum(ss, red) / (float)K + eps);
    }
    uint2 *dst = reinterpret_cast<uint2 *>(out + (size_t)row * K);
#pragma unroll 4
    for (int c = threadIdx.x; c < n4; c += kRowThreads) {
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
    if (fill) {
        for (int i = 0; i < pa.nmat; ++i) {
            float4 *o = reinterpret_cast<float4 *>(pa.out[i] + (size_t)row * pa.n[i]);
            const float4 *b = reinterpret_cast<const float4 *>(pa.bias[i]);
            const float4 *r = i == 0 && pa.residual ? reinterpret_cast<const float4 *>(pa.residual + (size_t)row * pa.n[0])
                                                    : nullptr;
#pragma unroll 4
            for (int c = threadIdx.x; c < pa.n[i] / 4; c += kRowThreads)
                o[c] = r ? r[c] : b ? b[c] : make_float4(0.f, 0.f, 0.f, 0.f);
        }
    }
}

// h = x + rmsnorm(h) in place, one block per row (Gemma-2's post-attention norm before the
// residual, kernels.ts:1733-1734).
__global__ void __launch_bounds__(kRowThreads) post_norm_residual_kernel(float *__restrict__ h,
                                                                         const float *__restrict__ x,
                                                                         const float *__restrict__ gain, float eps,
                                                                         int one_plus, int n) {
    __shared__ float red[kRowThreads / 32];
    const int row = blockIdx.x;
    float4 *p = reinterpret_cast<float4 *>(h + (size_t)row * n);
    const float4 *xr = reinterpret_cast<const float4 *>(x + (size_t)row * n);
    const int n4 = n / 4;
    float ss = 0.f;
#pragma unroll 4
    for (int c = threadIdx.x; c < n4; c += kRowThreads) {
        const float4 v = p[c];
        ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
    }
    const float inv = 1.f / sqrtf(block_row_sum(ss, red) / (float)n + eps);
#pragma unroll 4
    for (int c = threadIdx.x; c < n4; c += kRowThreads) {
        const float4 v = p[c], r = xr[c], g = reinterpret_cast<const float4 *>(gain)[c];
        p[c] = make_float4(r.x + v.x * inv * (one_plus ? 1.f + g.x : g.x), r.y + v.y * inv * (one_plus ? 1.f + g.y : g.y),
                           r.z + v.z * inv * (one_plus ? 1.f + g.z : g.z), r.w + v.w * inv * (one_plus ? 1.f + g.w : g.w));
    }
}

template <int NTOK>
__global__ void __launch_bounds__(kPThreads, 1)
    proj_kernel(const __grid_constant__ CUtensorMap tx, const __grid_constant__ CUtensorMap tw0,
                const __grid_constant__ CUtensorMap tw1, const __grid_constant__ CUtensorMap tw2,
                const __grid_constant__ CUtensorMap to0, const __grid_constant__ CUtensorMap to1,
                const __grid_constant__ CUtensorMap to2, const __grid_constant__ ProjArgs a) {
    using L = ProjLayout<NTOK>;
    constexpr int S = L::kStages;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + L::kBarOff);
    uint64_t *empty = full + S;
    uint64_t *done = empty + S;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(done + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int tile = blockIdx.x;
    int mi = 0;
    while (mi + 1 < a.nmat && tile >= a.tile_end[mi]) ++mi;
    const int f0 = (tile - (mi ? a.tile_end[mi - 1] : 0)) * kFM;   // first feature inside matrix mi
    const int ncols = a.n[mi];
    const CUtensorMap *tw = mi == 0 ? &tw0 : mi == 1 ? &tw1 : &tw2;
    const CUtensorMap *to = mi == 0 ? &to0 : mi == 1 ? &to1 : &to2;
    const int m0 = blockIdx.y * NTOK;
    const int split = blockIdx.z, splits = gridDim.z;
    const int nk = (a.K + L::kStepK - 1) / L::kStepK;
    const int kb = split * a.kps, ke = min(nk, kb + a.kps), nks = ke - kb;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(done, 1);
        fence_barrier_init();
    }
    __syncthreads();
    // The producer starts streaming at once; the MMA warp allocates the accumulator columns
    // meanwhile and hands their address to the epilogue warps (named barrier 1, 160 threads).
    uint32_t tmem = 0;
    if (warp == kPMma) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(tmem_slot)),
                     "r"((uint32_t)NTOK)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
        tc_fence_before();
        named_barrier_sync(1, 160);
        tc_fence_after();
        tmem = *tmem_slot;
    } else if (warp < 4) {
        named_barrier_sync(1, 160);
        tc_fence_after();
        tmem = *tmem_slot;
    }

    if (warp == kPProducer) {
        if (lane == 0) {
            tma_prefetch_desc(&tx);
            tma_prefetch_desc(tw);
            // Weights do not depend on the previous kernel: start the first ring before waiting.
            const int pre = min(S, nks);
            for (int j = 0; j < pre; ++j) {
                mbar_arrive_expect_tx(&full[j], L::kStageBytes);
                for (int b = 0; b < L::kKB; ++b)
                    tma_load_2d(smem + j * L::kStageBytes + b * L::kWBox, tw, (kb + j) * L::kStepK + b * kBoxK, f0,
                                &full[j]);
            }
            griddep_wait();
            for (int j = 0; j < pre; ++j)
                for (int b = 0; b < L::kKB; ++b)
                    tma_load_2d(smem + j * L::kStageBytes + L::kWBytes + b * L::kXBox, &tx,
                                (kb + j) * L::kStepK + b * kBoxK, m0, &full[j]);
            int issued = pre;
            for (int j = pre; j < nks; ++j) {
                const int s = j % S;
                if (!mbar_wait(&empty[s], ((j / S) - 1) & 1, a.err, kErrSlotTimeout)) break;
                uint8_t *st = smem + s * L::kStageBytes;
                mbar_arrive_expect_tx(&full[s], L::kStageBytes);
                for (int b = 0; b < L::kKB; ++b) {
                    tma_load_2d(st + b * L::kWBox, tw, (kb + j) * L::kStepK + b * kBoxK, f0, &full[s]);
                    tma_load_2d(st + L::kWBytes + b * L::kXBox, &tx, (kb + j) * L::kStepK + b * kBoxK, m0, &full[s]);
                }
                issued = j + 1;
            }
            // No copy may still be in flight when the ring is reused or the CTA exits.
            for (int j = issued > S ? issued - S : 0; j < issued; ++j)
                mbar_wait(&full[j % S], (j / S) & 1, a.err, kErrTmaTimeout);
        }
        __syncwarp();
    } else if (warp == kPMma) {
        if (lane == 0) {
            constexpr uint32_t idesc = f16_idesc(kFM, NTOK, 0, 0);
            for (int j = 0; j < nks; ++j) {
                const int s = j % S;
                if (!mbar_wait(&full[s], (j / S) & 1, a.err, kErrTmaTimeout)) break;
                tc_fence_after();
                const uint32_t w_base = smem_addr(smem + s * L::kStageBytes), x_base = w_base + L::kWBytes;
#pragma unroll
                for (int b = 0; b < L::kKB; ++b)
#pragma unroll
                    for (int ks = 0; ks < kBoxK / 16; ++ks)
                        tc_mma(tmem, sw128_desc(w_base + b * L::kWBox + ks * 32, 16, 1024),
                               sw128_desc(x_base + b * L::kXBox + ks * 32, 16, 1024), idesc, j > 0 || b > 0 || ks > 0);
                tc_commit(&empty[s]);  // the stage is free once these MMAs have read it
            }
            tc_commit(done);
            mbar_wait(done, 0, a.err, kErrMmaTimeout);
        }
        __syncwarp();
    }

    // Epilogue: thread r of warps 0-3 owns feature f0 + r (TMEM lane r).  Per 32 tokens: TMEM ->
    // registers (+ bias + residual with one split) -> staging tile -> one TMA store / reduce-add.
    if (warp < 4) {
        const int r = warp * 32 + lane;
        const int feat = f0 + r;
        const int ntok = min(NTOK, a.M - m0);
        const float *__restrict__ res =
            splits == 1 && a.residual && mi == 0 ? a.residual + (size_t)m0 * ncols + feat : nullptr;
        griddep_wait();   // outputs / residual may belong to the previous kernel
        const float bias = splits == 1 && feat < ncols && a.bias[mi] ? a.bias[mi][feat] : 0.f;
        mbar_wait(done, 0, a.err, kErrMmaTimeout);
        tc_fence_after();
        const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
#pragma unroll 1
        // Every warp runs every chunk (the named barriers count all four); after a timeout the
        // error word is set and the values are meaningless.
        for (int c = 0; c < NTOK / 32 && c * 32 < ntok; ++c) {
            float *stage = reinterpret_cast<float *>(smem + (c & 1) * L::kOutTile);
            if (c >= 2 && threadIdx.x == 0) bulk_wait_read_1();  // the TMA has read this buffer
            named_barrier_sync(2, 128);
            uint32_t v[32];
            tc_ld32_nowait(tmem + lane_base + c * 32, v);
            float x[32];
#pragma unroll
            for (int e = 0; e < 32; ++e)
                x[e] = res && feat < ncols && c * 32 + e < ntok ? res[(size_t)(c * 32 + e) * ncols] : 0.f;
            tc_wait_ld();
#pragma unroll
            for (int e = 0; e < 32; ++e) stage[e * kFM + r] = __uint_as_float(v[e]) + bias + x[e];
            fence_proxy_async_smem();  // generic writes -> visible to the TMA engine
            named_barrier_sync(2, 128);
            if (threadIdx.x == 0) {
                if (splits == 1)
                    tma_store_2d(to, stage, f0, m0 + c * 32);
                else
                    tma_reduce_add_2d(to, stage, f0, m0 + c * 32);
                bulk_commit();
            }
        }
        if (threadIdx.x == 0) bulk_wait_all();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == kPMma)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"((uint32_t)NTOK) : "memory");
}

template <int NTOK>
cudaError_t configure() {
    static unsigned long long configured = 0;
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 64 && (configured & (1ull << dev))) return cudaSuccess;
    cudaError_t e = cudaFuncSetAttribute(proj_kernel<NTOK>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         ProjLayout<NTOK>::kSmemBytes);
    if (e == cudaSuccess && dev < 64) configured |= 1ull << dev;
    return e;
}

template <int NTOK>
cudaError_t launch_t(const CUtensorMap &tx, const CUtensorMap *tw, const CUtensorMap *to, const ProjArgs &a,
                     cudaStream_t s) {
    cudaError_t e = configure<NTOK>();
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a.tile_end[a.nmat - 1], (a.M + NTOK - 1) / NTOK, a.splits);
    cfg.blockDim = dim3(kPThreads);
    cfg.dynamicSmemBytes = ProjLayout<NTOK>::kSmemBytes;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, proj_kernel<NTOK>, tx, tw[0], tw[1], tw[2], to[0], to[1], to[2], a);
}

template <int NTOK>
constexpr int ctas_per_sm() {
    return ProjLayout<NTOK>::kCtasPerSm;
}

}  // namespace

int proj_token_tile(int rows) { return rows <= 32 ? 32 : rows <= 64 ? 64 : rows <= 128 ? 128 : 256; }

// Split-K plan: when the output tiles leave most CTA slots idle, split the k steps (>= 2 per split)
// over up to 8 CTAs so that about one wave of slots is busy.
void proj_plan(ProjArgs &a, int ntok, int sms) {
    const int step = ProjLayout<32>::kStepK;
    const int nk = (a.K + step - 1) / step;
    const int tiles = a.tile_end[a.nmat - 1] * ((a.M + ntok - 1) / ntok);
    const int slots = sms * (ntok == 32 ? ctas_per_sm<32>() : ntok == 64 ? ctas_per_sm<64>()
                             : ntok == 128 ? ctas_per_sm<128>() : ctas_per_sm<256>());
    int splits = 1;
    if (tiles * 2 <= slots) splits = std::min(std::min(8, slots / tiles), std::max(1, nk / 2));
    a.kps = (nk + splits - 1) / splits;
    a.splits = (nk + a.kps - 1) / a.kps;  // no empty split
}

cudaError_t launch_norm_cast(const float *x, const float *gain, float eps, int one_plus, __half *out, int rows, int K,
                             const ProjArgs &a, cudaStream_t s) {
    if (rows == 0) return cudaSuccess;
    norm_cast_kernel<<<rows, kRowThreads, 0, s>>>(x, gain, eps, one_plus, out, K, a, a.splits > 1);
    return cudaGetLastError();
}

cudaError_t launch_post_norm_residual(float *h, const float *x, const float *gain, float eps, int one_plus, int rows,
                                      int n, cudaStream_t s) {
    if (rows == 0) return cudaSuccess;
    post_norm_residual_kernel<<<rows, kRowThreads, 0, s>>>(h, x, gain, eps, one_plus, n);
    return cudaGetLastError();
}

cudaError_t launch_proj(int ntok, const CUtensorMap &tx, const CUtensorMap *tw, const CUtensorMap *to,
                        const ProjArgs &a, cudaStream_t s) {
    switch (ntok) {
        case 32: return launch_t<32>(tx, tw, to, a, s);
        case 64: return launch_t<64>(tx, tw, to, a, s);
        case 128: return launch_t<128>(tx, tw, to, a, s);
        case 256: return launch_t<256>(tx, tw, to, a, s);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace brk
