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
//   - when the output tiles cannot fill the SMs (decode), K is split over a thread-block cluster of
//     up to 8 CTAs along z; each CTA parks its partial in its own shared memory and then sums one
//     slice of the tokens over all the cluster's partials through distributed shared memory, in
//     split order (deterministic, no global workspace, no atomics);
//   - warp 4 streams [128 features][64 k] weight boxes and [tokens][64 k] activation boxes
//     through a TMA ring (128-byte swizzle, CTA-local loads); the weight loads of the first ring
//     are issued before griddepcontrol.wait, so they overlap the kernel that produced the
//     activations (programmatic dependent launch);
//   - warp 5 issues tcgen05.mma (M 128, N tokens, K 16; fp16 in, fp32 in TMEM) and commits each
//     stage back to the producer; warps 0-3 (thread r <-> feature r) drain TMEM with tcgen05.ld and
//     store f32 outputs plus bias and residual, 32 consecutive features per warp store.
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
    // The split-K partial [NTOK][128] f32 reuses the ring once the MMAs are done.
    static_assert(NTOK * kFM * 4 <= kBarOff, "partial does not fit the ring");
};

// Cluster barrier without release semantics: orders nothing, only waits for every thread of the
// cluster (so pending global stores are not drained first).
__device__ __forceinline__ void cluster_sync_relaxed() {
    asm volatile("barrier.cluster.arrive.relaxed.aligned;\n\tbarrier.cluster.wait.aligned;" ::: "memory");
}

__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Generic address of the same shared-memory location in cluster CTA `rank` (plain loads then
// read that CTA's shared memory over the cluster's distributed shared memory).
__device__ __forceinline__ const float *map_cluster_ptr(const float *p, uint32_t rank) {
    uint64_t r;
    asm volatile("mapa.u64 %0, %1, %2;" : "=l"(r) : "l"(reinterpret_cast<uint64_t>(p)), "r"(rank));
    return reinterpret_cast<const float *>(r);
}

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
// so that they are in flight together.
__global__ void __launch_bounds__(kRowThreads) norm_cast_kernel(const float *__restrict__ x,
                                                                const float *__restrict__ gain, float eps,
                                                                int one_plus, __half *__restrict__ out, int K) {
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
                const __grid_constant__ ProjArgs a) {
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

    bool ok = true;
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

    // Epilogue: thread r of warps 0-3 owns feature f0 + r (TMEM lane r).  Every load of a group
    // of tokens is issued before the first of its stores, so the latencies overlap.
    const int r = warp * 32 + lane;
    const int feat = f0 + r;
    const bool epi = warp < 4;
    const int ntok = min(NTOK, a.M - m0);
    float *__restrict__ out = a.out[mi] + (size_t)m0 * ncols + feat;
    const float *__restrict__ res = a.residual && mi == 0 ? a.residual + (size_t)m0 * ncols + feat : nullptr;
    const int per = (ntok + splits - 1) / splits;   // split-K: tokens [t0, t1) are reduced here
    const int t0 = split * per, t1 = min(ntok, t0 + per);
    float bias = 0.f;
    if (epi) {
        griddep_wait();   // outputs / residual may belong to the previous kernel
        bias = feat < ncols && a.bias[mi] ? a.bias[mi][feat] : 0.f;
        ok = __all_sync(0xffffffffu, mbar_wait(done, 0, a.err, kErrMmaTimeout));  // tcgen05.ld is warp-wide
        tc_fence_after();
    }

    const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
    if (splits == 1) {
        if (epi && ok) {
#pragma unroll 1
            for (int c = 0; c < NTOK / 32 && c * 32 < ntok; ++c) {
                uint32_t v[32];
                tc_ld32_nowait(tmem + lane_base + c * 32, v);
                float x[32];
#pragma unroll
                for (int e = 0; e < 32; ++e)
                    x[e] = res && feat < ncols && c * 32 + e < ntok ? res[(size_t)(c * 32 + e) * ncols] : 0.f;
                tc_wait_ld();
                if (feat < ncols) {
#pragma unroll
                    for (int e = 0; e < 32; ++e)
                        if (c * 32 + e < ntok) out[(size_t)(c * 32 + e) * ncols] = __uint_as_float(v[e]) + bias + x[e];
                }
            }
        }
    } else {
        // Park the partial [token][feature] in this CTA's shared memory (the ring is idle now).
        float *part = reinterpret_cast<float *>(smem);
        if (epi) {
#pragma unroll 1
            for (int c = 0; c < NTOK / 32 && c * 32 < ntok; ++c) {
                uint32_t v[32];
                tc_ld32_nowait(tmem + lane_base + c * 32, v);
                tc_wait_ld();
#pragma unroll
                for (int e = 0; e < 32; ++e) part[(c * 32 + e) * kFM + r] = ok ? __uint_as_float(v[e]) : 0.f;
            }
        }
        cluster_sync_all();
        // This CTA sums tokens [t0, t1) over every split, in split order, four tokens per step.
        // The loop body stays small: each CTA runs it once, from a cold instruction cache.
        if (epi && feat < ncols) {
            const float *src[8];
#pragma unroll
            for (int q = 0; q < 8; ++q) src[q] = map_cluster_ptr(part + r, (uint32_t)min(q, splits - 1));
#pragma unroll 1
            for (int t = t0; t < t1; t += 4) {
                float pv[8][4], x[4];
#pragma unroll
                for (int u = 0; u < 4; ++u) x[u] = res && t + u < t1 ? res[(size_t)(t + u) * ncols] : 0.f;
#pragma unroll
                for (int q = 0; q < 8; ++q)
#pragma unroll
                    for (int u = 0; u < 4; ++u) pv[q][u] = q < splits && t + u < t1 ? src[q][(t + u) * kFM] : 0.f;
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    float acc = 0.f;
#pragma unroll
                    for (int q = 0; q < 8; ++q)
                        if (q < splits) acc += pv[q][u];
                    if (t + u < t1) out[(size_t)(t + u) * ncols] = acc + bias + x[u];
                }
            }
        }
        // No CTA leaves while another still reads its shared memory.  Those reads have returned
        // their values by now, so a relaxed arrive suffices (and the output stores need not drain).
        cluster_sync_relaxed();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == kPMma)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"((uint32_t)NTOK) : "memory");
}

template <int NTOK>
const void *proj_fn() {
    return reinterpret_cast<const void *>(proj_kernel<NTOK>);
}

template <int NTOK>
cudaError_t configure() {
    static unsigned long long configured = 0;
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 64 && (configured & (1ull << dev))) return cudaSuccess;
    cudaError_t e = cudaFuncSetAttribute(proj_kernel<NTOK>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         ProjLayout<NTOK>::kSmemBytes);
    if (e == cudaSuccess) e = cudaFuncSetAttribute(proj_kernel<NTOK>, cudaFuncAttributeNonPortableClusterSizeAllowed, 0);
    if (e == cudaSuccess && dev < 64) configured |= 1ull << dev;
    return e;
}

// Clusters of `splits` CTAs that can be resident at once (0 when the query fails).
template <int NTOK>
int max_clusters(int splits, int tiles) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(tiles, 1, splits);
    cfg.blockDim = dim3(kPThreads);
    cfg.dynamicSmemBytes = ProjLayout<NTOK>::kSmemBytes;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 1;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = splits;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, proj_kernel<NTOK>, &cfg) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    return n;
}

// Split count: the largest cluster size (<= 8, <= the k steps) whose clusters for all output tiles
// are resident in one wave, when one CTA per tile would leave most CTA slots idle.
template <int NTOK>
int choose_splits(int tiles, int nk, int slots) {
    static int cache[64][9];  // [device][splits] -> resident clusters (+1; 0 = unknown)
    int dev = 0;
    cudaGetDevice(&dev);
    if (tiles * 2 > slots || nk < 4) return 1;
    int best = 1;
    for (int s = 2; s <= 8 && s * 2 <= nk; ++s) {
        if (tiles * s > slots) break;
        int n;
        if (dev < 64 && cache[dev][s]) {
            n = cache[dev][s] - 1;
        } else {
            n = max_clusters<NTOK>(s, tiles);
            if (dev < 64) cache[dev][s] = n + 1;
        }
        if (n >= tiles) best = s;
    }
    return best;
}

template <int NTOK>
cudaError_t launch_t(const CUtensorMap &tx, const CUtensorMap *tw, ProjArgs a, int sms, cudaStream_t s) {
    cudaError_t e = configure<NTOK>();
    if (e != cudaSuccess) return e;
    const int tiles = a.tile_end[a.nmat - 1];
    const int nk = (a.K + ProjLayout<NTOK>::kStepK - 1) / ProjLayout<NTOK>::kStepK;
    int splits = choose_splits<NTOK>(tiles * ((a.M + NTOK - 1) / NTOK), nk, sms * ProjLayout<NTOK>::kCtasPerSm);
    a.kps = (nk + splits - 1) / splits;
    splits = (nk + a.kps - 1) / a.kps;  // no empty split
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(tiles, (a.M + NTOK - 1) / NTOK, splits);
    cfg.blockDim = dim3(kPThreads);
    cfg.dynamicSmemBytes = ProjLayout<NTOK>::kSmemBytes;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = 1;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = splits;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    return cudaLaunchKernelEx(&cfg, proj_kernel<NTOK>, tx, tw[0], tw[1], tw[2], a);
}

}  // namespace

int proj_token_tile(int rows) { return rows <= 32 ? 32 : rows <= 64 ? 64 : rows <= 128 ? 128 : 256; }

cudaError_t launch_norm_cast(const float *x, const float *gain, float eps, int one_plus, __half *out, int rows, int K,
                             cudaStream_t s) {
    if (rows == 0) return cudaSuccess;
    norm_cast_kernel<<<rows, kRowThreads, 0, s>>>(x, gain, eps, one_plus, out, K);
    return cudaGetLastError();
}

cudaError_t launch_post_norm_residual(float *h, const float *x, const float *gain, float eps, int one_plus, int rows,
                                      int n, cudaStream_t s) {
    if (rows == 0) return cudaSuccess;
    post_norm_residual_kernel<<<rows, kRowThreads, 0, s>>>(h, x, gain, eps, one_plus, n);
    return cudaGetLastError();
}

cudaError_t launch_proj(int ntok, const CUtensorMap &tx, const CUtensorMap *tw, const ProjArgs &a, int sms,
                        cudaStream_t s) {
    switch (ntok) {
        case 32: return launch_t<32>(tx, tw, a, sms, s);
        case 64: return launch_t<64>(tx, tw, a, sms, s);
        case 128: return launch_t<128>(tx, tw, a, sms, s);
        case 256: return launch_t<256>(tx, tw, a, sms, s);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace brk
