// Chunked causal prefill attention on the 5th-generation tensor cores (tcgen05 + TMEM).
//
// Replaces the reference's 2-pass thread-per-(token, head) `attention` kernel
// (shaders.ts:1482-1524) that recAttention dispatches for prefill chunks (kernels.ts:1634-1638).
//
// One CTA per (128-query tile, q head, sequence); keys stream in 128-key tiles from the fp16
// cache.  Roles (192 threads):
//   warps 0-3  softmax / epilogue: thread r owns query row r (TMEM lane r);
//   warp 4     TMA producer: K and V tiles (128-byte swizzled [keys][64] boxes, CTA-local loads)
//              into a 2-stage ring;
//   warp 5     TMEM allocator and MMA issuer (one elected lane).
// Per key tile j: S_j = Q K_j^T (M 128, N 128, fp16 -> fp32 in TMEM, double-buffered), the
// softmax warps read S_j, apply the causal / window mask, scale and online-softmax, write
// P_j = exp(S_j - m) as fp16 to shared memory, and the MMA warp issues O_j = P_j V_j into a
// TMEM tile that the softmax warps fold into their register accumulator o = o*alpha + O_j.
// S_{j+1} is computed while the softmax warps work on S_j.
#include <math_constants.h>

#include "common.cuh"
#include "internal.h"

namespace brk {

namespace {

constexpr int kTQ = 128;  // queries per CTA (the MMA's M)
constexpr int kTK = 128;  // keys per tile (N of QK^T, K of PV)
constexpr int kSoftmaxWarps = 4;
constexpr int kProducerWarp = 4;
constexpr int kMmaWarp = 5;
constexpr int kThreads = 6 * 32;
constexpr uint32_t kTmemCols = 512;  // S0 | S1 | O tile | unused
constexpr float kLn2f = 0.6931471805599453f;

template <int D>
struct PrefillLayout {
    static constexpr int kBlocks = D / 64;
    static constexpr uint32_t kQBlock = kTQ * 128;          // [128 rows][64] fp16 block
    static constexpr uint32_t kKVBlock = kTK * 128;
    static constexpr uint32_t kQBytes = kBlocks * kQBlock;
    static constexpr uint32_t kTileBytes = kBlocks * kKVBlock;  // one K (or V) tile
    static constexpr uint32_t kPBytes = 2 * kTQ * 128;          // [128 rows][128 keys] fp16
    static constexpr uint32_t kOffQ = 0;
    static constexpr uint32_t kOffK0 = kOffQ + kQBytes;
    static constexpr uint32_t kOffV0 = kOffK0 + kTileBytes;
    static constexpr uint32_t kOffK1 = kOffV0 + kTileBytes;
    static constexpr uint32_t kOffV1 = kOffK1 + kTileBytes;
    static constexpr uint32_t kOffP = kOffV1 + kTileBytes;
    static constexpr uint32_t kOffBar = kOffP + kPBytes;
    static constexpr uint32_t kNumBars = 16;
    static constexpr uint32_t kSmemBytes = 1024 + kOffBar + kNumBars * 8 + 16;
};

// Barrier slots.
enum : int {
    kBarKFull = 0,    // [2] TMA -> MMA
    kBarVFull = 2,    // [2] TMA -> MMA (and the softmax warps on the last tile)
    kBarKvEmpty = 4,  // [2] MMA commit -> producer
    kBarSFull = 6,    // [2] MMA commit -> softmax
    kBarSFree = 8,    // [2] softmax -> MMA
    kBarQFull = 10,   // softmax (q staged) -> MMA
    kBarPFull = 11,   // softmax (P written) -> MMA
    kBarOFull = 12,   // MMA commit (O tile ready, P consumed) -> softmax
    kBarOFree = 13,   // softmax (O tile read) -> MMA
    kBarMmaDone = 14, // MMA commit of everything -> teardown
};

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tc_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
                 : "memory");
}

// D[tmem] (+)= A[smem desc] * B[smem desc], kind::f16 (fp16 inputs, fp32 accumulators).
__device__ __forceinline__ void tc_mma(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                       bool accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"((uint32_t)accumulate)
        : "memory");
}

// 32 consecutive 32-bit TMEM columns of this thread's lane.
__device__ __forceinline__ void tc_ld32(uint32_t taddr, float (&v)[32]) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
          "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
          "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// Shared-memory matrix descriptor, 128-byte swizzle, sm_100 version field.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t addr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
    return (uint64_t)((addr >> 4) & 0x3FFFu) | ((uint64_t)((lbo_bytes >> 4) & 0x3FFFu) << 16) |
           ((uint64_t)((sbo_bytes >> 4) & 0x3FFFu) << 32) | (1ull << 46) | (2ull << 61);
}

// Instruction descriptor of kind::f16: fp16 A and B, fp32 D, M x N, operand majors.
__host__ __device__ constexpr uint32_t f16_idesc(int M, int N, int a_mn_major, int b_mn_major) {
    return (1u << 4) | ((uint32_t)a_mn_major << 15) | ((uint32_t)b_mn_major << 16) | ((uint32_t)(N >> 3) << 17) |
           ((uint32_t)(M >> 4) << 24);
}

template <int D>
__global__ void __launch_bounds__(kThreads, 1)
    prefill_attn_kernel(const __grid_constant__ CUtensorMap tmk, const __grid_constant__ CUtensorMap tmv,
                        const __grid_constant__ PrefillArgs a) {
    using L = PrefillLayout<D>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + L::kOffBar);
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + L::kOffBar + L::kNumBars * 8);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int h = blockIdx.x;
    const int qt = gridDim.y - 1 - blockIdx.y;  // heaviest (latest) query tiles first
    const int b = blockIdx.z;
    const int G = a.Hq / a.Hkv, kvh = h / G;
    const int T = a.T;
    const int q0 = qt * kTQ;
    const int past = a.past_len[b];
    const int nq = min(kTQ, T - q0);  // valid query rows of this tile

    // Key range (cache rows) of the whole tile: causal up to the last query, window from the first.
    int khi = past + q0 + nq - a.kv_offset;
    if (khi > a.cap) khi = a.cap;
    int klo = 0;
    if (a.window > 0) klo = max(0, past + q0 - a.window + 1 - a.kv_offset);
    const int nk = khi > klo ? (khi - klo + kTK - 1) / kTK : 0;
    const int seg_row = ((a.layer * a.B + b) * a.Hkv + kvh) * a.cap;

    if (threadIdx.x == 0) {
        for (int i = 0; i < 2; ++i) {
            mbar_init(&bars[kBarKFull + i], 1);
            mbar_init(&bars[kBarVFull + i], 1);
            mbar_init(&bars[kBarKvEmpty + i], 1);
            mbar_init(&bars[kBarSFull + i], 1);
            mbar_init(&bars[kBarSFree + i], kSoftmaxWarps * 32);
        }
        mbar_init(&bars[kBarQFull], kSoftmaxWarps * 32);
        mbar_init(&bars[kBarPFull], kSoftmaxWarps * 32);
        mbar_init(&bars[kBarOFull], 1);
        mbar_init(&bars[kBarOFree], kSoftmaxWarps * 32);
        mbar_init(&bars[kBarMmaDone], 1);
        fence_barrier_init();
    }
    if (warp == kMmaWarp) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(tmem_slot)),
                     "r"(kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const uint32_t tS0 = tmem, tO = tmem + 2 * kTK;

    uint8_t *sQ = smem + L::kOffQ;
    uint8_t *sP = smem + L::kOffP;
    uint8_t *sK[2] = {smem + L::kOffK0, smem + L::kOffK1};
    uint8_t *sV[2] = {smem + L::kOffV0, smem + L::kOffV1};

    if (warp == kProducerWarp) {
        if (lane == 0 && nk > 0) {
            tma_prefetch_desc(&tmk);
            tma_prefetch_desc(&tmv);
            int issued = 0;
            for (int j = 0; j < nk; ++j) {
                const int st = j & 1;
                if (j >= 2 && !mbar_wait(&bars[kBarKvEmpty + st], ((j >> 1) - 1) & 1, a.err, kErrSlotTimeout)) break;
                const int y = seg_row + klo + j * kTK;
                mbar_arrive_expect_tx(&bars[kBarKFull + st], L::kTileBytes);
#pragma unroll
                for (int blk = 0; blk < L::kBlocks; ++blk)
                    tma_load_2d(sK[st] + blk * L::kKVBlock, &tmk, blk * 64, y, &bars[kBarKFull + st]);
                mbar_arrive_expect_tx(&bars[kBarVFull + st], L::kTileBytes);
#pragma unroll
                for (int blk = 0; blk < L::kBlocks; ++blk)
                    tma_load_2d(sV[st] + blk * L::kKVBlock, &tmv, blk * 64, y, &bars[kBarVFull + st]);
                issued = j + 1;
            }
            for (int j = issued > 2 ? issued - 2 : 0; j < issued; ++j) {
                mbar_wait(&bars[kBarKFull + (j & 1)], (j >> 1) & 1, a.err, kErrTmaTimeout);
                mbar_wait(&bars[kBarVFull + (j & 1)], (j >> 1) & 1, a.err, kErrTmaTimeout);
            }
        }
        __syncwarp();
    } else if (warp == kMmaWarp) {
        if (lane == 0) {
            constexpr uint32_t idesc_qk = f16_idesc(kTQ, kTK, 0, 0);
            constexpr uint32_t idesc_pv = f16_idesc(kTQ, D, 0, 1);
            bool ok = nk > 0 && mbar_wait(&bars[kBarQFull], 0, a.err, kErrMmaTimeout);
            tc_fence_after();
            auto issue_pv = [&](int i) -> bool {
                const int st = i & 1;
                if (!mbar_wait(&bars[kBarPFull], i & 1, a.err, kErrMmaTimeout)) return false;
                if (!mbar_wait(&bars[kBarVFull + st], (i >> 1) & 1, a.err, kErrTmaTimeout)) return false;
                if (i >= 1 && !mbar_wait(&bars[kBarOFree], (i - 1) & 1, a.err, kErrMmaTimeout)) return false;
                tc_fence_after();
                const uint32_t p_base = smem_addr(sP), v_base = smem_addr(sV[st]);
#pragma unroll
                for (int kk = 0; kk < kTK / 16; ++kk) {
                    const uint64_t ad = sw128_desc(p_base + (kk >> 2) * (kTQ * 128) + (kk & 3) * 32, 16, 1024);
                    const uint64_t bd = sw128_desc(v_base + kk * 16 * 128, L::kKVBlock, 1024);
                    tc_mma(tO, ad, bd, idesc_pv, kk > 0);
                }
                tc_commit(&bars[kBarOFull]);
                tc_commit(&bars[kBarKvEmpty + st]);
                return true;
            };
            for (int j = 0; ok && j < nk; ++j) {
                const int st = j & 1;
                if (!mbar_wait(&bars[kBarKFull + st], (j >> 1) & 1, a.err, kErrTmaTimeout)) break;
                if (j >= 2 && !mbar_wait(&bars[kBarSFree + st], ((j >> 1) - 1) & 1, a.err, kErrMmaTimeout)) break;
                tc_fence_after();
                const uint32_t q_base = smem_addr(sQ), k_base = smem_addr(sK[st]);
#pragma unroll
                for (int ks = 0; ks < D / 16; ++ks) {
                    const uint64_t ad = sw128_desc(q_base + (ks >> 2) * L::kQBlock + (ks & 3) * 32, 16, 1024);
                    const uint64_t bd = sw128_desc(k_base + (ks >> 2) * L::kKVBlock + (ks & 3) * 32, 16, 1024);
                    tc_mma(tS0 + st * kTK, ad, bd, idesc_qk, ks > 0);
                }
                tc_commit(&bars[kBarSFull + st]);
                if (j >= 1 && !issue_pv(j - 1)) {
                    ok = false;
                    break;
                }
            }
            if (ok && nk > 0) issue_pv(nk - 1);
            // Every MMA this thread issued must finish before TMEM is released.
            tc_commit(&bars[kBarMmaDone]);
            mbar_wait(&bars[kBarMmaDone], 0, a.err, kErrMmaTimeout);
        }
        __syncwarp();
    } else {
        // ---- softmax warps: thread r <-> query row r.
        const int r = threadIdx.x;
        const int t = q0 + r;
        const bool row_ok = r < nq;
        // Stage q row r as fp16 in the 128-byte swizzled K-major layout of the MMA's A operand.
        {
            const float *src = a.q + (((size_t)b * T + (row_ok ? t : 0)) * a.Hq + h) * D;
#pragma unroll
            for (int c = 0; c < D / 8; ++c) {
                float4 x0 = make_float4(0.f, 0.f, 0.f, 0.f), x1 = x0;
                if (row_ok) {
                    x0 = *reinterpret_cast<const float4 *>(src + c * 8);
                    x1 = *reinterpret_cast<const float4 *>(src + c * 8 + 4);
                }
                uint4 pk;
                pk.x = pack_half2(x0.x, x0.y);
                pk.y = pack_half2(x0.z, x0.w);
                pk.z = pack_half2(x1.x, x1.y);
                pk.w = pack_half2(x1.z, x1.w);
                *reinterpret_cast<uint4 *>(sQ + (c >> 3) * L::kQBlock + sw128(r, c & 7)) = pk;
            }
            fence_proxy_async_smem();
            mbar_arrive(&bars[kBarQFull]);
        }
        const int pos = past + t;                         // absolute position of this query
        const int hi = row_ok ? pos - a.kv_offset : -1;   // last key (cache row) it attends
        const int lo = a.window > 0 ? pos - a.window + 1 - a.kv_offset : INT_MIN;
        const bool use_cap = a.softcap > 0.f;
        const uint32_t lane_base = (uint32_t)(warp * 32) << 16;

        float o[D];
#pragma unroll
        for (int d = 0; d < D; ++d) o[d] = 0.f;
        float m_run = -CUDART_INF_F, l_run = 0.f, alpha_prev = 1.f;
        bool ok = true;
        for (int j = 0; j < nk; ++j) {
            const int st = j & 1;
            const int kbase = klo + j * kTK;
            if (!mbar_wait(&bars[kBarSFull + st], (j >> 1) & 1, a.err, kErrMmaTimeout)) {
                ok = false;
                break;
            }
            tc_fence_after();
            const uint32_t ts = tS0 + st * kTK + lane_base;
            // Pass 1: masked, scaled scores (log2 units) -> tile row max.
            float mx = -CUDART_INF_F;
#pragma unroll
            for (int c = 0; c < kTK / 32; ++c) {
                float v[32];
                tc_ld32(ts + c * 32, v);
#pragma unroll
                for (int e = 0; e < 32; ++e) {
                    const int key = kbase + c * 32 + e;
                    float x = v[e];
                    if (use_cap) {
                        const float e2z = exp2f(x * a.cap_k1);
                        x = a.cap_k2 * (1.f - 2.f * __frcp_rn(1.f + e2z));
                    } else {
                        x *= a.scale_log2;
                    }
                    x = (key <= hi && key >= lo && key < khi) ? x : -CUDART_INF_F;
                    mx = fmaxf(mx, x);
                }
            }
            const float m_new = fmaxf(m_run, mx);
            const float m_use = m_new == -CUDART_INF_F ? 0.f : m_new;
            const float alpha = exp2f(m_run - m_use);
            m_run = m_new;
            // Fold the previous tile's PV result; afterwards P may be overwritten.
            if (j >= 1) {
                if (!mbar_wait(&bars[kBarOFull], (j - 1) & 1, a.err, kErrMmaTimeout)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
#pragma unroll
                for (int c = 0; c < D / 32; ++c) {
                    float v[32];
                    tc_ld32(tO + lane_base + c * 32, v);
#pragma unroll
                    for (int e = 0; e < 32; ++e) o[c * 32 + e] = o[c * 32 + e] * alpha_prev + v[e];
                }
                tc_fence_before();
                mbar_arrive(&bars[kBarOFree]);
            }
            // Pass 2: P = exp2(s - m) as fp16 into shared memory (K-major, swizzled), row sums.
            float rsum = 0.f;
#pragma unroll
            for (int c = 0; c < kTK / 32; ++c) {
                float v[32];
                tc_ld32(ts + c * 32, v);
                uint32_t pk[16];
#pragma unroll
                for (int e = 0; e < 32; e += 2) {
                    float pe[2];
#pragma unroll
                    for (int u = 0; u < 2; ++u) {
                        const int key = kbase + c * 32 + e + u;
                        float x = v[e + u];
                        if (use_cap) {
                            const float e2z = exp2f(x * a.cap_k1);
                            x = a.cap_k2 * (1.f - 2.f * __frcp_rn(1.f + e2z));
                        } else {
                            x *= a.scale_log2;
                        }
                        const bool valid = key <= hi && key >= lo && key < khi;
                        pe[u] = valid ? exp2f(x - m_use) : 0.f;
                        rsum += pe[u];
                    }
                    pk[e >> 1] = pack_half2(pe[0], pe[1]);
                }
#pragma unroll
                for (int q4 = 0; q4 < 4; ++q4) {
                    const int chunk = c * 4 + q4;  // 16-byte chunk over the 128 keys
                    *reinterpret_cast<uint4 *>(sP + (chunk >> 3) * (kTQ * 128) + sw128(r, chunk & 7)) =
                        make_uint4(pk[q4 * 4], pk[q4 * 4 + 1], pk[q4 * 4 + 2], pk[q4 * 4 + 3]);
                }
            }
            tc_fence_before();
            mbar_arrive(&bars[kBarSFree + st]);
            // Keys past the range end: zero their V rows so that 0 * (stale data) stays 0.
            if (kbase + kTK > khi) {
                if (!mbar_wait(&bars[kBarVFull + st], (j >> 1) & 1, a.err, kErrTmaTimeout)) {
                    ok = false;
                    break;
                }
                if (kbase + r >= khi) {
#pragma unroll
                    for (int blk = 0; blk < L::kBlocks; ++blk)
#pragma unroll
                        for (int c = 0; c < 8; ++c)
                            *reinterpret_cast<uint4 *>(sV[st] + blk * L::kKVBlock + sw128(r, c)) =
                                make_uint4(0u, 0u, 0u, 0u);
                }
            }
            fence_proxy_async_smem();
            mbar_arrive(&bars[kBarPFull]);
            l_run = l_run * alpha + rsum;
            alpha_prev = alpha;
        }
        if (ok && nk > 0) {
            if (mbar_wait(&bars[kBarOFull], (nk - 1) & 1, a.err, kErrMmaTimeout)) {
                tc_fence_after();
#pragma unroll
                for (int c = 0; c < D / 32; ++c) {
                    float v[32];
                    tc_ld32(tO + lane_base + c * 32, v);
#pragma unroll
                    for (int e = 0; e < 32; ++e) o[c * 32 + e] = o[c * 32 + e] * alpha_prev + v[e];
                }
                if (row_ok) {
                    const float inv = 1.f / l_run;
                    float *dst = a.out + (((size_t)b * T + t) * a.Hq + h) * D;
#pragma unroll
                    for (int d = 0; d < D; d += 4)
                        *reinterpret_cast<float4 *>(dst + d) =
                            make_float4(o[d] * inv, o[d + 1] * inv, o[d + 2] * inv, o[d + 3] * inv);
                }
            }
        }
        (void)kLn2f;
    }

    // Teardown: every TMEM read and MMA is complete; the allocating warp releases TMEM.
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == kMmaWarp)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
}

template <int D>
cudaError_t launch_prefill_t(const CUtensorMap &tmk, const CUtensorMap &tmv, const PrefillArgs &a, cudaStream_t s) {
    static unsigned long long configured = 0;
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 64 || !(configured & (1ull << dev))) {
        cudaError_t e = cudaFuncSetAttribute(prefill_attn_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             PrefillLayout<D>::kSmemBytes);
        if (e != cudaSuccess) return e;
        if (dev < 64) configured |= 1ull << dev;
    }
    const dim3 grid(a.Hq, (a.T + kTQ - 1) / kTQ, a.B);
    prefill_attn_kernel<D><<<grid, kThreads, PrefillLayout<D>::kSmemBytes, s>>>(tmk, tmv, a);
    return cudaGetLastError();
}

}  // namespace

cudaError_t launch_prefill(int head_dim, const CUtensorMap &tmk, const CUtensorMap &tmv, const PrefillArgs &a,
                           cudaStream_t s) {
    switch (head_dim) {
        case 64: return launch_prefill_t<64>(tmk, tmv, a, s);
        case 128: return launch_prefill_t<128>(tmk, tmv, a, s);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace brk
