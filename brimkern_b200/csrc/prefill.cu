// Chunked causal prefill attention on the 5th-generation tensor cores (tcgen05 + TMEM).
//
// Replaces the reference's 2-pass thread-per-(token, head) `attention` kernel
// (shaders.ts:1482-1524) that recAttention dispatches for prefill chunks (kernels.ts:1634-1638).
//
// One CTA runs two query streams that share every K/V tile: two q heads of the same kv head
// (even group size) or two consecutive 128-query tiles of one head (odd group size).  Roles
// (352 threads):
//   warps 0-3 / 4-7  softmax warpgroup of stream 0 / 1: thread r owns query row r (TMEM lane r);
//   warp 8           TMA producer: 64-key K and V tiles (128-byte swizzled [keys][64] boxes,
//                    CTA-local loads) into a 4-stage (D 64: 6-stage) ring;
//   warp 9 / 10      MMA issuer of stream 0 / 1 (one lane each); warp 9 also allocates TMEM.
// Per 64-key tile j and stream s: S_s = Q_s K_j^T (tcgen05.mma, M 128, N 64, fp16 -> fp32 in
// TMEM); the stream's warpgroup reads S_s once, masks (causal offset pastLen, window) only on
// boundary tiles, and writes P_s = exp2(s - m) as fp16 pairs into TMEM; the MMA warp
// accumulates O_s += P_s V_j in TMEM with P_s as the MMA's TMEM A operand.  The running max m is only raised (and O_s rescaled in
// TMEM) when a tile's max exceeds it by more than 2^8, so P stays <= 256 and rescaling is rare.
// The tensor core alternates between the streams: while one warpgroup works on its scores the
// other stream's MMAs run.  Stream 1 starts one tile late, which keeps the two warpgroups'
// exponential phases (MUFU-bound) apart.
#include <math_constants.h>

#include "common.cuh"
#include "internal.h"
#include "tcgen05.cuh"

namespace brk {

namespace {

constexpr int kTQ = kPrefillQRows;  // queries per stream (the MMA's M)
constexpr int kTK = 64;        // keys per tile (N of QK^T, K of PV)
constexpr int kProducerWarp = 8;
constexpr int kMmaWarp = 9;   // stream 0's MMA issuer (and the TMEM allocator)
constexpr int kMmaWarp1 = 10; // stream 1's MMA issuer
constexpr int kThreads = 11 * 32;
constexpr uint32_t kTmemCols = 512;  // S0 | S1 | O0 | O1
// Raise the running max (and rescale O) only when a tile's max exceeds it by more than 2^8.
constexpr float kRescaleLog2 = 8.f;
// Of every 8 pairs of a row's probabilities, this many take 2^x on the FMA pipe (ex2_poly2)
// instead of the MUFU unit, which the exponentials otherwise saturate.
constexpr int kPolyPairsPer8 = 2;

template <int D>
struct PrefillLayout {
    // K/V ring depth: TMA latency under a full chip (~2.7k cycles) exceeds one 64-key tile
    // period, so the ring keeps more tiles in flight (D 128: all the shared memory left).
    static constexpr int kStages = D == 64 ? 6 : 4;
    static constexpr int kBlocks = D / 64;
    static constexpr uint32_t kQBlock = kTQ * 128;             // [128 rows][64] fp16
    static constexpr uint32_t kKVBlock = kTK * 128;            // [64 keys][64] fp16
    static constexpr uint32_t kQBytes = kBlocks * kQBlock;     // one stream's q
    static constexpr uint32_t kTileBytes = kBlocks * kKVBlock; // one K (or V) tile
    static constexpr uint32_t kOffQ = 0;                       // 2 streams
    static constexpr uint32_t kOffKV = 2 * kQBytes;            // kStages x (K, V)
    static_assert(kStages <= 6, "barrier slots");
    static constexpr uint32_t kOffBar = kOffKV + kStages * 2 * kTileBytes;
    static constexpr uint32_t kNumBars = 25;
    static constexpr uint32_t kSmemBytes = 1024 + kOffBar + kNumBars * 8 + 16;
    static_assert(kSmemBytes <= 232448, "more than 227 KB of shared memory per CTA");
    // TMEM columns: S_s (f32) at s * 64, O_s (f32) at 128 + s * D, P_s (fp16 pairs) at 128 + 2D + s * 32.
    static constexpr uint32_t kColS = 0, kColO = 2 * kTK, kColP = 2 * kTK + 2 * D;
    static_assert(kColP + 2 * kTK / 2 <= kTmemCols, "TMEM columns");
};

// Barrier slots.
enum : int {
    kBarKvFull = 0,   // [kStages] TMA -> MMA
    kBarKvEmpty = 6,  // [kStages] MMA commit -> producer
    kBarSFull = 12,   // [2] MMA commit (S_s ready) -> softmax s
    kBarSFree = 14,   // [2] softmax s (S_s read) -> MMA
    kBarPFull = 16,   // [2] softmax s (P_s written, O_s rescaled) -> MMA
    kBarODone = 18,   // [2] MMA commit (PV_s done: P_s free, O_s stable) -> softmax s
    kBarQFull = 20,   // stream 0's q staged (by all eight softmax warps) -> MMA
    kBarMmaDone = 21, // [2] everything an issuer issued has completed -> teardown
    kBarStagger = 23, // stream 0's first P written -> stream 1's issuer starts
    kBarQFull1 = 24,  // stream 1's q staged -> MMA
};

// Score in log2 units from a raw q.k dot product (monotonic, so maxima commute with it).
template <bool CAP>
__device__ __forceinline__ float score_log2(float dot, const PrefillArgs &a) {
    if constexpr (CAP) {
        return softcap_log2(dot, a.cap_k1, a.cap_k2);
    } else {
        return dot * a.scale_log2;
    }
}

template <int D, bool CAP>
__global__ void __launch_bounds__(kThreads, 1)
    prefill_attn_kernel(const __grid_constant__ CUtensorMap tmk, const __grid_constant__ CUtensorMap tmv,
                        const __grid_constant__ CUtensorMap tmq,
                        const __grid_constant__ PrefillArgs a) {
    using L = PrefillLayout<D>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + L::kOffBar);
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + L::kOffBar + L::kNumBars * 8);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int G = a.Hq / a.Hkv;
    const int T = a.T;
    const int b = blockIdx.y;
    const int past = a.past_len[b];
    const int ntq = (T + kTQ - 1) / kTQ;
    // Streams: two heads of one kv group sharing a query tile, or (odd group) two query tiles of
    // one head.  Heaviest (latest) query tiles are scheduled first: the tile index is the grid's
    // slowest dimension (blocks start in x, y, z order), so every sequence's heaviest tiles
    // start before any lighter tile.
    const bool pair_heads = G % 2 == 0;
    const int head0 = pair_heads ? 2 * (int)blockIdx.x : (int)blockIdx.x;
    const int head1 = pair_heads ? head0 + 1 : head0;
    const int q00 = pair_heads ? (ntq - 1 - (int)blockIdx.z) * kTQ : 2 * ((ntq + 1) / 2 - 1 - (int)blockIdx.z) * kTQ;
    const int q01 = pair_heads ? q00 : q00 + kTQ;
    const int kvh = head0 / G;
    const int nq0 = max(0, min(kTQ, T - q00)), nq1 = max(0, min(kTQ, T - q01));
    const bool active1 = nq1 > 0;
    // Key range (cache rows) of the CTA: causal up to its last query, window from its first.
    const int q_last = (active1 ? q01 + nq1 : q00 + nq0) - 1;
    int khi = past + q_last + 1 - a.kv_offset;
    if (khi > a.cap) khi = a.cap;
    int klo = 0;
    if (a.window > 0) klo = max(0, past + q00 - a.window + 1 - a.kv_offset);
    const int nk = khi > klo ? (khi - klo + kTK - 1) / kTK : 0;
    const int seg_row = ((a.layer * a.B + b) * a.Hkv + kvh) * a.cap;

    if (threadIdx.x == 0) {
        for (int i = 0; i < L::kStages; ++i) {
            mbar_init(&bars[kBarKvFull + i], 1);
            mbar_init(&bars[kBarKvEmpty + i], active1 ? 2 : 1);  // one commit per MMA issuer
        }
        for (int s = 0; s < 2; ++s) {
            mbar_init(&bars[kBarSFull + s], 1);
            mbar_init(&bars[kBarSFree + s], 128);
            mbar_init(&bars[kBarPFull + s], 128);
            mbar_init(&bars[kBarODone + s], 1);
        }
        // q by TMA: the producer's one arrival with the copy's bytes; else all eight softmax warps.
        mbar_init(&bars[kBarQFull], a.q_tma ? 1 : 256);
        mbar_init(&bars[kBarQFull1], a.q_tma ? 1 : 256);
        mbar_init(&bars[kBarMmaDone], 1);
        mbar_init(&bars[kBarMmaDone + 1], 1);
        mbar_init(&bars[kBarStagger], 128);
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

    auto sQ = [&](int s) { return smem + L::kOffQ + s * L::kQBytes; };
    auto sK = [&](int st) { return smem + L::kOffKV + st * 2 * L::kTileBytes; };
    auto sV = [&](int st) { return smem + L::kOffKV + st * 2 * L::kTileBytes + L::kTileBytes; };

    if (warp == kProducerWarp) {
        if (lane == 0 && nk > 0) {
            tma_prefetch_desc(&tmk);
            tma_prefetch_desc(&tmv);
            if (a.q_tma) tma_prefetch_desc(&tmq);
            // Launched right behind the append of this chunk's K/V (programmatic dependent launch,
            // scheduled once the append has waited for its own predecessors, so the q projection
            // the prologue reads is complete): only these cache reads (and the rotated q the append
            // wrote) wait for the append.
            griddep_wait();
            if (a.q_tma) {
                // Both streams' q tiles: [128 tokens][64 dims] fp16 boxes of the [B*T][Hq*D] rows,
                // 128-byte swizzled -- the MMA's K-major A layout.  Rows past the chunk's end read
                // the next sequence's q (or zeros past the last): rows the softmax never writes.
#pragma unroll 1
                for (int sg = 0; sg < (active1 ? 2 : 1); ++sg) {
                    uint64_t *qb = &bars[sg ? kBarQFull1 : kBarQFull];
                    const int hs = sg ? head1 : head0, qs0 = sg ? q01 : q00;
                    mbar_arrive_expect_tx(qb, L::kQBytes);
#pragma unroll
                    for (int blk = 0; blk < L::kBlocks; ++blk)
                        tma_load_2d(sQ(sg) + blk * L::kQBlock, &tmq, hs * D + blk * 64, b * T + qs0, qb);
                }
            }
            int issued = 0;
            for (int j = 0; j < nk; ++j) {
                const int st = j % L::kStages;
                if (j >= L::kStages &&
                    !mbar_wait(&bars[kBarKvEmpty + st], ((j / L::kStages) - 1) & 1, a.err, kErrSlotTimeout))
                    break;
                const int y = seg_row + klo + j * kTK;
                mbar_arrive_expect_tx(&bars[kBarKvFull + st], 2 * L::kTileBytes);
#pragma unroll
                for (int blk = 0; blk < L::kBlocks; ++blk) {
                    tma_load_2d(sK(st) + blk * L::kKVBlock, &tmk, blk * 64, y, &bars[kBarKvFull + st]);
                    tma_load_2d(sV(st) + blk * L::kKVBlock, &tmv, blk * 64, y, &bars[kBarKvFull + st]);
                }
                issued = j + 1;
            }
            for (int j = issued > L::kStages ? issued - L::kStages : 0; j < issued; ++j)
                mbar_wait(&bars[kBarKvFull + j % L::kStages], (j / L::kStages) & 1, a.err, kErrTmaTimeout);
        }
        __syncwarp();
    } else if (warp == kMmaWarp || warp == kMmaWarp1) {
        // One issuing thread per stream: each stream's S and PV MMAs go out as soon as that
        // stream's softmax allows, independent of the other stream.
        const int s = warp - kMmaWarp;
        if (lane == 0 && nk > 0 && (s == 0 || active1)) {
            constexpr uint32_t idesc_qk = f16_idesc(kTQ, kTK, 0, 0);
            constexpr uint32_t idesc_pv = f16_idesc(kTQ, D, 0, 1);
            // Stream 0's softmax zeroes V rows past the key range in the last tile; stream 1's
            // PV of that tile waits for it too.
            const bool tail = klo + nk * kTK > khi;
            bool ok = mbar_wait(&bars[s ? kBarQFull1 : kBarQFull], 0, a.err, kErrMmaTimeout);
            auto issue_s = [&](int j) -> bool {
                const int st = j % L::kStages;
                if (!mbar_wait(&bars[kBarKvFull + st], (j / L::kStages) & 1, a.err, kErrTmaTimeout)) return false;
                if (j >= 1 && !mbar_wait(&bars[kBarSFree + s], (j - 1) & 1, a.err, kErrMmaTimeout)) return false;
                tc_fence_after();
                const uint32_t q_base = smem_addr(sQ(s)), k_base = smem_addr(sK(st));
#pragma unroll
                for (int ks = 0; ks < D / 16; ++ks) {
                    const uint64_t ad = sw128_desc(q_base + (ks >> 2) * L::kQBlock + (ks & 3) * 32, 16, 1024);
                    const uint64_t bd = sw128_desc(k_base + (ks >> 2) * L::kKVBlock + (ks & 3) * 32, 16, 1024);
                    tc_mma(tmem + L::kColS + s * kTK, ad, bd, idesc_qk, ks > 0);
                }
                tc_commit(&bars[kBarSFull + s]);
                return true;
            };
            auto issue_pv = [&](int j) -> bool {
                const int st = j % L::kStages;
                if (!mbar_wait(&bars[kBarPFull + s], j & 1, a.err, kErrMmaTimeout)) return false;
                if (s == 1 && tail && j == nk - 1 && !mbar_wait(&bars[kBarPFull], j & 1, a.err, kErrMmaTimeout))
                    return false;
                tc_fence_after();
                const uint32_t v_base = smem_addr(sV(st));
#pragma unroll
                for (int kk = 0; kk < kTK / 16; ++kk) {
                    const uint64_t bd = sw128_desc(v_base + kk * 16 * 128, L::kKVBlock, 1024);
                    tc_mma_ts(tmem + L::kColO + s * D, tmem + L::kColP + s * (kTK / 2) + kk * 8, bd, idesc_pv,
                              j > 0 || kk > 0);
                }
                tc_commit(&bars[kBarODone + s]);
                return true;
            };
            // S_s(j+1) only needs the softmax to have read S_s(j) (SFree), not its P: issuing it
            // before PV_s(j) lets it run under the softmax of tile j.
            // Stream 1 starts one tile behind stream 0, so that one warpgroup's exponentials (MUFU)
            // overlap the other's TMEM traffic and barrier waits instead of competing with them.
            if (ok && s == 1) ok = mbar_wait(&bars[kBarStagger], 0, a.err, kErrMmaTimeout);
            if (ok) ok = issue_s(0);
            for (int j = 0; ok && j < nk; ++j) {
                if (j + 1 < nk && !issue_s(j + 1)) break;
                if (!issue_pv(j)) break;
                tc_commit(&bars[kBarKvEmpty + j % L::kStages]);
            }
            // Every MMA this thread issued must finish before TMEM is released.
            tc_commit(&bars[kBarMmaDone + s]);
            mbar_wait(&bars[kBarMmaDone + s], 0, a.err, kErrMmaTimeout);
        }
        __syncwarp();
    } else {
        // ---- softmax warpgroups: stream s = warp / 4, thread r <-> query row r (TMEM lane r).
        const int s = warp >> 2;
        const int r = threadIdx.x & 127;
        const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
        const int h = s ? head1 : head0, q0 = s ? q01 : q00, nqs = s ? nq1 : nq0;
        const bool row_ok = r < nqs;
        const int t = q0 + r;
        // Stage both streams' q rows as fp16 in the 128-byte swizzled K-major layout of the MMA's
        // A operand (unless the producer loads them already rotated).
        if (a.q_tma) {
        } else if (a.q_raw) {
            // Fused q prologue: the per-head RMSNorm and NeoX rotation of the stream's query rows
            // (rmsnormCpu kernels.ts:3395, ropeCpu :3445) in f32 with the f32 copy of the table.
            // q only feeds the fp16 tensor-core operand, so the append's fp64 path (which the
            // cache rows need bit for bit) is not required here.  One warp per row: lane l holds
            // rotation pairs (i, i + D/2) for i in [l*P, l*P + P), so every load is coalesced and
            // the sum of squares is a warp reduction.
            constexpr int H2 = D / 2, P = H2 / 32;
            const int i0 = lane * P;
            float g0[P], g1[P];
#pragma unroll
            for (int p = 0; p < P; ++p) {
                const float w0 = a.q_norm ? a.q_norm[i0 + p] : 1.f, w1 = a.q_norm ? a.q_norm[i0 + p + H2] : 1.f;
                g0[p] = a.q_norm && a.one_plus ? 1.f + w0 : w0;
                g1[p] = a.q_norm && a.one_plus ? 1.f + w1 : w1;
            }
            // Stream 0's rows first, then stream 1's, each by all eight warps (rows w, w + 8, ...),
            // so that stream 0's MMAs start after half the staging.  Batches of kB rows: all loads
            // of a batch are issued before its first shared-memory store (stores through the
            // generic pointer would otherwise keep later loads behind them).  (16-row batches
            // measured slower here: 12.48 against 12.41 ms per prefill step.)
            constexpr int kB = 8;
#pragma unroll 1
            for (int sg = 0; sg < 2; ++sg) {
                const int hs = sg ? head1 : head0, qs0 = sg ? q01 : q00, nqss = sg ? nq1 : nq0;
                uint8_t *sqs = sQ(sg);
#pragma unroll 1
                for (int rb = 0; rb < kTQ / 8; rb += kB) {
                    float x0[kB][P], x1[kB][P], c[kB][P], sn[kB][P];
#pragma unroll
                    for (int u = 0; u < kB; ++u) {
                        const int rr = warp + 8 * (rb + u);
                        const bool ok_r = rr < nqss;
                        const int tr = qs0 + rr;
                        const float *src = a.q_raw + (((size_t)b * T + (ok_r ? tr : 0)) * a.Hq + hs) * D;
#pragma unroll
                        for (int p = 0; p < P; ++p) x0[u][p] = x1[u][p] = 0.f, c[u][p] = 1.f, sn[u][p] = 0.f;
                        if (ok_r) {
                            if constexpr (P == 2) {
                                const float2 lo = *reinterpret_cast<const float2 *>(src + i0);
                                const float2 hi = *reinterpret_cast<const float2 *>(src + i0 + H2);
                                x0[u][0] = lo.x, x0[u][1] = lo.y, x1[u][0] = hi.x, x1[u][1] = hi.y;
                                if (a.rope) {
                                    const float4 e = *reinterpret_cast<const float4 *>(a.rope + (size_t)(past + tr) * H2 + i0);
                                    c[u][0] = e.x, sn[u][0] = e.y, c[u][1] = e.z, sn[u][1] = e.w;
                                }
                            } else {
#pragma unroll
                                for (int p = 0; p < P; ++p) {
                                    x0[u][p] = src[i0 + p], x1[u][p] = src[i0 + p + H2];
                                    if (a.rope) {
                                        const float2 e = a.rope[(size_t)(past + tr) * H2 + i0 + p];
                                        c[u][p] = e.x, sn[u][p] = e.y;
                                    }
                                }
                            }
                        }
                    }
#pragma unroll
                    for (int u = 0; u < kB; ++u) {
                        const int rr = warp + 8 * (rb + u);
                        float inv = 1.f;
                        if (a.q_norm) {
                            float ss = 0.f;
#pragma unroll
                            for (int p = 0; p < P; ++p) ss = fmaf(x0[u][p], x0[u][p], fmaf(x1[u][p], x1[u][p], ss));
#pragma unroll
                            for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
                            inv = 1.f / sqrtf(ss / (float)D + a.eps);
                        }
                        float o0[P], o1[P];
#pragma unroll
                        for (int p = 0; p < P; ++p) {
                            const float y0 = x0[u][p] * inv * g0[p], y1 = x1[u][p] * inv * g1[p];
                            o0[p] = fmaf(y0, c[u][p], -(y1 * sn[u][p]));
                            o1[p] = fmaf(y1, c[u][p], y0 * sn[u][p]);
                        }
                        // Elements i0.. and i0 + D/2..: pieces of the row's swizzled 16-byte chunks.
                        const int j0 = i0 + H2;
                        uint8_t *d0 = sqs + (i0 >> 6) * L::kQBlock + sw128(rr, (i0 & 63) >> 3) + (i0 & 7) * 2;
                        uint8_t *d1 = sqs + (j0 >> 6) * L::kQBlock + sw128(rr, (j0 & 63) >> 3) + (j0 & 7) * 2;
                        if constexpr (P == 2) {
                            *reinterpret_cast<uint32_t *>(d0) = pack_half2(o0[0], o0[1]);
                            *reinterpret_cast<uint32_t *>(d1) = pack_half2(o1[0], o1[1]);
                        } else {
                            *reinterpret_cast<__half *>(d0) = __float2half_rn(o0[0]);
                            *reinterpret_cast<__half *>(d1) = __float2half_rn(o1[0]);
                        }
                    }
                }
                fence_proxy_async_smem();
                mbar_arrive(&bars[sg ? kBarQFull1 : kBarQFull]);
            }
        } else {
            // Pre-rotated f32 q: one warp per row (lane l: elements 4l.. of each 128-wide half),
            // stream by stream as above, 16 rows per warp loaded before their shared-memory stores.
            constexpr int kB = 16, PE = D / 32;  // elements per lane
#pragma unroll 1
            for (int sg = 0; sg < 2; ++sg) {
                const int hs = sg ? head1 : head0, qs0 = sg ? q01 : q00, nqss = sg ? nq1 : nq0;
                uint8_t *sqs = sQ(sg);
#pragma unroll 1
                for (int rb = 0; rb < kTQ / 8; rb += kB) {
                    float x[kB][PE];
#pragma unroll
                    for (int u = 0; u < kB; ++u) {
                        const int rr = warp + 8 * (rb + u);
                        const bool ok_r = rr < nqss;
                        const float *src = a.q + (((size_t)b * T + (ok_r ? qs0 + rr : 0)) * a.Hq + hs) * D;
                        if constexpr (PE == 4) {
                            const float4 v4 = ok_r ? *reinterpret_cast<const float4 *>(src + 4 * lane)
                                                   : make_float4(0.f, 0.f, 0.f, 0.f);
                            x[u][0] = v4.x, x[u][1] = v4.y, x[u][2] = v4.z, x[u][3] = v4.w;
                        } else {
                            const float2 v2 = ok_r ? *reinterpret_cast<const float2 *>(src + 2 * lane) : make_float2(0.f, 0.f);
                            x[u][0] = v2.x, x[u][1] = v2.y;
                        }
                    }
#pragma unroll
                    for (int u = 0; u < kB; ++u) {
                        const int rr = warp + 8 * (rb + u);
                        const int i = PE * lane;  // first element of this lane
                        uint8_t *d = sqs + (i >> 6) * L::kQBlock + sw128(rr, (i & 63) >> 3) + (i & 7) * 2;
                        if constexpr (PE == 4)
                            *reinterpret_cast<uint2 *>(d) = make_uint2(pack_half2(x[u][0], x[u][1]), pack_half2(x[u][2], x[u][3]));
                        else
                            *reinterpret_cast<uint32_t *>(d) = pack_half2(x[u][0], x[u][1]);
                    }
                }
                fence_proxy_async_smem();
                mbar_arrive(&bars[sg ? kBarQFull1 : kBarQFull]);
            }
        }
        if (s == 1 && !active1) {
            // Nothing to do for an empty second stream (odd group, last tile pair).
        } else {
            const int pos = past + t;                        // absolute position of this query
            const int hi = row_ok ? pos - a.kv_offset : -1;  // last key (cache row) it attends
            const int lo = a.window > 0 ? pos - a.window + 1 - a.kv_offset : INT_MIN;
            // Tiles that need no per-element mask: all 128 rows see all 64 keys.
            const int hi_min = past + q0 - a.kv_offset;
            const int lo_max = a.window > 0 ? past + q0 + nqs - 1 - a.window + 1 - a.kv_offset : INT_MIN;
            const uint32_t tS = tmem + L::kColS + s * kTK + lane_base;
            const uint32_t tO = tmem + L::kColO + s * D + lane_base;
            const uint32_t tP = tmem + L::kColP + s * (kTK / 2) + lane_base;
            float m_used = -CUDART_INF_F;  // max the probabilities are relative to (log2 units)
            float l_run = 0.f;
            bool ok = true;
            for (int j = 0; j < nk; ++j) {
                const int kbase = klo + j * kTK;
                if (!mbar_wait(&bars[kBarSFull + s], j & 1, a.err, kErrMmaTimeout)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                uint32_t raw[2][32];
                tc_ld32_nowait(tS, raw[0]);
                tc_ld32_nowait(tS + 32, raw[1]);
                tc_wait_ld();
                tc_fence_before();
                mbar_arrive(&bars[kBarSFree + s]);  // S_s may be overwritten by the next tile
                float v[64];
#pragma unroll
                for (int i = 0; i < 64; ++i) v[i] = __uint_as_float(raw[i >> 5][i & 31]);
                const bool full = kbase + kTK - 1 <= hi_min && kbase >= lo_max && kbase + kTK <= khi;
                if (!full) {
#pragma unroll
                    for (int i = 0; i < 64; ++i) {
                        const int key = kbase + i;
                        v[i] = (key <= hi && key >= lo && key < khi) ? v[i] : -CUDART_INF_F;
                    }
                }
                const float mraw = max_tree(v);
                const float mt = mraw == -CUDART_INF_F ? -CUDART_INF_F : score_log2<CAP>(mraw, a);
                // The row's max is raised when a tile's max exceeds it by more than 2^8 (or on its
                // first finite score); O_s (and l) of the row are then rescaled, except on that first
                // raise.  Rows decide separately, but tcgen05.ld / st / wait are warp-collective
                // (.sync.aligned), so the whole warp runs the rescale pass when any of its rows needs
                // it, the other rows with factor 1.
                const bool raise = mt > m_used + kRescaleLog2 || (m_used == -CUDART_INF_F && mt != -CUDART_INF_F);
                const bool rescale = raise && m_used != -CUDART_INF_F && j >= 1;
                bool waited_o = false;
                if (__any_sync(0xffffffffu, rescale)) {
                    // ... once PV_s(j-1) has landed (j >= 1 for the whole warp: j is uniform).
                    const bool got = mbar_wait(&bars[kBarODone + s], (j - 1) & 1, a.err, kErrMmaTimeout);
                    if (!__all_sync(0xffffffffu, got)) {
                        ok = false;
                        break;
                    }
                    waited_o = true;
                    tc_fence_after();
                    const float alpha = rescale ? ex2_fast(m_used - mt) : 1.f;
#pragma unroll 1
                    for (int c = 0; c < D / 32; ++c) {
                        uint32_t o[32];
                        tc_ld32_nowait(tO + c * 32, o);
                        tc_wait_ld();
#pragma unroll
                        for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
                        tc_st32(tO + c * 32, o);
                    }
                    tc_wait_st();
                    l_run *= alpha;
                }
                if (raise) m_used = mt;
                const float m_eff = m_used == -CUDART_INF_F ? 0.f : m_used;
                // P_s as packed fp16 in registers first, so that the exponentials overlap the
                // tensor core's PV_s(j-1); only the stores wait for it to stop reading P_s.
                // Packed f32x2 arithmetic and four independent row sums keep dependency chains short.
                float2 acc[4];
#pragma unroll
                for (int k = 0; k < 4; ++k) acc[k] = make_float2(0.f, 0.f);
                uint32_t pk[32];
                const float2 sc2 = make_float2(a.scale_log2, a.scale_log2), nm2 = make_float2(-m_eff, -m_eff);
#pragma unroll
                for (int u = 0; u < 32; ++u) {
                    float p0, p1;
                    if constexpr (CAP) {
                        p0 = v[2 * u] == -CUDART_INF_F ? 0.f : ex2_fast(score_log2<CAP>(v[2 * u], a) - m_eff);
                        p1 = v[2 * u + 1] == -CUDART_INF_F ? 0.f : ex2_fast(score_log2<CAP>(v[2 * u + 1], a) - m_eff);
                    } else {
                        const float2 x = ffma2(make_float2(v[2 * u], v[2 * u + 1]), sc2, nm2);
                        if ((u % 8) < kPolyPairsPer8) {
                            const float2 e = ex2_poly2(x);
                            p0 = e.x;
                            p1 = e.y;
                        } else {
                            p0 = ex2_fast(x.x);
                            p1 = ex2_fast(x.y);
                        }
                    }
                    acc[u & 3] = fadd2(acc[u & 3], make_float2(p0, p1));
                    pk[u] = pack_half2(p0, p1);
                }
                const float2 acc01 = fadd2(acc[0], acc[1]), acc23 = fadd2(acc[2], acc[3]);
                const float rsum = (acc01.x + acc01.y) + (acc23.x + acc23.y);
                if (j >= 1 && !waited_o) {
                    if (!mbar_wait(&bars[kBarODone + s], (j - 1) & 1, a.err, kErrMmaTimeout)) {
                        ok = false;
                        break;
                    }
                }
                tc_st32(tP, pk);
                // Keys past the range end: zero their V rows so that 0 * (stale data) stays 0
                // (stream 0's warpgroup does it; stream 1's PV of this tile also waits for P_0).
                // (Only some lanes zero a row; the warp leaves together on a timeout, since the
                // warp-collective tcgen05 instructions below need every lane.)
                if (s == 0 && kbase + kTK > khi) {
                    bool zok = true;
                    if (r < kTK && kbase + r >= khi) {
                        zok = mbar_wait(&bars[kBarKvFull + j % L::kStages], (j / L::kStages) & 1, a.err, kErrTmaTimeout);
                        if (zok) {
#pragma unroll
                            for (int blk = 0; blk < L::kBlocks; ++blk)
#pragma unroll
                                for (int c = 0; c < 8; ++c)
                                    *reinterpret_cast<uint4 *>(sV(j % L::kStages) + blk * L::kKVBlock + sw128(r, c)) =
                                        make_uint4(0u, 0u, 0u, 0u);
                        }
                    }
                    if (!__all_sync(0xffffffffu, zok)) {
                        ok = false;
                        break;
                    }
                    fence_proxy_async_smem();  // the zeroed V rows
                }
                tc_wait_st();
                tc_fence_before();
                mbar_arrive(&bars[kBarPFull + s]);
                if (s == 0 && j == 0) mbar_arrive(&bars[kBarStagger]);
                l_run += rsum;
            }
            bool fin = ok && nk > 0;
            if (fin) fin = mbar_wait(&bars[kBarODone + s], (nk - 1) & 1, a.err, kErrMmaTimeout);
            if (__all_sync(0xffffffffu, fin)) {
                tc_fence_after();
                const float inv = 1.f / l_run;
                float *dst = a.out + (((size_t)b * T + (row_ok ? t : 0)) * a.Hq + h) * D;
#pragma unroll 1
                for (int c = 0; c < D / 32; ++c) {
                    uint32_t o[32];
                    tc_ld32_nowait(tO + c * 32, o);
                    tc_wait_ld();
                    if (row_ok) {
#pragma unroll
                        for (int e = 0; e < 32; e += 4)
                            *reinterpret_cast<float4 *>(dst + c * 32 + e) =
                                make_float4(__uint_as_float(o[e]) * inv, __uint_as_float(o[e + 1]) * inv,
                                            __uint_as_float(o[e + 2]) * inv, __uint_as_float(o[e + 3]) * inv);
                    }
                }
            }
        }
    }

    // Teardown: every TMEM access and MMA is complete; the allocating warp releases TMEM.
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == kMmaWarp)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
}

template <int D, bool CAP>
cudaError_t launch_prefill_t(const CUtensorMap &tmk, const CUtensorMap &tmv, const CUtensorMap &tmq, const PrefillArgs &a,
                             cudaStream_t s,
                             bool pdl) {
    static unsigned long long configured = 0;
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 64 || !(configured & (1ull << dev))) {
        cudaError_t e = cudaFuncSetAttribute(prefill_attn_kernel<D, CAP>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             PrefillLayout<D>::kSmemBytes);
        if (e != cudaSuccess) return e;
        if (dev < 64) configured |= 1ull << dev;
    }
    const int G = a.Hq / a.Hkv;
    const int ntq = (a.T + kTQ - 1) / kTQ;
    const dim3 grid(G % 2 == 0 ? a.Hq / 2 : a.Hq, a.B, G % 2 == 0 ? ntq : (ntq + 1) / 2);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = PrefillLayout<D>::kSmemBytes;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, prefill_attn_kernel<D, CAP>, tmk, tmv, tmq, a);
}

}  // namespace

int prefill_tile_keys() { return kTK; }

cudaError_t launch_prefill(int head_dim, const CUtensorMap &tmk, const CUtensorMap &tmv, const PrefillArgs &a,
                           cudaStream_t s, bool pdl, const CUtensorMap *tmq) {
    const bool cap = a.softcap > 0.f;
    const CUtensorMap &q = tmq ? *tmq : tmk;  // unused unless a.q_tma
    switch (head_dim) {
        case 64:
            return cap ? launch_prefill_t<64, true>(tmk, tmv, q, a, s, pdl) : launch_prefill_t<64, false>(tmk, tmv, q, a, s, pdl);
        case 128:
            return cap ? launch_prefill_t<128, true>(tmk, tmv, q, a, s, pdl)
                       : launch_prefill_t<128, false>(tmk, tmv, q, a, s, pdl);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace brk
