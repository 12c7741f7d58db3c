// Decode attention over the resident KV cache, fp16 or int8 (replaces attention_decode and
// attention_decode_q8kv, shaders.ts:1768-1851 and 1856-1944, and their dispatch in recAttention /
// recAttentionQ8, kernels.ts:1626-1661).
//
// One CTA per (sequence, kv head, tile of 8 query rows, split).  The query rows of a tile are
// (token, q head) pairs of one kv head's group, so every K/V byte read from HBM serves the whole
// group.  A producer warp streams the CTA's key range through a shared-memory ring with 2-D TMA
// loads (CTA-local): fp16 rows as [keys][64 x fp16] boxes, int8 codes as [keys][<=128 B] boxes
// plus a [2][keys] box of f32 K / V scales.  Consumer warps come in key groups of 16 keys per
// stage (and, for head_dim 256, pairs that split the head dim and swap partial scores).
//
// Keys sit on the M dimension of the tensor-core tiles (mma.m16n8k16, fp16 in, fp32 accumulate)
// and the 8 query rows on N, so a decode step with a small GQA group wastes at most half of each
// tile instead of three quarters:
//   S^T [16 keys x 8 rows] = K [16 x D] Q^T [D x 8]
//   O^T [D x 8 rows]      += V^T [D x 16 keys] P^T [16 keys x 8 rows]
// P^T comes from the S^T accumulator fragment with one movmatrix transpose per 8 keys.
//
// int8 cache: each code is stored biased by +128 in one byte, so one byte permute turns two codes
// into the exact fp16 pair code + 1152 (codes_biased_half2); the bias is removed once per row
// instead of once per code: 1152 * sum(q) from each raw score, 1152 * sum(p') from each output.
// The K scale is constant over the head dim and factors out of the dot product
// (shaders.ts:1721-1726): s = scale_k[j] * sum_d q_d code_d; the V scale multiplies the
// probabilities, p'_j = p_j * scale_v[j], while the row sum keeps p_j.  Lanes read codes as
// 16-byte words; the head dim is permuted identically in q and K (k-step ks of lane quad qc covers
// head-dim bytes W qc + 4 ks + 0..3), and a lane's V fragment takes VW bytes at head-dim VW r of
// four keys, transposed 4 x 4 bytes at a time with byte permutes (output head-dim rows are
// permuted accordingly and restored at the merge).
//
// Tiles whose keys every row of the tile may attend (all but the causal / window edges and the
// range end) skip the per-score masks.
#include "decode_common.cuh"
#include "kv_q8.cuh"

namespace brk {

namespace {

constexpr int kRT = 8;  // query rows per CTA tile (the MMA N dimension)

// Ring stages, CTAs per SM (launch bound), head-dim split and key groups per (cache type, D),
// chosen by timing sweeps on B200: the int8 kernels run 4 CTAs per SM with shallower rings, the
// extra consumer warps hiding the code conversion.
template <bool Q8, int D>
struct DecodeCfg;
template <>
struct DecodeCfg<false, 64> {
    static constexpr int kStages = 4, kMinBlocks = 3, kDSplit = 1, kKeyGroups = 4;
};
template <>
struct DecodeCfg<false, 128> {
    static constexpr int kStages = 3, kMinBlocks = 2, kDSplit = 1, kKeyGroups = 4;
};
template <>
struct DecodeCfg<false, 256> {
    static constexpr int kStages = 2, kMinBlocks = 3, kDSplit = 2, kKeyGroups = 2;
};
template <>
struct DecodeCfg<true, 64> {
    static constexpr int kStages = 4, kMinBlocks = 4, kDSplit = 1, kKeyGroups = 4;
};
template <>
struct DecodeCfg<true, 128> {
    static constexpr int kStages = 2, kMinBlocks = 4, kDSplit = 1, kKeyGroups = 4;
};
template <>
struct DecodeCfg<true, 256> {
    static constexpr int kStages = 2, kMinBlocks = 4, kDSplit = 2, kKeyGroups = 2;
};

template <bool Q8, int D>
struct DecodeLayout {
    using C = DecodeCfg<Q8, D>;
    static constexpr int kDS = C::kDSplit;
    static constexpr int kKG = C::kKeyGroups;
    static constexpr int kStageKeys = 16 * kKG;
    static constexpr int kConsumers = kKG * kDS;
    static constexpr int kThreads = (kConsumers + 1) * 32;
    static constexpr int kRowBytes = Q8 ? D : 2 * D;                   // one key row of the cache
    static constexpr int kBoxCols = Q8 ? (D < 128 ? D : 128) : 128;     // bytes of one box row
    static constexpr int kBoxElems = Q8 ? kBoxCols : kBoxCols / 2;      // elements of one box row
    static constexpr int kBoxes = kRowBytes / kBoxCols;
    static constexpr uint32_t kBoxBytes = kStageKeys * kBoxCols;
    static constexpr uint32_t kTileBytes = kStageKeys * kRowBytes;      // K (or V) of one stage
    static constexpr uint32_t kScaleBytes = Q8 ? 2 * kStageKeys * 4 : 0;
    static constexpr uint32_t kLoadBytes = 2 * kTileBytes + kScaleBytes;
    static constexpr uint32_t kStageBytes = (kLoadBytes + 1023) / 1024 * 1024;
    static constexpr uint32_t kRingBytes = C::kStages * kStageBytes;
    // Score swap of the head-dim halves: [key group][parity][half][lane][4] floats.
    static constexpr uint32_t kSwapBytes = kDS > 1 ? kKG * 2 * 2 * 32 * 4 * 4 : 0;
    // Fused append: the tile's rotated q rows [kQRows][D + 8] f32 (padded against bank conflicts),
    // in the same bytes as the score swap (used only before the main loop).  head_dim 256 stages
    // up to 4 rows (GQA groups up to 4 fuse), the others a whole tile.
    static constexpr int kQRows = D == 256 ? 4 : 8;
    static constexpr uint32_t kQStride = D + 8;
    static constexpr uint32_t kQBytes = kQRows * kQStride * 4;
    static constexpr uint32_t kXBytes = kSwapBytes > kQBytes ? kSwapBytes : kQBytes;
    // Fused append into an int8 cache: the new K and V rows in f32, quantised from here.
    static constexpr uint32_t kNewRowBytes = Q8 ? 2 * D * 4 : 0;
    // Fused append: the new K and V rows as the cache stores them (fp16, or int8 codes and then
    // their two scales), patched into the ring stage that holds that row.
    static constexpr uint32_t kPatchBytes = Q8 ? 2 * D + 16 : 4 * D;
    static constexpr uint32_t kBarBytes = (2 * C::kStages + 2) * 8;  // full, empty, row load, row done
    static constexpr uint32_t kSmemBytes = 1024 + kRingBytes + kXBytes + kNewRowBytes + kPatchBytes + kBarBytes;
    static_assert(decode_epilogue_bytes<D, kKG, kRT>() <= kRingBytes, "merge buffers must fit in the ring");
};

// Fused append: a warp of its own computes the new rows while the producer streams (fp16 caches);
// the int8 kernels, whose four CTAs per SM leave no registers for a sixth warp, compute them in
// the producer warp after its first ring stages.
template <bool Q8, bool F>
struct DecodeRowWarp {
    static constexpr bool value = F && !Q8;
};
template <bool Q8, int D, bool F>
constexpr int decode_threads() { return DecodeLayout<Q8, D>::kThreads + (DecodeRowWarp<Q8, F>::value ? 32 : 0); }

// rmsnormCpu + ropeCpu (kernels.ts:3395, 3445) of one head row by one warp, in the append
// kernel's fp64 operations (append.cu; the same bits).  Lane l holds the row's pairs
// (i, i + D/2), i = l + 32 u, in x0 / x1, their norm gains in g0 / g1 and their rotation in e
// (all loaded by the caller, so that every input is in flight at once).  The sum of squares runs
// in the oracle's order d = 0 .. D-1 on every lane (the values come by shuffle), then
// y = f32(x * inv * g), rotated in double and rounded to f32 into o0 / o1.  has_gain false: no
// norm; has_cs false: no rotation.
template <int D>
__device__ __forceinline__ void rotate_row_regs(const float (&x0)[D / 64], const float (&x1)[D / 64],
                                                const float (&g0)[D / 64], const float (&g1)[D / 64], bool has_gain,
                                                double eps, int one_plus, const double2 (&e)[D / 64], bool has_cs,
                                                float (&o0)[D / 64], float (&o1)[D / 64]) {
    constexpr int NP = D / 64;
    double y0[NP], y1[NP];
#pragma unroll
    for (int u = 0; u < NP; ++u) {
        y0[u] = x0[u];
        y1[u] = x1[u];
    }
    if (has_gain) {
        double ss = 0.0;
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
            for (int u = 0; u < NP; ++u)
#pragma unroll 8
                for (int l = 0; l < 32; ++l) {
                    // Element d = h * D/2 + 32 u + l, in ascending d.
                    const double xd = (double)__shfl_sync(0xffffffffu, h ? x1[u] : x0[u], l);
                    ss = __fma_rn(xd, xd, ss);  // x^2 is exact in double: one rounding, as ss + x*x
                }
        const double inv = __ddiv_rn(1.0, __dsqrt_rn(__dadd_rn(__ddiv_rn(ss, (double)D), eps)));
#pragma unroll
        for (int u = 0; u < NP; ++u) {
            const double w0 = g0[u], w1 = g1[u];
            const double ga = one_plus ? __dadd_rn(1.0, w0) : w0, gb = one_plus ? __dadd_rn(1.0, w1) : w1;
            y0[u] = (double)(float)__dmul_rn(__dmul_rn(y0[u], inv), ga);
            y1[u] = (double)(float)__dmul_rn(__dmul_rn(y1[u], inv), gb);
        }
    }
#pragma unroll
    for (int u = 0; u < NP; ++u) {
        if (has_cs) {
            o0[u] = (float)__dsub_rn(__dmul_rn(y0[u], e[u].x), __dmul_rn(y1[u], e[u].y));
            o1[u] = (float)__dadd_rn(__dmul_rn(y1[u], e[u].x), __dmul_rn(y0[u], e[u].y));
        } else {
            o0[u] = (float)y0[u];
            o1[u] = (float)y1[u];
        }
    }
}

// The new token's K (QK-norm + RoPE with the append kernel's fp64 operations, hence its bits) and
// V rows of the fused append, computed and stored in the cache by the producer warp (after it
// has put the first ring stages in flight, before the stage that holds the new row): fp16
// rounded to nearest even, or quantised as quantize_kv does.  Each lane fences its stores for
// the async proxy, which the warp's next TMA load of that row requires.
template <bool Q8, int D>
__device__ __noinline__ void fused_kv_rows(const DecodeArgs &a, int b, int kvh, int past, int seg, float *newrow,
                                           uint8_t *patch, int lane) {
    constexpr int H2 = D / 2, NP = D / 64;
    const double2 *cs = a.rope ? a.rope + (size_t)past * H2 : nullptr;
    const size_t crow = (size_t)seg * a.cap + (size_t)(past - a.kv_offset);
    // Every input of both rows in flight at once: the K and V pairs, k's norm gains and the
    // rotation of this position (one round trip to memory instead of one per input).
    const float *ksrc = a.k_in + ((size_t)b * a.Hkv + kvh) * D, *vsrc = a.v_in + ((size_t)b * a.Hkv + kvh) * D;
    float in0[2][NP], in1[2][NP], g0[NP], g1[NP];
    double2 e[NP];
#pragma unroll
    for (int u = 0; u < NP; ++u) {
        const int i = lane + 32 * u;
        in0[0][u] = ksrc[i];
        in1[0][u] = ksrc[i + H2];
        in0[1][u] = vsrc[i];
        in1[1][u] = vsrc[i + H2];
        g0[u] = a.k_norm ? a.k_norm[i] : 0.f;
        g1[u] = a.k_norm ? a.k_norm[i + H2] : 0.f;
        e[u] = cs ? cs[i] : make_double2(1.0, 0.0);
    }
#pragma unroll
    for (int which = 0; which < 2; ++which) {
        const bool is_k = which == 0;
        float o0[NP], o1[NP];
        rotate_row_regs<D>(in0[which], in1[which], g0, g1, is_k && a.k_norm, a.eps, a.one_plus, e, is_k && cs, o0, o1);
        if constexpr (Q8) {
            float *x = newrow + which * D;
#pragma unroll
            for (int u = 0; u < NP; ++u) {
                x[lane + 32 * u] = o0[u];
                x[lane + 32 * u + H2] = o1[u];
            }
            __syncwarp();
            quantize_row_warp(x, D, (is_k ? a.kc8 : a.vc8) + crow * D,
                              a.scales + ((size_t)seg * 2 + which) * a.scale_pitch + (size_t)(past - a.kv_offset),
                              lane);
            quantize_row_warp(x, D, patch + which * D, reinterpret_cast<float *>(patch + 2 * D) + which, lane);
        } else {
            __half *dst = (is_k ? a.kc : a.vc) + crow * D;
            __half *pd = reinterpret_cast<__half *>(patch) + which * D;
#pragma unroll
            for (int u = 0; u < NP; ++u) {
                const __half h0 = __float2half_rn(o0[u]), h1 = __float2half_rn(o1[u]);
                dst[lane + 32 * u] = h0;
                dst[lane + 32 * u + H2] = h1;
                pd[lane + 32 * u] = h0;
                pd[lane + 32 * u + H2] = h1;
            }
        }
    }
}

// Fused append, by the producer's elected lane: the new rows from `patch` into the ring stage `st`
// (whose copy of the cache has landed) at row `rpos`, in the stage's swizzled layouts, fp16 rows
// or int8 codes plus their scales.
template <bool Q8, int D>
__device__ __forceinline__ void patch_new_row(uint8_t *st, int rpos, const uint8_t *patch) {
    using L = DecodeLayout<Q8, D>;
#pragma unroll 1
    for (int which = 0; which < 2; ++which) {
        uint8_t *base = st + which * L::kTileBytes;
        if constexpr (Q8) {
            for (int b0 = 0; b0 < D; b0 += 16) {
                const int j = b0 / L::kBoxCols, cb = (b0 % L::kBoxCols) / 16;
                const uint32_t off = L::kBoxCols == 128 ? sw128(rpos, cb) : sw64(rpos, cb);
                *reinterpret_cast<uint4 *>(base + j * L::kBoxBytes + off) =
                    *reinterpret_cast<const uint4 *>(patch + which * D + b0);
            }
        } else {
            for (int d0 = 0; d0 < D; d0 += 8) {
                const int j = d0 / 64, c = (d0 % 64) / 8;
                *reinterpret_cast<uint4 *>(base + j * L::kBoxBytes + sw128(rpos, c)) =
                    *reinterpret_cast<const uint4 *>(patch + (which * D + d0) * 2);
            }
        }
    }
    if constexpr (Q8) {
        float *sc = reinterpret_cast<float *>(st + 2 * L::kTileBytes);
        const float *ps = reinterpret_cast<const float *>(patch + 2 * D);
        sc[rpos] = ps[0];
        sc[L::kStageKeys + rpos] = ps[1];
    }
}

// F: the fused-append form (brk_attn_step with one token); a separate instantiation, so that the
// plain kernel's code and registers stay as they are.
template <bool Q8, int D, bool F>
__global__ void __launch_bounds__(decode_threads<Q8, D, F>(), DecodeCfg<Q8, D>::kMinBlocks)
    decode_kernel(const __grid_constant__ CUtensorMap tmk, const __grid_constant__ CUtensorMap tmv,
                   const __grid_constant__ CUtensorMap tms, const __grid_constant__ DecodeArgs a) {
    using L = DecodeLayout<Q8, D>;
    constexpr int S = DecodeCfg<Q8, D>::kStages;
    constexpr int DS = L::kDS;
    constexpr int NC = L::kConsumers;
    constexpr int KG = L::kKG;
    constexpr int SK = L::kStageKeys;
    constexpr int DH = D / DS;  // head-dim slice of one warp: 64 or 128
    constexpr int KS = DH / 16; // k-steps of S^T = K Q^T
    constexpr int MT = DH / 16; // m-tiles (16 head-dim rows) of O^T
    constexpr int W = DH / 4;   // int8: K bytes of a key row per lane-quad member
    constexpr int VW = DH / 8;  // int8: V bytes of a key row per lane
    constexpr int NG = VW / 4;  // int8: V words of a key row per lane
    static_assert(DH == 64 || DH == 128, "per-warp head-dim slice");

    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *ring = smem;
    float *xbuf = reinterpret_cast<float *>(ring + L::kRingBytes);
    float *newrow = reinterpret_cast<float *>(ring + L::kRingBytes + L::kXBytes);  // int8: [2][D]
    uint8_t *patch = ring + L::kRingBytes + L::kXBytes + L::kNewRowBytes;
    uint64_t *full = reinterpret_cast<uint64_t *>(patch + L::kPatchBytes);
    uint64_t *empty = full + S;
    uint64_t *rowbar = empty + S;    // fused append: the copy of the stage that holds the new row
    uint64_t *rowdone = rowbar + 1;  // fused append: the new rows are in `patch`

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int split = blockIdx.x;
    const int kvh = blockIdx.y / a.mtiles, mtile = blockIdx.y % a.mtiles;
    const int b = blockIdx.z;
    const int G = a.G, T = a.T;
    const int nrows = T * G;
    const int row0 = mtile * kRT;
    const int past = a.past_len[b];

    // Key range; for int8 a window's first key is rounded down to a multiple of 4 (16-byte scale
    // boxes) -- the extra keys are below every row's window and masked.
    const KeyRange kr = decode_key_range(a, past, row0, nrows, split, SK, Q8 ? 4 : 1, kRT);
    const int k_begin = kr.k_begin, k_end = kr.k_end, ntiles = kr.ntiles;
    const int seg = (a.layer * a.B + b) * a.Hkv + kvh;
    // Fused append: this CTA writes the new token's K / V rows (cache row past - kv_offset) when
    // its key range holds them, before its ring loads that row.
    const int new_row = past - a.kv_offset;
    const bool writes_row = F && new_row >= k_begin && new_row < k_end;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], NC);
        }
        mbar_init(rowbar, 1);
        mbar_init(rowdone, 1);
        fence_barrier_init();
    }
    __syncthreads();

    if (warp == NC) {
        // ---- producer: one elected lane streams the stages through the ring.
        // Fused append: the stage that holds the new row (tile rt) is loaded as usual but counted
        // on `rowbar`; once that copy has landed and the row warp has the new rows ready, the rows
        // are patched into the stage and only then is the stage released to the consumers.  So the
        // copy of that stage does not wait for the new rows, and the rows do not make a round trip
        // through memory before the consumers see them.
        constexpr bool kRowWarp = DecodeRowWarp<Q8, F>::value;
        const int rt = writes_row ? (new_row - k_begin) / SK : -1;
        int issued = 0;
        bool ok = true;
        bool row_ready = kRowWarp;  // the patch may be applied as soon as the stage is issued
        auto issue = [&](int i_end) {
            for (int i = issued; i < i_end && ok; ++i) {
                const int s = i % S;
                const int key = k_begin + i * SK;
                if (i >= S && !mbar_wait(&empty[s], ((i / S) - 1) & 1, a.err, kErrSlotTimeout)) {
                    ok = false;
                    break;
                }
                uint64_t *bar = i == rt ? rowbar : &full[s];
                mbar_arrive_expect_tx(bar, L::kLoadBytes);
                uint8_t *st = ring + s * L::kStageBytes;
                const int y = seg * a.cap + key;
#pragma unroll
                for (int j = 0; j < L::kBoxes; ++j) tma_load_2d(st + j * L::kBoxBytes, &tmk, j * L::kBoxElems, y, bar);
#pragma unroll
                for (int j = 0; j < L::kBoxes; ++j)
                    tma_load_2d(st + L::kTileBytes + j * L::kBoxBytes, &tmv, j * L::kBoxElems, y, bar);
                if constexpr (Q8) tma_load_2d(st + 2 * L::kTileBytes, &tms, key, seg * 2, bar);
                issued = i + 1;
                if constexpr (F) {
                    if (i == rt && row_ready) {
                        // Bounded waits; on a timeout the error word is set and the stage still
                        // goes to the consumers (whose results are then meaningless).
                        if ((!kRowWarp || mbar_wait(rowdone, 0, a.err, kErrMmaTimeout)) &&
                            mbar_wait(rowbar, 0, a.err, kErrTmaTimeout))
                            patch_new_row<Q8, D>(st, new_row - key, patch);
                        mbar_arrive(&full[s]);
                    }
                }
            }
        };
        if (ntiles > 0) {
            if (lane == 0) {
                tma_prefetch_desc(&tmk);
                tma_prefetch_desc(&tmv);
                if constexpr (Q8) tma_prefetch_desc(&tms);
            }
            // As a programmatic dependent this CTA may start before the preceding kernel has
            // finished; cache rows (and the fused append's inputs) may come from it or, as kernels
            // that trigger their dependents early wait for their own predecessors before they
            // finish, from anything the stream ran before.  The CTA's set-up has overlapped it.
            griddep_wait();
            if constexpr (F && !kRowWarp) {
                if (writes_row) {
                    // The first ring stages (the new row's among them, unpatched, if it is that
                    // early), then the rows, then the patch of that stage if it is already issued.
                    if (lane == 0) issue(min(ntiles, S));
                    __syncwarp();
                    fused_kv_rows<Q8, D>(a, b, kvh, past, seg, newrow, patch, lane);
                    __syncwarp();
                    row_ready = true;
                    if (lane == 0 && issued > rt) {
                        uint8_t *st = ring + (rt % S) * L::kStageBytes;
                        if (mbar_wait(rowbar, 0, a.err, kErrTmaTimeout))
                            patch_new_row<Q8, D>(st, new_row - (k_begin + rt * SK), patch);
                        mbar_arrive(&full[rt % S]);
                    }
                }
            }
            if (lane == 0) {
                issue(ntiles);
                // Before leaving, make sure every copy this lane started has landed (bounded).
                for (int i = issued > S ? issued - S : 0; i < issued; ++i)
                    mbar_wait(&full[i % S], (i / S) & 1, a.err, kErrTmaTimeout);
            }
        }
        if (a.cluster) {
            __syncwarp();
            decode_cluster_idle();  // the cluster merge's two barriers count every thread
        }
        return;
    }
    if constexpr (DecodeRowWarp<Q8, F>::value) {
        if (warp == NC + 1) {
            // ---- fused append: the row warp computes the new K / V rows (the append kernel's fp64
            // operations, hence its bits), stores them in the cache for later steps and leaves them
            // in `patch` for the producer, while the producer streams the other stages.
            if (writes_row) {
                griddep_wait();  // k_in / v_in may come from the preceding kernel
                fused_kv_rows<Q8, D>(a, b, kvh, past, seg, newrow, patch, lane);
                __syncwarp();
                if (lane == 0) mbar_arrive(rowdone);  // release: the patch bytes before the producer's wait
            }
            if (a.cluster) {
                __syncwarp();
                decode_cluster_idle();
            }
            return;
        }
    }

    griddep_wait();  // q (or, fused, q_in / k_in / v_in) may come from the preceding kernel
    const int kg = warp % KG;  // key group: keys [16 kg, 16 kg + 16) of every stage
    const int dh = warp / KG;  // head-dim slice [DH dh, DH dh + DH)
    const int qr = lane >> 2, qc = lane & 3;

    if constexpr (F) {
        // Fused append: the tile's q rows rotated from the raw projection (QK-norm + RoPE in f32:
        // q only becomes the fp16 tensor-core operand), a warp per row, into shared memory; split 0
        // also writes them to q_rot (the caller's q_work).
        constexpr int H2 = D / 2;
        float *qstage = xbuf;
        const int nvalid = min(kRT, nrows - row0);
        const float2 *cs = a.rope32 ? a.rope32 + (size_t)past * H2 : nullptr;
        // The gains and the rotation are the same for every row of the tile (one token): loaded
        // once, together with the first row, instead of after each row's sum of squares.
        float gq0[H2 / 32], gq1[H2 / 32];
        float2 cq[H2 / 32];
#pragma unroll
        for (int u = 0; u < H2 / 32; ++u) {
            const int i = lane + 32 * u;
            const float w0 = a.q_norm ? a.q_norm[i] : 1.f, w1 = a.q_norm ? a.q_norm[i + H2] : 1.f;
            gq0[u] = a.q_norm && a.one_plus ? 1.f + w0 : w0;
            gq1[u] = a.q_norm && a.one_plus ? 1.f + w1 : w1;
            cq[u] = cs ? cs[i] : make_float2(1.f, 0.f);
        }
        for (int j = warp; j < nvalid; j += NC) {
            const size_t R = (size_t)b * a.Hq + kvh * G + (row0 + j) % G;  // one token
            const float *src = a.q_in + R * D;
            float x0[H2 / 32], x1[H2 / 32];
            float ss = 0.f;
#pragma unroll
            for (int u = 0; u < H2 / 32; ++u) {
                x0[u] = src[lane + 32 * u];
                x1[u] = src[lane + 32 * u + H2];
                ss = fmaf(x0[u], x0[u], fmaf(x1[u], x1[u], ss));
            }
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
            const float inv = a.q_norm ? 1.f / sqrtf(ss / (float)D + (float)a.eps) : 1.f;
            float *dst = qstage + j * L::kQStride;
#pragma unroll
            for (int u = 0; u < H2 / 32; ++u) {
                const int i = lane + 32 * u;
                float y0 = x0[u], y1 = x1[u];
                if (a.q_norm) {
                    y0 *= inv * gq0[u];
                    y1 *= inv * gq1[u];
                }
                float o0 = y0, o1 = y1;
                if (cs) {
                    const float2 c = cq[u];
                    o0 = y0 * c.x - y1 * c.y;
                    o1 = y1 * c.x + y0 * c.y;
                }
                dst[i] = o0;
                dst[i + H2] = o1;
                if (split == 0) {
                    a.q_rot[R * D + i] = o0;
                    a.q_rot[R * D + i + H2] = o1;
                }
            }
        }
        named_barrier_sync(1, NC * 32);
    }

    // Q^T fragments (B operand, column qr = query row row0 + qr), fp32 -> fp16: from global
    // memory, or (fused) from the staged rows.
    uint32_t qf[KS][2];
    {
        const int rq = row0 + qr;
        const float *qrow = nullptr;
        if (rq < nrows)
            qrow = F ? xbuf + qr * L::kQStride + dh * DH
                     : a.q + (((size_t)b * T + rq / G) * a.Hq + kvh * G + rq % G) * D + dh * DH;
#pragma unroll
        for (int ks = 0; ks < KS; ++ks) {
            if constexpr (Q8) {
                const float4 x = qrow ? *reinterpret_cast<const float4 *>(qrow + W * qc + 4 * ks)
                                      : make_float4(0.f, 0.f, 0.f, 0.f);
                qf[ks][0] = pack_half2(x.x, x.y);
                qf[ks][1] = pack_half2(x.z, x.w);
            } else {
                const float2 x0 = qrow ? *reinterpret_cast<const float2 *>(qrow + ks * 16 + 2 * qc) : make_float2(0.f, 0.f);
                const float2 x1 =
                    qrow ? *reinterpret_cast<const float2 *>(qrow + ks * 16 + 8 + 2 * qc) : make_float2(0.f, 0.f);
                qf[ks][0] = pack_half2(x0.x, x0.y);
                qf[ks][1] = pack_half2(x1.x, x1.y);
            }
        }
    }
    if constexpr (F) named_barrier_sync(1, NC * 32);  // the staging bytes become the score swap

    // int8: 1152 * (sum of the fp16 q over this slice) for rows 2qc, 2qc + 1 -- the bias of the
    // raw scores against biased codes.
    float qbias[2] = {0.f, 0.f};
    if constexpr (Q8) {
        float part = 0.f;
#pragma unroll
        for (int ks = 0; ks < KS; ++ks) {
            const float2 f0 = __half22float2(*reinterpret_cast<const __half2 *>(&qf[ks][0]));
            const float2 f1 = __half22float2(*reinterpret_cast<const __half2 *>(&qf[ks][1]));
            part += (f0.x + f0.y) + (f1.x + f1.y);
        }
        part += __shfl_xor_sync(0xffffffffu, part, 1);
        part += __shfl_xor_sync(0xffffffffu, part, 2);  // row qr's sum, in every lane of quad qr
        qbias[0] = kCodeBias * __shfl_sync(0xffffffffu, part, 8 * qc);
        qbias[1] = kCodeBias * __shfl_sync(0xffffffffu, part, 8 * qc + 4);
    }

    // This lane's scores are keys (qr, qr + 8) x rows (2qc, 2qc + 1): causal / window limits.
    int hi[2], lo[2];
#pragma unroll
    for (int j = 0; j < 2; ++j) {
        const int r = row0 + 2 * qc + j;
        hi[j] = r < nrows ? past + r / G - a.kv_offset : -1;
        lo[j] = a.window > 0 ? past + r / G - a.window + 1 - a.kv_offset : INT_MIN;
    }
    const bool use_cap = a.softcap > 0.f;
    // Keys every valid row of the tile attends: [kin_lo, kin_hi).
    const int t_first = row0 / G, t_last = (min(row0 + kRT, nrows) - 1) / G;
    const int kin_hi = min(k_end, past + t_first + 1 - a.kv_offset);
    const int kin_lo = a.window > 0 ? past + t_last - a.window + 1 - a.kv_offset : INT_MIN;

    float o[MT][4];
#pragma unroll
    for (int m = 0; m < MT; ++m) o[m][0] = o[m][1] = o[m][2] = o[m][3] = 0.f;
    float m2[2] = {-CUDART_INF_F, -CUDART_INF_F};  // running max per row, log2 units
    float lsum[2] = {0.f, 0.f};                    // this lane's share of the running sums
    float psum[2] = {0.f, 0.f};                    // int8: same for the fp16 p' fed to the tensor cores

    for (int i = 0; i < ntiles; ++i) {
        const int s = i % S;
        if (!mbar_wait(&full[s], (i / S) & 1, a.err, kErrTmaTimeout)) break;
        uint8_t *kt = ring + s * L::kStageBytes;
        uint8_t *vt = kt + L::kTileBytes;
        const int key0 = k_begin + i * SK + kg * 16;

        // ---- S^T = K Q^T for the warp's 16 keys over its head-dim slice (two accumulators, even
        // and odd k-steps, to halve the dependent MMA chain).
        float sacc[4];
        float sacc2[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
        if constexpr (Q8) {
            const uint8_t *kb = kt + dh * L::kBoxBytes;
            const int rA = kg * 16 + qr, rB = rA + 8;
            uint32_t wa[KS], wb[KS];
            if constexpr (DH == 128) {
                const uint4 a0 = *reinterpret_cast<const uint4 *>(kb + sw128(rA, 2 * qc));
                const uint4 a1 = *reinterpret_cast<const uint4 *>(kb + sw128(rA, 2 * qc + 1));
                const uint4 b0 = *reinterpret_cast<const uint4 *>(kb + sw128(rB, 2 * qc));
                const uint4 b1 = *reinterpret_cast<const uint4 *>(kb + sw128(rB, 2 * qc + 1));
                wa[0] = a0.x, wa[1] = a0.y, wa[2] = a0.z, wa[3] = a0.w, wa[4] = a1.x, wa[5] = a1.y, wa[6] = a1.z;
                wa[7] = a1.w;
                wb[0] = b0.x, wb[1] = b0.y, wb[2] = b0.z, wb[3] = b0.w, wb[4] = b1.x, wb[5] = b1.y, wb[6] = b1.z;
                wb[7] = b1.w;
            } else {
                const uint4 a0 = *reinterpret_cast<const uint4 *>(kb + sw64(rA, qc));
                const uint4 b0 = *reinterpret_cast<const uint4 *>(kb + sw64(rB, qc));
                wa[0] = a0.x, wa[1] = a0.y, wa[2] = a0.z, wa[3] = a0.w;
                wb[0] = b0.x, wb[1] = b0.y, wb[2] = b0.z, wb[3] = b0.w;
            }
#pragma unroll
            for (int ks = 0; ks < KS; ++ks)
                mma_16816(sacc2[ks & 1], codes_biased_half2(wa[ks], 0x4140u), codes_biased_half2(wb[ks], 0x4140u),
                          codes_biased_half2(wa[ks], 0x4342u), codes_biased_half2(wb[ks], 0x4342u), qf[ks][0],
                          qf[ks][1]);
#pragma unroll
            for (int e = 0; e < 4; ++e) sacc[e] = (sacc2[0][e] + sacc2[1][e]) - qbias[e & 1];
        } else {
            const int krow = kg * 16 + (lane & 15);
#pragma unroll
            for (int ks = 0; ks < KS; ++ks) {
                const int chunk = dh * (DH / 8) + ks * 2 + (lane >> 4);
                uint32_t a0, a1, a2, a3;
                ldsm_x4(smem_addr(kt + (chunk >> 3) * L::kBoxBytes + sw128(krow, chunk & 7)), a0, a1, a2, a3);
                mma_16816(sacc2[ks & 1], a0, a1, a2, a3, qf[ks][0], qf[ks][1]);
            }
#pragma unroll
            for (int e = 0; e < 4; ++e) sacc[e] = sacc2[0][e] + sacc2[1][e];
        }
        if constexpr (DS > 1) {
            // Swap partial scores with the warp holding the other head-dim half (double-buffered by
            // tile parity: one pair barrier per tile); add in a fixed order so both agree.
            float *mine = xbuf + (((kg * 2 + (i & 1)) * 2 + dh) * 32 + lane) * 4;
            const float *theirs = xbuf + (((kg * 2 + (i & 1)) * 2 + (dh ^ 1)) * 32 + lane) * 4;
            *reinterpret_cast<float4 *>(mine) = make_float4(sacc[0], sacc[1], sacc[2], sacc[3]);
            named_barrier_sync(2 + kg, 64);
            const float4 t = *reinterpret_cast<const float4 *>(theirs);
            if (dh == 0) {
                sacc[0] += t.x, sacc[1] += t.y, sacc[2] += t.z, sacc[3] += t.w;
            } else {
                sacc[0] = t.x + sacc[0], sacc[1] = t.y + sacc[1], sacc[2] = t.z + sacc[2], sacc[3] = t.w + sacc[3];
            }
        }

        // ---- scaled scores (log2 units), masked on edge tiles, and the online softmax per row.
        float ksc[2] = {1.f, 1.f}, vsc[2] = {1.f, 1.f};
        if constexpr (Q8) {
            const float *sc = reinterpret_cast<const float *>(kt + 2 * L::kTileBytes);
            ksc[0] = sc[kg * 16 + qr];
            ksc[1] = sc[kg * 16 + qr + 8];
            vsc[0] = sc[SK + kg * 16 + qr];
            vsc[1] = sc[SK + kg * 16 + qr + 8];
        }
        const bool interior = key0 >= kin_lo && key0 + 16 <= kin_hi;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            float x = sacc[e];
            if constexpr (Q8) x *= ksc[e >> 1];
            if (use_cap) {
                x = softcap_log2(x, a.cap_k1, a.cap_k2);
            } else {
                x *= a.scale_log2;
            }
            sacc[e] = x;
        }
        bool valid[4] = {true, true, true, true};
        if (!interior) {
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int key = key0 + qr + (e >> 1) * 8;
                const int j = e & 1;  // row 2qc + j
                valid[e] = key >= lo[j] && key <= hi[j] && key < k_end;
                sacc[e] = valid[e] ? sacc[e] : -CUDART_INF_F;
            }
        }
        float mx[2] = {fmaxf(sacc[0], sacc[2]), fmaxf(sacc[1], sacc[3])};
        float muse[2];
        bool grew = false;
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            mx[j] = fmaxf(mx[j], __shfl_xor_sync(0xffffffffu, mx[j], 4));
            mx[j] = fmaxf(mx[j], __shfl_xor_sync(0xffffffffu, mx[j], 8));
            mx[j] = fmaxf(mx[j], __shfl_xor_sync(0xffffffffu, mx[j], 16));
            const float mnew = fmaxf(m2[j], mx[j]);
            grew |= mnew > m2[j];
            muse[j] = mnew == -CUDART_INF_F ? 0.f : mnew;
        }
        // Rescale the running sums and outputs only when some row's maximum grew.
        if (__any_sync(0xffffffffu, grew)) {
            float alpha[2];
#pragma unroll
            for (int j = 0; j < 2; ++j) {
                alpha[j] = ex2_fast(m2[j] - muse[j]);
                lsum[j] *= alpha[j];
                if constexpr (Q8) psum[j] *= alpha[j];
            }
#pragma unroll
            for (int m = 0; m < MT; ++m) {
                o[m][0] *= alpha[0];
                o[m][1] *= alpha[1];
                o[m][2] *= alpha[0];
                o[m][3] *= alpha[1];
            }
        }
#pragma unroll
        for (int j = 0; j < 2; ++j) m2[j] = fmaxf(m2[j], mx[j]);
        float p[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            p[e] = ex2_fast(sacc[e] - muse[e & 1]);
            lsum[e & 1] += p[e];
            if constexpr (Q8) p[e] = valid[e] ? p[e] * vsc[e >> 1] : 0.f;
        }
        const uint32_t pt0 = pack_half2(p[0], p[1]), pt1 = pack_half2(p[2], p[3]);
        if constexpr (Q8) {
            // The fp16 p' the tensor cores see, per row: the bias 1152 * sum(p') of the outputs.
            const float2 f0 = __half22float2(*reinterpret_cast<const __half2 *>(&pt0));
            const float2 f1 = __half22float2(*reinterpret_cast<const __half2 *>(&pt1));
            psum[0] += f0.x + f1.x;
            psum[1] += f0.y + f1.y;
        }
        // P^T fragments -> P fragments (B operand of O^T += V^T P^T): keys 0-7 and 8-15.
        const uint32_t pb0 = movmatrix_t(pt0);
        const uint32_t pb1 = movmatrix_t(pt1);

        // ---- O^T += V^T P^T over the warp's head-dim slice.
        if constexpr (Q8) {
            const uint8_t *vb = vt + dh * L::kBoxBytes;
            const int vr = kg * 16 + 2 * qc;
            uint32_t vw[4][NG];
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const int r = vr + (k & 1) + (k >> 1) * 8;  // keys 2qc, 2qc+1, 2qc+8, 2qc+9
                if constexpr (DH == 128) {
                    const uint4 w = *reinterpret_cast<const uint4 *>(vb + sw128(r, qr));
                    vw[k][0] = w.x, vw[k][1] = w.y, vw[k][2] = w.z, vw[k][3] = w.w;
                } else {
                    const uint2 w = *reinterpret_cast<const uint2 *>(vb + sw64(r, qr >> 1) + (qr & 1) * 8);
                    vw[k][0] = w.x, vw[k][1] = w.y;
                }
            }
#pragma unroll
            for (int g = 0; g < NG; ++g) {
                // Pairs (key 2qc, key 2qc+1) / (2qc+8, 2qc+9) of head-dim bytes 4g+t: t = 0, 1 in
                // lo, t = 2, 3 in hi.  m-tile 2g+u takes bytes 4g+2u (its row qr) and 4g+2u+1 (row qr+8).
                const uint32_t lo01 = prmt(vw[0][g], vw[1][g], 0x5140u), hi01 = prmt(vw[0][g], vw[1][g], 0x7362u);
                const uint32_t lo23 = prmt(vw[2][g], vw[3][g], 0x5140u), hi23 = prmt(vw[2][g], vw[3][g], 0x7362u);
                mma_16816(o[2 * g], codes_biased_half2(lo01, 0x4140u), codes_biased_half2(lo01, 0x4342u),
                          codes_biased_half2(lo23, 0x4140u), codes_biased_half2(lo23, 0x4342u), pb0, pb1);
                mma_16816(o[2 * g + 1], codes_biased_half2(hi01, 0x4140u), codes_biased_half2(hi01, 0x4342u),
                          codes_biased_half2(hi23, 0x4140u), codes_biased_half2(hi23, 0x4342u), pb0, pb1);
            }
        } else {
            // Keys past the range end get zero V (in this warp's slice), so that 0 * (whatever
            // the tile holds there) stays 0.
            const bool tail = key0 + 16 > k_end;
            if (tail) {
                const int first = max(k_end - key0, 0);
                for (int idx = lane; idx < (16 - first) * (DH / 8); idx += 32) {
                    const int rl = first + idx / (DH / 8), ch = dh * (DH / 8) + idx % (DH / 8);
                    *reinterpret_cast<uint4 *>(vt + (ch >> 3) * L::kBoxBytes + sw128(kg * 16 + rl, ch & 7)) =
                        make_uint4(0u, 0u, 0u, 0u);
                }
                __syncwarp();
            }
            const int j8 = lane >> 3;
            const int vrow = kg * 16 + (j8 >> 1) * 8 + (lane & 7);
#pragma unroll
            for (int m = 0; m < MT; ++m) {
                const int chunk = dh * (DH / 8) + m * 2 + (j8 & 1);
                uint32_t a0, a1, a2, a3;
                ldsm_x4_t(smem_addr(vt + (chunk >> 3) * L::kBoxBytes + sw128(vrow, chunk & 7)), a0, a1, a2, a3);
                mma_16816(o[m], a0, a1, a2, a3, pb0, pb1);
            }
        }
        // Every lane's reads of this slot (and the tail's zero stores) are generic-proxy accesses;
        // the next TMA into the slot writes through the async proxy, which the mbarrier's
        // release / acquire alone does not order after them.  Without this fence, int8 launches
        // with two or more CTAs per SM read bytes of the following tile now and then (whole
        // (sequence, kv head) outputs off by 1e-3..3e-2, different from launch to launch).
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
    }

    // ---- merge the key groups' (m, l, O) in shared memory (the ring is free now).
#pragma unroll
    for (int j = 0; j < 2; ++j) {
        lsum[j] += __shfl_xor_sync(0xffffffffu, lsum[j], 4);
        lsum[j] += __shfl_xor_sync(0xffffffffu, lsum[j], 8);
        lsum[j] += __shfl_xor_sync(0xffffffffu, lsum[j], 16);
        if constexpr (Q8) {
            psum[j] += __shfl_xor_sync(0xffffffffu, psum[j], 4);
            psum[j] += __shfl_xor_sync(0xffffffffu, psum[j], 8);
            psum[j] += __shfl_xor_sync(0xffffffffu, psum[j], 16);
        }
    }
    if constexpr (Q8) {
        // Remove the code bias: O^T[d][row] -= 1152 * sum of the row's p'.
#pragma unroll
        for (int m = 0; m < MT; ++m) {
            o[m][0] -= kCodeBias * psum[0];
            o[m][1] -= kCodeBias * psum[1];
            o[m][2] -= kCodeBias * psum[0];
            o[m][3] -= kCodeBias * psum[1];
        }
    }
    named_barrier_sync(1, NC * 32);
    float *cm = reinterpret_cast<float *>(ring);  // [key group][kRT]
    float *cl = cm + KG * kRT;                    // [key group][kRT]
    float *co = cl + KG * kRT;                    // [key group][kRT][D]
    if (qr == 0 && dh == 0) {
        cm[kg * kRT + 2 * qc] = m2[0];
        cm[kg * kRT + 2 * qc + 1] = m2[1];
        cl[kg * kRT + 2 * qc] = lsum[0];
        cl[kg * kRT + 2 * qc + 1] = lsum[1];
    }
    float *c0 = co + (kg * kRT + 2 * qc) * D;  // row 2qc; row 2qc + 1 is D further
#pragma unroll
    for (int m = 0; m < MT; ++m) {
        // Head-dim rows of m-tile m held by this lane: dA (fragment row qr), dB (row qr + 8).
        int dA, dB;
        if constexpr (Q8) {
            dA = dh * DH + VW * qr + 4 * (m >> 1) + 2 * (m & 1);
            dB = dA + 1;
        } else {
            dA = dh * DH + m * 16 + qr;
            dB = dA + 8;
        }
        c0[dA] = o[m][0];
        c0[D + dA] = o[m][1];
        c0[dB] = o[m][2];
        c0[D + dB] = o[m][3];
    }
    named_barrier_sync(1, NC * 32);

    if (a.cluster)
        decode_epilogue_cluster<D, KG, NC, kRT>(a, ring, row0, nrows, kvh, b, split);
    else
        decode_epilogue<D, KG, NC, kRT>(a, ring, row0, nrows, kvh, mtile, b, split);
}

// Log-sum-exp merge of one row's partials by one warp (brk_attn_combine: partials gathered from
// several GPUs); the row's maximum and sum are reduced across the lanes first.
__device__ __forceinline__ void combine_row(const CombineArgs &a, int row, int lane) {
    float M = -CUDART_INF_F;
    for (int p = lane; p < a.n_parts; p += 32) M = fmaxf(M, a.part_ml[(size_t)p * a.stride_ml + (size_t)row * 2]);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, off));
    float Lsum = 0.f;
    if (M != -CUDART_INF_F)
        for (int p = lane; p < a.n_parts; p += 32) {
            const float m = a.part_ml[(size_t)p * a.stride_ml + (size_t)row * 2];
            if (m != -CUDART_INF_F) Lsum += a.part_ml[(size_t)p * a.stride_ml + (size_t)row * 2 + 1] * expf(m - M);
        }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) Lsum += __shfl_xor_sync(0xffffffffu, Lsum, off);
    for (int d = lane; d < a.D; d += 32) {
        float O = 0.f;
        if (M != -CUDART_INF_F)
            for (int p = 0; p < a.n_parts; ++p) {
                const float m = a.part_ml[(size_t)p * a.stride_ml + (size_t)row * 2];
                if (m != -CUDART_INF_F) O += a.part_o[(size_t)p * a.stride_o + (size_t)row * a.D + d] * expf(m - M);
            }
        if (a.out) {
            a.out[(size_t)row * a.D + d] = O / Lsum;
        } else {
            a.out_o[(size_t)row * a.D + d] = O;
            if (d == 0) {
                a.out_ml[(size_t)row * 2] = M;
                a.out_ml[(size_t)row * 2 + 1] = Lsum;
            }
        }
    }
}

__global__ void combine_kernel(const __grid_constant__ CombineArgs a) {
    const int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (row < a.rows) combine_row(a, row, lane);
}

// The combine of a sequence-sharded decode over peer memory: one thread per block waits until
// every rank's flag holds `epoch` (each rank's decode launch stores it after its last partial
// landed here), bounded by wait_ns; on timeout the context's error word records
// kErrPeerTimeout and the block writes nothing.
__global__ void combine_peers_kernel(const __grid_constant__ CombineArgs a, const unsigned *flags, int world,
                                     unsigned epoch, unsigned long long wait_ns, int *err) {
    __shared__ int ready;
    if (threadIdx.x == 0) {
        int ok = 1;
        const unsigned long long t0 = global_timer_ns();
        for (int p = 0; p < world && ok; ++p) {
            uint32_t polls = 0;
            while (ld_acquire_sys(flags + p) != epoch) {
                if ((++polls & 63u) == 0 && (global_timer_ns() - t0 > wait_ns || polls >= kWaitPolls)) {
                    ok = 0;
                    break;
                }
            }
        }
        if (!ok && err) atomicCAS(err, 0, kErrPeerTimeout);
        ready = ok;
    }
    __syncthreads();
    if (!ready) return;
    const int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (row < a.rows) combine_row(a, row, lane);
}

template <bool Q8, int D, bool F>
cudaError_t launch_t(const CUtensorMap &tmk, const CUtensorMap &tmv, const CUtensorMap &tms, const DecodeArgs &a,
                      dim3 grid, cudaStream_t s, bool pdl) {
    static unsigned long long configured = 0;  // one bit per device: the opt-in is per device
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 64 || !(configured & (1ull << dev))) {
        cudaError_t e = cudaFuncSetAttribute(decode_kernel<Q8, D, F>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             DecodeLayout<Q8, D>::kSmemBytes);
        if (e == cudaSuccess) e = cudaFuncSetAttribute(decode_kernel<Q8, D, F>,
                                                       cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
        if (e != cudaSuccess) return e;
        if (dev < 64) configured |= 1ull << dev;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(decode_threads<Q8, D, F>());
    cfg.dynamicSmemBytes = DecodeLayout<Q8, D>::kSmemBytes;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    int n = 0;
    if (pdl) {
        attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[n++].val.programmaticStreamSerializationAllowed = 1;
    }
    if (a.cluster) {
        attr[n].id = cudaLaunchAttributeClusterDimension;
        attr[n].val.clusterDim.x = grid.x;  // the splits of a tile
        attr[n].val.clusterDim.y = 1;
        attr[n++].val.clusterDim.z = 1;
    }
    cfg.attrs = attr;
    cfg.numAttrs = n;
    return cudaLaunchKernelEx(&cfg, decode_kernel<Q8, D, F>, tmk, tmv, tms, a);
}

template <int D>
cudaError_t launch_dt(bool q8, bool fused, const CUtensorMap &tmk, const CUtensorMap &tmv, const CUtensorMap &tms,
                      const DecodeArgs &a, dim3 grid, cudaStream_t s, bool pdl) {
    if (q8) return fused ? launch_t<true, D, true>(tmk, tmv, tms, a, grid, s, pdl)
                         : launch_t<true, D, false>(tmk, tmv, tms, a, grid, s, pdl);
    return fused ? launch_t<false, D, true>(tmk, tmv, tms, a, grid, s, pdl)
                 : launch_t<false, D, false>(tmk, tmv, tms, a, grid, s, pdl);
}

template <bool Q8, int D>
int ctas_t() {
    static int n = 0;
    if (n == 0) {
        cudaFuncSetAttribute(decode_kernel<Q8, D, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             DecodeLayout<Q8, D>::kSmemBytes);
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, decode_kernel<Q8, D, false>, DecodeLayout<Q8, D>::kThreads,
                                                          DecodeLayout<Q8, D>::kSmemBytes) != cudaSuccess ||
            n < 1)
            n = 1;
    }
    return n;
}

}  // namespace

int decode_rows_per_tile() { return kRT; }

namespace {
template <bool Q8, int D>
int clusters_t(int size) {
    static int cache[17] = {};  // per cluster size; the GPU's partition into GPCs is fixed
    if (size < 2 || size > 16) return 0;
    if (cache[size] == 0) {
        cudaFuncSetAttribute(decode_kernel<Q8, D, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             DecodeLayout<Q8, D>::kSmemBytes);
        cudaFuncSetAttribute(decode_kernel<Q8, D, false>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(size, 64, 1);
        cfg.blockDim = dim3(DecodeLayout<Q8, D>::kThreads);
        cfg.dynamicSmemBytes = DecodeLayout<Q8, D>::kSmemBytes;
        cudaLaunchAttribute attr;
        attr.id = cudaLaunchAttributeClusterDimension;
        attr.val.clusterDim.x = size;
        attr.val.clusterDim.y = 1;
        attr.val.clusterDim.z = 1;
        cfg.attrs = &attr;
        cfg.numAttrs = 1;
        int n = 0;
        if (cudaOccupancyMaxActiveClusters(&n, decode_kernel<Q8, D, false>, &cfg) != cudaSuccess) {
            cudaGetLastError();
            n = 0;
        }
        cache[size] = n > 0 ? n : -1;
    }
    return cache[size] > 0 ? cache[size] : 0;
}
}  // namespace

int decode_max_clusters(int head_dim, bool q8, int size) {
    switch (head_dim) {
        case 64: return q8 ? clusters_t<true, 64>(size) : clusters_t<false, 64>(size);
        case 128: return q8 ? clusters_t<true, 128>(size) : clusters_t<false, 128>(size);
        case 256: return q8 ? clusters_t<true, 256>(size) : clusters_t<false, 256>(size);
        default: return 0;
    }
}

cudaError_t preload_decode_kernels() {
    // With lazy module loading a kernel's code is loaded, and its device memory taken, at the
    // first launch; asking for its attributes loads it now.
    const void *fns[] = {(const void *)decode_kernel<false, 64, false>, (const void *)decode_kernel<false, 128, false>,
                         (const void *)decode_kernel<false, 256, false>, (const void *)decode_kernel<true, 64, false>,
                         (const void *)decode_kernel<true, 128, false>,  (const void *)decode_kernel<true, 256, false>,
                         (const void *)decode_kernel<false, 64, true>,  (const void *)decode_kernel<false, 128, true>,
                         (const void *)decode_kernel<false, 256, true>, (const void *)decode_kernel<true, 64, true>,
                         (const void *)decode_kernel<true, 128, true>,  (const void *)decode_kernel<true, 256, true>,
                         (const void *)combine_kernel,            (const void *)combine_peers_kernel};
    for (const void *f : fns) {
        cudaFuncAttributes fa;
        cudaError_t e = cudaFuncGetAttributes(&fa, f);
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

int decode_ctas_per_sm(int head_dim, bool q8) {
    switch (head_dim) {
        case 64: return q8 ? ctas_t<true, 64>() : ctas_t<false, 64>();
        case 128: return q8 ? ctas_t<true, 128>() : ctas_t<false, 128>();
        case 256: return q8 ? ctas_t<true, 256>() : ctas_t<false, 256>();
        default: return 1;
    }
}

cudaError_t launch_decode(bool q8, int head_dim, const CUtensorMap &tmk, const CUtensorMap &tmv,
                           const CUtensorMap &tms, const DecodeArgs &a, int grid_x, int grid_y, int grid_z,
                           cudaStream_t s, bool pdl) {
    static_assert(DecodeLayout<false, 64>::kStageKeys == 64 && DecodeLayout<false, 128>::kStageKeys == 64 &&
                      DecodeLayout<false, 256>::kStageKeys == 32 && DecodeLayout<true, 64>::kStageKeys == 64 &&
                      DecodeLayout<true, 128>::kStageKeys == 64 && DecodeLayout<true, 256>::kStageKeys == 32,
                  "stage keys must match decode_stage_keys()");
    const dim3 grid(grid_x, grid_y, grid_z);
    switch (head_dim) {
        case 64: return launch_dt<64>(q8, a.fuse != 0, tmk, tmv, tms, a, grid, s, pdl);
        case 128: return launch_dt<128>(q8, a.fuse != 0, tmk, tmv, tms, a, grid, s, pdl);
        case 256: return launch_dt<256>(q8, a.fuse != 0, tmk, tmv, tms, a, grid, s, pdl);
        default: return cudaErrorInvalidValue;
    }
}

int decode_stage_keys(int head_dim) {
    switch (head_dim) {
        case 64: return DecodeLayout<false, 64>::kStageKeys;
        case 128: return DecodeLayout<false, 128>::kStageKeys;
        case 256: return DecodeLayout<false, 256>::kStageKeys;
        default: return 64;
    }
}

cudaError_t launch_combine_peers(const CombineArgs &a, const unsigned *flags, int world, unsigned epoch,
                                 unsigned long long wait_ns, int *err, cudaStream_t s) {
    if (a.rows == 0) return cudaSuccess;
    const int threads = 256;
    const long long blocks = ((long long)a.rows * 32 + threads - 1) / threads;
    combine_peers_kernel<<<(unsigned)blocks, threads, 0, s>>>(a, flags, world, epoch, wait_ns, err);
    return cudaGetLastError();
}

cudaError_t launch_combine(const CombineArgs &a, cudaStream_t s) {
    if (a.rows == 0) return cudaSuccess;
    const int threads = 256;
    const long long blocks = ((long long)a.rows * 32 + threads - 1) / threads;
    combine_kernel<<<(unsigned)blocks, threads, 0, s>>>(a);
    return cudaGetLastError();
}

}  // namespace brk
