// Decode attention over the resident fp16 KV cache (replaces attention_decode,
// shaders.ts:1768-1851, and its dispatch in recAttention, kernels.ts:1626-1641).
//
// One CTA per (sequence, kv head, row tile, split).  The rows of a CTA are up to 16 (token,
// q head) pairs of one kv head's query group, so every K/V byte read from HBM serves the whole
// group (the reference re-reads K/V once per q head).  A producer warp streams the CTA's key
// range through a ring of shared-memory stages with 2-D TMA loads (128-byte swizzled
// [keys][64 x fp16] boxes, CTA-local).  Consumer warps come in key groups (four, or two for
// head_dim 256), each taking 16 keys of every stage; with the head-dim split DS = 2 (head_dim
// 256) each key group is a warp pair that owns one half of the head dimension and swaps partial
// QK^T scores through shared memory.  QK^T and PV run on the tensor cores (mma.m16n8k16, fp16 in, fp32 accumulate) with an
// online softmax per warp (quad shuffles).  The key groups merge their (max, sum, output) in
// shared memory; with split-KV the last CTA of a (sequence, kv head, row tile) merges the splits.
#include "decode_common.cuh"

namespace brk {

namespace {

constexpr int kKeysPerWarp = 16;

template <int D>
struct DecodeCfg;
template <>
struct DecodeCfg<64> {
    static constexpr int kStages = 6, kMinBlocks = 2, kDSplit = 1, kKeyGroups = 4;
};
template <>
struct DecodeCfg<128> {
    static constexpr int kStages = 3, kMinBlocks = 2, kDSplit = 1, kKeyGroups = 4;
};
// head_dim 256: two key groups (32-key stages) x two head-dim halves, so that two CTAs fit per SM.
template <>
struct DecodeCfg<256> {
    static constexpr int kStages = 3, kMinBlocks = 2, kDSplit = 2, kKeyGroups = 2;
};

template <int D>
struct DecodeLayout {
    static constexpr int kDS = DecodeCfg<D>::kDSplit;
    static constexpr int kKG = DecodeCfg<D>::kKeyGroups;
    static constexpr int kStageKeys = kKeysPerWarp * kKG;           // keys per ring stage
    static constexpr int kConsumers = kKG * kDS;                    // consumer warps
    static constexpr int kThreads = (kConsumers + 1) * 32;          // + one producer warp
    static constexpr int kBlocks = D / 64;                          // 128-byte column blocks per row
    static constexpr uint32_t kBoxBytes = kStageKeys * 128;         // one [keys][64] fp16 box
    static constexpr uint32_t kTileBytes = kBlocks * kBoxBytes;     // K (or V) of one stage
    static constexpr uint32_t kStageBytes = 2 * kTileBytes;
    static constexpr uint32_t kRingBytes = DecodeCfg<D>::kStages * kStageBytes;
    static constexpr uint32_t kQBytes = kBlocks * 16 * 128;         // 16 rows of q, fp16, swizzled
    // Score swap of the head-dim halves, [key group][parity][half][lane][8] floats; it reuses
    // the q staging area once every warp holds its q fragments.
    static constexpr uint32_t kXBytes = kDS > 1 ? kKG * 2 * 2 * 32 * 8 * 4 : 0;
    static_assert(kXBytes <= kQBytes, "score swap must fit in the q staging area");
    static constexpr uint32_t kBarBytes = 2 * DecodeCfg<D>::kStages * 8;
    static constexpr uint32_t kSmemBytes = 1024 + kRingBytes + kQBytes + kBarBytes;
    static_assert(decode_epilogue_bytes<D, kKG>() <= kRingBytes, "merge buffers must fit in the ring");
};

template <int D>
__global__ void __launch_bounds__(DecodeLayout<D>::kThreads, DecodeCfg<D>::kMinBlocks)
    decode_attn_kernel(const __grid_constant__ CUtensorMap tmk, const __grid_constant__ CUtensorMap tmv,
                       const __grid_constant__ DecodeArgs a) {
    using L = DecodeLayout<D>;
    constexpr int S = DecodeCfg<D>::kStages;
    constexpr int DS = L::kDS;
    constexpr int NC = L::kConsumers;
    constexpr int KG = L::kKG;
    constexpr int kStageKeys = L::kStageKeys;
    constexpr int DH = D / DS;     // head-dim slice of one warp
    constexpr int KS = DH / 16;    // k-steps of QK^T per warp
    constexpr int NTO = DH / 8;    // output n-tiles per warp
    static_assert(DH <= 128, "per-warp head-dim slice");

    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *ring = smem;
    uint8_t *qs = ring + L::kRingBytes;
    float *xbuf = reinterpret_cast<float *>(qs);  // score swap, after the q fragments are loaded
    uint64_t *full = reinterpret_cast<uint64_t *>(qs + L::kQBytes);
    uint64_t *empty = full + S;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int split = blockIdx.x;
    const int kvh = blockIdx.y / a.mtiles, mt = blockIdx.y % a.mtiles;
    const int b = blockIdx.z;
    const int G = a.G, T = a.T;
    const int nrows = T * G;
    const int row0 = mt * 16;
    const int past = a.past_len[b];

    // Key range of this CTA, in cache rows.
    const KeyRange kr = decode_key_range(a, past, row0, nrows, split, kStageKeys, 1);
    const int k_begin = kr.k_begin, k_end = kr.k_end, ntiles = kr.ntiles;
    const int seg_row = ((a.layer * a.B + b) * a.Hkv + kvh) * a.cap;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], NC);
        }
        fence_barrier_init();
    }
    __syncthreads();  // barrier initialisation visible to every warp

    if (warp == NC) {
        // ---- producer: one elected lane streams K/V tiles through the ring.
        if (lane == 0 && ntiles > 0) {
            tma_prefetch_desc(&tmk);
            tma_prefetch_desc(&tmv);
            int issued = 0;
            bool waited = false;
            // Rows from dep_row on may be written by a preceding kernel (the append, when this
            // launch is its programmatic dependent): tiles touching them wait for it to finish.
            const int dep_row = past - a.kv_offset;
            for (int i = 0; i < ntiles; ++i) {
                const int s = i % S;
                if (!waited && k_begin + (i + 1) * kStageKeys > dep_row) {
                    griddep_wait();
                    waited = true;
                }
                if (i >= S && !mbar_wait(&empty[s], ((i / S) - 1) & 1, a.err, kErrSlotTimeout)) break;
                mbar_arrive_expect_tx(&full[s], L::kStageBytes);
                uint8_t *st = ring + s * L::kStageBytes;
                const int y = seg_row + k_begin + i * kStageKeys;
#pragma unroll
                for (int j = 0; j < L::kBlocks; ++j) tma_load_2d(st + j * L::kBoxBytes, &tmk, j * 64, y, &full[s]);
#pragma unroll
                for (int j = 0; j < L::kBlocks; ++j)
                    tma_load_2d(st + L::kTileBytes + j * L::kBoxBytes, &tmv, j * 64, y, &full[s]);
                issued = i + 1;
            }
            // Before leaving, make sure every copy this lane started has landed (bounded).
            for (int i = issued > S ? issued - S : 0; i < issued; ++i)
                mbar_wait(&full[i % S], (i / S) & 1, a.err, kErrTmaTimeout);
        }
        return;
    }

    // ---- consumers: stage this CTA's 16 q rows as fp16, in the same swizzled layout as the K
    // boxes (q comes from the preceding append when launched as its dependent).
    griddep_wait();
    for (int idx = threadIdx.x; idx < 16 * (D / 8); idx += NC * 32) {
        const int r = idx / (D / 8), ch = idx % (D / 8);
        const int rr = row0 + r;
        float4 x0 = make_float4(0.f, 0.f, 0.f, 0.f), x1 = x0;
        if (rr < nrows) {
            const int t = rr / G, h = kvh * G + rr % G;
            const float *src = a.q + (((size_t)b * T + t) * a.Hq + h) * D + ch * 8;
            x0 = *reinterpret_cast<const float4 *>(src);
            x1 = *reinterpret_cast<const float4 *>(src + 4);
        }
        uint4 pk;
        pk.x = pack_half2(x0.x, x0.y);
        pk.y = pack_half2(x0.z, x0.w);
        pk.z = pack_half2(x1.x, x1.y);
        pk.w = pack_half2(x1.z, x1.w);
        *reinterpret_cast<uint4 *>(qs + (ch >> 3) * 2048 + sw128(r, ch & 7)) = pk;
    }
    named_barrier_sync(1, NC * 32);

    const int kg = warp % KG;  // key group: keys [16 kg, 16 kg + 16) of every stage
    const int dh = warp / KG;  // head-dim slice [DH dh, DH dh + DH)
    const int qr = lane >> 2, qc = lane & 3;
    uint32_t qf[KS][4];
#pragma unroll
    for (int k = 0; k < KS; ++k) {
        const int ks = dh * KS + k;  // global k-step over D
        ldsm_x4(smem_addr(qs + (ks >> 2) * 2048 + sw128(lane & 15, (ks & 3) * 2 + (lane >> 4))), qf[k][0], qf[k][1],
                qf[k][2], qf[k][3]);
    }
    if constexpr (DS > 1) named_barrier_sync(1, NC * 32);  // q staging area becomes the score swap

    // Causal / window limits of this lane's two rows (rows rA and rA + 8 of the tile).
    const int rA = row0 + qr, rB = rA + 8;
    const int hiA = rA < nrows ? past + rA / G - a.kv_offset : -1;
    const int hiB = rB < nrows ? past + rB / G - a.kv_offset : -1;
    const int loA = a.window > 0 ? past + rA / G - a.window + 1 - a.kv_offset : INT_MIN;
    const int loB = a.window > 0 ? past + rB / G - a.window + 1 - a.kv_offset : INT_MIN;
    const bool use_cap = a.softcap > 0.f;

    float o[NTO][4];
#pragma unroll
    for (int n = 0; n < NTO; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
    float m2[2] = {-CUDART_INF_F, -CUDART_INF_F};  // running max, log2 units
    float lsum[2] = {0.f, 0.f};                    // this lane's share of the running sum

    for (int i = 0; i < ntiles; ++i) {
        const int s = i % S;
        if (!mbar_wait(&full[s], (i / S) & 1, a.err, kErrTmaTimeout)) break;
        uint8_t *kt = ring + s * L::kStageBytes;
        uint8_t *vt = kt + L::kTileBytes;
        const int key0 = k_begin + i * kStageKeys + kg * kKeysPerWarp;

        // S = Q K^T over this warp's head-dim slice for its 16 keys (two n-tiles of 8 keys).
        float sacc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
        const int krow = kg * kKeysPerWarp + ((lane >> 4) << 3) + (lane & 7);
#pragma unroll
        for (int k = 0; k < KS; ++k) {
            const int ks = dh * KS + k;
            uint32_t b0, b1, b2, b3;
            ldsm_x4(smem_addr(kt + (ks >> 2) * L::kBoxBytes + sw128(krow, (ks & 3) * 2 + ((lane >> 3) & 1))), b0, b1,
                    b2, b3);
            mma_16816(sacc[0], qf[k][0], qf[k][1], qf[k][2], qf[k][3], b0, b1);
            mma_16816(sacc[1], qf[k][0], qf[k][1], qf[k][2], qf[k][3], b2, b3);
        }
        if constexpr (DS > 1) {
            // Swap partial scores with the warp that holds the other half of the head dim
            // (double-buffered by tile parity, so one pair barrier per tile suffices).
            float *mine = xbuf + (((kg * 2 + (i & 1)) * 2 + dh) * 32 + lane) * 8;
            float *theirs = xbuf + (((kg * 2 + (i & 1)) * 2 + (dh ^ 1)) * 32 + lane) * 8;
            *reinterpret_cast<float4 *>(mine) = make_float4(sacc[0][0], sacc[0][1], sacc[0][2], sacc[0][3]);
            *reinterpret_cast<float4 *>(mine + 4) = make_float4(sacc[1][0], sacc[1][1], sacc[1][2], sacc[1][3]);
            named_barrier_sync(2 + kg, 64);
            const float4 t0 = *reinterpret_cast<const float4 *>(theirs);
            const float4 t1 = *reinterpret_cast<const float4 *>(theirs + 4);
            // Add in a fixed order (slice 0 + slice 1) so both warps hold identical scores.
            const float4 lo0 = dh == 0 ? make_float4(sacc[0][0], sacc[0][1], sacc[0][2], sacc[0][3]) : t0;
            const float4 lo1 = dh == 0 ? make_float4(sacc[1][0], sacc[1][1], sacc[1][2], sacc[1][3]) : t1;
            const float4 hi0 = dh == 0 ? t0 : make_float4(sacc[0][0], sacc[0][1], sacc[0][2], sacc[0][3]);
            const float4 hi1 = dh == 0 ? t1 : make_float4(sacc[1][0], sacc[1][1], sacc[1][2], sacc[1][3]);
            sacc[0][0] = lo0.x + hi0.x, sacc[0][1] = lo0.y + hi0.y, sacc[0][2] = lo0.z + hi0.z;
            sacc[0][3] = lo0.w + hi0.w;
            sacc[1][0] = lo1.x + hi1.x, sacc[1][1] = lo1.y + hi1.y, sacc[1][2] = lo1.z + hi1.z;
            sacc[1][3] = lo1.w + hi1.w;
        }

        // Scores -> masked, scaled (log2 units), online softmax per row.
        float mx[2] = {-CUDART_INF_F, -CUDART_INF_F};
#pragma unroll
        for (int nt = 0; nt < 2; ++nt)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int key = key0 + nt * 8 + 2 * qc + (e & 1);
                const int hi = e < 2 ? hiA : hiB, lo = e < 2 ? loA : loB;
                float x = sacc[nt][e];
                if (use_cap) {
                    // c*tanh(s/c) (shaders.ts:1490) in log2 units, with tanh(z) = 1 - 2/(1 + e^{2z}):
                    // one exp2 and one reciprocal; saturates to +-1 for large |z|.
                    const float e2z = exp2f(x * a.cap_k1);
                    x = a.cap_k2 * (1.f - 2.f * __frcp_rn(1.f + e2z));
                } else {
                    x = x * a.scale_log2;
                }
                x = (key >= lo && key <= hi && key < k_end) ? x : -CUDART_INF_F;
                sacc[nt][e] = x;
                mx[e >> 1] = fmaxf(mx[e >> 1], x);
            }
        float muse[2];
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 1));
            mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 2));
            const float mnew = fmaxf(m2[r], mx[r]);
            muse[r] = mnew == -CUDART_INF_F ? 0.f : mnew;
            const float alpha = exp2f(m2[r] - muse[r]);
            m2[r] = mnew;
            lsum[r] *= alpha;
#pragma unroll
            for (int n = 0; n < NTO; ++n) {
                o[n][2 * r] *= alpha;
                o[n][2 * r + 1] *= alpha;
            }
        }
        float p[2][4];
#pragma unroll
        for (int nt = 0; nt < 2; ++nt)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                p[nt][e] = exp2f(sacc[nt][e] - muse[e >> 1]);
                lsum[e >> 1] += p[nt][e];
            }
        const uint32_t pa0 = pack_half2(p[0][0], p[0][1]);
        const uint32_t pa1 = pack_half2(p[0][2], p[0][3]);
        const uint32_t pa2 = pack_half2(p[1][0], p[1][1]);
        const uint32_t pa3 = pack_half2(p[1][2], p[1][3]);

        // Keys past the range end get zero V (in this warp's head-dim slice), so that
        // 0 * (whatever the tile read there) stays 0.
        const bool tail = key0 + kKeysPerWarp > k_end;
        if (tail) {
            const int first = max(k_end - key0, 0);
            for (int idx = lane; idx < (kKeysPerWarp - first) * (DH / 8); idx += 32) {
                const int rl = first + idx / (DH / 8), ch = dh * (DH / 8) + idx % (DH / 8);
                *reinterpret_cast<uint4 *>(vt + (ch >> 3) * L::kBoxBytes + sw128(kg * kKeysPerWarp + rl, ch & 7)) =
                    make_uint4(0u, 0u, 0u, 0u);
            }
            __syncwarp();
        }

        // O += P V over this warp's head-dim slice (16 keys), V fragments through ldmatrix.trans.
        const int vrow = kg * kKeysPerWarp + (((lane >> 3) & 1) << 3) + (lane & 7);
#pragma unroll
        for (int np = 0; np < NTO / 2; ++np) {
            const int chunk = dh * (DH / 8) + np * 2 + (lane >> 4);
            uint32_t b0, b1, b2, b3;
            ldsm_x4_t(smem_addr(vt + (chunk >> 3) * L::kBoxBytes + sw128(vrow, chunk & 7)), b0, b1, b2, b3);
            mma_16816(o[2 * np], pa0, pa1, pa2, pa3, b0, b1);
            mma_16816(o[2 * np + 1], pa0, pa1, pa2, pa3, b2, b3);
        }
        if (tail) fence_proxy_async_smem();  // generic writes before the next TMA into this slot
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
    }

    // ---- merge the key groups' (m, l, O) in shared memory (the ring is free now).
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        lsum[r] += __shfl_xor_sync(0xffffffffu, lsum[r], 1);
        lsum[r] += __shfl_xor_sync(0xffffffffu, lsum[r], 2);
    }
    named_barrier_sync(1, NC * 32);
    float *cm = reinterpret_cast<float *>(ring);  // [key group][16]
    float *cl = cm + KG * 16;                     // [key group][16]
    float *co = cl + KG * 16;                     // [key group][16][D]
    if (qc == 0 && dh == 0) {
        cm[kg * 16 + qr] = m2[0];
        cm[kg * 16 + qr + 8] = m2[1];
        cl[kg * 16 + qr] = lsum[0];
        cl[kg * 16 + qr + 8] = lsum[1];
    }
#pragma unroll
    for (int n = 0; n < NTO; ++n) {
        const int d = dh * DH + n * 8 + 2 * qc;
        *reinterpret_cast<float2 *>(co + (kg * 16 + qr) * D + d) = make_float2(o[n][0], o[n][1]);
        *reinterpret_cast<float2 *>(co + (kg * 16 + qr + 8) * D + d) = make_float2(o[n][2], o[n][3]);
    }
    named_barrier_sync(1, NC * 32);

    decode_epilogue<D, KG, NC>(a, ring, row0, nrows, kvh, mt, b, split);
}

// Log-sum-exp merge of partials (brk_attn_combine: partials gathered from several GPUs): one
// warp per row; the row's maximum and sum are reduced across the lanes first.
__global__ void combine_kernel(const __grid_constant__ CombineArgs a) {
    const int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (row >= a.rows) return;
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

template <int D>
cudaError_t launch_decode_t(const CUtensorMap &tmk, const CUtensorMap &tmv, const DecodeArgs &a, dim3 grid,
                            cudaStream_t s, bool pdl) {
    static unsigned long long configured = 0;  // one bit per device: the opt-in is per device
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 64 || !(configured & (1ull << dev))) {
        cudaError_t e = cudaFuncSetAttribute(decode_attn_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             DecodeLayout<D>::kSmemBytes);
        if (e != cudaSuccess) return e;
        if (dev < 64) configured |= 1ull << dev;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(DecodeLayout<D>::kThreads);
    cfg.dynamicSmemBytes = DecodeLayout<D>::kSmemBytes;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, decode_attn_kernel<D>, tmk, tmv, a);
}

template <int D>
int ctas_per_sm_t() {
    static int n = 0;
    if (n == 0) {
        cudaFuncSetAttribute(decode_attn_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             DecodeLayout<D>::kSmemBytes);
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, decode_attn_kernel<D>, DecodeLayout<D>::kThreads,
                                                          DecodeLayout<D>::kSmemBytes) != cudaSuccess ||
            n < 1)
            n = 1;
    }
    return n;
}

}  // namespace

int decode_stage_keys(int head_dim) {
    switch (head_dim) {
        case 64: return DecodeLayout<64>::kStageKeys;
        case 128: return DecodeLayout<128>::kStageKeys;
        case 256: return DecodeLayout<256>::kStageKeys;
        default: return 64;
    }
}

int decode_ctas_per_sm(int head_dim, bool q8) {
    if (q8) return decode_q8_ctas_per_sm(head_dim);
    switch (head_dim) {
        case 64: return ctas_per_sm_t<64>();
        case 128: return ctas_per_sm_t<128>();
        case 256: return ctas_per_sm_t<256>();
        default: return 1;
    }
}

cudaError_t launch_decode(int head_dim, const CUtensorMap &tmk, const CUtensorMap &tmv, const DecodeArgs &a,
                          int grid_x, int grid_y, int grid_z, cudaStream_t s, bool pdl) {
    const dim3 grid(grid_x, grid_y, grid_z);
    switch (head_dim) {
        case 64: return launch_decode_t<64>(tmk, tmv, a, grid, s, pdl);
        case 128: return launch_decode_t<128>(tmk, tmv, a, grid, s, pdl);
        case 256: return launch_decode_t<256>(tmk, tmv, a, grid, s, pdl);
        default: return cudaErrorInvalidValue;
    }
}

cudaError_t launch_combine(const CombineArgs &a, cudaStream_t s) {
    if (a.rows == 0) return cudaSuccess;
    const int threads = 256;
    const long long blocks = ((long long)a.rows * 32 + threads - 1) / threads;
    combine_kernel<<<(unsigned)blocks, threads, 0, s>>>(a);
    return cudaGetLastError();
}

}  // namespace brk
