// Decode attention over the int8 KV cache (replaces attention_decode_q8kv / attention_q8kv,
// shaders.ts:1711-1756 and 1856-1944, and their dispatch in recAttentionQ8, kernels.ts:1650-1661).
//
// Same CTA decomposition, ring and epilogue as the fp16 decode kernel (decode.cu): one CTA per
// (sequence, kv head, row tile, split), a producer warp streaming [keys][<=128 B] code boxes and
// a [2][keys] box of f32 scales per stage by TMA, consumer warps in key groups of 16 keys.  The
// cache holds each code biased by +128 (one byte), so a code becomes an exact fp16 value with one
// byte permute and one fp16x2 subtraction (codes_to_half2), and both products run on the tensor
// cores (mma.m16n8k16, fp16 in, fp32 accumulate):
//   - QK^T: the K scale is constant over the head dim, so it factors out of the dot product
//     (shaders.ts:1721-1726): s = scale_k[j] * sum_d q_d code_d.  Each lane reads its K bytes as
//     16-byte words and the head dim is permuted identically in q and K (the dot product does not
//     depend on the order of its terms): k-step ks of lane quad qc covers head-dim bytes
//     W*qc + 4*ks + (0..3), with W = DH/4 the bytes a quad holds.
//   - PV: the V scale varies per key, so it multiplies the probabilities, p'_j = p_j * scale_v[j];
//     the row sum keeps the unscaled p.  A lane's V fragment holds four keys (2qc, 2qc+1, 2qc+8,
//     2qc+9: the keys of its P fragment) at one head-dim index; it reads each key's 16 (DH 128) or
//     8 (DH 64) bytes as one word and transposes the 4 x 4 byte blocks with byte permutes.  The
//     output tile columns are permuted accordingly (column c of group g, byte t <-> head-dim
//     index VW*c + 4g + t) and un-permuted when the key groups merge.
// Both layouts are bank-conflict free for DH 128 (128-byte swizzle); DH 64 uses the 64-byte
// swizzle (conflict free for K, two-way for V).
#include "decode_common.cuh"

namespace brk {

namespace {

template <int D>
struct Q8Cfg;
template <>
struct Q8Cfg<64> {
    static constexpr int kStages = 6, kMinBlocks = 2, kDSplit = 1, kKeyGroups = 4;
};
template <>
struct Q8Cfg<128> {
    static constexpr int kStages = 4, kMinBlocks = 2, kDSplit = 1, kKeyGroups = 4;
};
// head_dim 256: two head-dim halves (one 128-byte code box each) x two key groups.
template <>
struct Q8Cfg<256> {
    static constexpr int kStages = 4, kMinBlocks = 2, kDSplit = 2, kKeyGroups = 2;
};

template <int D>
struct Q8Layout {
    static constexpr int kDS = Q8Cfg<D>::kDSplit;
    static constexpr int kKG = Q8Cfg<D>::kKeyGroups;
    static constexpr int kStageKeys = 16 * kKG;
    static constexpr int kConsumers = kKG * kDS;
    static constexpr int kThreads = (kConsumers + 1) * 32;
    static constexpr int kBoxCols = D < 128 ? D : 128;               // bytes per box row
    static constexpr uint32_t kBoxBytes = kStageKeys * kBoxCols;
    static constexpr uint32_t kTileBytes = kStageKeys * D;           // codes of K (or V) per stage
    static constexpr uint32_t kScaleBytes = 2 * kStageKeys * 4;      // [K, V][keys] f32
    static constexpr uint32_t kLoadBytes = 2 * kTileBytes + kScaleBytes;
    static constexpr uint32_t kStageBytes = (kLoadBytes + 1023) / 1024 * 1024;
    static constexpr uint32_t kRingBytes = Q8Cfg<D>::kStages * kStageBytes;
    // Score swap of the head-dim halves: [key group][parity][half][lane][8] floats.
    static constexpr uint32_t kXBytes = kDS > 1 ? kKG * 2 * 2 * 32 * 8 * 4 : 0;
    static constexpr uint32_t kBarBytes = 2 * Q8Cfg<D>::kStages * 8;
    static constexpr uint32_t kSmemBytes = 1024 + kRingBytes + kXBytes + kBarBytes;
    static_assert(decode_epilogue_bytes<D, kKG>() <= kRingBytes, "merge buffers must fit in the ring");
};

template <int D>
__global__ void __launch_bounds__(Q8Layout<D>::kThreads, Q8Cfg<D>::kMinBlocks)
    decode_q8_kernel(const __grid_constant__ CUtensorMap tmk, const __grid_constant__ CUtensorMap tmv,
                     const __grid_constant__ CUtensorMap tms, const __grid_constant__ DecodeArgs a) {
    using L = Q8Layout<D>;
    constexpr int S = Q8Cfg<D>::kStages;
    constexpr int DS = L::kDS;
    constexpr int NC = L::kConsumers;
    constexpr int KG = L::kKG;
    constexpr int kStageKeys = L::kStageKeys;
    constexpr int DH = D / DS;   // head-dim slice of one warp: 64 or 128
    constexpr int KS = DH / 16;  // k-steps of QK^T
    constexpr int W = DH / 4;    // K bytes of one key row held by a lane quad member
    constexpr int VW = DH / 8;   // V bytes of one key row read by a lane
    constexpr int NG = VW / 4;   // V words per key row per lane
    constexpr int NTO = DH / 8;  // output n-tiles (NG * 4)
    static_assert(DH == 64 || DH == 128, "per-warp head-dim slice");

    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *ring = smem;
    float *xbuf = reinterpret_cast<float *>(ring + L::kRingBytes);
    uint64_t *full = reinterpret_cast<uint64_t *>(ring + L::kRingBytes + L::kXBytes);
    uint64_t *empty = full + S;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int split = blockIdx.x;
    const int kvh = blockIdx.y / a.mtiles, mt = blockIdx.y % a.mtiles;
    const int b = blockIdx.z;
    const int G = a.G, T = a.T;
    const int nrows = T * G;
    const int row0 = mt * 16;
    const int past = a.past_len[b];

    // Key range; a window's first key is rounded down to a multiple of 4 (16-byte scale boxes).
    const KeyRange kr = decode_key_range(a, past, row0, nrows, split, kStageKeys, 4);
    const int k_begin = kr.k_begin, k_end = kr.k_end, ntiles = kr.ntiles;
    const int seg = (a.layer * a.B + b) * a.Hkv + kvh;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], NC);
        }
        fence_barrier_init();
    }
    __syncthreads();

    if (warp == NC) {
        // ---- producer: K codes, V codes and their scales of each stage through the ring.
        if (lane == 0 && ntiles > 0) {
            tma_prefetch_desc(&tmk);
            tma_prefetch_desc(&tmv);
            tma_prefetch_desc(&tms);
            int issued = 0;
            bool waited = false;
            const int dep_row = past - a.kv_offset;  // rows from here on may be the append's
            for (int i = 0; i < ntiles; ++i) {
                const int s = i % S;
                const int key = k_begin + i * kStageKeys;
                if (!waited && key + kStageKeys > dep_row) {
                    griddep_wait();
                    waited = true;
                }
                if (i >= S && !mbar_wait(&empty[s], ((i / S) - 1) & 1, a.err, kErrSlotTimeout)) break;
                mbar_arrive_expect_tx(&full[s], L::kLoadBytes);
                uint8_t *st = ring + s * L::kStageBytes;
                const int y = seg * a.cap + key;
#pragma unroll
                for (int j = 0; j < D / L::kBoxCols; ++j) tma_load_2d(st + j * L::kBoxBytes, &tmk, j * 128, y, &full[s]);
#pragma unroll
                for (int j = 0; j < D / L::kBoxCols; ++j)
                    tma_load_2d(st + L::kTileBytes + j * L::kBoxBytes, &tmv, j * 128, y, &full[s]);
                tma_load_2d(st + 2 * L::kTileBytes, &tms, key, seg * 2, &full[s]);
                issued = i + 1;
            }
            for (int i = issued > S ? issued - S : 0; i < issued; ++i)
                mbar_wait(&full[i % S], (i / S) & 1, a.err, kErrTmaTimeout);
        }
        return;
    }

    griddep_wait();  // q comes from the preceding append when launched as its dependent
    const int kg = warp % KG;  // key group: keys [16 kg, 16 kg + 16) of every stage
    const int dh = warp / KG;  // head-dim slice [DH dh, DH dh + DH)
    const int qr = lane >> 2, qc = lane & 3;

    // q fragments straight from global memory in the codes' k order: k-step ks of this lane
    // covers head-dim indices d0 .. d0+3 with d0 = DH dh + W qc + 4 ks (rows qr and qr + 8).
    uint32_t qf[KS][4];
    {
        const int rA = row0 + qr, rB = rA + 8;
        const float *qa = rA < nrows ? a.q + (((size_t)b * T + rA / G) * a.Hq + kvh * G + rA % G) * D : nullptr;
        const float *qb = rB < nrows ? a.q + (((size_t)b * T + rB / G) * a.Hq + kvh * G + rB % G) * D : nullptr;
#pragma unroll
        for (int ks = 0; ks < KS; ++ks) {
            const int d0 = dh * DH + W * qc + 4 * ks;
            const float4 xa = qa ? *reinterpret_cast<const float4 *>(qa + d0) : make_float4(0.f, 0.f, 0.f, 0.f);
            const float4 xb = qb ? *reinterpret_cast<const float4 *>(qb + d0) : make_float4(0.f, 0.f, 0.f, 0.f);
            qf[ks][0] = pack_half2(xa.x, xa.y);
            qf[ks][1] = pack_half2(xb.x, xb.y);
            qf[ks][2] = pack_half2(xa.z, xa.w);
            qf[ks][3] = pack_half2(xb.z, xb.w);
        }
    }

    const int rA = row0 + qr, rB = rA + 8;
    const int hiA = rA < nrows ? past + rA / G - a.kv_offset : -1;
    const int hiB = rB < nrows ? past + rB / G - a.kv_offset : -1;
    const int loA = a.window > 0 ? past + rA / G - a.window + 1 - a.kv_offset : INT_MIN;
    const int loB = a.window > 0 ? past + rB / G - a.window + 1 - a.kv_offset : INT_MIN;
    const bool use_cap = a.softcap > 0.f;

    float o[NTO][4];
#pragma unroll
    for (int n = 0; n < NTO; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
    float m2[2] = {-CUDART_INF_F, -CUDART_INF_F};
    float lsum[2] = {0.f, 0.f};

    for (int i = 0; i < ntiles; ++i) {
        const int s = i % S;
        if (!mbar_wait(&full[s], (i / S) & 1, a.err, kErrTmaTimeout)) break;
        const uint8_t *st = ring + s * L::kStageBytes;
        const uint8_t *kb = st + dh * L::kBoxBytes;  // the code box of this warp's head-dim slice
        const uint8_t *vb = kb + L::kTileBytes;
        const float *sc = reinterpret_cast<const float *>(st + 2 * L::kTileBytes);
        const int key0 = k_begin + i * kStageKeys + kg * 16;

        // Raw scores sum_d q_d code_d for the warp's 16 keys (two n-tiles of 8).
        float sacc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
        for (int nt = 0; nt < 2; ++nt) {
            const int r = kg * 16 + nt * 8 + qr;
            uint32_t kw[KS];
            if constexpr (DH == 128) {
                const uint4 w0 = *reinterpret_cast<const uint4 *>(kb + sw128(r, 2 * qc));
                const uint4 w1 = *reinterpret_cast<const uint4 *>(kb + sw128(r, 2 * qc + 1));
                kw[0] = w0.x, kw[1] = w0.y, kw[2] = w0.z, kw[3] = w0.w;
                kw[4] = w1.x, kw[5] = w1.y, kw[6] = w1.z, kw[7] = w1.w;
            } else {
                const uint4 w0 = *reinterpret_cast<const uint4 *>(kb + sw64(r, qc));
                kw[0] = w0.x, kw[1] = w0.y, kw[2] = w0.z, kw[3] = w0.w;
            }
#pragma unroll
            for (int ks = 0; ks < KS; ++ks)
                mma_16816(sacc[nt], qf[ks][0], qf[ks][1], qf[ks][2], qf[ks][3], codes_to_half2(kw[ks], 0x4140u),
                          codes_to_half2(kw[ks], 0x4342u));
        }
        if constexpr (DS > 1) {
            float *mine = xbuf + (((kg * 2 + (i & 1)) * 2 + dh) * 32 + lane) * 8;
            float *theirs = xbuf + (((kg * 2 + (i & 1)) * 2 + (dh ^ 1)) * 32 + lane) * 8;
            *reinterpret_cast<float4 *>(mine) = make_float4(sacc[0][0], sacc[0][1], sacc[0][2], sacc[0][3]);
            *reinterpret_cast<float4 *>(mine + 4) = make_float4(sacc[1][0], sacc[1][1], sacc[1][2], sacc[1][3]);
            named_barrier_sync(2 + kg, 64);
            const float4 t0 = *reinterpret_cast<const float4 *>(theirs);
            const float4 t1 = *reinterpret_cast<const float4 *>(theirs + 4);
            // Fixed order (slice 0 + slice 1) so that both warps hold identical scores.
            const float4 lo0 = dh == 0 ? make_float4(sacc[0][0], sacc[0][1], sacc[0][2], sacc[0][3]) : t0;
            const float4 lo1 = dh == 0 ? make_float4(sacc[1][0], sacc[1][1], sacc[1][2], sacc[1][3]) : t1;
            const float4 hi0 = dh == 0 ? t0 : make_float4(sacc[0][0], sacc[0][1], sacc[0][2], sacc[0][3]);
            const float4 hi1 = dh == 0 ? t1 : make_float4(sacc[1][0], sacc[1][1], sacc[1][2], sacc[1][3]);
            sacc[0][0] = lo0.x + hi0.x, sacc[0][1] = lo0.y + hi0.y, sacc[0][2] = lo0.z + hi0.z;
            sacc[0][3] = lo0.w + hi0.w;
            sacc[1][0] = lo1.x + hi1.x, sacc[1][1] = lo1.y + hi1.y, sacc[1][2] = lo1.z + hi1.z;
            sacc[1][3] = lo1.w + hi1.w;
        }

        // Scales of this lane's keys kg*16 + {2qc, 2qc+1} (n-tile 0) and + 8 (n-tile 1).
        const float2 ks0 = *reinterpret_cast<const float2 *>(sc + kg * 16 + 2 * qc);
        const float2 ks1 = *reinterpret_cast<const float2 *>(sc + kg * 16 + 8 + 2 * qc);
        const float2 vs0 = *reinterpret_cast<const float2 *>(sc + kStageKeys + kg * 16 + 2 * qc);
        const float2 vs1 = *reinterpret_cast<const float2 *>(sc + kStageKeys + kg * 16 + 8 + 2 * qc);
        const float kscale[2][2] = {{ks0.x, ks0.y}, {ks1.x, ks1.y}};
        const float vscale[2][2] = {{vs0.x, vs0.y}, {vs1.x, vs1.y}};

        float mx[2] = {-CUDART_INF_F, -CUDART_INF_F};
#pragma unroll
        for (int nt = 0; nt < 2; ++nt)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int key = key0 + nt * 8 + 2 * qc + (e & 1);
                const int hi = e < 2 ? hiA : hiB, lo = e < 2 ? loA : loB;
                float x = sacc[nt][e] * kscale[nt][e & 1];
                if (use_cap) {
                    // c*tanh(s/c) in log2 units, tanh(z) = 1 - 2/(1 + e^{2z}) (as in decode.cu).
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
        float pv[2][4];
#pragma unroll
        for (int nt = 0; nt < 2; ++nt)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const float p = exp2f(sacc[nt][e] - muse[e >> 1]);
                lsum[e >> 1] += p;
                pv[nt][e] = p * vscale[nt][e & 1];
            }
        const uint32_t pa0 = pack_half2(pv[0][0], pv[0][1]);
        const uint32_t pa1 = pack_half2(pv[0][2], pv[0][3]);
        const uint32_t pa2 = pack_half2(pv[1][0], pv[1][1]);
        const uint32_t pa3 = pack_half2(pv[1][2], pv[1][3]);

        // O += P' V: this lane's keys kg*16 + {2qc, 2qc+1, 2qc+8, 2qc+9}, its VW bytes at
        // head-dim VW*qr of each, transposed 4 x 4 bytes at a time into fp16 fragments.
        const int vr = kg * 16 + 2 * qc;
        uint32_t vw[4][NG];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const int r = vr + (k & 1) + (k >> 1) * 8;
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
            // Byte t of lo01 / hi01 pairs: keys (2qc, 2qc+1) at head-dim byte t (lo: t = 0, 1; hi: 2, 3).
            const uint32_t lo01 = prmt(vw[0][g], vw[1][g], 0x5140u), hi01 = prmt(vw[0][g], vw[1][g], 0x7362u);
            const uint32_t lo23 = prmt(vw[2][g], vw[3][g], 0x5140u), hi23 = prmt(vw[2][g], vw[3][g], 0x7362u);
            mma_16816(o[g * 4 + 0], pa0, pa1, pa2, pa3, codes_to_half2(lo01, 0x4140u), codes_to_half2(lo23, 0x4140u));
            mma_16816(o[g * 4 + 1], pa0, pa1, pa2, pa3, codes_to_half2(lo01, 0x4342u), codes_to_half2(lo23, 0x4342u));
            mma_16816(o[g * 4 + 2], pa0, pa1, pa2, pa3, codes_to_half2(hi01, 0x4140u), codes_to_half2(hi23, 0x4140u));
            mma_16816(o[g * 4 + 3], pa0, pa1, pa2, pa3, codes_to_half2(hi01, 0x4342u), codes_to_half2(hi23, 0x4342u));
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
    }

    // ---- merge the key groups (ring reused), un-permuting the output columns.
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        lsum[r] += __shfl_xor_sync(0xffffffffu, lsum[r], 1);
        lsum[r] += __shfl_xor_sync(0xffffffffu, lsum[r], 2);
    }
    named_barrier_sync(1, NC * 32);
    float *cm = reinterpret_cast<float *>(ring);
    float *cl = cm + KG * 16;
    float *co = cl + KG * 16;
    if (qc == 0 && dh == 0) {
        cm[kg * 16 + qr] = m2[0];
        cm[kg * 16 + qr + 8] = m2[1];
        cl[kg * 16 + qr] = lsum[0];
        cl[kg * 16 + qr + 8] = lsum[1];
    }
#pragma unroll
    for (int g = 0; g < NG; ++g)
#pragma unroll
        for (int t = 0; t < 4; ++t) {
            const int n = g * 4 + t;
            const int dA = dh * DH + VW * (2 * qc) + 4 * g + t;
            const int dB = dA + VW;
            co[(kg * 16 + qr) * D + dA] = o[n][0];
            co[(kg * 16 + qr) * D + dB] = o[n][1];
            co[(kg * 16 + qr + 8) * D + dA] = o[n][2];
            co[(kg * 16 + qr + 8) * D + dB] = o[n][3];
        }
    named_barrier_sync(1, NC * 32);

    decode_epilogue<D, KG, NC>(a, ring, row0, nrows, kvh, mt, b, split);
}

template <int D>
cudaError_t launch_q8_t(const CUtensorMap &tmk, const CUtensorMap &tmv, const CUtensorMap &tms, const DecodeArgs &a,
                        dim3 grid, cudaStream_t s, bool pdl) {
    static unsigned long long configured = 0;  // one bit per device: the opt-in is per device
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 64 || !(configured & (1ull << dev))) {
        cudaError_t e = cudaFuncSetAttribute(decode_q8_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             Q8Layout<D>::kSmemBytes);
        if (e != cudaSuccess) return e;
        if (dev < 64) configured |= 1ull << dev;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(Q8Layout<D>::kThreads);
    cfg.dynamicSmemBytes = Q8Layout<D>::kSmemBytes;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, decode_q8_kernel<D>, tmk, tmv, tms, a);
}

template <int D>
int q8_ctas_per_sm_t() {
    static int n = 0;
    if (n == 0) {
        cudaFuncSetAttribute(decode_q8_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, Q8Layout<D>::kSmemBytes);
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, decode_q8_kernel<D>, Q8Layout<D>::kThreads,
                                                          Q8Layout<D>::kSmemBytes) != cudaSuccess ||
            n < 1)
            n = 1;
    }
    return n;
}

}  // namespace

int decode_q8_ctas_per_sm(int head_dim) {
    switch (head_dim) {
        case 64: return q8_ctas_per_sm_t<64>();
        case 128: return q8_ctas_per_sm_t<128>();
        case 256: return q8_ctas_per_sm_t<256>();
        default: return 1;
    }
}

cudaError_t launch_decode_q8(int head_dim, const CUtensorMap &tmk, const CUtensorMap &tmv, const CUtensorMap &tms,
                             const DecodeArgs &a, int grid_x, int grid_y, int grid_z, cudaStream_t s, bool pdl) {
    static_assert(Q8Layout<64>::kStageKeys == 64 && Q8Layout<128>::kStageKeys == 64 && Q8Layout<256>::kStageKeys == 32,
                  "stage keys must match decode_stage_keys()");
    const dim3 grid(grid_x, grid_y, grid_z);
    switch (head_dim) {
        case 64: return launch_q8_t<64>(tmk, tmv, tms, a, grid, s, pdl);
        case 128: return launch_q8_t<128>(tmk, tmv, tms, a, grid, s, pdl);
        case 256: return launch_q8_t<256>(tmk, tmv, tms, a, grid, s, pdl);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace brk
