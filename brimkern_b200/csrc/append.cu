// KV append with the q/k prologue fused: per-head RMSNorm (QK-norm), NeoX RoPE, fp16 store (or,
// for an int8 cache, the quantize_kv quantisation of shaders.ts:1673-1705, kernels.ts:1721-1725).
//
// Replaces, for one layer, the reference's chain rmsnorm(q), rmsnorm(k) (kernels.ts:1707-1709,
// shaders.ts:580-598) -> rope / rope_factors (kernels.ts:1710-1718, shaders.ts:1361-1408) ->
// copyBufferToBuffer of K and V into the cache at row pastLen (kernels.ts:1727-1730).
//
// Bit-exactness: the reference's CPU functions (rmsnormCpu kernels.ts:3395, ropeCpu :3445,
// ropeFactorsCpu :3428) compute in double and round to f32 on each Float32Array store.  This
// kernel does the same in fp64 with explicitly rounded operations (no FMA contraction), the
// sum of squares in the same sequential order, and cos/sin taken from a table the host built
// with the same libm expression, so each stored f32 equals the oracle's; K and V are then
// rounded f32 -> fp16 to nearest even, or quantised to int8 from those same f32 values.
#include "common.cuh"
#include "internal.h"
#include "kv_q8.cuh"

namespace brk {

namespace {

constexpr int kRowsPerBlock = 4;  // one warp per head-vector row

// DT: the head dim as a compile-time constant (64 / 128 / 256), or 0 for any other even size.
template <int DT>
__global__ void __launch_bounds__(kRowsPerBlock * 32) append_kernel(const __grid_constant__ AppendArgs a) {
    // This grid waits for whatever the stream ran before it, then lets its dependent (the decode
    // or prefill kernel of the same step) be scheduled: that kernel may read what the earlier
    // kernels wrote (the q projection, cache rows) before this grid finishes, and waits for this
    // grid only before the rows it writes.
    griddep_wait();
    griddep_launch_dependents();
    extern __shared__ double sq_all[];  // per warp: D squares (double), then D values (float)
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int D = DT ? DT : a.D, half = D >> 1;
    const int per_tok = a.Hq + 2 * a.Hkv;
    const long long row = (long long)blockIdx.x * kRowsPerBlock + warp;
    if (row >= (long long)a.B * a.T * per_tok) return;
    const int bt = (int)(row / per_tok), kind = (int)(row % per_tok);
    const int b = bt / a.T, t = bt % a.T;
    const int pos = a.past_len[b] + t;

    const float *src;
    const float *gain = nullptr;
    bool rotate = a.rope != nullptr;
    float *qdst = nullptr;
    __half *cdst = nullptr;
    uint8_t *c8dst = nullptr;  // int8 cache: codes of this row, and its scale slot
    float *sdst = nullptr;
    if (kind < a.Hq) {
        if (!a.q_out) return;
        src = a.q_in + ((size_t)bt * a.Hq + kind) * D;
        gain = a.q_norm;
        qdst = a.q_out + ((size_t)bt * a.Hq + kind) * D;
    } else {
        const bool is_k = kind < a.Hq + a.Hkv;
        const int h = is_k ? kind - a.Hq : kind - a.Hq - a.Hkv;
        const float *in = is_k ? a.k_in : a.v_in;
        if (!in) return;
        src = in + ((size_t)bt * a.Hkv + h) * D;
        const size_t seg = (size_t)(a.layer * a.B + b) * a.Hkv + h;
        const size_t crow = seg * a.cap + (size_t)(pos - a.kv_offset);
        if (a.kc) {
            cdst = (is_k ? a.kc : a.vc) + crow * D;
        } else {
            c8dst = (is_k ? a.kc8 : a.vc8) + crow * D;
            sdst = a.scales + (seg * 2 + (is_k ? 0 : 1)) * a.scale_pitch + (size_t)(pos - a.kv_offset);
        }
        if (is_k) {
            gain = a.k_norm;
        } else {
            rotate = false;  // V is neither normalised nor rotated
        }
    }

    double *sq = sq_all + (size_t)warp * D * 3 / 2;  // D doubles + D floats per warp
    float *xs = reinterpret_cast<float *>(sq + D);
    for (int d = lane; d < D; d += 32) {
        const float x = src[d];
        xs[d] = x;
        sq[d] = __dmul_rn((double)x, (double)x);  // exact: an f32 square fits a double
    }
    __syncwarp();

    if (gain) {
        // rmsnormCpu (kernels.ts:3395): ss = sum of x^2 in index order (double), inv = 1/sqrt(ss/dim + eps),
        // y = f32(x*inv*g).  Only the ordered additions are sequential.
        double inv = 0.0;
        if (lane == 0) {
            double ss = 0.0;
            if constexpr (DT > 0) {
#pragma unroll
                for (int d = 0; d < DT; ++d) ss = __dadd_rn(ss, sq[d]);
            } else {
                for (int d = 0; d < D; ++d) ss = __dadd_rn(ss, sq[d]);
            }
            inv = __ddiv_rn(1.0, __dsqrt_rn(__dadd_rn(__ddiv_rn(ss, (double)D), a.eps)));
        }
        inv = __shfl_sync(0xffffffffu, inv, 0);
        for (int d = lane; d < D; d += 32) {
            const double w = gain[d];
            const double g = a.one_plus ? __dadd_rn(1.0, w) : w;
            xs[d] = (float)__dmul_rn(__dmul_rn((double)xs[d], inv), g);
        }
        __syncwarp();
    }

    if (rotate) {
        // ropeCpu (kernels.ts:3445): o_i = f32(x_i c - x_{i+D/2} s), o_{i+D/2} = f32(x_{i+D/2} c + x_i s).
        const double2 *cs = a.rope + (size_t)pos * half;
        for (int i = lane; i < half; i += 32) {
            const double2 e = cs[i];
            const double x0 = xs[i], x1 = xs[i + half];
            const float o0 = (float)__dsub_rn(__dmul_rn(x0, e.x), __dmul_rn(x1, e.y));
            const float o1 = (float)__dadd_rn(__dmul_rn(x1, e.x), __dmul_rn(x0, e.y));
            if (qdst) {
                qdst[i] = o0;
                qdst[i + half] = o1;
            } else if (cdst) {
                cdst[i] = __float2half_rn(o0);
                cdst[i + half] = __float2half_rn(o1);
            } else {
                xs[i] = o0;  // int8: quantised below from the final f32 row
                xs[i + half] = o1;
            }
        }
    } else if (!c8dst) {
        for (int d = lane; d < D; d += 32) {
            if (qdst)
                qdst[d] = xs[d];
            else
                cdst[d] = __float2half_rn(xs[d]);
        }
    }
    if (c8dst) {
        __syncwarp();
        quantize_row_warp(xs, D, c8dst, sdst, lane);
    }
}

// Row-block form of the same append for head_dim 64 / 128 / 256: ROWS head rows per block of 256
// threads.  The rows are staged in shared memory with coalesced loads (padded stride D + 1, so
// that one thread walking one row and its neighbours walking theirs hit distinct banks); one
// thread per row then runs the ordered double sum of squares, all threads apply the norm and the
// rotation element by element (coalesced gains, table and stores), and an int8 cache quantises
// each K / V row from its final f32 values.  Same operations in the same order as append_kernel,
// so the outputs are the same bits.
template <int D, int ROWS>
__global__ void __launch_bounds__(256) append_block_kernel(const __grid_constant__ AppendArgs a) {
    griddep_wait();  // then the dependent may start (see append_kernel)
    griddep_launch_dependents();
    constexpr int kStride = D + 1;
    constexpr int H2 = D / 2;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    double *inv_s = reinterpret_cast<double *>(smem_raw);                 // [ROWS]
    int4 *meta = reinterpret_cast<int4 *>(smem_raw + ROWS * sizeof(double));  // [ROWS] kind, bt, head, pos
    float *xs = reinterpret_cast<float *>(smem_raw + ROWS * (sizeof(double) + sizeof(int4)));  // [ROWS][D+1]
    // Only the rows asked for (q with q_out, k with k_in, v with v_in) are enumerated, per token
    // in that order, so that a K / V-only append (prefill chunks) spends no blocks on q rows.
    const int nq = a.q_out ? a.Hq : 0, nkh = a.k_in ? a.Hkv : 0, nvh = a.v_in ? a.Hkv : 0;
    const int per_tok = nq + nkh + nvh;
    const long long total = (long long)a.B * a.T * per_tok;
    const long long row0 = (long long)blockIdx.x * ROWS;
    const int nrow = (int)min((long long)ROWS, total - row0);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    // Row descriptors: kind 0 = q, 1 = k, 2 = v.
    if (threadIdx.x < nrow) {
        const long long row = row0 + threadIdx.x;
        const int bt = (int)(row / per_tok), kind_h = (int)(row % per_tok);
        const int kind = kind_h < nq ? 0 : kind_h < nq + nkh ? 1 : 2;
        const int h = kind == 0 ? kind_h : kind == 1 ? kind_h - nq : kind_h - nq - nkh;
        meta[threadIdx.x] = make_int4(kind, bt, h, a.past_len[bt / a.T] + bt % a.T);
    }
    __syncthreads();
    auto source = [&](int4 m) -> const float * {
        return m.x == 0 ? a.q_in + ((size_t)m.y * a.Hq + m.z) * D
                        : (m.x == 1 ? a.k_in : a.v_in) + ((size_t)m.y * a.Hkv + m.z) * D;
    };
    // 1. Coalesced loads: one warp per row at a time.
    for (int lr = warp; lr < nrow; lr += 8) {
        const int4 m = meta[lr];
        if (m.x < 0) continue;
        const float4 *src = reinterpret_cast<const float4 *>(source(m));
        for (int c = lane; c < D / 4; c += 32) {
            const float4 x = src[c];
            float *dst = xs + lr * kStride + 4 * c;
            dst[0] = x.x, dst[1] = x.y, dst[2] = x.z, dst[3] = x.w;
        }
    }
    __syncthreads();
    // 2. rmsnormCpu's ordered sum (kernels.ts:3395), one thread per row: inv = 1/sqrt(ss/D + eps).
    if (threadIdx.x < nrow) {
        const int4 m = meta[threadIdx.x];
        const float *gain = m.x == 0 ? a.q_norm : m.x == 1 ? a.k_norm : nullptr;
        double inv = 0.0;
        if (m.x >= 0 && gain) {
            const float *x = xs + threadIdx.x * kStride;
            // x^2 is exact in double, so one rounding of x^2 + ss (fma) is the oracle's ss + x*x.
            double ss = 0.0;
#pragma unroll 16
            for (int d = 0; d < D; ++d) {
                const double xd = (double)x[d];
                ss = __fma_rn(xd, xd, ss);
            }
            inv = __ddiv_rn(1.0, __dsqrt_rn(__dadd_rn(__ddiv_rn(ss, (double)D), a.eps)));
        }
        inv_s[threadIdx.x] = inv;
    }
    __syncthreads();
    // 3. Norm and rotation (ropeCpu kernels.ts:3445) per element pair (i, i + D/2), and the stores:
    // one warp per row, lane l always owning pairs i = l + 32u, so that its gains are converted
    // once per block and a row's addresses once per row.
    constexpr int NP = H2 / 32;  // pairs per lane
    const bool q8 = a.kc == nullptr && a.kc8 != nullptr;
    double gq[NP][2], gk[NP][2];
#pragma unroll
    for (int u = 0; u < NP; ++u) {
        const int i = lane + 32 * u;
#pragma unroll
        for (int e = 0; e < 2; ++e) {
            const double wq = a.q_norm ? (double)a.q_norm[i + e * H2] : 0.0;
            const double wk = a.k_norm ? (double)a.k_norm[i + e * H2] : 0.0;
            gq[u][e] = a.one_plus ? __dadd_rn(1.0, wq) : wq;
            gk[u][e] = a.one_plus ? __dadd_rn(1.0, wk) : wk;
        }
    }
    for (int lr = warp; lr < nrow; lr += 8) {
        const int4 m = meta[lr];
        if (m.x < 0) continue;
        float *xr = xs + lr * kStride;
        const bool norm = m.x == 0 ? a.q_norm != nullptr : m.x == 1 && a.k_norm != nullptr;
        const double inv = inv_s[lr];
        const bool rotate = a.rope && m.x < 2;
        const double2 *cs = rotate ? a.rope + (size_t)m.w * H2 : nullptr;
        float *qdst = nullptr;
        __half *cdst = nullptr;
        if (m.x == 0) {
            qdst = a.q_out + ((size_t)m.y * a.Hq + m.z) * D;
        } else if (!q8) {
            const size_t crow =
                ((size_t)(a.layer * a.B + m.y / a.T) * a.Hkv + m.z) * a.cap + (size_t)(m.w - a.kv_offset);
            cdst = (m.x == 1 ? a.kc : a.vc) + crow * D;
        }
        if (m.x == 2 && cdst) {
            // V into an fp16 cache: a plain round to nearest.
#pragma unroll
            for (int u = 0; u < NP; ++u) {
                const int i = lane + 32 * u;
                cdst[i] = __float2half_rn(xr[i]);
                cdst[i + H2] = __float2half_rn(xr[i + H2]);
            }
            continue;
        }
#pragma unroll
        for (int u = 0; u < NP; ++u) {
            const int i = lane + 32 * u;
            double y0 = xr[i], y1 = xr[i + H2];
            if (norm) {
                const double g0 = m.x == 0 ? gq[u][0] : gk[u][0], g1 = m.x == 0 ? gq[u][1] : gk[u][1];
                y0 = (double)(float)__dmul_rn(__dmul_rn(y0, inv), g0);
                y1 = (double)(float)__dmul_rn(__dmul_rn(y1, inv), g1);
            }
            float o0 = (float)y0, o1 = (float)y1;
            if (rotate) {
                const double2 e = cs[i];
                o0 = (float)__dsub_rn(__dmul_rn(y0, e.x), __dmul_rn(y1, e.y));
                o1 = (float)__dadd_rn(__dmul_rn(y1, e.x), __dmul_rn(y0, e.y));
            }
            if (qdst) {
                qdst[i] = o0;
                qdst[i + H2] = o1;
            } else if (cdst) {
                cdst[i] = __float2half_rn(o0);
                cdst[i + H2] = __float2half_rn(o1);
            } else {
                xr[i] = o0;  // int8: quantised below from the final row
                xr[i + H2] = o1;
            }
        }
    }
    if (q8) {
        __syncthreads();
        for (int lr = warp; lr < nrow; lr += 8) {
            const int4 m = meta[lr];
            if (m.x < 1) continue;
            const int b = m.y / a.T;
            const size_t seg = (size_t)(a.layer * a.B + b) * a.Hkv + m.z;
            const size_t r = (size_t)(m.w - a.kv_offset);
            quantize_row_warp(xs + lr * kStride, D, (m.x == 1 ? a.kc8 : a.vc8) + (seg * a.cap + r) * D,
                              a.scales + (seg * 2 + (m.x == 1 ? 0 : 1)) * a.scale_pitch + r, lane);
        }
    }
}

// K / V rows of a multi-token append (prefill chunks) into an fp16 cache, no q: one block per
// (32 tokens, kv head, sequence), so the block's cache rows are contiguous.  Warps load their
// rows (all loads of a warp issued before its first store), V rows go straight to the cache
// (round to nearest), K rows are staged in shared memory; one thread per K row runs the ordered
// double sum of squares; then a warp per K row applies the norm and the rotation with exactly
// append_block_kernel's double operations (same bits; it only spends far fewer instructions on
// row bookkeeping).
//
// With a.q16 the grid has Hq more blocks along y: those rotate the chunk's q rows instead (one
// warp per row, RMSNorm and NeoX rotation in f32 with the f32 table, exactly the prefill kernel's
// q prologue: q only feeds its fp16 tensor-core operand) and store them as fp16 for the prefill
// kernel's TMA loads.
template <int D>
__device__ __forceinline__ void q16_rows(const AppendArgs &a, int hq, int b, int t0, int nt, int warp, int lane) {
    constexpr int TT = 32, RPW = TT / 8, H2 = D / 2, P = H2 / 32;
    const int i0 = lane * P;
    const int pos0 = a.past_len[b] + t0;
    float g0[P], g1[P];
#pragma unroll
    for (int p = 0; p < P; ++p) {
        const float w0 = a.q_norm ? a.q_norm[i0 + p] : 1.f, w1 = a.q_norm ? a.q_norm[i0 + p + H2] : 1.f;
        g0[p] = a.q_norm && a.one_plus ? 1.f + w0 : w0;
        g1[p] = a.q_norm && a.one_plus ? 1.f + w1 : w1;
    }
    float x0[RPW][P], x1[RPW][P], c[RPW][P], sn[RPW][P];
#pragma unroll
    for (int u = 0; u < RPW; ++u) {
        const int tl = warp + 8 * u;
        const bool ok = tl < nt;
        const float *src = a.q_in + ((size_t)(b * a.T + t0 + (ok ? tl : 0)) * a.Hq + hq) * D;
#pragma unroll
        for (int p = 0; p < P; ++p) {
            x0[u][p] = ok ? src[i0 + p] : 0.f;
            x1[u][p] = ok ? src[i0 + p + H2] : 0.f;
            const float2 e = ok && a.rope32 ? a.rope32[(size_t)(pos0 + tl) * H2 + i0 + p] : make_float2(1.f, 0.f);
            c[u][p] = e.x, sn[u][p] = e.y;
        }
    }
#pragma unroll
    for (int u = 0; u < RPW; ++u) {
        const int tl = warp + 8 * u;
        float inv = 1.f;
        if (a.q_norm) {
            float ss = 0.f;
#pragma unroll
            for (int p = 0; p < P; ++p) ss = fmaf(x0[u][p], x0[u][p], fmaf(x1[u][p], x1[u][p], ss));
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
            inv = 1.f / sqrtf(ss / (float)D + (float)a.eps);
        }
        float o0[P], o1[P];
#pragma unroll
        for (int p = 0; p < P; ++p) {
            const float y0 = x0[u][p] * inv * g0[p], y1 = x1[u][p] * inv * g1[p];
            o0[p] = fmaf(y0, c[u][p], -(y1 * sn[u][p]));
            o1[p] = fmaf(y1, c[u][p], y0 * sn[u][p]);
        }
        if (tl < nt) {
            __half *dst = a.q16 + ((size_t)(b * a.T + t0 + tl) * a.Hq + hq) * D;
            if constexpr (P == 2) {
                *reinterpret_cast<uint32_t *>(dst + i0) = pack_half2(o0[0], o0[1]);
                *reinterpret_cast<uint32_t *>(dst + i0 + H2) = pack_half2(o1[0], o1[1]);
            } else {
#pragma unroll
                for (int p = 0; p < P; ++p) {
                    dst[i0 + p] = __float2half_rn(o0[p]);
                    dst[i0 + p + H2] = __float2half_rn(o1[p]);
                }
            }
        }
    }
}

template <int D>
__global__ void __launch_bounds__(256) kv_append_kernel(const __grid_constant__ AppendArgs a) {
    griddep_wait();  // then the dependent may start (see append_kernel)
    griddep_launch_dependents();
    constexpr int TT = 32, RPW = TT / 8;         // tokens per block, rows per warp
    constexpr int H2 = D / 2, NP = H2 / 32;      // rotation pairs per lane
    constexpr int C4 = D / 4 >= 32 ? D / 128 : 1;  // float4 per lane per row
    constexpr int kStride = D + 1;
    __shared__ float xs[TT * kStride];
    __shared__ double inv_s[TT];
    const int t0 = blockIdx.x * TT, h = blockIdx.y, b = blockIdx.z;
    const int nt = min(TT, a.T - t0);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (h >= a.Hkv) {
        q16_rows<D>(a, h - a.Hkv, b, t0, nt, warp, lane);
        return;
    }
    const int pos0 = a.past_len[b] + t0;
    const size_t crow0 = ((size_t)(a.layer * a.B + b) * a.Hkv + h) * a.cap + (size_t)(pos0 - a.kv_offset);
    __half *kc = a.kc + crow0 * D, *vc = a.vc + crow0 * D;

    // 1. Loads: K -> shared memory, V -> cache.
    {
        float4 kx[RPW][C4], vx[RPW][C4];
#pragma unroll
        for (int u = 0; u < RPW; ++u) {
            const int tl = warp + 8 * u;
            const size_t in_row = ((size_t)(b * a.T + t0 + (tl < nt ? tl : 0)) * a.Hkv + h) * D;
#pragma unroll
            for (int c = 0; c < C4; ++c) {
                const int col = lane + 32 * c;
                const bool ok = tl < nt && col < D / 4;
                kx[u][c] = ok ? reinterpret_cast<const float4 *>(a.k_in + in_row)[col] : make_float4(0.f, 0.f, 0.f, 0.f);
                vx[u][c] = ok ? reinterpret_cast<const float4 *>(a.v_in + in_row)[col] : make_float4(0.f, 0.f, 0.f, 0.f);
            }
        }
#pragma unroll
        for (int u = 0; u < RPW; ++u) {
            const int tl = warp + 8 * u;
#pragma unroll
            for (int c = 0; c < C4; ++c) {
                const int col = lane + 32 * c;
                if (tl < nt && col < D / 4) {
                    float *dst = xs + tl * kStride + 4 * col;
                    dst[0] = kx[u][c].x, dst[1] = kx[u][c].y, dst[2] = kx[u][c].z, dst[3] = kx[u][c].w;
                    *reinterpret_cast<uint2 *>(vc + (size_t)tl * D + 4 * col) =
                        make_uint2(pack_half2(vx[u][c].x, vx[u][c].y), pack_half2(vx[u][c].z, vx[u][c].w));
                }
            }
        }
    }
    __syncthreads();
    // 2. rmsnormCpu's ordered sum (kernels.ts:3395), one thread per K row.
    if (a.k_norm && threadIdx.x < nt) {
        const float *x = xs + threadIdx.x * kStride;
        double ss = 0.0;
#pragma unroll 16
        for (int d = 0; d < D; ++d) {
            const double xd = (double)x[d];
            ss = __fma_rn(xd, xd, ss);  // x^2 is exact in double: one rounding, as ss + x*x
        }
        inv_s[threadIdx.x] = __ddiv_rn(1.0, __dsqrt_rn(__dadd_rn(__ddiv_rn(ss, (double)D), a.eps)));
    }
    __syncthreads();
    // 3. Norm and rotation (ropeCpu kernels.ts:3445), a warp per K row, lane l owning the pairs
    //    (i, i + D/2) for i = l + 32u; the table entries of the warp's rows are loaded first.
    double g0[NP], g1[NP];
#pragma unroll
    for (int u = 0; u < NP; ++u) {
        const int i = lane + 32 * u;
        const double w0 = a.k_norm ? (double)a.k_norm[i] : 1.0, w1 = a.k_norm ? (double)a.k_norm[i + H2] : 1.0;
        g0[u] = a.k_norm && a.one_plus ? __dadd_rn(1.0, w0) : w0;
        g1[u] = a.k_norm && a.one_plus ? __dadd_rn(1.0, w1) : w1;
    }
    double2 cs[RPW][NP];
#pragma unroll
    for (int r = 0; r < RPW; ++r) {
        const int tl = warp + 8 * r;
#pragma unroll
        for (int u = 0; u < NP; ++u)
            cs[r][u] = a.rope && tl < nt ? a.rope[(size_t)(pos0 + tl) * H2 + lane + 32 * u] : make_double2(1.0, 0.0);
    }
#pragma unroll
    for (int r = 0; r < RPW; ++r) {
        const int tl = warp + 8 * r;
        if (tl >= nt) break;
        const float *xr = xs + tl * kStride;
        const double inv = a.k_norm ? inv_s[tl] : 0.0;
        __half *dst = kc + (size_t)tl * D;
#pragma unroll
        for (int u = 0; u < NP; ++u) {
            const int i = lane + 32 * u;
            double y0 = xr[i], y1 = xr[i + H2];
            if (a.k_norm) {
                y0 = (double)(float)__dmul_rn(__dmul_rn(y0, inv), g0[u]);
                y1 = (double)(float)__dmul_rn(__dmul_rn(y1, inv), g1[u]);
            }
            float o0 = (float)y0, o1 = (float)y1;
            if (a.rope) {
                o0 = (float)__dsub_rn(__dmul_rn(y0, cs[r][u].x), __dmul_rn(y1, cs[r][u].y));
                o1 = (float)__dadd_rn(__dmul_rn(y1, cs[r][u].x), __dmul_rn(y0, cs[r][u].y));
            }
            dst[i] = __float2half_rn(o0);
            dst[i + H2] = __float2half_rn(o1);
        }
    }
}

template <int D, int ROWS>
constexpr size_t append_block_smem() {
    return ROWS * (sizeof(double) + sizeof(int4)) + (size_t)ROWS * (D + 1) * sizeof(float);
}

// Plain f32 -> fp16 row store into one (layer, sequence) segment: rows [row0, row0+n) of every
// kv head.  kc/vc point at row row0 of kv head 0 of the segment; heads are `cap` rows apart.
__global__ void kv_write_rows_kernel(__half *kc, __half *vc, const float *k, const float *v, int n_rows, int Hkv,
                                     int D, int cap) {
    const long long n = (long long)n_rows * Hkv * D;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
        const int d = (int)(i % D);
        const int h = (int)((i / D) % Hkv);
        const int r = (int)(i / ((long long)D * Hkv));
        const size_t dst = ((size_t)h * cap + r) * D + d;
        if (k) kc[dst] = __float2half_rn(k[i]);
        if (v) vc[dst] = __float2half_rn(v[i]);
    }
}

__global__ void kv_read_rows_kernel(const __half *kc, const __half *vc, uint16_t *k, uint16_t *v, int n_rows, int Hkv,
                                    int D, int cap) {
    const long long n = (long long)n_rows * Hkv * D;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
        const int d = (int)(i % D);
        const int h = (int)((i / D) % Hkv);
        const int r = (int)(i / ((long long)D * Hkv));
        const size_t src = ((size_t)h * cap + r) * D + d;
        if (k) k[i] = __half_as_ushort(kc[src]);
        if (v) v[i] = __half_as_ushort(vc[src]);
    }
}

}  // namespace

template <int D, int ROWS>
cudaError_t launch_block(cudaLaunchConfig_t cfg, const AppendArgs &a, long long rows) {
    cfg.gridDim = dim3((unsigned)((rows + ROWS - 1) / ROWS));
    cfg.dynamicSmemBytes = append_block_smem<D, ROWS>();
    return cudaLaunchKernelEx(&cfg, append_block_kernel<D, ROWS>, a);
}

cudaError_t launch_append(const AppendArgs &a, cudaStream_t s, bool pdl) {
    long long rows = (long long)a.B * a.T * (a.Hq + 2 * a.Hkv);
    if (rows == 0) return cudaSuccess;
    // The row-block kernels enumerate only the rows asked for.
    const long long block_rows =
        (long long)a.B * a.T * ((a.q_out ? a.Hq : 0) + (a.k_in ? a.Hkv : 0) + (a.v_in ? a.Hkv : 0));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)((rows + kRowsPerBlock - 1) / kRowsPerBlock));
    cfg.blockDim = dim3(kRowsPerBlock * 32);
    cfg.dynamicSmemBytes = (size_t)kRowsPerBlock * a.D * 12;  // squares (double) + values (float)
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    // Head dims 64 / 128 / 256: row blocks (large appends: 8 KB of rows per block; decode-sized
    // ones: 16 rows per block, so that the rows spread over the SMs).
    if (a.D == 64 || a.D == 128 || a.D == 256) {
        if (block_rows == 0) return cudaSuccess;
        rows = block_rows;
        // K / V only into an fp16 cache (prefill chunks): the dedicated kernel.
        if (!a.q_out && a.k_in && a.v_in && a.kc && a.T >= 8) {
            cfg.gridDim = dim3((unsigned)((a.T + 31) / 32), (unsigned)(a.Hkv + (a.q16 ? a.Hq : 0)), (unsigned)a.B);
            cfg.blockDim = dim3(256);
            cfg.dynamicSmemBytes = 0;
            switch (a.D) {
                case 64: return cudaLaunchKernelEx(&cfg, kv_append_kernel<64>, a);
                case 128: return cudaLaunchKernelEx(&cfg, kv_append_kernel<128>, a);
                default: return cudaLaunchKernelEx(&cfg, kv_append_kernel<256>, a);
            }
        }
    }
    const bool big = rows >= 148LL * 2 * (8192 / (a.D > 0 ? a.D : 1));
    cfg.blockDim = dim3(256);
    switch (a.D) {
        case 64:
            return big ? launch_block<64, 128>(cfg, a, rows) : launch_block<64, 16>(cfg, a, rows);
        case 128:
            return big ? launch_block<128, 64>(cfg, a, rows) : launch_block<128, 16>(cfg, a, rows);
        case 256:
            return big ? launch_block<256, 32>(cfg, a, rows) : launch_block<256, 16>(cfg, a, rows);
        default:
            cfg.blockDim = dim3(kRowsPerBlock * 32);
            return cudaLaunchKernelEx(&cfg, append_kernel<0>, a);
    }
}

cudaError_t launch_kv_write_rows(__half *kc, __half *vc, const float *k, const float *v, int n_rows, int Hkv, int D,
                                 int cap, cudaStream_t s) {
    const long long n = (long long)n_rows * Hkv * D;
    if (n == 0) return cudaSuccess;
    const unsigned grid = (unsigned)((n + 255) / 256 < 4096 ? (n + 255) / 256 : 4096);
    kv_write_rows_kernel<<<grid, 256, 0, s>>>(kc, vc, k, v, n_rows, Hkv, D, cap);
    return cudaGetLastError();
}

cudaError_t launch_kv_read_rows(const __half *kc, const __half *vc, uint16_t *k, uint16_t *v, int n_rows, int Hkv,
                                int D, int cap, cudaStream_t s) {
    const long long n = (long long)n_rows * Hkv * D;
    if (n == 0) return cudaSuccess;
    const unsigned grid = (unsigned)((n + 255) / 256 < 4096 ? (n + 255) / 256 : 4096);
    kv_read_rows_kernel<<<grid, 256, 0, s>>>(kc, vc, k, v, n_rows, Hkv, D, cap);
    return cudaGetLastError();
}

}  // namespace brk
