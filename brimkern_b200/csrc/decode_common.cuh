// Pieces of the decode kernel (decode.cu) kept apart from its main loop: the key range of a CTA
// and the epilogue that merges the key groups and, with split-KV, the splits (the last CTA of a
// (sequence, kv head, row tile) merges every split's partial).
#pragma once

#include <math_constants.h>

#include "common.cuh"
#include "internal.h"

namespace brk {

constexpr float kLn2 = 0.6931471805599453f;

// Cache rows [k_begin, k_end) that one CTA attends, in stage-sized tiles.  Token t of the CTA's
// rows attends [pos_t - W + 1, pos_t] (W <= 0: from 0).  `align` rounds the window's first key
// down (the int8 kernel loads scales in 16-byte boxes); keys below a row's own limit are masked.
struct KeyRange {
    int k_begin, k_end, ntiles;
};

__device__ __forceinline__ KeyRange decode_key_range(const DecodeArgs &a, int past, int row0, int nrows, int split,
                                                     int stage_keys, int align, int rows_per_tile) {
    const int G = a.G;
    const int t_lo = row0 / G;
    const int t_hi = min(row0 + rows_per_tile - 1, nrows - 1) / G;
    int kv_hi = past + t_hi + 1 - a.kv_offset;
    if (kv_hi > a.cap) kv_hi = a.cap;
    int kv_lo = 0;
    if (a.window > 0) kv_lo = max(0, past + t_lo - a.window + 1 - a.kv_offset) / align * align;
    KeyRange r;
    r.k_begin = kv_lo + split * a.keys_per_split;
    r.k_end = min(kv_hi, r.k_begin + a.keys_per_split);
    r.ntiles = r.k_begin < r.k_end ? (r.k_end - r.k_begin + stage_keys - 1) / stage_keys : 0;
    return r;
}

// Push mode: element d of row R's final partial (m in natural-log units) to every rank.
template <int D>
__device__ __forceinline__ void push_partial(const DecodeArgs &a, size_t R, int d, float o, float m, float l) {
    for (int p = 0; p < a.push_world; ++p) {
        a.push_o[p][R * D + d] = o;
        if (d == 0) {
            a.push_ml[p][R * 2] = m;
            a.push_ml[p][R * 2 + 1] = l;
        }
    }
}

// Push mode: after a tile's rows went out, count the tile; the launch's last tile publishes the
// epoch to every rank.  Each writer fences its remote stores at system scope before the count, so
// the flag (a system-scope release) is ordered after every tile's data.
template <int NC>
__device__ __forceinline__ void push_finish(const DecodeArgs &a) {
    __threadfence_system();
    named_barrier_sync(1, NC * 32);
    if (threadIdx.x == 0) {
        const int prev = atomicAdd(a.push_done, 1);
        if (prev == a.push_tiles - 1) {
            *a.push_done = 0;  // every tile is in: ready for the next launch
            __threadfence_system();
            for (int p = 0; p < a.push_world; ++p) st_release_sys(a.push_flag[p], a.epoch);
        }
    }
}

// After every consumer warp has written its key group's running max (log2 units), sum and
// unnormalised output rows into cm [KG][RT], cl [KG][RT] and co [KG][RT][D] at the start of
// `ring` (RT query rows per tile): writes this CTA's rows (final output, or its split's partial),
// then, with split-KV, lets the last CTA of the tile merge all splits.  Called by the NC
// consumer warps only.
template <int D, int KG, int NC, int RT>
__device__ __forceinline__ void decode_epilogue(const DecodeArgs &a, uint8_t *ring, int row0, int nrows, int kvh,
                                                int mt, int b, int split) {
    const float *cm = reinterpret_cast<const float *>(ring);
    const float *cl = cm + KG * RT;
    const float *co = cl + KG * RT;
    const int G = a.G, T = a.T;
    const int nvalid = min(RT, nrows - row0);
    const int rows_total = a.B * T * a.Hq;
    // (a) This CTA's (m, l, o) per row.  Single split: the final output (or the caller's
    // partial); several splits: this split's partial in the workspace.
    for (int idx = threadIdx.x; idx < nvalid * D; idx += NC * 32) {
        const int r = idx / D, d = idx % D;
        float M = -CUDART_INF_F;
#pragma unroll
        for (int w = 0; w < KG; ++w) M = fmaxf(M, cm[w * RT + r]);
        float Lsum = 0.f, O = 0.f;
        if (M != -CUDART_INF_F) {
#pragma unroll
            for (int w = 0; w < KG; ++w) {
                const float f = exp2f(cm[w * RT + r] - M);
                Lsum += cl[w * RT + r] * f;
                O += co[(w * RT + r) * D + d] * f;
            }
        }
        const int rr = row0 + r;
        const int t = rr / G, h = kvh * G + rr % G;
        const size_t R = ((size_t)b * T + t) * a.Hq + h;
        if (a.nsplit == 1 && a.out) {
            a.out[R * D + d] = O / Lsum;
        } else if (a.nsplit == 1 && a.push_world) {
            push_partial<D>(a, R, d, O, M == -CUDART_INF_F ? -CUDART_INF_F : M * kLn2, Lsum);
        } else {
            const size_t PR = (size_t)split * rows_total + R;
            a.part_o[PR * D + d] = O;
            if (d == 0) {
                a.part_ml[PR * 2] = M == -CUDART_INF_F ? -CUDART_INF_F : M * kLn2;
                a.part_ml[PR * 2 + 1] = Lsum;
            }
        }
    }
    griddep_launch_dependents();
    if (a.nsplit == 1) {
        if (a.push_world) push_finish<NC>(a);
        return;
    }

    // (b) Split-KV: the last CTA to finish for this (sequence, kv head, row tile) merges every
    // split's partial (threadfence-reduction pattern: release fence, counter, acquire fence).
    __threadfence();
    named_barrier_sync(1, NC * 32);
    int *flag = reinterpret_cast<int *>(const_cast<float *>(co) + KG * RT * D);
    float *row_l = reinterpret_cast<float *>(flag + 4);  // [RT]
    float *row_m = row_l + RT;                            // [RT]
    float *wts = row_m + RT;                              // [RT][nsplit]
    if (threadIdx.x == 0) {
        const int tile = (b * a.Hkv + kvh) * a.mtiles + mt;
        const int prev = atomicAdd(&a.counters[tile], 1);
        flag[0] = prev == a.nsplit - 1;
        if (prev == a.nsplit - 1) a.counters[tile] = 0;  // every arrival is in: ready for the next launch
    }
    named_barrier_sync(1, NC * 32);
    if (!flag[0]) return;
    __threadfence();
    // Row statistics: a warp per row, its lanes over the splits (one round of loads per row).
    const int mw = threadIdx.x >> 5, ml = threadIdx.x & 31;
    for (int r = mw; r < nvalid; r += NC) {
        const int rr = row0 + r;
        const size_t R = ((size_t)b * T + rr / G) * a.Hq + kvh * G + rr % G;
        float mloc = -CUDART_INF_F;
        for (int sp = ml; sp < a.nsplit; sp += 32)
            mloc = fmaxf(mloc, __ldcg(&a.part_ml[((size_t)sp * rows_total + R) * 2]));
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) mloc = fmaxf(mloc, __shfl_xor_sync(0xffffffffu, mloc, off));
        const float M = mloc;
        float lloc = 0.f;
        for (int sp = ml; sp < a.nsplit; sp += 32) {
            const float2 ml2 = __ldcg(reinterpret_cast<const float2 *>(&a.part_ml[((size_t)sp * rows_total + R) * 2]));
            const float w = ml2.x == -CUDART_INF_F ? 0.f : expf(ml2.x - M);
            wts[r * a.nsplit + sp] = w;
            lloc += w * ml2.y;
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) lloc += __shfl_xor_sync(0xffffffffu, lloc, off);
        if (ml == 0) {
            row_l[r] = lloc;
            row_m[r] = M;
        }
    }
    named_barrier_sync(1, NC * 32);
    // Outputs: a thread per (row, 4 head-dim values); eight splits' loads in flight at a time.
    for (int idx = threadIdx.x; idx < nvalid * (D / 4); idx += NC * 32) {
        const int r = idx / (D / 4), d4 = idx % (D / 4);
        const int rr = row0 + r;
        const size_t R = ((size_t)b * T + rr / G) * a.Hq + kvh * G + rr % G;
        float4 O = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int sp0 = 0; sp0 < a.nsplit; sp0 += 8) {
            float4 v[8];
#pragma unroll
            for (int u = 0; u < 8; ++u)
                v[u] = sp0 + u < a.nsplit
                           ? __ldcg(reinterpret_cast<const float4 *>(&a.part_o[((size_t)(sp0 + u) * rows_total + R) * D]) + d4)
                           : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                const float w = sp0 + u < a.nsplit ? wts[r * a.nsplit + sp0 + u] : 0.f;
                O.x = fmaf(w, v[u].x, O.x), O.y = fmaf(w, v[u].y, O.y), O.z = fmaf(w, v[u].z, O.z),
                O.w = fmaf(w, v[u].w, O.w);
            }
        }
        const float o4[4] = {O.x, O.y, O.z, O.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int d = 4 * d4 + e;
            if (a.out) {
                a.out[R * D + d] = o4[e] / row_l[r];
            } else if (a.push_world) {
                push_partial<D>(a, R, d, o4[e], row_m[r], row_l[r]);
            } else {
                a.res_o[R * D + d] = o4[e];
                if (d == 0) {
                    a.res_ml[R * 2] = row_m[r];
                    a.res_ml[R * 2 + 1] = row_l[r];
                }
            }
        }
    }
    if (a.push_world) push_finish<NC>(a);
}

// Split-KV merge across a thread-block cluster (the splits of one (sequence, kv head, row
// tile) launched as one cluster, split = rank): each CTA keeps its split's (m, l, o) rows in its
// own shared memory behind cm / cl / co, the cluster synchronises, every CTA merges a slice of
// the tile's (row, head-dim) elements reading all splits' partials through distributed shared
// memory and writes them, and a second cluster barrier keeps every CTA's shared memory alive
// until the last remote read.  No global partials, no fences or arrival counters, and the merge
// is spread over the cluster instead of falling to one last CTA.  Called by the NC consumer
// warps; the producer warp takes the two cluster barriers on its own (decode_cluster_idle).
template <int D, int KG, int NC, int RT>
__device__ __forceinline__ void decode_epilogue_cluster(const DecodeArgs &a, uint8_t *ring, int row0, int nrows,
                                                        int kvh, int b, int split) {
    const float *cm = reinterpret_cast<const float *>(ring);
    const float *cl = cm + KG * RT;
    const float *co = cl + KG * RT;
    float *sp_ml = const_cast<float *>(co) + KG * RT * D;  // [RT][2] this split's (m log2 units, l)
    float *sp_o = sp_ml + 2 * RT;                          // [RT][D] this split's unnormalised o
    const int G = a.G, T = a.T;
    const int nvalid = min(RT, nrows - row0);
    for (int idx = threadIdx.x; idx < nvalid * D; idx += NC * 32) {
        const int r = idx / D, d = idx % D;
        float M = -CUDART_INF_F;
#pragma unroll
        for (int w = 0; w < KG; ++w) M = fmaxf(M, cm[w * RT + r]);
        float Lsum = 0.f, O = 0.f;
        if (M != -CUDART_INF_F) {
#pragma unroll
            for (int w = 0; w < KG; ++w) {
                const float f = exp2f(cm[w * RT + r] - M);
                Lsum += cl[w * RT + r] * f;
                O += co[(w * RT + r) * D + d] * f;
            }
        }
        sp_o[r * D + d] = O;
        if (d == 0) {
            sp_ml[2 * r] = M;
            sp_ml[2 * r + 1] = Lsum;
        }
    }
    griddep_launch_dependents();
    cluster_sync_all();  // every split's partial is in its CTA's shared memory
    const int nsplit = a.nsplit;
    // Every CTA merges an equal contiguous share of the tile's elements (consecutive threads on
    // consecutive head-dim elements: conflict-free reads of every split's shared memory), so that
    // all of them work even when the tile has few rows.
    const int total = nvalid * D, chunk = (total + nsplit - 1) / nsplit;
    const int e_end = min(total, (split + 1) * chunk);
    for (int idx = split * chunk + threadIdx.x; idx < e_end; idx += NC * 32) {
        const int r = idx / D, d = idx % D;
        // Every split's (m, l, o) of this output requested at once: the loads cross the cluster's
        // network, and one round trip per split in turn cost microseconds at 16 splits.
        float mv[kMaxClusterSplits], lv[kMaxClusterSplits], ov[kMaxClusterSplits];
#pragma unroll
        for (int sp = 0; sp < kMaxClusterSplits; ++sp) {
            const bool in = sp < nsplit;
            mv[sp] = in ? ld_cluster_f32(sp_ml + 2 * r, sp) : -CUDART_INF_F;
            lv[sp] = in ? ld_cluster_f32(sp_ml + 2 * r + 1, sp) : 0.f;
            ov[sp] = in ? ld_cluster_f32(sp_o + r * D + d, sp) : 0.f;
        }
        float M = -CUDART_INF_F;
#pragma unroll
        for (int sp = 0; sp < kMaxClusterSplits; ++sp) M = fmaxf(M, mv[sp]);
        float Lsum = 0.f, O = 0.f;
        if (M != -CUDART_INF_F) {
#pragma unroll
            for (int sp = 0; sp < kMaxClusterSplits; ++sp) {
                if (sp < nsplit) {
                    const float w = mv[sp] == -CUDART_INF_F ? 0.f : exp2f(mv[sp] - M);
                    Lsum += w * lv[sp];
                    O += w * ov[sp];
                }
            }
        }
        const int rr = row0 + r;
        const size_t R = ((size_t)b * T + rr / G) * a.Hq + kvh * G + rr % G;
        if (a.out) {
            a.out[R * D + d] = O / Lsum;
        } else {
            a.res_o[R * D + d] = O;
            if (d == 0) {
                a.res_ml[R * 2] = M == -CUDART_INF_F ? -CUDART_INF_F : M * kLn2;
                a.res_ml[R * 2 + 1] = Lsum;
            }
        }
    }
    cluster_sync_all();  // no CTA leaves while another may still read its shared memory
}

// The producer warp's part of decode_epilogue_cluster: the same two cluster barriers.
__device__ __forceinline__ void decode_cluster_idle() {
    cluster_sync_all();
    cluster_sync_all();
}

// Bytes of `ring` the epilogue needs: cm, cl, co, then the larger of the flag word with the
// split-merge rows (up to 64 splits, global merge) and the split's partial (cluster merge).
template <int D, int KG, int RT>
constexpr uint32_t decode_epilogue_bytes() {
    return KG * RT * D * 4 + 2 * KG * RT * 4 +
           (16 + 2 * RT * 4 + RT * 64 * 4 > 2 * RT * 4 + RT * D * 4 ? 16 + 2 * RT * 4 + RT * 64 * 4
                                                                     : 2 * RT * 4 + RT * D * 4);
}

}  // namespace brk
