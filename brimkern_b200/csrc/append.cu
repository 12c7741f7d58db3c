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
    // The dependent decode may be scheduled now (it waits for this grid before reading q or the
    // new rows); this grid itself waits for whatever the stream ran before it.
    griddep_launch_dependents();
    griddep_wait();
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

cudaError_t launch_append(const AppendArgs &a, cudaStream_t s, bool pdl) {
    const long long rows = (long long)a.B * a.T * (a.Hq + 2 * a.Hkv);
    if (rows == 0) return cudaSuccess;
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
    switch (a.D) {
        case 64: return cudaLaunchKernelEx(&cfg, append_kernel<64>, a);
        case 128: return cudaLaunchKernelEx(&cfg, append_kernel<128>, a);
        case 256: return cudaLaunchKernelEx(&cfg, append_kernel<256>, a);
        default: return cudaLaunchKernelEx(&cfg, append_kernel<0>, a);
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
