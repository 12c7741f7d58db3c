// Internal structures of libbrk_attn: the objects behind the opaque C-ABI handles and the
// argument blocks of each kernel.  Argument blocks travel by value as kernel parameters
// (positions included), so a launch needs no host->device copy.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "brk_attn.h"

struct brk_ctx {
    int device = 0;
    int num_sms = 0;
    int *d_err = nullptr;      // device error word written by bounded waits (brk::DeviceError)
    void *ws = nullptr;        // split-KV workspace
    size_t ws_bytes = 0;
    uint64_t launches = 0;     // kernels launched through this context
};

struct brk_rope {
    brk_ctx *ctx = nullptr;
    int head_dim = 0;
    int max_pos = 0;
    double2 *table = nullptr;  // [max_pos][head_dim/2] (cos, sin)
};

struct brk_kv {
    brk_ctx *ctx = nullptr;
    brk_kv_desc desc{};
    int cap = 0;
    __half *k = nullptr;       // [layer][seq][kv head][cap][D]
    __half *v = nullptr;
    CUtensorMap tm_dec_k{}, tm_dec_v{};  // boxes for the decode kernel
    CUtensorMap tm_pre_k{}, tm_pre_v{};  // boxes for the prefill kernel
};

namespace brk {

struct AppendArgs {
    const float *q_in, *k_in, *v_in;
    float *q_out;
    __half *kc, *vc;
    const double2 *rope;
    int rope_max;
    const float *q_norm, *k_norm;
    double eps;
    int one_plus;
    int B, T, Hq, Hkv, D, layer, cap, kv_offset;
    int past_len[BRK_MAX_BATCH];
};

struct DecodeArgs {
    const float *q;       // [B][T][Hq][D] f32
    float *out;           // [B][T][Hq][D] f32 final output, or nullptr (partial mode)
    float *part_ml;       // per-split partials [nsplit][B*T*Hq][2]: workspace, or with a single
    float *part_o;        //   split in partial mode the caller's buffer; [nsplit][B*T*Hq][D]
    float *res_ml;        // partial mode with splits: the caller's buffer for the merged partial
    float *res_o;
    int *counters;        // [B*Hkv*mtiles] split arrival counters, zero between launches
    int *err;
    int B, T, Hq, Hkv, G;
    int layer, cap, mtiles, nsplit, keys_per_split;
    int kv_offset, window;
    float scale, scale_log2, softcap;
    float cap_k1;           // softcap: 2 * scale * log2(e) / softcap  (exp2 argument of e^{2z})
    float cap_k2;           // softcap: softcap * log2(e)              (score in log2 units)
    int past_len[BRK_MAX_BATCH];
};

struct PrefillArgs {
    const float *q;  // [B][T][Hq][D] f32 (rotated), or nullptr when q_raw is given
    float *out;      // [B][T][Hq][D] f32
    // Fused q prologue (brk_attn_prefill_step): raw projection q, gain, rope table.
    const float *q_raw;
    const float *q_norm;
    const double2 *rope;
    double eps;
    int one_plus;
    int *err;
    int B, T, Hq, Hkv, layer, cap, kv_offset, window;
    float scale_log2, softcap, cap_k1, cap_k2;
    int past_len[BRK_MAX_BATCH];
};

struct CombineArgs {
    const float *part_ml, *part_o;
    size_t stride_ml, stride_o;  // floats between consecutive parts
    float *out;             // normalised output, or nullptr
    float *out_ml, *out_o;  // combined partial (m, l, o), or nullptr
    int n_parts, rows, D;
};

// Keys per pipeline stage of the decode kernel for a head dim.
int decode_stage_keys(int head_dim);
int prefill_tile_keys();

// pdl: launch so that the next (dependent) decode kernel may start during this one.
cudaError_t launch_append(const AppendArgs &a, cudaStream_t s, bool pdl);
// pdl: launch as a programmatic dependent of the preceding kernel (the append of brk_attn_step).
cudaError_t launch_decode(int head_dim, const CUtensorMap &tmk, const CUtensorMap &tmv, const DecodeArgs &a,
                          int grid_x, int grid_y, int grid_z, cudaStream_t s, bool pdl);
cudaError_t launch_combine(const CombineArgs &a, cudaStream_t s);
// Tensor-core prefill (head_dim 64 or 128); maps with prefill_tile_keys()-row boxes.
cudaError_t launch_prefill(int head_dim, const CUtensorMap &tmk, const CUtensorMap &tmv, const PrefillArgs &a,
                           cudaStream_t s);
// Concurrent CTAs per SM of the decode kernel for a head dim (occupancy query).
int decode_ctas_per_sm(int head_dim);

// kc/vc point at row row0 of kv head 0 of one (layer, sequence) segment; heads are cap rows apart.
cudaError_t launch_kv_write_rows(__half *kc, __half *vc, const float *k, const float *v, int n_rows, int n_kv_heads,
                                 int head_dim, int cap, cudaStream_t s);
cudaError_t launch_kv_read_rows(const __half *kc, const __half *vc, uint16_t *k, uint16_t *v, int n_rows,
                                int n_kv_heads, int head_dim, int cap, cudaStream_t s);

}  // namespace brk
