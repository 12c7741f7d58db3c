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
    void *ws = nullptr;        // split-KV partials: (m, l) pairs, then the outputs
    size_t ws_bytes = 0;
    // Split-KV arrival counters, one per (sequence, kv head, row tile) of a launch; each launch's
    // last arriver puts its counter back to zero.  A buffer of their own: were they part of the
    // partials' workspace, a launch with fewer tiles would write partials over the counters of
    // tiles that a later, larger launch counts on being zero.
    int *counters = nullptr;
    size_t counters_n = 0;
    void *stage = nullptr;     // fp16 staging of an int8 cache layer for the prefill kernel
    size_t stage_bytes = 0;
    void *act = nullptr;       // fp16 activations of the projection GEMMs
    size_t act_bytes = 0;
    uint64_t launches = 0;     // kernels launched through this context
};

// This rank's exchange area for sequence-sharded decode over peer memory (brk_attn_decode_push /
// brk_attn_combine_peers): [2 parities][world sources][stride floats] of packed partials
// [rows*2 | rows*D], then [2 parities][world] uint32 epoch flags.  peers[p] is rank p's area as
// seen from this device (own area included), mapped through CUDA IPC or attached in-process.
struct brk_peer {
    brk_ctx *ctx = nullptr;
    int world = 0, rank = 0, max_rows = 0, head_dim = 0;
    size_t stride = 0;          // floats per (parity, source) block
    size_t flags_offset = 0;    // bytes from the area base to the flags
    void *area = nullptr;
    void *peers[8] = {};
    bool opened[8] = {};        // mapped with cudaIpcOpenMemHandle (closed on destroy)
    int *done = nullptr;        // tiles of this rank's current push launch that have finished
};

struct brk_rope {
    brk_ctx *ctx = nullptr;
    int head_dim = 0;
    int max_pos = 0;
    double2 *table = nullptr;  // [max_pos][head_dim/2] (cos, sin), the K / q rotation of the append
    float2 *table32 = nullptr; // the same rounded to f32: the prefill kernel's q prologue
};

struct brk_kv {
    brk_ctx *ctx = nullptr;
    brk_kv_desc desc{};
    int cap = 0;
    // BRK_KV_F16: fp16 rows [layer][seq][kv head][cap][D].
    __half *k = nullptr;
    __half *v = nullptr;
    // BRK_KV_I8: codes biased by +128 as bytes, [layer][seq][kv head][cap][D], and f32 scales
    // [layer][seq][kv head][2 (K, V)][scale_pitch] (scale_pitch = cap rounded up to 4, so that a
    // TMA box of scales may start at any 4-aligned key).
    uint8_t *k8 = nullptr;
    uint8_t *v8 = nullptr;
    float *scales = nullptr;
    int scale_pitch = 0;
    CUtensorMap tm_dec_k{}, tm_dec_v{};  // boxes for the decode kernel (fp16 rows or int8 codes)
    CUtensorMap tm_dec_s{};              // int8 mode: [2][keys] scale boxes for the decode kernel
    CUtensorMap tm_pre_k{}, tm_pre_v{};  // fp16 mode: boxes for the prefill kernel
    bool q8() const { return desc.dtype == BRK_KV_I8; }
};

namespace brk {

struct AppendArgs {
    const float *q_in, *k_in, *v_in;
    float *q_out;
    __half *kc, *vc;          // fp16 cache, or nullptr in int8 mode
    uint8_t *kc8, *vc8;       // int8 cache: biased codes, and
    float *scales;            //   [seg][2][scale_pitch] scales
    int scale_pitch;
    const double2 *rope;
    int rope_max;
    const float *q_norm, *k_norm;
    double eps;
    int one_plus;
    int B, T, Hq, Hkv, D, layer, cap, kv_offset;
    // Prefill chunks into an fp16 cache: q rotated in f32 (as the prefill kernel's own q
    // prologue does) into fp16 [B][T][Hq][D] for the prefill kernel's TMA loads, or nullptr.
    __half *q16;
    const float2 *rope32;
    int past_len[BRK_MAX_BATCH];
};

// Query rows per stream of the tensor-core prefill kernel (its q tiles' TMA box height).
constexpr int kPrefillQRows = 128;

// Most splits of one (sequence, kv head, row tile) that merge through a thread-block cluster.
constexpr int kMaxClusterSplits = 16;

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
    // Push mode (push_world > 0, partial mode only): the final partial of every row goes to
    // push_ml[p] / push_o[p] on each of the push_world ranks; the last tile of the launch to
    // finish then stores `epoch` into push_flag[p] on every rank (system-scope release).
    // Split-KV merge through a thread-block cluster (the nsplit CTAs of a tile are one cluster):
    // no workspace partials or counters (decode_epilogue_cluster).
    int cluster;
    int push_world;
    unsigned epoch;
    int push_tiles;         // tiles of this launch (B * Hkv * mtiles)
    int *push_done;         // finished-tile counter, zero between launches
    float *push_ml[8];
    float *push_o[8];
    unsigned *push_flag[8];
    // Fused append (fuse != 0, one new token per sequence, brk_attn_step): every CTA rotates the
    // q rows of its tile from q_in (QK-norm + RoPE in f32: q only feeds the fp16 operand) straight
    // into its fragments, split 0 also writing them to q_rot (the caller's q_work), and the CTA
    // whose key range holds position past_len[b] computes that position's K / V rows from
    // k_in / v_in (the append's fp64 operations) and stores them in the cache before its ring
    // loads them.
    int fuse;
    float *q_rot;           // = q, the rotated rows' destination
    const float *q_in, *k_in, *v_in;
    __half *kc, *vc;        // fp16 cache, or
    uint8_t *kc8, *vc8;     //   int8 codes (biased) and
    float *scales;          //   [seg][2][scale_pitch] scales
    int scale_pitch;
    const double2 *rope;    // [positions][D/2] (cos, sin) in double (the K row), or nullptr
    const float2 *rope32;   // the same rounded to f32 (the q rows)
    const float *q_norm, *k_norm;
    double eps;
    int one_plus;
    int past_len[BRK_MAX_BATCH];
};

struct PrefillArgs {
    const float *q;  // [B][T][Hq][D] f32 (rotated), or nullptr when q_raw is given
    float *out;      // [B][T][Hq][D] f32
    // Fused q prologue (brk_attn_prefill_step): raw projection q, gain, f32 rope table.
    const float *q_raw;
    const float *q_norm;
    const float2 *rope;
    // q already rotated to fp16 [B][T][Hq][D] (the append of the chunk wrote it): the producer
    // loads both streams' q tiles with TMA (map `tmq`) and the softmax warps stage nothing.
    int q_tma;
    float eps;
    int one_plus;
    int *err;
    int B, T, Hq, Hkv, layer, cap, kv_offset, window;
    float scale_log2, softcap, cap_k1, cap_k2;
    int past_len[BRK_MAX_BATCH];
};

// Projection GEMM (proj.cu): out[i] [M][n_i] = A [M][K] . W_i^T (+ bias_i) (+ residual for
// matrix 0), for up to three weight matrices W_i [n_i][K] concatenated along the output columns
// (n_end: cumulative ends).
struct ProjArgs {
    int M, K, nmat;
    int tile_end[3];          // cumulative 128-feature tiles per weight matrix
    int n[3];                 // output features of each matrix
    float *out[3];            // [M][n[i]] f32
    const float *bias[3];     // [n[i]] or null
    const float *residual;    // [M][n[0]] added to matrix 0 (or null)
    int splits, kps;          // split-K factor and k steps (of 64) per split (proj_plan)
    int *err;
};

struct CombineArgs {
    const float *part_ml, *part_o;
    size_t stride_ml, stride_o;  // floats between consecutive parts
    float *out;             // normalised output, or nullptr
    float *out_ml, *out_o;  // combined partial (m, l, o), or nullptr
    int n_parts, rows, D;
};

// Keys per pipeline stage of the decode kernel for a head dim (the same for both cache types).
int decode_stage_keys(int head_dim);
int prefill_tile_keys();

// pdl: launch so that the next (dependent) decode kernel may start during this one.
cudaError_t launch_append(const AppendArgs &a, cudaStream_t s, bool pdl);
// Decode kernel for both cache types: tmk / tmv map fp16 rows or int8 codes, tms the int8 scales
// (ignored for fp16); grid (splits, kv heads x row tiles of decode_rows_per_tile() query rows,
// sequences).  pdl: launch as a programmatic dependent of the preceding kernel (the append of
// brk_attn_step).
cudaError_t launch_decode(bool q8, int head_dim, const CUtensorMap &tmk, const CUtensorMap &tmv,
                          const CUtensorMap &tms, const DecodeArgs &a, int grid_x, int grid_y, int grid_z,
                          cudaStream_t s, bool pdl);
int decode_rows_per_tile();
// How many clusters of `size` decode CTAs fit on the GPU at once (0: clusters of that size cannot
// be launched).
int decode_max_clusters(int head_dim, bool q8, int size);
// Loads every decode / combine kernel on the current device now instead of at its first launch.
cudaError_t preload_decode_kernels();
cudaError_t launch_combine(const CombineArgs &a, cudaStream_t s);
// Combine after a bounded wait (wait_ns) until flags[p] == epoch for every p < world.
cudaError_t launch_combine_peers(const CombineArgs &a, const unsigned *flags, int world, unsigned epoch,
                                 unsigned long long wait_ns, int *err, cudaStream_t s);
// Tensor-core prefill (head_dim 64 or 128); maps with prefill_tile_keys()-row boxes.
cudaError_t launch_prefill(int head_dim, const CUtensorMap &tmk, const CUtensorMap &tmv, const PrefillArgs &a,
                           cudaStream_t s, bool pdl = false, const CUtensorMap *tmq = nullptr);
// Concurrent CTAs per SM of the decode kernel for a head dim and cache type (occupancy query).
int decode_ctas_per_sm(int head_dim, bool q8);

// kc/vc point at row row0 of kv head 0 of one (layer, sequence) segment; heads are cap rows apart.
cudaError_t launch_kv_write_rows(__half *kc, __half *vc, const float *k, const float *v, int n_rows, int n_kv_heads,
                                 int head_dim, int cap, cudaStream_t s);
cudaError_t launch_kv_read_rows(const __half *kc, const __half *vc, uint16_t *k, uint16_t *v, int n_rows,
                                int n_kv_heads, int head_dim, int cap, cudaStream_t s);

// int8 mode.  kc/vc: codes at row row0 of kv head 0 of one (layer, sequence) segment; sc: that
// segment's scales ([kv head][2][pitch]) offset by row0.  write_q8 quantises f32 rows
// (quantize_kv); store_codes writes given codes and scales; read returns codes and scales in the
// reference's token-major layout.
cudaError_t launch_kv_write_q8(uint8_t *kc, uint8_t *vc, float *sc, const float *k, const float *v, int n_rows,
                               int n_kv_heads, int head_dim, int cap, int pitch, cudaStream_t s);
cudaError_t launch_kv_store_codes(uint8_t *kc, uint8_t *vc, float *sc, const int8_t *k, const float *ks,
                                  const int8_t *v, const float *vs, int n_rows, int n_kv_heads, int head_dim, int cap,
                                  int pitch, cudaStream_t s);
cudaError_t launch_kv_read_q8(const uint8_t *kc, const uint8_t *vc, const float *sc, int8_t *k, float *ks, int8_t *v,
                              float *vs, int n_rows, int n_kv_heads, int head_dim, int cap, int pitch, cudaStream_t s);
// Dequantise rows [0, rows) of every (sequence, kv head) of one layer into fp16 staging
// [B][Hkv][rows][D] (K and V), for the tensor-core prefill kernel.
cudaError_t launch_kv_dequant(const uint8_t *kc, const uint8_t *vc, const float *sc, __half *k, __half *v, int layer,
                              int B, int n_kv_heads, int head_dim, int cap, int pitch, int rows, cudaStream_t s);

// Projections (proj.cu).  proj_token_tile: tokens per CTA (the MMA N) for M rows: 32..256;
// proj_plan sets a.splits / a.kps; launch_norm_cast also pre-fills the outputs when a.splits > 1.
int proj_token_tile(int rows);
void proj_plan(ProjArgs &a, int ntok, int sms);
cudaError_t launch_norm_cast(const float *x, const float *gain, float eps, int one_plus, __half *out, int rows, int K,
                             const ProjArgs &a, cudaStream_t s);
cudaError_t launch_post_norm_residual(float *h, const float *x, const float *gain, float eps, int one_plus, int rows,
                                      int n, cudaStream_t s);
cudaError_t launch_proj(int ntok, const CUtensorMap &tx, const CUtensorMap *tw, const CUtensorMap *to,
                        const ProjArgs &a, cudaStream_t s);

// Non-causal attention staging (full.cu): token-major f32 [B][L][H][D] K/V -> head-major fp16
// [B][H][L][Dp] (zero-padded head dim), and f32 rows [rows][D] -> [rows][Dp] zero-padded.
cudaError_t launch_stage_kv(const float *k, const float *v, __half *ks, __half *vs, int B, int L, int H, int D, int Dp,
                            cudaStream_t s);
cudaError_t launch_pad_rows(const float *src, float *dst, long long rows, int D, int Dp, cudaStream_t s);

}  // namespace brk
