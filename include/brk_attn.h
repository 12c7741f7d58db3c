/*
 * brk_attn.h — C ABI of the B200 (sm_100a) attention operator for the Brimkern engine.
 *
 * Replaces the engine's attention / KV-cache operator path (RomainKH/Brimkern,
 * src/lib/webgpu/kernels.ts): recAttention / recAttentionQ8 dispatch (:1626-1661), the f32 KV
 * append (:1727-1730), the per-layer KV manager (:1749-1806) and the readback twins used by
 * selfValidate (:556-704).  The WGSL kernels they launch (src/lib/webgpu/shaders.ts:1361-1944)
 * are replaced by hand-written CUDA for sm_100a.
 *
 * Conventions
 *   - Every entry point returns an int status: BRK_OK (0) or a negative BRK_ERR_* code; the
 *     message of the last failure on the calling thread is brk_last_error().  Nothing aborts
 *     and no C++ exception crosses the ABI.
 *   - All tensor pointers are DEVICE pointers unless the parameter says "host".  Layouts are the
 *     reference's (kernels.ts:608-609): q / out [batch][n_tokens][n_heads][head_dim] f32,
 *     k / v inputs [batch][n_tokens][n_kv_heads][head_dim] f32.
 *   - `stream` is a cudaStream_t passed as void* (NULL = legacy default stream).  Work is
 *     stream-ordered; calls on one context come from one host thread at a time.
 *   - Positions: token t of sequence b sits at absolute position past_len[b] + t and attends
 *     keys [0, past_len[b] + t] (kernels.ts:1816, shaders.ts:1500), or the last `window` of
 *     them when params->window > 0.
 */
#ifndef BRK_ATTN_H
#define BRK_ATTN_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define BRK_ABI_VERSION 2
#define BRK_MAX_BATCH 512 /* sequences per call (positions travel in the kernel parameters) */

enum {
    BRK_OK = 0,
    BRK_ERR_INVALID = -1,     /* bad argument or unsupported shape */
    BRK_ERR_CUDA = -2,        /* a CUDA runtime call failed */
    BRK_ERR_CAPACITY = -3,    /* a position or row is beyond the cache / rope table */
    BRK_ERR_UNSUPPORTED = -4, /* head_dim or dtype without a kernel */
    BRK_ERR_DEVICE = -5       /* a kernel reported a bounded-wait timeout (brk_ctx_check) */
};

/* KV cache element types.  BRK_KV_I8 is the reference's int8 mode (setKvQuant(true),
 * kernels.ts:1755-1760): symmetric int8 codes with one f32 scale per (row, kv head) for K and for
 * V (quantize_kv, shaders.ts:1673-1705), half the bytes of fp16. */
enum { BRK_KV_F16 = 0, BRK_KV_I8 = 1 };

typedef struct brk_ctx brk_ctx;   /* one per GPU: device id, error flag, workspace */
typedef struct brk_kv brk_kv;     /* persistent KV cache of n_layers layers (KvEntry, kernels.ts:93) */
typedef struct brk_rope brk_rope; /* RoPE cos/sin table in HBM */

typedef struct {
    int n_layers;   /* layers held (the reference keys KvEntry by layer, kernels.ts:1749) */
    int batch;      /* independent sequences */
    int n_kv_heads;
    int head_dim;   /* 64, 128 or 256 */
    int capacity;   /* rows per (layer, sequence, kv head); brk_kv_grow enlarges it */
    int dtype;      /* BRK_KV_F16 or BRK_KV_I8 */
} brk_kv_desc;

/* Per-layer attention configuration: LayerCfg's attention fields (kernels.ts:24-56). */
typedef struct {
    int n_heads;
    int n_kv_heads;      /* n_heads % n_kv_heads == 0 (GQA group = n_heads / n_kv_heads) */
    int head_dim;
    float scale;         /* attnScale; <= 0 selects 1/sqrt(head_dim) (kernels.ts:1627) */
    float softcap;       /* attnLogitSoftcap; <= 0 disables s -> c*tanh(s/c) (shaders.ts:1490) */
    int window;          /* sliding window in keys; <= 0 = global attention (extension) */
    int kv_offset;       /* absolute position of cache row 0 (sequence-sharded caches); else 0 */
    int norm_one_plus;   /* RMSNorm gain convention x*(1+w) (rmsGainOnePlus) */
    double eps;          /* QK-norm epsilon (LayerCfg.eps) */
    const float *q_norm; /* device [head_dim] per-head q RMSNorm gain, or NULL (kernels.ts:1708) */
    const float *k_norm; /* device [head_dim] per-head k RMSNorm gain, or NULL (kernels.ts:1709) */
    const brk_rope *rope; /* NeoX RoPE table, or NULL for no rotary embedding */
} brk_attn_params;

/* ---- errors / version -------------------------------------------------------------------- */
const char *brk_last_error(void);
int brk_abi_version(void);

/* ---- context (the WebGpuEngine instance, kernels.ts:100) ------------------------------- */
int brk_ctx_create(int device, brk_ctx **out);
int brk_ctx_destroy(brk_ctx *ctx);
/* Synchronises `stream` and reports BRK_ERR_DEVICE if any kernel of this context hit a wait
 * limit since the last check (then clears the flag).  Mirrors the engine's health flags. */
int brk_ctx_check(brk_ctx *ctx, void *stream);
/* Pre-sizes the split-KV workspace (bytes) so that later calls allocate nothing. */
int brk_ctx_reserve(brk_ctx *ctx, size_t bytes);
/* Pre-sizes the context's fp16 staging buffer (bytes), which three paths fill per call:
 * brk_attn_prefill_step over an fp16 cache (8+ tokens) stages the rotated q, 2 * batch *
 * n_tokens * n_heads * head_dim bytes; prefill over an int8 cache stages the layer's
 * dequantised rows, 2 * batch * n_kv_heads * rows * head_dim * 2 bytes with rows = max over
 * the batch of past_len + n_tokens - kv_offset; non-
 * causal attention stages its K/V (and, for head dims other than 64 / 128 / 256, q and out):
 * 4 * batch * n_kv_heads * kv_len * Dp + 8 * batch * n_tokens * n_heads * Dp + 256 bytes with
 * Dp the head dim rounded up to 64 / 128 / 256 (the q term only when Dp != head_dim).  A call
 * whose staging fits allocates nothing; one that does not grows the buffer (after a device
 * synchronise, as queued kernels may still read it). */
int brk_ctx_reserve_stage(brk_ctx *ctx, size_t bytes);
/* Number of kernels this context has launched so far (diagnostics / benchmarks). */
uint64_t brk_ctx_launches(const brk_ctx *ctx);

/* ---- RoPE tables (rope / rope_factors, shaders.ts:1361-1408; ropeCpu kernels.ts:3428-3460) -
 * cos/sin of pos / (base^(2i/D) * ff[i]) for pos in [0, max_positions), computed on the host in
 * double exactly as the reference's CPU function does, so the device append reproduces it
 * bit for bit.  ff_host: host [head_dim/2] divisors (rope_freqs.weight, model.ts:590-597) or
 * NULL. */
int brk_rope_create(brk_ctx *ctx, int head_dim, double base, const float *ff_host,
                    int max_positions, brk_rope **out);
int brk_rope_destroy(brk_rope *rope);
int brk_rope_max_positions(const brk_rope *rope);
/* Meta's published llama3 frequency scaling as divisors ff[i] (the values llama.cpp stores as
 * rope_freqs.weight, which the reference reads at model.ts:590-597).  ff_out: host [head_dim/2]. */
int brk_llama3_rope_factors(int head_dim, double base, double factor, double low_freq_factor,
                            double high_freq_factor, int original_context, float *ff_out);

/* ---- KV cache (ensureKv / resetKvGpu / clearKvCache, kernels.ts:1766-1806) ------------------
 * Stored head-major, [layer][sequence][kv head][capacity][head_dim], zero-initialised: fp16, or
 * for BRK_KV_I8 one byte per code plus per-(row, kv head) K and V scales.  Every attention entry
 * point below works on both types; the int8 prefill dequantises the layer to fp16 staging held by
 * the context (so two streams must not run int8 prefill on one context at the same time). */
int brk_kv_create(brk_ctx *ctx, const brk_kv_desc *desc, brk_kv **out);
int brk_kv_destroy(brk_kv *kv);
int brk_kv_capacity(const brk_kv *kv);
/* ensureKv (kernels.ts:1782-1806): if rows > capacity, grow to max(rows, capacity+1024, 1024)
 * with a device-side copy of the existing rows. */
int brk_kv_grow(brk_kv *kv, int rows, void *stream);
/* clearKvCache / resetKvGpu (kernels.ts:1766-1777) and the session restart of runDecodeGpu
 * (kernels.ts:1817-1825: a new session or pastLen 0 starts the cache over): zero the rows of
 * sequence `seq` in every layer, leaving the other sequences' rows untouched, or of every
 * sequence when seq == -1 (the reference holds a single session; a batch holds one per
 * sequence).  Stream-ordered, no allocation. */
int brk_kv_reset(brk_kv *kv, int seq, void *stream);
/* Plain row store, no norm or rotation: the f32 copy of kernels.ts:1729-1730 for callers that
 * already hold final K/V, f32 -> fp16 (round to nearest even); for an int8 cache the quantize_kv
 * pass of recQuantizeKv (kernels.ts:1644-1648).  k, v: [n_rows][n_kv_heads][D] f32 (either may
 * be NULL). */
int brk_kv_write_rows(brk_kv *kv, int layer, int seq, int row0, int n_rows, const float *k,
                      const float *v, void *stream);
/* Test hook: copy rows back in the reference's token-major layout as fp16 bit patterns.
 * k_out, v_out: device [n_rows][n_kv_heads][D] uint16.  fp16 caches only. */
int brk_kv_read_rows(const brk_kv *kv, int layer, int seq, int row0, int n_rows,
                     uint16_t *k_out, uint16_t *v_out, void *stream);
/* int8 caches: store given codes and scales (the inputs of the attentionQ8Kv readback twin,
 * kernels.ts:681), and read them back (quantizeKvReadback, kernels.ts:664), in the reference's
 * layout: codes [n_rows][n_kv_heads][D] int8, scales [n_rows][n_kv_heads] f32 (K and V pairs may
 * each be NULL). */
int brk_kv_write_codes(brk_kv *kv, int layer, int seq, int row0, int n_rows, const int8_t *k_codes,
                       const float *k_scales, const int8_t *v_codes, const float *v_scales, void *stream);
int brk_kv_read_codes(const brk_kv *kv, int layer, int seq, int row0, int n_rows, int8_t *k_codes,
                      float *k_scales, int8_t *v_codes, float *v_scales, void *stream);

/* ---- hot path ----------------------------------------------------------------------------- */
/* KV append with the q/k prologue fused (kernels.ts:1707-1730): per-head RMSNorm of q and k
 * (if gains are given), NeoX RoPE (if a table is given) at position past_len[b]+t, K and V
 * stored at cache row past_len[b]+t-kv_offset (fp16, or quantised as quantize_kv does for an
 * int8 cache, kernels.ts:1721-1725); the rotated q is written to q_out f32
 * [B][T][Hq][D] for the attention call.  With kv == NULL only q is processed (the rope / rmsnorm
 * readback twins, any even head_dim up to 1024).  past_len: HOST [batch]. */
int brk_attn_append(brk_ctx *ctx, brk_kv *kv, int layer, const brk_attn_params *p, int batch,
                    int n_tokens, const int32_t *past_len, const float *q_in, const float *k_in,
                    const float *v_in, float *q_out, void *stream);

/* One decode step of a layer's attention slice (recordLayerKV, kernels.ts:1707-1731): the
 * append above followed by the decode kernel, launched so that the decode kernel starts
 * streaming the cache rows that the append does not touch while the append still runs
 * (programmatic dependent launch).  q_work receives the rotated q; out [B][T][Hq][D] f32.
 * Decode shapes only (n_tokens * group <= 64).  past_len: HOST [batch]. */
int brk_attn_step(brk_ctx *ctx, brk_kv *kv, int layer, const brk_attn_params *p, int batch,
                  int n_tokens, const int32_t *past_len, const float *q_in, const float *k_in,
                  const float *v_in, float *q_work, float *out, void *stream);

/* recAttention (kernels.ts:1626-1641): attention of q [B][T][Hq][D] (already rotated) over
 * cache rows [0, past_len[b]+t] -> out [B][T][Hq][D] f32.  Picks the decode kernel for small
 * T*group, the tensor-core prefill kernel otherwise (env BRK_ATTN_DECODE=0 forces the latter,
 * like ?attndecode=0, kernels.ts:181-215).  past_len: HOST [batch]. */
int brk_attn_forward(brk_ctx *ctx, const brk_kv *kv, int layer, const brk_attn_params *p,
                     int batch, int n_tokens, const int32_t *past_len, const float *q, float *out,
                     void *stream);
/* The decode kernel alone (attention_decode, shaders.ts:1768-1851): one CTA per (sequence,
 * kv head[, split]) so the whole query group shares each K/V read, split-KV + LSE combine. */
int brk_attn_decode(brk_ctx *ctx, const brk_kv *kv, int layer, const brk_attn_params *p,
                    int batch, int n_tokens, const int32_t *past_len, const float *q, float *out,
                    void *stream);
/* The number of key-range splits (CTAs per (sequence, kv head, row tile)) that brk_attn_decode
 * and brk_attn_step pick for this call: an automatic choice from the GPU's CTA slots and the
 * longest attended range, or BRK_DECODE_SPLITS when set.  Returns the count (>= 1) or a
 * negative BRK_ERR_* code.  Launches nothing (diagnostics, tests and benchmarks).  No reference
 * counterpart (the reference never splits the key range). */
int brk_attn_decode_splits(brk_ctx *ctx, const brk_kv *kv, const brk_attn_params *p, int batch,
                           int n_tokens, const int32_t *past_len);
/* No-allocation variant of brk_attn_decode.  No counterpart in the reference: it exists for
 * callers of this library that cannot allocate device memory while they run attention -- for
 * example serving hosts that hand nearly all of HBM to their own KV-cache pool at start-up (a
 * later cudaMalloc would fail), or hosts whose decode loop must not stall on the device-wide
 * synchronisation that cudaMalloc / cudaFree imply.  brk_attn_decode may grow the context's
 * workspace the first time a call needs more split-KV partials; this entry point instead keeps
 * the partials in a fixed array compiled into the library and calls no allocator.
 *   - Same arguments, outputs and split choice as brk_attn_decode.  The caller still provides
 *     q and out.
 *   - The array holds BRK_DECODE_STATIC_SCRATCH_BYTES.  A call that splits the key range
 *     (brk_attn_decode_splits > 1) needs, with rows = batch * n_tokens * n_heads and
 *     tiles = batch * n_kv_heads * ceil(n_tokens * n_heads / n_kv_heads / 8):
 *       round_up(4 * tiles, 256) + 4 * (round_up(2 * nsplit * rows, 4) + nsplit * rows * head_dim)
 *     bytes (arrival counters, (m, l) pairs, partial outputs); a call that needs more fails with
 *     BRK_ERR_CAPACITY and a message giving both sizes.  A one-split call uses none of it.
 *   - The array and the decode kernels are loaded on a device by the first brk_ctx_create for
 *     that device (the array's memory is taken then and held until the process exits), so
 *     create the context before handing the rest of HBM to a pool; the calls themselves do no
 *     set-up and allocate nothing.
 *   - All calls on a device share the array and it keeps the last call's contents.  Each call
 *     clears its arrival counters with one cudaMemsetAsync on the caller's stream before the
 *     kernel, and the kernel writes every partial before reading it.  Calls whose kernels
 *     overlap on the GPU (other streams, other contexts on the same device) race on the array:
 *     serialise them. */
#define BRK_DECODE_STATIC_SCRATCH_BYTES (8u << 20)
int brk_attn_decode_static(brk_ctx *ctx, const brk_kv *kv, int layer, const brk_attn_params *p,
                           int batch, int n_tokens, const int32_t *past_len, const float *q,
                           float *out, void *stream);
/* The tensor-core prefill kernel alone (replaces the 2-pass `attention`, shaders.ts:1482-1524):
 * tcgen05.mma / TMEM tiles for QK^T and PV, causal with the chunk offset past_len. */
int brk_attn_prefill(brk_ctx *ctx, const brk_kv *kv, int layer, const brk_attn_params *p,
                     int batch, int n_tokens, const int32_t *past_len, const float *q, float *out,
                     void *stream);
/* The same with q already rotated and rounded to fp16 (IEEE half bits, [B][T][Hq][D], 16-byte
 * aligned), which the kernel loads with TMA instead of staging it (the form brk_attn_prefill_step
 * uses for fp16 caches).  fp16 caches only. */
int brk_attn_prefill_h(brk_ctx *ctx, const brk_kv *kv, int layer, const brk_attn_params *p,
                       int batch, int n_tokens, const int32_t *past_len, const uint16_t *q16, float *out,
                       void *stream);

/* One prefill chunk of a layer's attention slice (recordLayerKV, kernels.ts:1707-1731, as the
 * chunked prefill of lfm2Model.ts:320-333): K/V appended as by brk_attn_append, then the
 * tensor-core kernel.  q gets QK-norm + RoPE in f32 (q only feeds the fp16 tensor-core operand):
 * for an fp16 cache and 8+ tokens in the append kernel, which leaves it as fp16 rows in the
 * context's staging buffer for the tensor-core kernel's TMA loads; otherwise inside the
 * tensor-core kernel's q staging.  The cache rows equal brk_attn_append's bit for bit.  head_dim
 * 64 or 128.
 * q_in [B][T][Hq][D], k_in / v_in [B][T][Hkv][D] f32 projections; out [B][T][Hq][D] f32. */
int brk_attn_prefill_step(brk_ctx *ctx, brk_kv *kv, int layer, const brk_attn_params *p,
                          int batch, int n_tokens, const int32_t *past_len, const float *q_in,
                          const float *k_in, const float *v_in, float *out, void *stream);

/* Non-causal attention (attention_full / attention_full_wg, shaders.ts:1530-1667, dispatched by
 * recAttentionFull, kernels.ts:1277-1290; UNet / ViT self- and cross-attention): every query
 * attends all kv_len keys, kv_len independent of n_tokens.  q [B][n_tokens][n_heads][head_dim],
 * k / v [B][kv_len][n_kv_heads][head_dim], out [B][n_tokens][n_heads][head_dim] f32; head_dim
 * 1..256.  K/V are staged as fp16 in the context (so two streams must not run this on one
 * context at the same time).  p->scale (<= 0: 1/sqrt(head_dim)) and p->softcap apply; rope,
 * norm gains, window and kv_offset must be unset. */
int brk_attn_full(brk_ctx *ctx, const brk_attn_params *p, int batch, int n_tokens, int kv_len,
                  const float *q, const float *k, const float *v, float *out, void *stream);

/* Split-KV partial over this cache's rows (extension, no reference counterpart; used to shard
 * a long context across GPUs): per row R = (b*T + t)*Hq + h, part_ml[2R] = max score m (natural
 * log units, -inf if no key), part_ml[2R+1] = sum l of exp(s - m), part_o[R*D..] = sum of
 * exp(s - m) * v (unnormalised).  Keys are cache rows r at absolute position kv_offset + r. */
int brk_attn_decode_partial(brk_ctx *ctx, const brk_kv *kv, int layer,
                            const brk_attn_params *p, int batch, int n_tokens,
                            const int32_t *past_len, const float *q, float *part_ml,
                            float *part_o, void *stream);
/* Log-sum-exp combine of n_parts partials -> out [rows][head_dim] = sum e^{m-M} o / sum e^{m-M} l.
 * Part p's (m, l) pairs start at part_ml + p * part_stride and its outputs at
 * part_o + p * part_stride (floats); part_stride 0 means the dense layouts [n_parts][rows][2]
 * and [n_parts][rows][head_dim].  A packed per-GPU buffer [rows*2 | rows*head_dim] gathered from
 * N GPUs is combined with part_ml = buf, part_o = buf + 2*rows, part_stride = rows*(2+head_dim). */
int brk_attn_combine(brk_ctx *ctx, int n_parts, int rows, int head_dim, const float *part_ml,
                     const float *part_o, size_t part_stride, float *out, void *stream);

/* ---- the projections either side of the operator (recordLayerKV, kernels.ts:1700-1736) -------
 * The layer-input RMSNorm with the q / k / v projections that feed brk_attn_append / step, and
 * the output projection with the residual add that consumes the attention output, as tensor-core
 * GEMMs.  Weights are the engine's fp16 matrices [n][k] (matmul_t_f16w: C = A W^T), passed as
 * raw fp16 bits; activations are f32 [rows][width] (rows = batch * n_tokens) and are cast to
 * fp16 for the tensor cores.  Widths: d_model / q_dim multiples of 8 as inputs, projection
 * outputs multiples of 4; all pointers 16-byte aligned.  Small row counts (decode) split K over
 * several CTAs whose f32 partials are added in L2 in no fixed order, so those outputs may differ
 * in the last bit from run to run.  One context runs one projection at a time (its activation
 * staging buffer is shared).
 *   brk_proj_qkv: n1 = rmsnorm(x, attn_norm) (attn_norm NULL: no norm), q = n1 wq^T (+ bq), k, v
 *   likewise (biases may be NULL).
 *   brk_proj_out: h = x + o where o = attn wo^T, or rmsnorm(o, post_norm) when post_norm is given
 *   (Gemma-2's post-attention norm).  h may not alias x. */
int brk_proj_qkv(brk_ctx *ctx, int rows, int d_model, int q_dim, int kv_dim, const float *x,
                 const float *attn_norm, double eps, int norm_one_plus, const uint16_t *wq,
                 const uint16_t *wk, const uint16_t *wv, const float *bq, const float *bk,
                 const float *bv, float *q, float *k, float *v, void *stream);
int brk_proj_out(brk_ctx *ctx, int rows, int q_dim, int d_model, const float *attn, const uint16_t *wo,
                 const float *post_norm, double eps, int norm_one_plus, const float *x, float *h,
                 void *stream);

/* ---- sequence-sharded decode over peer memory (extension, no reference counterpart) ---------
 * The fused form of decode_partial + all-gather + combine for one process per GPU: each rank's
 * decode kernel stores its final partials straight into every rank's exchange area (plain
 * stores through NVLink into memory mapped with CUDA IPC) and publishes an epoch flag there;
 * each rank's combine waits for every rank's flag, then merges.
 *   - The exchange area holds two epochs (parity epoch & 1).  Every rank makes the same calls with
 *     the same epochs (1, 2, 3, ... one per layer step), decode_push(e) then combine_peers(e) on
 *     one stream; then no rank can overwrite data another rank has yet to combine.
 *   - A rank whose partials do not arrive within timeout_s makes the combine write nothing and
 *     record a device error (brk_ctx_check -> BRK_ERR_DEVICE); recreate the areas after that.
 *   - Destroy an area only after every rank has finished its last combine (a host barrier). */
#define BRK_MAX_PEERS 8
#define BRK_PEER_HANDLE_BYTES 64
typedef struct brk_peer brk_peer;
/* This rank's exchange area for `world` ranks of up to max_rows rows (B * n_tokens * n_heads). */
int brk_peer_create(brk_ctx *ctx, int world, int rank, int max_rows, int head_dim, brk_peer **out);
/* The area's IPC handle (BRK_PEER_HANDLE_BYTES opaque bytes) for the other ranks' brk_peer_open. */
int brk_peer_handle(const brk_peer *peer, void *handle, size_t handle_bytes);
int brk_peer_open(brk_peer *peer, int peer_rank, const void *handle, size_t handle_bytes);
/* In-process form of brk_peer_open: rank peer_rank's area `other` (same device, or a device with
 * peer access). */
int brk_peer_attach(brk_peer *peer, int peer_rank, const brk_peer *other);
int brk_peer_destroy(brk_peer *peer);
/* brk_attn_decode_partial over this rank's cache rows, pushed into every rank's area. */
int brk_attn_decode_push(brk_ctx *ctx, const brk_kv *kv, int layer, const brk_attn_params *p,
                         int batch, int n_tokens, const int32_t *past_len, const float *q,
                         brk_peer *peer, uint32_t epoch, void *stream);
/* brk_attn_decode_push for one new token per sequence with the append fused into the launch, as
 * brk_attn_step does it: q_in is the raw q projection (rotated in the kernel; q_work receives the
 * rotated q), and the rank whose cache holds position past_len[b] (row past_len[b] - kv_offset
 * below the capacity) stores that position's K / V rows from k_in / v_in, which the other ranks
 * may pass as NULL.  Extension, no reference counterpart. */
int brk_attn_step_push(brk_ctx *ctx, brk_kv *kv, int layer, const brk_attn_params *p, int batch,
                       const int32_t *past_len, const float *q_in, const float *k_in, const float *v_in,
                       float *q_work, brk_peer *peer, uint32_t epoch, void *stream);
/* Waits (at most timeout_s) for every rank's partials of `epoch`, then out [rows][head_dim] =
 * their log-sum-exp combine. */
int brk_attn_combine_peers(brk_ctx *ctx, brk_peer *peer, int rows, uint32_t epoch, double timeout_s,
                           float *out, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* BRK_ATTN_H */
