// C-ABI implementation of libbrk_attn (declared in include/brk_attn.h): contexts, RoPE tables,
// the KV cache manager and the dispatch of the attention kernels.  Host code only.
#include <cudaTypedefs.h>

#include <algorithm>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "internal.h"

namespace {

thread_local std::string g_last_error;

int fail(int code, const char *fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return code;
}

int cuda_fail(cudaError_t e, const char *what) {
    return fail(BRK_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}

#define BRK_CUDA(call)                                         \
    do {                                                       \
        cudaError_t e_ = (call);                               \
        if (e_ != cudaSuccess) return cuda_fail(e_, #call);    \
    } while (0)

// Makes `device` current for the scope of a call and restores the caller's device afterwards.
struct DeviceGuard {
    int prev = -1;
    bool changed = false;
    explicit DeviceGuard(int device) {
        if (cudaGetDevice(&prev) == cudaSuccess && prev != device) {
            changed = cudaSetDevice(device) == cudaSuccess;
        }
    }
    ~DeviceGuard() {
        if (changed) cudaSetDevice(prev);
    }
};

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (!fn) {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }
    return fn;
}

// 2-D map over a row-major [rows][cols] buffer with box [box_rows][box_cols].
int make_map(CUtensorMap *m, CUtensorMapDataType type, size_t esize, const void *base, uint64_t rows, uint64_t cols,
             uint32_t box_cols, uint32_t box_rows, CUtensorMapSwizzle swizzle) {
    auto enc = tensor_map_encoder();
    if (!enc) return fail(BRK_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
    cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)(cols * esize)};
    cuuint32_t box[2] = {box_cols, box_rows};
    cuuint32_t estr[2] = {1u, 1u};
    CUresult r = enc(m, type, 2, const_cast<void *>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                     swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(BRK_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    return BRK_OK;
}

// fp16 cache rows [rows][head_dim], box = [box_rows][64] with the 128-byte swizzle that the
// kernels' shared-memory addressing assumes.
int make_cache_map(CUtensorMap *m, const __half *base, uint64_t rows, int head_dim, int box_rows) {
    return make_map(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, sizeof(__half), base, rows, (uint64_t)head_dim, 64u,
                    (uint32_t)box_rows, CU_TENSOR_MAP_SWIZZLE_128B);
}

// int8 code rows [rows][head_dim] bytes, box = [box_rows][min(head_dim, 128) B]: 128-byte swizzle,
// or the 64-byte one for head_dim 64 (the addressing of the decode kernel, decode.cu).
int make_code_map(CUtensorMap *m, const uint8_t *base, uint64_t rows, int head_dim, int box_rows) {
    const bool narrow = head_dim < 128;
    return make_map(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, base, rows, (uint64_t)head_dim, narrow ? 64u : 128u,
                    (uint32_t)box_rows, narrow ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B);
}

bool supported_head_dim(int d) { return d == 64 || d == 128 || d == 256; }

size_t kv_elems(const brk_kv_desc &d, int cap) {
    return (size_t)d.n_layers * d.batch * d.n_kv_heads * (size_t)cap * d.head_dim;
}

size_t kv_segments(const brk_kv_desc &d) { return (size_t)d.n_layers * d.batch * d.n_kv_heads; }

// Zeroes every buffer of the cache: fp16 rows, or int8 codes (byte 0x80 = code 0, the storage
// being biased by +128) and scales.
cudaError_t kv_zero(brk_kv *kv, cudaStream_t s) {
    const size_t elems = kv_elems(kv->desc, kv->cap);
    cudaError_t e = cudaSuccess;
    if (kv->q8()) {
        e = cudaMemsetAsync(kv->k8, 0x80, elems, s);
        if (e == cudaSuccess) e = cudaMemsetAsync(kv->v8, 0x80, elems, s);
        if (e == cudaSuccess)
            e = cudaMemsetAsync(kv->scales, 0, kv_segments(kv->desc) * 2 * kv->scale_pitch * sizeof(float), s);
    } else {
        e = cudaMemsetAsync(kv->k, 0, elems * sizeof(__half), s);
        if (e == cudaSuccess) e = cudaMemsetAsync(kv->v, 0, elems * sizeof(__half), s);
    }
    return e;
}

// Allocates zeroed buffers for capacity `cap` into kv (the previous pointers are overwritten, not
// freed).  On failure the buffers that were allocated stay in kv for kv_free.
cudaError_t kv_alloc(brk_kv *kv, int cap) {
    kv->k = kv->v = nullptr;
    kv->k8 = kv->v8 = nullptr;
    kv->scales = nullptr;
    const int saved_cap = kv->cap;
    kv->cap = cap;
    const size_t elems = kv_elems(kv->desc, cap);
    cudaError_t e;
    if (kv->q8()) {
        kv->scale_pitch = (cap + 3) / 4 * 4;
        e = cudaMalloc(&kv->k8, elems);
        if (e == cudaSuccess) e = cudaMalloc(&kv->v8, elems);
        if (e == cudaSuccess) e = cudaMalloc(&kv->scales, kv_segments(kv->desc) * 2 * kv->scale_pitch * sizeof(float));
    } else {
        e = cudaMalloc(&kv->k, elems * sizeof(__half));
        if (e == cudaSuccess) e = cudaMalloc(&kv->v, elems * sizeof(__half));
    }
    if (e == cudaSuccess) e = kv_zero(kv, 0);
    if (e == cudaSuccess) e = cudaStreamSynchronize(0);
    kv->cap = saved_cap;
    return e;
}

void kv_free(brk_kv *kv) {
    cudaFree(kv->k);
    cudaFree(kv->v);
    cudaFree(kv->k8);
    cudaFree(kv->v8);
    cudaFree(kv->scales);
    kv->k = kv->v = nullptr;
    kv->k8 = kv->v8 = nullptr;
    kv->scales = nullptr;
}

int kv_build_maps(brk_kv *kv) {
    const uint64_t rows = (uint64_t)kv->desc.n_layers * kv->desc.batch * kv->desc.n_kv_heads * kv->cap;
    int rc;
    if (kv->q8()) {
        const int sk = brk::decode_stage_keys(kv->desc.head_dim);
        if ((rc = make_code_map(&kv->tm_dec_k, kv->k8, rows, kv->desc.head_dim, sk))) return rc;
        if ((rc = make_code_map(&kv->tm_dec_v, kv->v8, rows, kv->desc.head_dim, sk))) return rc;
        // Scales [segment][K, V][pitch]: one box = both scale rows of a stage's keys.
        return make_map(&kv->tm_dec_s, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, sizeof(float), kv->scales,
                        kv_segments(kv->desc) * 2, (uint64_t)kv->scale_pitch, (uint32_t)sk, 2u,
                        CU_TENSOR_MAP_SWIZZLE_NONE);
    }
    if ((rc = make_cache_map(&kv->tm_dec_k, kv->k, rows, kv->desc.head_dim, brk::decode_stage_keys(kv->desc.head_dim))))
        return rc;
    if ((rc = make_cache_map(&kv->tm_dec_v, kv->v, rows, kv->desc.head_dim, brk::decode_stage_keys(kv->desc.head_dim))))
        return rc;
    if ((rc = make_cache_map(&kv->tm_pre_k, kv->k, rows, kv->desc.head_dim, brk::prefill_tile_keys()))) return rc;
    if ((rc = make_cache_map(&kv->tm_pre_v, kv->v, rows, kv->desc.head_dim, brk::prefill_tile_keys()))) return rc;
    return BRK_OK;
}

// Shape checks shared by every attention entry point.
int check_call(const brk_ctx *ctx, const brk_kv *kv, int layer, const brk_attn_params *p, int batch, int n_tokens,
               const int32_t *past_len) {
    if (!ctx || !kv || !p || !past_len) return fail(BRK_ERR_INVALID, "null handle or argument");
    if (kv->ctx != ctx) return fail(BRK_ERR_INVALID, "kv cache belongs to another context");
    if (layer < 0 || layer >= kv->desc.n_layers)
        return fail(BRK_ERR_INVALID, "layer %d outside [0, %d)", layer, kv->desc.n_layers);
    if (batch != kv->desc.batch) return fail(BRK_ERR_INVALID, "batch %d != cache batch %d", batch, kv->desc.batch);
    if (batch < 1 || batch > BRK_MAX_BATCH) return fail(BRK_ERR_INVALID, "batch %d outside [1, %d]", batch, BRK_MAX_BATCH);
    if (n_tokens < 1) return fail(BRK_ERR_INVALID, "n_tokens %d < 1", n_tokens);
    if (p->n_kv_heads != kv->desc.n_kv_heads || p->head_dim != kv->desc.head_dim)
        return fail(BRK_ERR_INVALID, "params (%d kv heads, dim %d) do not match the cache (%d, %d)", p->n_kv_heads,
                    p->head_dim, kv->desc.n_kv_heads, kv->desc.head_dim);
    if (p->n_heads < 1 || p->n_kv_heads < 1 || p->n_heads % p->n_kv_heads)
        return fail(BRK_ERR_INVALID, "n_heads %d is not a multiple of n_kv_heads %d", p->n_heads, p->n_kv_heads);
    if (!supported_head_dim(p->head_dim)) return fail(BRK_ERR_UNSUPPORTED, "head_dim %d (64, 128 or 256)", p->head_dim);
    if (p->kv_offset < 0) return fail(BRK_ERR_INVALID, "kv_offset %d < 0", p->kv_offset);
    for (int b = 0; b < batch; ++b)
        if (past_len[b] < p->kv_offset)
            return fail(BRK_ERR_INVALID, "past_len[%d] = %d is before the cache's first position %d", b, past_len[b],
                        p->kv_offset);
    return BRK_OK;
}

float effective_scale(const brk_attn_params *p) {
    return p->scale > 0.f ? p->scale : (float)(1.0 / std::sqrt((double)p->head_dim));
}

// Splits of the key range per (sequence, kv head, row tile); BRK_DECODE_SPLITS overrides.
//  - Grids of one wave or less: a CTA streams its range at a bounded rate (its ring holds a few
//    stages), so the grid needs about 1.5 CTAs per SM in flight to keep HBM busy, and every CTA
//    beyond that only adds fixed cost (ring ramp, partial, merge).  The fewest splits that reach
//    that many CTAs, within one wave.  Measured on B200 (Qwen3-4B shapes, head_dim 128, L 4096,
//    cluster merge): B 8 kernel 30.4 / 28.0 / 24.8 / 26.8 us at 2 / 3 / 4 / 6 splits; B 16 44.0 /
//    44.8 / 53.6 us at 2 / 3 / 4 splits.
//  - Larger grids: enough CTAs to fill the GPU's concurrent slots without leaving a mostly-empty
//    last wave, each CTA's fixed cost counted as four stages.
int choose_splits(const brk_ctx *ctx, int head_dim, bool q8, int units, int span) {
    const int tk = brk::decode_stage_keys(head_dim);
    const int max_split = std::max(1, std::min(64, (span + tk - 1) / tk));
    if (const char *env = getenv("BRK_DECODE_SPLITS")) {
        int n = atoi(env);
        if (n >= 1) return std::min(n, max_split);
    }
    const long long slots = (long long)ctx->num_sms * brk::decode_ctas_per_sm(head_dim, q8);
    // No split shorter than four ring stages: a shorter one does not amortise its CTA's fixed cost
    // (pipeline ramp, partial write, its share of the merge).  Measured on B200 at B 1, L 4096,
    // head_dim 128: 16 splits of 256 keys ran 1.51 TB/s, 32 of 128 keys 1.40, 64 of 64 keys 0.93.
    const int max_auto = std::max(1, std::min(max_split, span / (4 * tk)));
    // int8 caches are issue-bound (a CTA converts every code), so their CTAs stream slowly and the
    // multi-wave model below suits them at every size; head_dim 256 splits the head dim over warp
    // pairs and streams slower per CTA than 64 / 128 (Gemma-2 B 32: 3 splits 6554 GB/s, 2 splits
    // 6428 GB/s).
    if (units < slots && !q8) {
        const long long target = head_dim > 128 ? (5LL * ctx->num_sms + 1) / 2 : (3LL * ctx->num_sms + 1) / 2;
        int n = (int)std::min<long long>(max_auto, (target + units - 1) / units);
        while (n > 1 && (long long)units * n > slots) --n;
        return std::max(1, n);
    }
    double best = 1e30;
    int best_n = 1;
    for (int n = 1; n <= max_auto; ++n) {
        const long long ctas = (long long)units * n;
        const long long waves = (ctas + slots - 1) / slots;
        const int keys = ((span + n - 1) / n + tk - 1) / tk * tk;
        // + the fixed cost of a CTA (pipeline ramp, merge epilogue) in key units: measured on B200
        // it is worth about four stages, so short CTAs in many waves lose to fewer, longer ones.
        double cost = (double)waves * (keys + 4 * tk);
        if (n > 1) cost += 4 * tk;  // the split merge
        if (cost < best - 1e-9) {
            best = cost;
            best_n = n;
        }
    }
    return best_n;
}

// Split plan of a decode call: the longest attended range over the batch (rows beyond the cache
// capacity are an error unless clamp_rows), the split count and the keys per split (a multiple
// of the ring's stage keys).
int decode_split_plan(const brk_ctx *ctx, const brk_kv *kv, const brk_attn_params *p, int batch, int n_tokens,
                      const int32_t *past_len, bool clamp_rows, int *nsplit_out, int *keys_per_split_out) {
    const int D = p->head_dim;
    const int window = p->window > 0 ? p->window : 0;
    int span = 1;
    for (int b = 0; b < batch; ++b) {
        int hi = past_len[b] + n_tokens - p->kv_offset;
        if (hi > kv->cap) {
            if (!clamp_rows)
                return fail(BRK_ERR_CAPACITY, "sequence %d needs %d cache rows, capacity is %d (grow the cache)", b, hi,
                            kv->cap);
            hi = kv->cap;
        }
        int lo = window > 0 ? std::max(0, past_len[b] - window + 1 - p->kv_offset) : 0;
        span = std::max(span, hi - lo);
    }
    const int G = p->n_heads / p->n_kv_heads;
    const int rt = brk::decode_rows_per_tile();
    const int units = batch * p->n_kv_heads * ((n_tokens * G + rt - 1) / rt);
    int nsplit = choose_splits(ctx, D, kv->q8(), units, span);
    const int tk = brk::decode_stage_keys(D);
    const int kps = ((span + nsplit - 1) / nsplit + tk - 1) / tk * tk;
    *keys_per_split_out = kps;
    *nsplit_out = (span + kps - 1) / kps;
    return BRK_OK;
}

// The decode path (final output or a partial), splitting the key range over CTAs.
// Static split-KV scratch layout: arrival counters (cleared by each call), then the partials.
size_t counters_bytes(int units) { return ((size_t)units * sizeof(int) + 255) / 256 * 256; }

// Split-KV arrival counters for at least n tiles (zeroed; a larger buffer replaces a smaller one
// after the device is idle, so that no queued kernel still counts in the old one).
constexpr size_t kInitialCounters = 1u << 16;
int ensure_counters(brk_ctx *ctx, size_t n) {
    if (n <= ctx->counters_n) return BRK_OK;
    const size_t want = std::max(n, 2 * ctx->counters_n);
    DeviceGuard g(ctx->device);
    BRK_CUDA(cudaDeviceSynchronize());
    cudaFree(ctx->counters);
    ctx->counters = nullptr;
    ctx->counters_n = 0;
    BRK_CUDA(cudaMalloc(&ctx->counters, want * sizeof(int)));
    BRK_CUDA(cudaMemset(ctx->counters, 0, want * sizeof(int)));
    ctx->counters_n = want;
    return BRK_OK;
}

// fixed_ws / fixed_bytes: when set, the split-KV scratch goes there and nothing is allocated
// (brk_attn_decode_static); otherwise the context workspace is used and grown on demand.
// pdl: the decode kernel is a programmatic dependent of the append launched just before it.
// The append fused into the decode launch (brk_attn_step with one token): raw projections in,
// rotated q out.
struct FusedAppend {
    const float *q_in, *k_in, *v_in;
    float *q_work;
};

int run_decode(brk_ctx *ctx, const brk_kv *kv, int layer, const brk_attn_params *p, int batch, int n_tokens,
               const int32_t *past_len, const float *q, float *out, float *part_ml, float *part_o, bool clamp_rows,
               cudaStream_t stream, void *fixed_ws = nullptr, size_t fixed_bytes = 0, bool pdl = false,
               brk_peer *push = nullptr, uint32_t epoch = 0, const FusedAppend *fused = nullptr) {
    const int D = p->head_dim, G = p->n_heads / p->n_kv_heads;
    brk::DecodeArgs a;
    memset(&a, 0, sizeof(a));
    a.q = q;
    a.err = ctx->d_err;
    a.B = batch;
    a.T = n_tokens;
    a.Hq = p->n_heads;
    a.Hkv = p->n_kv_heads;
    a.G = G;
    a.layer = layer;
    a.cap = kv->cap;
    const int rt = brk::decode_rows_per_tile();
    a.mtiles = (n_tokens * G + rt - 1) / rt;
    a.kv_offset = p->kv_offset;
    a.window = p->window > 0 ? p->window : 0;
    a.scale = effective_scale(p);
    a.scale_log2 = a.scale * 1.4426950408889634f;
    a.softcap = p->softcap > 0.f ? p->softcap : 0.f;
    if (a.softcap > 0.f) {
        const double log2e = 1.4426950408889634;
        a.cap_k1 = (float)(2.0 * (double)a.scale * log2e / (double)a.softcap);
        a.cap_k2 = (float)((double)a.softcap * log2e);
    }
    for (int b = 0; b < batch; ++b) a.past_len[b] = past_len[b];
    int nsplit = 1;
    int rc = decode_split_plan(ctx, kv, p, batch, n_tokens, past_len, clamp_rows, &nsplit, &a.keys_per_split);
    if (rc) return rc;
    const int units = batch * p->n_kv_heads * a.mtiles;
    a.nsplit = nsplit;
    const int rows = batch * n_tokens * p->n_heads;

    // Small grids (every CTA resident at once) merge their splits through a thread-block cluster
    // instead of global partials and a last-arriver merge; the static entry point keeps the
    // workspace merge (its scratch array is what it is for), and so do push launches.
    const bool cluster = nsplit > 1 && nsplit <= brk::kMaxClusterSplits && !fixed_ws && !push && !getenv("BRK_DECODE_NO_CLUSTER") &&
                         units <= brk::decode_max_clusters(D, kv->q8(), nsplit);
    if (nsplit == 1) {
        a.out = out;  // final output, or (out == nullptr) the caller's partial buffer directly
        a.part_ml = part_ml;
        a.part_o = part_o;
    } else if (cluster) {
        a.cluster = 1;
        a.out = out;
        a.res_ml = part_ml;
        a.res_o = part_o;
    } else {
        // (m, l) pairs, then the outputs from a 16-byte boundary (the merge reads them as float4).
        const size_t ml_floats = ((size_t)nsplit * rows * 2 + 3) / 4 * 4;
        const size_t part_bytes = (ml_floats + (size_t)nsplit * rows * D) * sizeof(float);
        char *ws;
        if (fixed_ws) {
            // The static array holds the counters too, cleared by every call.
            const size_t cbytes = counters_bytes(units);
            const size_t need = cbytes + part_bytes;
            if (need > fixed_bytes)
                return fail(BRK_ERR_CAPACITY,
                            "%d-way split-KV partials of %d rows need %zu bytes of scratch; the library's static "
                            "scratch holds %zu (use brk_attn_decode, or fewer sequences per call)",
                            nsplit, rows, need, fixed_bytes);
            ws = static_cast<char *>(fixed_ws);
            // The counters must start at zero; the array keeps whatever the last call left.
            cudaError_t e = cudaMemsetAsync(ws, 0, cbytes, stream);
            if (e != cudaSuccess) return cuda_fail(e, "clearing the static split counters");
            a.counters = reinterpret_cast<int *>(ws);
            ws += cbytes;
        } else {
            if (part_bytes > ctx->ws_bytes) {
                rc = brk_ctx_reserve(ctx, part_bytes);
                if (rc) return rc;
            }
            rc = ensure_counters(ctx, (size_t)units);
            if (rc) return rc;
            ws = static_cast<char *>(ctx->ws);
            a.counters = ctx->counters;
        }
        a.part_ml = reinterpret_cast<float *>(ws);
        a.part_o = a.part_ml + ml_floats;
        a.out = out;
        a.res_ml = part_ml;
        a.res_o = part_o;
    }
    if (fused) {
        a.fuse = 1;
        a.q = fused->q_work;
        a.q_rot = fused->q_work;
        a.q_in = fused->q_in;
        a.k_in = fused->k_in;
        a.v_in = fused->v_in;
        a.kc = kv->k;
        a.vc = kv->v;
        a.kc8 = kv->k8;
        a.vc8 = kv->v8;
        a.scales = kv->scales;
        a.scale_pitch = kv->scale_pitch;
        a.rope = p->rope ? p->rope->table : nullptr;
        a.rope32 = p->rope ? p->rope->table32 : nullptr;
        a.q_norm = p->q_norm;
        a.k_norm = p->k_norm;
        a.eps = p->eps;
        a.one_plus = p->norm_one_plus ? 1 : 0;
    }
    if (push) {
        // This rank's block (parity epoch & 1, source `rank`) of every rank's exchange area.
        const int par = (int)(epoch & 1u);
        a.push_world = push->world;
        a.epoch = epoch;
        a.push_tiles = units;
        a.push_done = push->done;
        for (int r = 0; r < push->world; ++r) {
            float *blk = static_cast<float *>(push->peers[r]) + ((size_t)par * push->world + push->rank) * push->stride;
            a.push_ml[r] = blk;
            a.push_o[r] = blk + (size_t)rows * 2;
            a.push_flag[r] = reinterpret_cast<unsigned *>(static_cast<char *>(push->peers[r]) + push->flags_offset) +
                             par * push->world + push->rank;
        }
    }
    cudaError_t e = brk::launch_decode(kv->q8(), D, kv->tm_dec_k, kv->tm_dec_v, kv->q8() ? kv->tm_dec_s : kv->tm_dec_k,
                                       a, nsplit, p->n_kv_heads * a.mtiles, batch, stream, pdl);
    if (e != cudaSuccess) return cuda_fail(e, "decode kernel launch");
    ++ctx->launches;
    return BRK_OK;
}

}  // namespace

namespace {

// Split-KV partials of brk_attn_decode_static.  A file-scope device array: every GPU that loads
// this library holds BRK_DECODE_STATIC_SCRATCH_BYTES of it until the process exits, and all
// calls on one GPU share it.
static __device__ __align__(256) unsigned char g_decode_static_scratch[BRK_DECODE_STATIC_SCRATCH_BYTES];

// Device address of the array on the current device.  In host code the symbol only names a
// host-side stand-in, so the real address is looked up once per device (with that device
// current) and cached.
int static_scratch_address(void **out) {
    static std::mutex mu;
    static void *addr[64] = {};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
    if (dev < 0 || dev >= 64) return fail(BRK_ERR_UNSUPPORTED, "device %d: static scratch supports devices 0..63", dev);
    std::lock_guard<std::mutex> lock(mu);
    if (!addr[dev]) {
        void *p = nullptr;
        e = cudaGetSymbolAddress(&p, g_decode_static_scratch);
        if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(static decode scratch)");
        addr[dev] = p;
    }
    *out = addr[dev];
    return BRK_OK;
}

}  // namespace

extern "C" {

const char *brk_last_error(void) { return g_last_error.c_str(); }

int brk_abi_version(void) { return BRK_ABI_VERSION; }

int brk_ctx_create(int device, brk_ctx **out) {
    if (!out) return fail(BRK_ERR_INVALID, "out is null");
    *out = nullptr;
    int n = 0;
    BRK_CUDA(cudaGetDeviceCount(&n));
    if (device < 0 || device >= n) return fail(BRK_ERR_INVALID, "device %d outside [0, %d)", device, n);
    DeviceGuard g(device);
    cudaDeviceProp prop;
    BRK_CUDA(cudaGetDeviceProperties(&prop, device));
    if (prop.major != 10) return fail(BRK_ERR_UNSUPPORTED, "device %d is sm_%d%d; this build targets sm_100a", device, prop.major, prop.minor);
    brk_ctx *c = new brk_ctx();
    c->device = device;
    c->num_sms = prop.multiProcessorCount;
    cudaError_t e = cudaMalloc(&c->d_err, sizeof(int));
    if (e == cudaSuccess) e = cudaMemset(c->d_err, 0, sizeof(int));
    if (e != cudaSuccess) {
        cudaFree(c->d_err);
        delete c;
        return cuda_fail(e, "context error word");
    }
    // Everything brk_attn_decode_static needs on this device is taken here, so that its calls
    // allocate nothing: the decode kernels are loaded (lazy module loading would load them, and
    // take their device memory, at the first launch) and the static scratch array's module is
    // loaded (its BRK_DECODE_STATIC_SCRATCH_BYTES are taken then) with its address cached.
    e = brk::preload_decode_kernels();
    if (e != cudaSuccess) {
        cudaFree(c->d_err);
        delete c;
        return cuda_fail(e, "loading the decode kernels");
    }
    void *scratch = nullptr;
    int rc = static_scratch_address(&scratch);
    if (rc == BRK_OK) rc = ensure_counters(c, kInitialCounters);
    if (rc) {
        cudaFree(c->counters);
        cudaFree(c->d_err);
        delete c;
        return rc;
    }
    *out = c;
    return BRK_OK;
}

int brk_ctx_destroy(brk_ctx *ctx) {
    if (!ctx) return BRK_OK;
    DeviceGuard g(ctx->device);
    cudaDeviceSynchronize();
    cudaFree(ctx->d_err);
    cudaFree(ctx->counters);
    cudaFree(ctx->ws);
    cudaFree(ctx->stage);
    cudaFree(ctx->act);
    delete ctx;
    return BRK_OK;
}

int brk_ctx_check(brk_ctx *ctx, void *stream) {
    if (!ctx) return fail(BRK_ERR_INVALID, "null context");
    DeviceGuard g(ctx->device);
    BRK_CUDA(cudaStreamSynchronize(static_cast<cudaStream_t>(stream)));
    int err = 0;
    BRK_CUDA(cudaMemcpy(&err, ctx->d_err, sizeof(int), cudaMemcpyDeviceToHost));
    if (err) {
        BRK_CUDA(cudaMemset(ctx->d_err, 0, sizeof(int)));
        // A kernel that gave up may have left split counters mid-count: start them from zero.
        if (ctx->counters) BRK_CUDA(cudaMemset(ctx->counters, 0, ctx->counters_n * sizeof(int)));
        return fail(BRK_ERR_DEVICE, "a kernel gave up on a bounded wait (code %d)", err);
    }
    return BRK_OK;
}

uint64_t brk_ctx_launches(const brk_ctx *ctx) { return ctx ? ctx->launches : 0; }

int brk_ctx_reserve(brk_ctx *ctx, size_t bytes) {
    if (!ctx) return fail(BRK_ERR_INVALID, "null context");
    if (bytes <= ctx->ws_bytes) return BRK_OK;
    DeviceGuard g(ctx->device);
    BRK_CUDA(cudaDeviceSynchronize());  // queued kernels may still read the old workspace
    cudaFree(ctx->ws);
    ctx->ws = nullptr;
    ctx->ws_bytes = 0;
    BRK_CUDA(cudaMalloc(&ctx->ws, bytes));
    ctx->ws_bytes = bytes;
    return BRK_OK;
}

namespace {
int ensure_stage(brk_ctx *ctx, size_t bytes);
}  // namespace

int brk_ctx_reserve_stage(brk_ctx *ctx, size_t bytes) {
    if (!ctx) return fail(BRK_ERR_INVALID, "null context");
    DeviceGuard g(ctx->device);
    return ensure_stage(ctx, bytes);
}

int brk_rope_create(brk_ctx *ctx, int head_dim, double base, const float *ff_host, int max_positions,
                    brk_rope **out) {
    if (!ctx || !out) return fail(BRK_ERR_INVALID, "null argument");
    *out = nullptr;
    if (head_dim < 2 || head_dim % 2) return fail(BRK_ERR_INVALID, "head_dim %d must be even", head_dim);
    if (max_positions < 1) return fail(BRK_ERR_INVALID, "max_positions %d < 1", max_positions);
    const int half = head_dim / 2;
    // ropeCpu / ropeFactorsCpu (kernels.ts:3428-3460): freq = pos / (base ** (2i/D) [* ff[i]]).
    std::vector<double> denom(half);
    for (int i = 0; i < half; ++i) {
        double dn = std::pow(base, (2.0 * i) / (double)head_dim);
        if (ff_host) dn = dn * (double)ff_host[i];
        denom[i] = dn;
    }
    std::vector<double2> table((size_t)max_positions * half);
    for (int pos = 0; pos < max_positions; ++pos)
        for (int i = 0; i < half; ++i) {
            const double freq = (double)pos / denom[i];
            table[(size_t)pos * half + i] = make_double2(std::cos(freq), std::sin(freq));
        }
    DeviceGuard g(ctx->device);
    brk_rope *r = new brk_rope();
    r->ctx = ctx;
    r->head_dim = head_dim;
    r->max_pos = max_positions;
    std::vector<float2> table32(table.size());
    for (size_t i = 0; i < table.size(); ++i) table32[i] = make_float2((float)table[i].x, (float)table[i].y);
    cudaError_t e = cudaMalloc(&r->table, table.size() * sizeof(double2));
    if (e == cudaSuccess) e = cudaMemcpy(r->table, table.data(), table.size() * sizeof(double2), cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMalloc(&r->table32, table32.size() * sizeof(float2));
    if (e == cudaSuccess)
        e = cudaMemcpy(r->table32, table32.data(), table32.size() * sizeof(float2), cudaMemcpyHostToDevice);
    if (e != cudaSuccess) {
        cudaFree(r->table);
        cudaFree(r->table32);
        delete r;
        return cuda_fail(e, "rope table");
    }
    *out = r;
    return BRK_OK;
}

int brk_rope_destroy(brk_rope *rope) {
    if (!rope) return BRK_OK;
    DeviceGuard g(rope->ctx->device);
    cudaFree(rope->table);
    cudaFree(rope->table32);
    delete rope;
    return BRK_OK;
}

int brk_rope_max_positions(const brk_rope *rope) { return rope ? rope->max_pos : 0; }

int brk_llama3_rope_factors(int head_dim, double base, double factor, double low_freq_factor,
                            double high_freq_factor, int original_context, float *ff_out) {
    if (!ff_out || head_dim < 2 || head_dim % 2 || factor <= 0 || high_freq_factor <= low_freq_factor ||
        original_context <= 0)
        return fail(BRK_ERR_INVALID, "invalid llama3 rope scaling arguments");
    // Published llama3 scaling: keep high frequencies, divide low frequencies by `factor`, and
    // interpolate in between on orig_ctx / wavelength.  Stored as divisors of the frequency.
    const double pi = 3.14159265358979323846;
    const double low_wavelen = original_context / low_freq_factor;
    const double high_wavelen = original_context / high_freq_factor;
    for (int i = 0; i < head_dim / 2; ++i) {
        const double freq = 1.0 / std::pow(base, (2.0 * i) / head_dim);
        const double wavelen = 2.0 * pi / freq;
        double scaled;
        if (wavelen < high_wavelen) {
            scaled = freq;
        } else if (wavelen > low_wavelen) {
            scaled = freq / factor;
        } else {
            const double smooth = (original_context / wavelen - low_freq_factor) / (high_freq_factor - low_freq_factor);
            scaled = (1.0 - smooth) * freq / factor + smooth * freq;
        }
        ff_out[i] = (float)(freq / scaled);
    }
    return BRK_OK;
}

int brk_kv_create(brk_ctx *ctx, const brk_kv_desc *desc, brk_kv **out) {
    if (!ctx || !desc || !out) return fail(BRK_ERR_INVALID, "null argument");
    *out = nullptr;
    const brk_kv_desc &d = *desc;
    if (d.dtype != BRK_KV_F16 && d.dtype != BRK_KV_I8)
        return fail(BRK_ERR_UNSUPPORTED, "kv dtype %d (BRK_KV_F16 or BRK_KV_I8)", d.dtype);
    if (!supported_head_dim(d.head_dim)) return fail(BRK_ERR_UNSUPPORTED, "head_dim %d (64, 128 or 256)", d.head_dim);
    if (d.n_layers < 1 || d.batch < 1 || d.batch > BRK_MAX_BATCH || d.n_kv_heads < 1 || d.capacity < 1)
        return fail(BRK_ERR_INVALID, "invalid kv descriptor");
    if ((long long)d.n_layers * d.batch * d.n_kv_heads * (long long)d.capacity >= (1ll << 31))
        return fail(BRK_ERR_CAPACITY, "layers * batch * kv_heads * capacity must stay below 2^31 rows");
    DeviceGuard g(ctx->device);
    brk_kv *kv = new brk_kv();
    kv->ctx = ctx;
    kv->desc = d;
    kv->cap = d.capacity;
    cudaError_t e = kv_alloc(kv, kv->cap);
    if (e != cudaSuccess) {
        kv_free(kv);
        delete kv;
        return cuda_fail(e, "kv cache allocation");
    }
    int rc = kv_build_maps(kv);
    if (rc) {
        kv_free(kv);
        delete kv;
        return rc;
    }
    *out = kv;
    return BRK_OK;
}

int brk_kv_destroy(brk_kv *kv) {
    if (!kv) return BRK_OK;
    DeviceGuard g(kv->ctx->device);
    cudaDeviceSynchronize();
    kv_free(kv);
    delete kv;
    return BRK_OK;
}

int brk_kv_capacity(const brk_kv *kv) { return kv ? kv->cap : 0; }

int brk_kv_grow(brk_kv *kv, int rows, void *stream) {
    if (!kv) return fail(BRK_ERR_INVALID, "null kv");
    if (rows <= kv->cap) return BRK_OK;
    const int cap = std::max(rows, std::max(kv->cap + 1024, 1024));  // ensureKv, kernels.ts:1785
    const brk_kv_desc &d = kv->desc;
    if ((long long)d.n_layers * d.batch * d.n_kv_heads * (long long)cap >= (1ll << 31))
        return fail(BRK_ERR_CAPACITY, "growing to %d rows exceeds 2^31 cache rows", cap);
    DeviceGuard g(kv->ctx->device);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    brk_kv old = *kv;  // the current buffers, copied from below
    // On failure: drop the new buffers and keep the cache as it was.
    auto restore = [&](cudaError_t err, const char *what) {
        kv_free(kv);
        kv->k = old.k, kv->v = old.v, kv->k8 = old.k8, kv->v8 = old.v8, kv->scales = old.scales;
        kv->scale_pitch = old.scale_pitch;
        return cuda_fail(err, what);
    };
    cudaError_t e = kv_alloc(kv, cap);  // zeroed buffers of the new capacity
    if (e != cudaSuccess) return restore(e, "kv cache growth");
    const size_t segs = kv_segments(d);
    const size_t esz = kv->q8() ? 1 : sizeof(__half);
    const size_t old_pitch = (size_t)old.cap * d.head_dim * esz;
    const size_t new_pitch = (size_t)cap * d.head_dim * esz;
    void *dk = kv->q8() ? (void *)kv->k8 : (void *)kv->k, *dv = kv->q8() ? (void *)kv->v8 : (void *)kv->v;
    const void *sk = kv->q8() ? (const void *)old.k8 : (const void *)old.k;
    const void *sv = kv->q8() ? (const void *)old.v8 : (const void *)old.v;
    e = cudaMemcpy2DAsync(dk, new_pitch, sk, old_pitch, old_pitch, segs, cudaMemcpyDeviceToDevice, s);
    if (e == cudaSuccess) e = cudaMemcpy2DAsync(dv, new_pitch, sv, old_pitch, old_pitch, segs, cudaMemcpyDeviceToDevice, s);
    if (e == cudaSuccess && kv->q8())
        e = cudaMemcpy2DAsync(kv->scales, (size_t)kv->scale_pitch * sizeof(float), old.scales,
                              (size_t)old.scale_pitch * sizeof(float), (size_t)old.cap * sizeof(float), segs * 2,
                              cudaMemcpyDeviceToDevice, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) return restore(e, "kv cache growth copy");
    kv_free(&old);
    kv->cap = cap;
    return kv_build_maps(kv);
}

int brk_kv_reset(brk_kv *kv, int seq, void *stream) {
    if (!kv) return fail(BRK_ERR_INVALID, "null kv");
    const brk_kv_desc &d = kv->desc;
    if (seq < -1 || seq >= d.batch) return fail(BRK_ERR_INVALID, "sequence %d outside [-1, %d)", seq, d.batch);
    DeviceGuard g(kv->ctx->device);
    const cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (seq < 0) {
        cudaError_t e = kv_zero(kv, s);
        return e == cudaSuccess ? BRK_OK : cuda_fail(e, "kv reset");
    }
    // One sequence: for every layer its n_kv_heads segments are contiguous, [layer][seq][head]
    // -> a 2-D memset with one row per layer, pitched by the batch's segments.
    const size_t esz = kv->q8() ? 1 : sizeof(__half);
    const size_t width = (size_t)d.n_kv_heads * kv->cap * d.head_dim * esz;
    const size_t pitch = width * d.batch;
    const size_t off = width * seq;
    cudaError_t e;
    if (kv->q8()) {
        e = cudaMemset2DAsync(kv->k8 + off, pitch, 0x80, width, d.n_layers, s);
        if (e == cudaSuccess) e = cudaMemset2DAsync(kv->v8 + off, pitch, 0x80, width, d.n_layers, s);
        const size_t swidth = (size_t)d.n_kv_heads * 2 * kv->scale_pitch * sizeof(float);
        if (e == cudaSuccess)
            e = cudaMemset2DAsync(reinterpret_cast<char *>(kv->scales) + swidth * seq, swidth * d.batch, 0, swidth,
                                  d.n_layers, s);
    } else {
        e = cudaMemset2DAsync(reinterpret_cast<char *>(kv->k) + off, pitch, 0, width, d.n_layers, s);
        if (e == cudaSuccess) e = cudaMemset2DAsync(reinterpret_cast<char *>(kv->v) + off, pitch, 0, width, d.n_layers, s);
    }
    return e == cudaSuccess ? BRK_OK : cuda_fail(e, "kv reset of one sequence");
}

static int check_rows(const brk_kv *kv, int layer, int seq, int row0, int n_rows) {
    if (!kv) return fail(BRK_ERR_INVALID, "null kv");
    if (layer < 0 || layer >= kv->desc.n_layers || seq < 0 || seq >= kv->desc.batch)
        return fail(BRK_ERR_INVALID, "layer %d / sequence %d out of range", layer, seq);
    if (row0 < 0 || n_rows < 0 || (long long)row0 + n_rows > kv->cap)
        return fail(BRK_ERR_CAPACITY, "rows [%d, %d) outside the capacity %d", row0, row0 + n_rows, kv->cap);
    return BRK_OK;
}

int brk_kv_write_rows(brk_kv *kv, int layer, int seq, int row0, int n_rows, const float *k, const float *v,
                      void *stream) {
    int rc = check_rows(kv, layer, seq, row0, n_rows);
    if (rc) return rc;
    DeviceGuard g(kv->ctx->device);
    const brk_kv_desc &d = kv->desc;
    const size_t seg0 = (size_t)(layer * d.batch + seq) * d.n_kv_heads;
    const size_t off = (seg0 * kv->cap + row0) * d.head_dim;
    cudaError_t e;
    if (kv->q8())
        e = brk::launch_kv_write_q8(kv->k8 + off, kv->v8 + off, kv->scales + seg0 * 2 * kv->scale_pitch + row0, k, v,
                                    n_rows, d.n_kv_heads, d.head_dim, kv->cap, kv->scale_pitch,
                                    static_cast<cudaStream_t>(stream));
    else
        e = brk::launch_kv_write_rows(kv->k + off, kv->v + off, k, v, n_rows, d.n_kv_heads, d.head_dim, kv->cap,
                                      static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? BRK_OK : cuda_fail(e, "kv write");
}

int brk_kv_read_rows(const brk_kv *kv, int layer, int seq, int row0, int n_rows, uint16_t *k_out, uint16_t *v_out,
                     void *stream) {
    int rc = check_rows(kv, layer, seq, row0, n_rows);
    if (rc) return rc;
    if (kv->q8()) return fail(BRK_ERR_UNSUPPORTED, "int8 cache: read codes and scales with brk_kv_read_codes");
    DeviceGuard g(kv->ctx->device);
    const brk_kv_desc &d = kv->desc;
    const size_t off = ((size_t)(layer * d.batch + seq) * d.n_kv_heads * kv->cap + row0) * d.head_dim;
    cudaError_t e = brk::launch_kv_read_rows(kv->k + off, kv->v + off, k_out, v_out, n_rows, d.n_kv_heads, d.head_dim,
                                             kv->cap, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? BRK_OK : cuda_fail(e, "kv read");
}

int brk_kv_write_codes(brk_kv *kv, int layer, int seq, int row0, int n_rows, const int8_t *k_codes,
                       const float *k_scales, const int8_t *v_codes, const float *v_scales, void *stream) {
    int rc = check_rows(kv, layer, seq, row0, n_rows);
    if (rc) return rc;
    if (!kv->q8()) return fail(BRK_ERR_UNSUPPORTED, "brk_kv_write_codes needs an int8 cache");
    if (!k_codes != !k_scales || !v_codes != !v_scales) return fail(BRK_ERR_INVALID, "codes and scales go together");
    DeviceGuard g(kv->ctx->device);
    const brk_kv_desc &d = kv->desc;
    const size_t seg0 = (size_t)(layer * d.batch + seq) * d.n_kv_heads;
    const size_t off = (seg0 * kv->cap + row0) * d.head_dim;
    cudaError_t e = brk::launch_kv_store_codes(kv->k8 + off, kv->v8 + off, kv->scales + seg0 * 2 * kv->scale_pitch + row0,
                                               k_codes, k_scales, v_codes, v_scales, n_rows, d.n_kv_heads, d.head_dim,
                                               kv->cap, kv->scale_pitch, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? BRK_OK : cuda_fail(e, "kv code store");
}

int brk_kv_read_codes(const brk_kv *kv, int layer, int seq, int row0, int n_rows, int8_t *k_codes, float *k_scales,
                      int8_t *v_codes, float *v_scales, void *stream) {
    int rc = check_rows(kv, layer, seq, row0, n_rows);
    if (rc) return rc;
    if (!kv->q8()) return fail(BRK_ERR_UNSUPPORTED, "brk_kv_read_codes needs an int8 cache");
    DeviceGuard g(kv->ctx->device);
    const brk_kv_desc &d = kv->desc;
    const size_t seg0 = (size_t)(layer * d.batch + seq) * d.n_kv_heads;
    const size_t off = (seg0 * kv->cap + row0) * d.head_dim;
    cudaError_t e = brk::launch_kv_read_q8(kv->k8 + off, kv->v8 + off, kv->scales + seg0 * 2 * kv->scale_pitch + row0,
                                           k_codes, k_scales, v_codes, v_scales, n_rows, d.n_kv_heads, d.head_dim,
                                           kv->cap, kv->scale_pitch, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? BRK_OK : cuda_fail(e, "kv code read");
}

namespace {
int append_impl(brk_ctx *ctx, brk_kv *kv, int layer, const brk_attn_params *p, int batch, int n_tokens,
                const int32_t *past_len, const float *q_in, const float *k_in, const float *v_in, float *q_out,
                void *stream, bool pdl, __half *q16 = nullptr) {
    if ((q_in != nullptr) != (q_out != nullptr || q16 != nullptr))
        return fail(BRK_ERR_INVALID, "q_in and q_out go together");
    if ((k_in == nullptr) != (v_in == nullptr)) return fail(BRK_ERR_INVALID, "k_in and v_in go together");
    if (kv) {
        int rc = check_call(ctx, kv, layer, p, batch, n_tokens, past_len);
        if (rc) return rc;
    } else {
        // q-only prologue (norm + rotation of q, no cache): any even head_dim up to 1024.
        if (!ctx || !p || !past_len) return fail(BRK_ERR_INVALID, "null handle or argument");
        if (k_in) return fail(BRK_ERR_INVALID, "k_in / v_in need a kv cache");
        if (p->head_dim < 2 || p->head_dim % 2 || p->head_dim > 1024 || p->n_heads < 1)
            return fail(BRK_ERR_INVALID, "q-only append needs an even head_dim <= 1024 and n_heads >= 1");
        if (batch < 1 || batch > BRK_MAX_BATCH || n_tokens < 1)
            return fail(BRK_ERR_INVALID, "batch %d / n_tokens %d out of range", batch, n_tokens);
        for (int b = 0; b < batch; ++b)
            if (past_len[b] < 0) return fail(BRK_ERR_INVALID, "past_len[%d] < 0", b);
    }
    if (p->rope && (p->rope->head_dim != p->head_dim || p->rope->ctx != ctx))
        return fail(BRK_ERR_INVALID, "rope table head_dim %d != %d", p->rope->head_dim, p->head_dim);
    brk::AppendArgs a;
    memset(&a, 0, sizeof(a));
    if ((long long)batch * n_tokens * (p->n_heads + 2LL * p->n_kv_heads) >= (1LL << 31))
        return fail(BRK_ERR_INVALID, "batch * n_tokens * (n_heads + 2 n_kv_heads) must stay below 2^31 rows");
    for (int b = 0; b < batch; ++b) {
        const int last = past_len[b] + n_tokens;
        if (p->rope && last > p->rope->max_pos)
            return fail(BRK_ERR_CAPACITY, "position %d beyond the rope table (%d positions)", last - 1, p->rope->max_pos);
        if (k_in && last - p->kv_offset > kv->cap)
            return fail(BRK_ERR_CAPACITY, "sequence %d appends up to row %d, capacity is %d (grow the cache)", b,
                        last - p->kv_offset, kv->cap);
        a.past_len[b] = past_len[b];
    }
    DeviceGuard g(ctx->device);
    a.q_in = q_in;
    a.k_in = k_in;
    a.v_in = v_in;
    a.q_out = q_out;
    a.q16 = q16;
    a.rope32 = q16 && p->rope ? p->rope->table32 : nullptr;
    a.kc = kv ? kv->k : nullptr;
    a.vc = kv ? kv->v : nullptr;
    a.kc8 = kv ? kv->k8 : nullptr;
    a.vc8 = kv ? kv->v8 : nullptr;
    a.scales = kv ? kv->scales : nullptr;
    a.scale_pitch = kv ? kv->scale_pitch : 0;
    a.rope = p->rope ? p->rope->table : nullptr;
    a.rope_max = p->rope ? p->rope->max_pos : 0;
    a.q_norm = p->q_norm;
    a.k_norm = p->k_norm;
    a.eps = p->eps;
    a.one_plus = p->norm_one_plus ? 1 : 0;
    a.B = batch;
    a.T = n_tokens;
    a.Hq = p->n_heads;
    a.Hkv = kv ? p->n_kv_heads : 0;
    a.D = p->head_dim;
    a.layer = layer;
    a.cap = kv ? kv->cap : 0;
    a.kv_offset = p->kv_offset;
    cudaError_t e = brk::launch_append(a, static_cast<cudaStream_t>(stream), pdl);
    if (e != cudaSuccess) return cuda_fail(e, "append kernel launch");
    ++ctx->launches;
    return BRK_OK;
}
}  // namespace

int brk_attn_append(brk_ctx *ctx, brk_kv *kv, int layer, const brk_attn_params *p, int batch, int n_tokens,
                    const int32_t *past_len, const float *q_in, const float *k_in, const float *v_in, float *q_out,
                    void *stream) {
    return append_impl(ctx, kv, layer, p, batch, n_tokens, past_len, q_in, k_in, v_in, q_out, stream, false);
}

int brk_attn_step(brk_ctx *ctx, brk_kv *kv, int layer, const brk_attn_params *p, int batch, int n_tokens,
                  const int32_t *past_len, const float *q_in, const float *k_in, const float *v_in, float *q_work,
                  float *out, void *stream) {
    if (!q_in || !k_in || !v_in || !q_work || !out) return fail(BRK_ERR_INVALID, "null tensor argument");
    int rc = check_call(ctx, kv, layer, p, batch, n_tokens, past_len);
    if (rc) return rc;
    if (n_tokens * (p->n_heads / p->n_kv_heads) > 64)
        return fail(BRK_ERR_UNSUPPORTED, "brk_attn_step covers decode (n_tokens * group <= 64); use append + forward");
    for (int b = 0; b < batch; ++b)
        if (past_len[b] + n_tokens - p->kv_offset > kv->cap)
            return fail(BRK_ERR_CAPACITY, "sequence %d needs %d cache rows, capacity is %d (grow the cache)", b,
                        past_len[b] + n_tokens - p->kv_offset, kv->cap);
    if (n_tokens == 1 && (p->head_dim != 256 || p->n_heads / p->n_kv_heads <= 4)) {
        // One token: the append runs inside the decode launch (no second kernel, no dependency
        // between launches; head_dim 256 stages up to 4 q rows per tile); the same checks as
        // brk_attn_append.
        if (p->rope && (p->rope->head_dim != p->head_dim || p->rope->ctx != ctx))
            return fail(BRK_ERR_INVALID, "rope table head_dim %d != %d", p->rope->head_dim, p->head_dim);
        for (int b = 0; b < batch; ++b)
            if (p->rope && past_len[b] + 1 > p->rope->max_pos)
                return fail(BRK_ERR_CAPACITY, "position %d beyond the rope table (%d positions)", past_len[b],
                            p->rope->max_pos);
        DeviceGuard g(ctx->device);
        const FusedAppend f{q_in, k_in, v_in, q_work};
        return run_decode(ctx, kv, layer, p, batch, n_tokens, past_len, q_work, out, nullptr, nullptr, false,
                          static_cast<cudaStream_t>(stream), nullptr, 0, true, nullptr, 0, &f);
    }
    rc = append_impl(ctx, kv, layer, p, batch, n_tokens, past_len, q_in, k_in, v_in, q_work, stream, true);
    if (rc) return rc;
    DeviceGuard g(ctx->device);
    return run_decode(ctx, kv, layer, p, batch, n_tokens, past_len, q_work, out, nullptr, nullptr, false,
                      static_cast<cudaStream_t>(stream), nullptr, 0, true);
}

int brk_attn_decode(brk_ctx *ctx, const brk_kv *kv, int layer, const brk_attn_params *p, int batch, int n_tokens,
                    const int32_t *past_len, const float *q, float *out, void *stream) {
    int rc = check_call(ctx, kv, layer, p, batch, n_tokens, past_len);
    if (rc) return rc;
    if (!q || !out) return fail(BRK_ERR_INVALID, "null q or out");
    DeviceGuard g(ctx->device);
    return run_decode(ctx, kv, layer, p, batch, n_tokens, past_len, q, out, nullptr, nullptr, false,
                      static_cast<cudaStream_t>(stream));
}

int brk_attn_decode_splits(brk_ctx *ctx, const brk_kv *kv, const brk_attn_params *p, int batch, int n_tokens,
                           const int32_t *past_len) {
    int rc = check_call(ctx, kv, 0, p, batch, n_tokens, past_len);
    if (rc) return rc;
    int nsplit = 1, kps = 0;
    rc = decode_split_plan(ctx, kv, p, batch, n_tokens, past_len, false, &nsplit, &kps);
    return rc ? rc : nsplit;
}

// No-allocation variant of brk_attn_decode (declared in brk_attn.h with the reasons).
int brk_attn_decode_static(brk_ctx *ctx, const brk_kv *kv, int layer, const brk_attn_params *p, int batch,
                           int n_tokens, const int32_t *past_len, const float *q, float *out, void *stream) {
    int rc = check_call(ctx, kv, layer, p, batch, n_tokens, past_len);
    if (rc) return rc;
    if (!q || !out) return fail(BRK_ERR_INVALID, "null q or out");
    DeviceGuard g(ctx->device);
    void *scratch = nullptr;
    rc = static_scratch_address(&scratch);
    if (rc) return rc;
    return run_decode(ctx, kv, layer, p, batch, n_tokens, past_len, q, out, nullptr, nullptr, false,
                      static_cast<cudaStream_t>(stream), scratch, BRK_DECODE_STATIC_SCRATCH_BYTES);
}

namespace {
// Grows the context's prefill staging buffer to at least `bytes` (int8 caches only).
int ensure_stage(brk_ctx *ctx, size_t bytes) {
    if (bytes <= ctx->stage_bytes) return BRK_OK;
    BRK_CUDA(cudaDeviceSynchronize());  // queued kernels may still read the old buffer
    cudaFree(ctx->stage);
    ctx->stage = nullptr;
    ctx->stage_bytes = 0;
    BRK_CUDA(cudaMalloc(&ctx->stage, bytes));
    ctx->stage_bytes = bytes;
    return BRK_OK;
}

// The tensor-core prefill launch: q rotated (q) or raw with the prologue fused (q_raw).
// clamp_rows: positions may run past the cache capacity (the kernel attends rows below it), for
// the non-causal path whose rows all sit at the last key.
int prefill_impl(brk_ctx *ctx, const brk_kv *kv, int layer, const brk_attn_params *p, int batch, int n_tokens,
                 const int32_t *past_len, const float *q, const float *q_raw, float *out, void *stream,
                 bool clamp_rows = false, bool pdl = false, const __half *q16 = nullptr) {
    int rc = check_call(ctx, kv, layer, p, batch, n_tokens, past_len);
    if (rc) return rc;
    if ((!q && !q_raw && !q16) || !out) return fail(BRK_ERR_INVALID, "null q or out");
    if (q_raw && p->rope) {
        if (p->rope->head_dim != p->head_dim || p->rope->ctx != ctx)
            return fail(BRK_ERR_INVALID, "rope table head_dim %d != %d", p->rope->head_dim, p->head_dim);
        for (int b = 0; b < batch; ++b)
            if (past_len[b] + n_tokens > p->rope->max_pos)
                return fail(BRK_ERR_CAPACITY, "position %d beyond the rope table (%d positions)",
                            past_len[b] + n_tokens - 1, p->rope->max_pos);
    }
    if (p->head_dim != 64 && p->head_dim != 128)
        return fail(BRK_ERR_UNSUPPORTED, "tensor-core prefill covers head_dim 64 and 128 (got %d)", p->head_dim);
    brk::PrefillArgs a;
    memset(&a, 0, sizeof(a));
    for (int b = 0; b < batch; ++b) {
        if (!clamp_rows && past_len[b] + n_tokens - p->kv_offset > kv->cap)
            return fail(BRK_ERR_CAPACITY, "sequence %d needs %d cache rows, capacity is %d (grow the cache)", b,
                        past_len[b] + n_tokens - p->kv_offset, kv->cap);
        a.past_len[b] = past_len[b];
    }
    if ((n_tokens + 127) / 128 > 65535) return fail(BRK_ERR_INVALID, "n_tokens %d too large", n_tokens);
    DeviceGuard g(ctx->device);
    a.q = q_raw || q16 ? nullptr : q;
    a.q_raw = q16 ? nullptr : q_raw;
    a.q_tma = q16 ? 1 : 0;
    a.q_norm = q_raw ? p->q_norm : nullptr;
    a.rope = q_raw && p->rope ? p->rope->table32 : nullptr;
    a.eps = (float)p->eps;
    a.one_plus = p->norm_one_plus ? 1 : 0;
    a.out = out;
    a.err = ctx->d_err;
    a.B = batch;
    a.T = n_tokens;
    a.Hq = p->n_heads;
    a.Hkv = p->n_kv_heads;
    a.layer = layer;
    a.cap = kv->cap;
    a.kv_offset = p->kv_offset;
    a.window = p->window > 0 ? p->window : 0;
    const float scale = effective_scale(p);
    a.scale_log2 = scale * 1.4426950408889634f;
    a.softcap = p->softcap > 0.f ? p->softcap : 0.f;
    if (a.softcap > 0.f) {
        const double log2e = 1.4426950408889634;
        a.cap_k1 = (float)(2.0 * (double)scale * log2e / (double)a.softcap);
        a.cap_k2 = (float)((double)a.softcap * log2e);
    }
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (kv->q8()) {
        // int8 cache: dequantise this layer's rows [0, rows) to fp16 staging (one pass over the
        // codes, small next to the tensor-core work of a prefill chunk) and attend over it.
        int rows = 1;
        for (int b = 0; b < batch; ++b) rows = std::max(rows, past_len[b] + n_tokens - p->kv_offset);
        const size_t half_elems = (size_t)batch * p->n_kv_heads * rows * p->head_dim;
        rc = ensure_stage(ctx, 2 * half_elems * sizeof(__half));
        if (rc) return rc;
        __half *sk = static_cast<__half *>(ctx->stage), *sv = sk + half_elems;
        cudaError_t e = brk::launch_kv_dequant(kv->k8, kv->v8, kv->scales, sk, sv, layer, batch, p->n_kv_heads,
                                               p->head_dim, kv->cap, kv->scale_pitch, rows, st);
        if (e != cudaSuccess) return cuda_fail(e, "kv dequantise launch");
        ++ctx->launches;
        CUtensorMap mk, mv;
        const uint64_t srows = (uint64_t)batch * p->n_kv_heads * rows;
        if ((rc = make_cache_map(&mk, sk, srows, p->head_dim, brk::prefill_tile_keys()))) return rc;
        if ((rc = make_cache_map(&mv, sv, srows, p->head_dim, brk::prefill_tile_keys()))) return rc;
        a.layer = 0;
        a.cap = rows;
        e = brk::launch_prefill(p->head_dim, mk, mv, a, st);
        if (e != cudaSuccess) return cuda_fail(e, "prefill kernel launch");
        ++ctx->launches;
        return BRK_OK;
    }
    CUtensorMap tmq;
    if (q16 && (rc = make_map(&tmq, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, sizeof(__half), q16, (uint64_t)batch * n_tokens,
                              (uint64_t)p->n_heads * p->head_dim, 64u, (uint32_t)brk::kPrefillQRows,
                              CU_TENSOR_MAP_SWIZZLE_128B)))
        return rc;
    cudaError_t e = brk::launch_prefill(p->head_dim, kv->tm_pre_k, kv->tm_pre_v, a, st, pdl, q16 ? &tmq : nullptr);
    if (e != cudaSuccess) return cuda_fail(e, "prefill kernel launch");
    ++ctx->launches;
    return BRK_OK;
}
}  // namespace

int brk_attn_prefill(brk_ctx *ctx, const brk_kv *kv, int layer, const brk_attn_params *p, int batch, int n_tokens,
                     const int32_t *past_len, const float *q, float *out, void *stream) {
    return prefill_impl(ctx, kv, layer, p, batch, n_tokens, past_len, q, nullptr, out, stream);
}

int brk_attn_prefill_h(brk_ctx *ctx, const brk_kv *kv, int layer, const brk_attn_params *p, int batch, int n_tokens,
                       const int32_t *past_len, const uint16_t *q16, float *out, void *stream) {
    if (!q16) return fail(BRK_ERR_INVALID, "null q");
    if (reinterpret_cast<uintptr_t>(q16) % 16) return fail(BRK_ERR_INVALID, "q must be 16-byte aligned");
    if (kv && kv->q8()) return fail(BRK_ERR_UNSUPPORTED, "fp16 q into the prefill kernel covers fp16 caches");
    return prefill_impl(ctx, kv, layer, p, batch, n_tokens, past_len, nullptr, nullptr, out, stream, false, false,
                        reinterpret_cast<const __half *>(q16));
}

int brk_attn_prefill_step(brk_ctx *ctx, brk_kv *kv, int layer, const brk_attn_params *p, int batch, int n_tokens,
                          const int32_t *past_len, const float *q_in, const float *k_in, const float *v_in, float *out,
                          void *stream) {
    if (!q_in || !k_in || !v_in || !out) return fail(BRK_ERR_INVALID, "null tensor argument");
    int rc = check_call(ctx, kv, layer, p, batch, n_tokens, past_len);
    if (rc) return rc;
    // fp16 caches, chunks of 8+ tokens: the K/V append kernel also rotates q (f32, the prefill
    // kernel's own q arithmetic) into fp16 rows in the context's staging buffer, which the prefill
    // kernel loads with TMA -- its q prologue would otherwise sit before each CTA's first MMA.
    // Otherwise the append stores K/V only and the q prologue runs inside the prefill kernel.
    // Either way the prefill kernel is launched as a programmatic dependent of the append.
    if (!kv->q8() && (p->head_dim == 64 || p->head_dim == 128) && n_tokens >= 8) {
        if (p->rope && (p->rope->head_dim != p->head_dim || p->rope->ctx != ctx))
            return fail(BRK_ERR_INVALID, "rope table head_dim %d != %d", p->rope->head_dim, p->head_dim);
        rc = ensure_stage(ctx, (size_t)batch * n_tokens * p->n_heads * p->head_dim * sizeof(__half));
        if (rc) return rc;
        __half *q16 = static_cast<__half *>(ctx->stage);
        rc = append_impl(ctx, kv, layer, p, batch, n_tokens, past_len, q_in, k_in, v_in, nullptr, stream, false, q16);
        if (rc) return rc;
        return prefill_impl(ctx, kv, layer, p, batch, n_tokens, past_len, nullptr, nullptr, out, stream, false, true,
                            q16);
    }
    rc = append_impl(ctx, kv, layer, p, batch, n_tokens, past_len, nullptr, k_in, v_in, nullptr, stream, false);
    if (rc) return rc;
    return prefill_impl(ctx, kv, layer, p, batch, n_tokens, past_len, nullptr, q_in, out, stream, false, true);
}

int brk_attn_forward(brk_ctx *ctx, const brk_kv *kv, int layer, const brk_attn_params *p, int batch, int n_tokens,
                     const int32_t *past_len, const float *q, float *out, void *stream) {
    // recAttention's choice (kernels.ts:1634): the decode kernel for few (token, head) rows per kv
    // head, the tensor-core kernel for prefill chunks.  BRK_ATTN_DECODE=0 forces the latter where
    // it exists (the reference's ?attndecode=0 kill switch).
    if (p && p->n_kv_heads > 0 && (p->head_dim == 64 || p->head_dim == 128)) {
        const char *env = getenv("BRK_ATTN_DECODE");
        const bool decode_off = env && env[0] == '0';
        const int rows = n_tokens * (p->n_heads / p->n_kv_heads);
        if (decode_off || rows > 128)
            return brk_attn_prefill(ctx, kv, layer, p, batch, n_tokens, past_len, q, out, stream);
    }
    return brk_attn_decode(ctx, kv, layer, p, batch, n_tokens, past_len, q, out, stream);
}

int brk_attn_decode_partial(brk_ctx *ctx, const brk_kv *kv, int layer, const brk_attn_params *p, int batch,
                            int n_tokens, const int32_t *past_len, const float *q, float *part_ml, float *part_o,
                            void *stream) {
    int rc = check_call(ctx, kv, layer, p, batch, n_tokens, past_len);
    if (rc) return rc;
    if (!q || !part_ml || !part_o) return fail(BRK_ERR_INVALID, "null q or partial buffers");
    DeviceGuard g(ctx->device);
    return run_decode(ctx, kv, layer, p, batch, n_tokens, past_len, q, nullptr, part_ml, part_o, true,
                      static_cast<cudaStream_t>(stream));
}

int brk_attn_combine(brk_ctx *ctx, int n_parts, int rows, int head_dim, const float *part_ml, const float *part_o,
                     size_t part_stride, float *out, void *stream) {
    if (!ctx || !part_ml || !part_o || !out) return fail(BRK_ERR_INVALID, "null argument");
    if (n_parts < 1 || rows < 0 || head_dim < 1) return fail(BRK_ERR_INVALID, "invalid combine shape");
    DeviceGuard g(ctx->device);
    brk::CombineArgs c;
    c.part_ml = part_ml;
    c.part_o = part_o;
    c.stride_ml = part_stride ? part_stride : (size_t)rows * 2;
    c.stride_o = part_stride ? part_stride : (size_t)rows * head_dim;
    c.out = out;
    c.out_ml = nullptr;
    c.out_o = nullptr;
    c.n_parts = n_parts;
    c.rows = rows;
    c.D = head_dim;
    cudaError_t e = brk::launch_combine(c, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "combine kernel launch");
    ++ctx->launches;
    return BRK_OK;
}

int brk_attn_full(brk_ctx *ctx, const brk_attn_params *p, int batch, int n_tokens, int kv_len, const float *q,
                  const float *k, const float *v, float *out, void *stream) {
    if (!ctx || !p || !q || !k || !v || !out) return fail(BRK_ERR_INVALID, "null argument");
    if (p->n_heads < 1 || p->n_kv_heads < 1 || p->n_heads % p->n_kv_heads)
        return fail(BRK_ERR_INVALID, "n_heads %d is not a multiple of n_kv_heads %d", p->n_heads, p->n_kv_heads);
    if (p->head_dim < 1 || p->head_dim > 256)
        return fail(BRK_ERR_UNSUPPORTED, "non-causal attention covers head_dim 1..256 (got %d)", p->head_dim);
    if (p->rope || p->q_norm || p->k_norm || p->window > 0 || p->kv_offset)
        return fail(BRK_ERR_INVALID, "non-causal attention takes no rope, norm gains, window or kv_offset");
    if (batch < 1 || batch > BRK_MAX_BATCH || n_tokens < 1 || kv_len < 1)
        return fail(BRK_ERR_INVALID, "batch %d / n_tokens %d / kv_len %d out of range", batch, n_tokens, kv_len);
    if ((long long)batch * p->n_kv_heads * kv_len >= (1ll << 31) ||
        (long long)batch * n_tokens * p->n_heads >= (1ll << 31))
        return fail(BRK_ERR_CAPACITY, "rows beyond 2^31");
    DeviceGuard g(ctx->device);
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    const int D = p->head_dim, Dp = D <= 64 ? 64 : D <= 128 ? 128 : 256;
    const int G = p->n_heads / p->n_kv_heads;
    const size_t kv_elems = (size_t)batch * p->n_kv_heads * kv_len * Dp;
    const size_t q_elems = D == Dp ? 0 : (size_t)batch * n_tokens * p->n_heads * Dp;
    int rc = ensure_stage(ctx, kv_elems * 2 * sizeof(__half) + q_elems * 2 * sizeof(float) + 256);
    if (rc) return rc;
    __half *sk = static_cast<__half *>(ctx->stage), *sv = sk + kv_elems;
    float *qp = const_cast<float *>(q), *op = out;
    if (q_elems) {
        qp = reinterpret_cast<float *>(reinterpret_cast<uintptr_t>(sv + kv_elems + 127) & ~uintptr_t(127));
        op = qp + q_elems;
    }
    cudaError_t e = brk::launch_stage_kv(k, v, sk, sv, batch, kv_len, p->n_kv_heads, D, Dp, st);
    if (e == cudaSuccess && q_elems)
        e = brk::launch_pad_rows(q, qp, (long long)batch * n_tokens * p->n_heads, D, Dp, st);
    if (e != cudaSuccess) return cuda_fail(e, "non-causal staging launch");
    ctx->launches += q_elems ? 2 : 1;
    // The staged rows as a one-layer cache whose every query sits at its last key.
    brk_kv view;
    view.ctx = ctx;
    view.desc = brk_kv_desc{1, batch, p->n_kv_heads, Dp, kv_len, BRK_KV_F16};
    view.cap = kv_len;
    view.k = sk;
    view.v = sv;
    if ((rc = kv_build_maps(&view))) return rc;
    brk_attn_params pp = *p;
    pp.head_dim = Dp;
    pp.scale = effective_scale(p);  // 1/sqrt of the caller's head_dim, not the padded one
    std::vector<int32_t> past(batch, kv_len - 1);
    if ((Dp == 64 || Dp == 128) && (long long)n_tokens * G > 64)
        rc = prefill_impl(ctx, &view, 0, &pp, batch, n_tokens, past.data(), qp, nullptr, op, stream, true);
    else
        rc = run_decode(ctx, &view, 0, &pp, batch, n_tokens, past.data(), qp, op, nullptr, nullptr, true, st);
    if (rc) return rc;
    if (q_elems) {
        e = cudaMemcpy2DAsync(out, (size_t)D * sizeof(float), op, (size_t)Dp * sizeof(float), (size_t)D * sizeof(float),
                              (size_t)batch * n_tokens * p->n_heads, cudaMemcpyDeviceToDevice, st);
        if (e != cudaSuccess) return cuda_fail(e, "non-causal output copy");
    }
    return BRK_OK;
}

namespace {
// fp16 weight matrix [n][k] (K-major), boxes [nt][64].
int make_weight_map(CUtensorMap *m, const uint16_t *w, int n, int k, int nt) {
    return make_map(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, w, (uint64_t)n, (uint64_t)k, 64u, (uint32_t)nt,
                    CU_TENSOR_MAP_SWIZZLE_128B);
}

int ensure_act(brk_ctx *ctx, size_t bytes) {
    if (bytes <= ctx->act_bytes) return BRK_OK;
    BRK_CUDA(cudaDeviceSynchronize());  // queued kernels may still read the old buffer
    cudaFree(ctx->act);
    ctx->act = nullptr;
    ctx->act_bytes = 0;
    BRK_CUDA(cudaMalloc(&ctx->act, bytes));
    ctx->act_bytes = bytes;
    return BRK_OK;
}

// Casts `rows` x K activations to fp16 (RMSNorm fused when gain is given) and runs the GEMM over
// up to three weight matrices.
int run_proj(brk_ctx *ctx, int rows, int K, const float *x, const float *gain, double eps, int one_plus, int nmat,
             const int *n, const uint16_t *const *w, float *const *out, const float *const *bias,
             const float *residual, cudaStream_t st) {
    const int ntok = brk::proj_token_tile(rows);
    for (int i = 0; i < nmat; ++i)
        if (n[i] < 4 || n[i] % 4) return fail(BRK_ERR_INVALID, "projection width %d (a multiple of 4)", n[i]);
    int rc = ensure_act(ctx, (size_t)rows * K * sizeof(__half));
    if (rc) return rc;
    __half *act = static_cast<__half *>(ctx->act);
    CUtensorMap tx, tw[3], to[3];
    if ((rc = make_map(&tx, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, act, (uint64_t)rows, (uint64_t)K, 64u, (uint32_t)ntok,
                       CU_TENSOR_MAP_SWIZZLE_128B)))
        return rc;
    brk::ProjArgs a;
    memset(&a, 0, sizeof(a));
    a.M = rows;
    a.K = K;
    a.nmat = nmat;
    a.residual = residual;
    a.err = ctx->d_err;
    int end = 0;
    for (int i = 0; i < 3; ++i) {
        const int j = i < nmat ? i : 0;
        if ((rc = make_weight_map(&tw[i], w[j], n[j], K, 128))) return rc;
        // Output [rows][n] f32, box [32 tokens][128 features], no swizzle (the staging layout).
        if ((rc = make_map(&to[i], CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, out[j], (uint64_t)rows, (uint64_t)n[j], 128u, 32u,
                           CU_TENSOR_MAP_SWIZZLE_NONE)))
            return rc;
        if (i < nmat) {
            end += (n[i] + 127) / 128;
            a.tile_end[i] = end;
            a.n[i] = n[i];
            a.out[i] = out[i];
            a.bias[i] = bias[i];
        }
    }
    brk::proj_plan(a, ntok, ctx->num_sms);
    cudaError_t e = brk::launch_norm_cast(x, gain, (float)eps, one_plus, act, rows, K, a, st);
    if (e != cudaSuccess) return cuda_fail(e, "activation cast launch");
    ++ctx->launches;
    e = brk::launch_proj(ntok, tx, tw, to, a, st);
    if (e != cudaSuccess) return cuda_fail(e, "projection GEMM launch");
    ++ctx->launches;
    return BRK_OK;
}

int check_proj(const brk_ctx *ctx, int rows, int K, const float *x, const void *out) {
    if (!ctx || !x || !out) return fail(BRK_ERR_INVALID, "null argument");
    if (rows < 1 || K < 8 || K % 8) return fail(BRK_ERR_INVALID, "rows %d / input width %d (a multiple of 8)", rows, K);
    if ((long long)rows * K >= (1ll << 31)) return fail(BRK_ERR_CAPACITY, "rows * width beyond 2^31");
    return BRK_OK;
}
}  // namespace

int brk_proj_qkv(brk_ctx *ctx, int rows, int d_model, int q_dim, int kv_dim, const float *x, const float *attn_norm,
                 double eps, int norm_one_plus, const uint16_t *wq, const uint16_t *wk, const uint16_t *wv,
                 const float *bq, const float *bk, const float *bv, float *q, float *k, float *v, void *stream) {
    int rc = check_proj(ctx, rows, d_model, x, q);
    if (rc) return rc;
    if (!wq || !wk || !wv || !k || !v) return fail(BRK_ERR_INVALID, "null weight or output");
    DeviceGuard g(ctx->device);
    const int n[3] = {q_dim, kv_dim, kv_dim};
    const uint16_t *w[3] = {wq, wk, wv};
    float *out[3] = {q, k, v};
    const float *bias[3] = {bq, bk, bv};
    return run_proj(ctx, rows, d_model, x, attn_norm, eps, norm_one_plus, 3, n, w, out, bias, nullptr,
                    static_cast<cudaStream_t>(stream));
}

int brk_proj_out(brk_ctx *ctx, int rows, int q_dim, int d_model, const float *attn, const uint16_t *wo,
                 const float *post_norm, double eps, int norm_one_plus, const float *x, float *h, void *stream) {
    int rc = check_proj(ctx, rows, q_dim, attn, h);
    if (rc) return rc;
    if (!wo || !x) return fail(BRK_ERR_INVALID, "null weight or residual");
    if (d_model % 4) return fail(BRK_ERR_INVALID, "d_model %d must be a multiple of 4", d_model);
    DeviceGuard g(ctx->device);
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    const int n[1] = {d_model};
    const uint16_t *w[1] = {wo};
    float *out[1] = {h};
    const float *bias[1] = {nullptr};
    rc = run_proj(ctx, rows, q_dim, attn, nullptr, 0.0, 0, 1, n, w, out, bias, post_norm ? nullptr : x, st);
    if (rc || !post_norm) return rc;
    cudaError_t e = brk::launch_post_norm_residual(h, x, post_norm, (float)eps, norm_one_plus, rows, d_model, st);
    if (e != cudaSuccess) return cuda_fail(e, "post-norm launch");
    ++ctx->launches;
    return BRK_OK;
}

int brk_peer_create(brk_ctx *ctx, int world, int rank, int max_rows, int head_dim, brk_peer **out) {
    if (!ctx || !out) return fail(BRK_ERR_INVALID, "null argument");
    *out = nullptr;
    if (world < 1 || world > BRK_MAX_PEERS || rank < 0 || rank >= world)
        return fail(BRK_ERR_INVALID, "rank %d of world %d (1..%d ranks)", rank, world, BRK_MAX_PEERS);
    if (max_rows < 1 || head_dim < 1) return fail(BRK_ERR_INVALID, "max_rows %d / head_dim %d", max_rows, head_dim);
    DeviceGuard g(ctx->device);
    brk_peer *pr = new brk_peer();
    pr->ctx = ctx;
    pr->world = world;
    pr->rank = rank;
    pr->max_rows = max_rows;
    pr->head_dim = head_dim;
    pr->stride = ((size_t)max_rows * (2 + head_dim) + 63) / 64 * 64;  // 256-byte aligned blocks
    pr->flags_offset = 2 * (size_t)world * pr->stride * sizeof(float);
    const size_t bytes = pr->flags_offset + 256;
    cudaError_t e = cudaMalloc(&pr->area, bytes);
    if (e == cudaSuccess) e = cudaMemset(pr->area, 0, bytes);
    if (e == cudaSuccess) e = cudaMalloc(&pr->done, sizeof(int));
    if (e == cudaSuccess) e = cudaMemset(pr->done, 0, sizeof(int));
    if (e != cudaSuccess) {
        cudaFree(pr->area);
        cudaFree(pr->done);
        delete pr;
        return cuda_fail(e, "peer exchange area");
    }
    pr->peers[rank] = pr->area;
    *out = pr;
    return BRK_OK;
}

int brk_peer_handle(const brk_peer *peer, void *handle, size_t handle_bytes) {
    if (!peer || !handle) return fail(BRK_ERR_INVALID, "null argument");
    if (handle_bytes < sizeof(cudaIpcMemHandle_t))
        return fail(BRK_ERR_INVALID, "handle buffer of %zu bytes (needs %zu)", handle_bytes, sizeof(cudaIpcMemHandle_t));
    DeviceGuard g(peer->ctx->device);
    cudaIpcMemHandle_t h;
    BRK_CUDA(cudaIpcGetMemHandle(&h, peer->area));
    memcpy(handle, &h, sizeof(h));
    return BRK_OK;
}

int brk_peer_open(brk_peer *peer, int peer_rank, const void *handle, size_t handle_bytes) {
    if (!peer || !handle) return fail(BRK_ERR_INVALID, "null argument");
    if (peer_rank < 0 || peer_rank >= peer->world || peer_rank == peer->rank)
        return fail(BRK_ERR_INVALID, "peer rank %d (world %d, own rank %d)", peer_rank, peer->world, peer->rank);
    if (handle_bytes < sizeof(cudaIpcMemHandle_t)) return fail(BRK_ERR_INVALID, "short handle");
    if (peer->peers[peer_rank]) return fail(BRK_ERR_INVALID, "peer rank %d is already mapped", peer_rank);
    DeviceGuard g(peer->ctx->device);
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof(h));
    void *ptr = nullptr;
    BRK_CUDA(cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess));
    peer->peers[peer_rank] = ptr;
    peer->opened[peer_rank] = true;
    return BRK_OK;
}

int brk_peer_attach(brk_peer *peer, int peer_rank, const brk_peer *other) {
    if (!peer || !other) return fail(BRK_ERR_INVALID, "null argument");
    if (peer_rank < 0 || peer_rank >= peer->world || peer_rank == peer->rank || other->rank != peer_rank ||
        other->world != peer->world || other->max_rows != peer->max_rows || other->head_dim != peer->head_dim)
        return fail(BRK_ERR_INVALID, "attaching rank %d: areas of different shapes or ranks", peer_rank);
    if (peer->peers[peer_rank]) return fail(BRK_ERR_INVALID, "peer rank %d is already mapped", peer_rank);
    if (other->ctx->device != peer->ctx->device) {
        DeviceGuard g(peer->ctx->device);
        cudaError_t e = cudaDeviceEnablePeerAccess(other->ctx->device, 0);
        if (e == cudaErrorPeerAccessAlreadyEnabled) {
            cudaGetLastError();
        } else if (e != cudaSuccess) {
            return cuda_fail(e, "enabling peer access");
        }
    }
    peer->peers[peer_rank] = other->area;
    return BRK_OK;
}

int brk_peer_destroy(brk_peer *peer) {
    if (!peer) return BRK_OK;
    DeviceGuard g(peer->ctx->device);
    cudaDeviceSynchronize();
    for (int r = 0; r < peer->world; ++r)
        if (peer->opened[r]) cudaIpcCloseMemHandle(peer->peers[r]);
    cudaFree(peer->area);
    cudaFree(peer->done);
    delete peer;
    return BRK_OK;
}

int brk_attn_decode_push(brk_ctx *ctx, const brk_kv *kv, int layer, const brk_attn_params *p, int batch,
                         int n_tokens, const int32_t *past_len, const float *q, brk_peer *peer, uint32_t epoch,
                         void *stream) {
    int rc = check_call(ctx, kv, layer, p, batch, n_tokens, past_len);
    if (rc) return rc;
    if (!q || !peer) return fail(BRK_ERR_INVALID, "null q or peer area");
    if (peer->ctx != ctx) return fail(BRK_ERR_INVALID, "peer area belongs to another context");
    if (epoch == 0) return fail(BRK_ERR_INVALID, "epoch 0 is reserved (flags start at 0)");
    const long long rows = (long long)batch * n_tokens * p->n_heads;
    if (rows > peer->max_rows || p->head_dim != peer->head_dim)
        return fail(BRK_ERR_INVALID, "%lld rows of head_dim %d exceed the peer area (%d rows of %d)", rows, p->head_dim,
                    peer->max_rows, peer->head_dim);
    for (int r = 0; r < peer->world; ++r)
        if (!peer->peers[r]) return fail(BRK_ERR_INVALID, "rank %d's area is not mapped (brk_peer_open)", r);
    DeviceGuard g(ctx->device);
    return run_decode(ctx, kv, layer, p, batch, n_tokens, past_len, q, nullptr, nullptr, nullptr, true,
                      static_cast<cudaStream_t>(stream), nullptr, 0, false, peer, epoch);
}

int brk_attn_step_push(brk_ctx *ctx, brk_kv *kv, int layer, const brk_attn_params *p, int batch,
                       const int32_t *past_len, const float *q_in, const float *k_in, const float *v_in,
                       float *q_work, brk_peer *peer, uint32_t epoch, void *stream) {
    int rc = check_call(ctx, kv, layer, p, batch, 1, past_len);
    if (rc) return rc;
    if (!q_in || !q_work || !peer) return fail(BRK_ERR_INVALID, "null q_in, q_work or peer area");
    if (peer->ctx != ctx) return fail(BRK_ERR_INVALID, "peer area belongs to another context");
    if (epoch == 0) return fail(BRK_ERR_INVALID, "epoch 0 is reserved (flags start at 0)");
    if (p->head_dim == 256 && p->n_heads / p->n_kv_heads > 4)
        return fail(BRK_ERR_UNSUPPORTED, "head_dim 256 with a GQA group above 4: use brk_attn_append + decode_push");
    const long long rows = (long long)batch * p->n_heads;
    if (rows > peer->max_rows || p->head_dim != peer->head_dim)
        return fail(BRK_ERR_INVALID, "%lld rows of head_dim %d exceed the peer area (%d rows of %d)", rows, p->head_dim,
                    peer->max_rows, peer->head_dim);
    for (int r = 0; r < peer->world; ++r)
        if (!peer->peers[r]) return fail(BRK_ERR_INVALID, "rank %d's area is not mapped (brk_peer_open)", r);
    if (p->rope && (p->rope->head_dim != p->head_dim || p->rope->ctx != ctx))
        return fail(BRK_ERR_INVALID, "rope table head_dim %d != %d", p->rope->head_dim, p->head_dim);
    for (int b = 0; b < batch; ++b) {
        if (p->rope && past_len[b] + 1 > p->rope->max_pos)
            return fail(BRK_ERR_CAPACITY, "position %d beyond the rope table (%d positions)", past_len[b],
                        p->rope->max_pos);
        // This rank stores the new row when its cache holds that position (the last shard).
        if (past_len[b] - p->kv_offset < kv->cap && (!k_in || !v_in))
            return fail(BRK_ERR_INVALID, "sequence %d's new position is in this cache: k_in and v_in are needed", b);
    }
    DeviceGuard g(ctx->device);
    const FusedAppend f{q_in, k_in, v_in, q_work};
    return run_decode(ctx, kv, layer, p, batch, 1, past_len, q_work, nullptr, nullptr, nullptr, true,
                      static_cast<cudaStream_t>(stream), nullptr, 0, false, peer, epoch, &f);
}

int brk_attn_combine_peers(brk_ctx *ctx, brk_peer *peer, int rows, uint32_t epoch, double timeout_s, float *out,
                           void *stream) {
    if (!ctx || !peer || !out) return fail(BRK_ERR_INVALID, "null argument");
    if (peer->ctx != ctx) return fail(BRK_ERR_INVALID, "peer area belongs to another context");
    if (rows < 0 || rows > peer->max_rows) return fail(BRK_ERR_INVALID, "rows %d outside [0, %d]", rows, peer->max_rows);
    if (epoch == 0) return fail(BRK_ERR_INVALID, "epoch 0 is reserved (flags start at 0)");
    if (!(timeout_s > 0.0) || timeout_s > 60.0) return fail(BRK_ERR_INVALID, "timeout %g s outside (0, 60]", timeout_s);
    DeviceGuard g(ctx->device);
    const int par = (int)(epoch & 1u);
    float *base = static_cast<float *>(peer->area) + (size_t)par * peer->world * peer->stride;
    brk::CombineArgs c;
    c.part_ml = base;
    c.part_o = base + (size_t)rows * 2;
    c.stride_ml = c.stride_o = peer->stride;
    c.out = out;
    c.out_ml = nullptr;
    c.out_o = nullptr;
    c.n_parts = peer->world;
    c.rows = rows;
    c.D = peer->head_dim;
    const unsigned *flags =
        reinterpret_cast<const unsigned *>(static_cast<const char *>(peer->area) + peer->flags_offset) + par * peer->world;
    cudaError_t e = brk::launch_combine_peers(c, flags, peer->world, epoch, (unsigned long long)(timeout_s * 1e9),
                                              ctx->d_err, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "combine kernel launch");
    ++ctx->launches;
    return BRK_OK;
}

}  // extern "C"
