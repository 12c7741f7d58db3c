/*
 * CPU oracle for the Brimkern attention path — TEST INFRASTRUCTURE ONLY (see oracle.h).
 *
 * JS semantics restated in C:
 *   - a JS `number` is an IEEE double, so every intermediate here is a `double`;
 *   - a store into a Float32Array rounds to f32, which is the `(float)` cast at each store;
 *   - compiled with -ffp-contract=off so that no a*b+c is fused (JS never fuses).
 * Math.exp / Math.tanh / Math.cos / Math.sin / Math.sqrt / `**` map to libm's exp, tanh,
 * cos, sin, sqrt, pow.
 */
#include "oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* kernels.ts:3395-3404 (rmsnormCpu). */
void brk_oracle_rmsnorm(const float *x, const float *w, int rows, int dim, double eps,
                        int one_plus, float *o) {
    for (int r = 0; r < rows; r++) {
        const float *xr = x + (long long)r * dim;
        double ss = 0;
        for (int i = 0; i < dim; i++) {
            double xi = xr[i];
            ss += xi * xi; /* x ** 2: exact in double for an f32 x */
        }
        double inv = 1.0 / sqrt(ss / dim + eps);
        for (int i = 0; i < dim; i++) {
            double g = one_plus ? 1.0 + (double)w[i] : (double)w[i];
            o[(long long)r * dim + i] = (float)((double)xr[i] * inv * g);
        }
    }
}

/* Shared body of ropeCpu (kernels.ts:3445-3460) and ropeFactorsCpu (kernels.ts:3428-3443):
 * freq = pos / (base ** ((2*i)/headDim) [* ff[i]]). */
static void rope_body(const float *x, const float *ff, int rows, int head_dim, int n_heads,
                      int past_len, double base, float *o) {
    int half = head_dim / 2;
    for (int r = 0; r < rows; r++) {
        double pos = (double)past_len + floor((double)r / (double)n_heads);
        long long b = (long long)r * head_dim;
        for (int i = 0; i < half; i++) {
            double denom = pow(base, (2.0 * i) / (double)head_dim);
            if (ff) denom = denom * (double)ff[i];
            double freq = pos / denom;
            double c = cos(freq), s = sin(freq);
            double x0 = x[b + i], x1 = x[b + i + half];
            o[b + i] = (float)(x0 * c - x1 * s);
            o[b + i + half] = (float)(x1 * c + x0 * s);
        }
    }
}

void brk_oracle_rope(const float *x, int rows, int head_dim, int n_heads, int past_len,
                     double base, float *o) {
    rope_body(x, NULL, rows, head_dim, n_heads, past_len, base, o);
}

void brk_oracle_rope_factors(const float *x, const float *ff, int rows, int head_dim,
                             int n_heads, int past_len, double base, float *o) {
    rope_body(x, ff, rows, head_dim, n_heads, past_len, base, o);
}

/* The score closure of attentionCpu (kernels.ts:3469): cap(s) = softcap*tanh(s/softcap). */
static inline double cap_score(double s, double softcap) {
    return softcap > 0 ? softcap * tanh(s / softcap) : s;
}

/* One (t, h) row of attentionCpu (kernels.ts:3472-3493) over keys [lo, last].
 * scores: scratch of at least last+1 doubles.  o_row is accumulated with an f32 store at
 * every step, exactly as `o[qB + dd] += w * v[vB + dd]` on a Float32Array. */
static void attend_row(const float *q_row, const float *k, const float *v, int kvh,
                       int n_kv_heads, int head_dim, int lo, int last, double scale,
                       double softcap, double *scores, float *o_row) {
    double mx = -INFINITY;
    for (int j = lo; j <= last; j++) {
        const float *kr = k + ((long long)j * n_kv_heads + kvh) * head_dim;
        double dot = 0;
        for (int dd = 0; dd < head_dim; dd++) dot += (double)q_row[dd] * (double)kr[dd];
        double s = cap_score(dot * scale, softcap);
        scores[j] = s;
        if (s > mx) mx = s;
    }
    double denom = 0;
    for (int j = lo; j <= last; j++) {
        scores[j] = exp(scores[j] - mx);
        denom += scores[j];
    }
    for (int dd = 0; dd < head_dim; dd++) o_row[dd] = 0.0f;
    for (int j = lo; j <= last; j++) {
        double w = scores[j] / denom;
        const float *vr = v + ((long long)j * n_kv_heads + kvh) * head_dim;
        for (int dd = 0; dd < head_dim; dd++)
            o_row[dd] = (float)((double)o_row[dd] + w * (double)vr[dd]);
    }
}

static inline int window_lo(int last, int window) {
    if (window <= 0) return 0;
    int lo = last - window + 1;
    return lo > 0 ? lo : 0;
}

static inline double default_scale(double scale, int head_dim) {
    return isnan(scale) ? 1.0 / sqrt((double)head_dim) : scale;
}

/* kernels.ts:3466-3495 (attentionCpu) + sliding-window extension. */
void brk_oracle_attention(const float *q, const float *k, const float *v, int n_tokens,
                          int n_heads, int n_kv_heads, int head_dim, int past_len,
                          double scale, double softcap, int window, float *o) {
    scale = default_scale(scale, head_dim);
    double group = (double)n_heads / (double)n_kv_heads;
    double *scores = (double *)malloc(sizeof(double) * (size_t)(past_len + n_tokens + 1));
    for (int t = 0; t < n_tokens; t++)
        for (int h = 0; h < n_heads; h++) {
            int kvh = (int)floor((double)h / group);
            long long qb = ((long long)t * n_heads + h) * head_dim;
            int last = past_len + t;
            attend_row(q + qb, k, v, kvh, n_kv_heads, head_dim, window_lo(last, window), last,
                       scale, softcap, scores, o + qb);
        }
    free(scores);
}

void brk_oracle_attention_partial(const float *q, const float *k, const float *v,
                                  int n_tokens, int n_heads, int n_kv_heads, int head_dim,
                                  int past_len, double scale, double softcap, int window,
                                  int key_lo, int key_hi, double *m, double *l, double *o) {
    scale = default_scale(scale, head_dim);
    double group = (double)n_heads / (double)n_kv_heads;
    for (int t = 0; t < n_tokens; t++)
        for (int h = 0; h < n_heads; h++) {
            int kvh = (int)floor((double)h / group);
            long long row = (long long)t * n_heads + h;
            const float *qr = q + row * head_dim;
            int last = past_len + t;
            int lo = window_lo(last, window);
            if (lo < key_lo) lo = key_lo;
            int hi = last < key_hi - 1 ? last : key_hi - 1;
            double mx = -INFINITY;
            for (int j = lo; j <= hi; j++) {
                const float *kr = k + ((long long)j * n_kv_heads + kvh) * head_dim;
                double dot = 0;
                for (int dd = 0; dd < head_dim; dd++) dot += (double)qr[dd] * (double)kr[dd];
                double s = cap_score(dot * scale, softcap);
                if (s > mx) mx = s;
            }
            double sum = 0;
            double *orow = o + row * head_dim;
            for (int dd = 0; dd < head_dim; dd++) orow[dd] = 0;
            for (int j = lo; j <= hi; j++) {
                const float *kr = k + ((long long)j * n_kv_heads + kvh) * head_dim;
                double dot = 0;
                for (int dd = 0; dd < head_dim; dd++) dot += (double)qr[dd] * (double)kr[dd];
                double p = exp(cap_score(dot * scale, softcap) - mx);
                sum += p;
                const float *vr = v + ((long long)j * n_kv_heads + kvh) * head_dim;
                for (int dd = 0; dd < head_dim; dd++) orow[dd] += p * (double)vr[dd];
            }
            m[row] = mx;
            l[row] = sum;
        }
}

void brk_oracle_combine(const double *m, const double *l, const double *o, int n_parts,
                        int rows, int head_dim, float *out) {
    for (int r = 0; r < rows; r++) {
        double M = -INFINITY;
        for (int s = 0; s < n_parts; s++)
            if (m[(long long)s * rows + r] > M) M = m[(long long)s * rows + r];
        double L = 0;
        for (int s = 0; s < n_parts; s++) {
            double ms = m[(long long)s * rows + r];
            if (ms == -INFINITY) continue;
            L += l[(long long)s * rows + r] * exp(ms - M);
        }
        for (int dd = 0; dd < head_dim; dd++) {
            double acc = 0;
            for (int s = 0; s < n_parts; s++) {
                double ms = m[(long long)s * rows + r];
                if (ms == -INFINITY) continue;
                acc += o[((long long)s * rows + r) * head_dim + dd] * exp(ms - M);
            }
            out[(long long)r * head_dim + dd] = (float)(acc / L);
        }
    }
}

/* Non-causal attention (attention_full, shaders.ts:1530-1570) as the reference's own gate computes
 * it (kernels.ts:3168-3177): per (head, query) the score s_j = f32(dot * scale) with the dot in
 * double, mx = max s_j, s_j = f32(exp(s_j - mx)), sum in double, o = f32(sum_j (s_j / sum) v_j)
 * accumulated in double.  Every query attends all kv_len keys.  Extensions that reduce to the gate
 * in its case (n_kv_heads == n_heads, no softcap): GQA (kvh = floor(h / group)) and the softcap
 * c * tanh(s / c) of attentionCpu (kernels.ts:3469) applied before the f32 store. */
void brk_oracle_attention_full(const float *q, const float *k, const float *v, int n_tokens,
                               int n_heads, int n_kv_heads, int head_dim, int kv_len,
                               double scale, double softcap, float *o) {
    scale = default_scale(scale, head_dim);
    double group = (double)n_heads / (double)n_kv_heads;
    float *s = (float *)malloc(sizeof(float) * (size_t)(kv_len > 0 ? kv_len : 1));
    double *acc = (double *)malloc(sizeof(double) * (size_t)head_dim);
    for (int h = 0; h < n_heads; h++)
        for (int t = 0; t < n_tokens; t++) {
            int kvh = (int)floor((double)h / group);
            const float *qr = q + ((long long)t * n_heads + h) * head_dim;
            float mx = -INFINITY;
            for (int j = 0; j < kv_len; j++) {
                const float *kr = k + ((long long)j * n_kv_heads + kvh) * head_dim;
                double d2 = 0;
                for (int e = 0; e < head_dim; e++) d2 += (double)qr[e] * (double)kr[e];
                s[j] = (float)cap_score(d2 * scale, softcap);
                if (s[j] > mx) mx = s[j];
            }
            double sum = 0;
            for (int j = 0; j < kv_len; j++) {
                s[j] = (float)exp((double)s[j] - (double)mx);
                sum += (double)s[j];
            }
            for (int e = 0; e < head_dim; e++) {
                double a = 0;
                for (int j = 0; j < kv_len; j++)
                    a += ((double)s[j] / sum) * (double)v[((long long)j * n_kv_heads + kvh) * head_dim + e];
                acc[e] = a;
            }
            float *orow = o + ((long long)t * n_heads + h) * head_dim;
            for (int e = 0; e < head_dim; e++) orow[e] = (float)acc[e];
        }
    free(acc);
    free(s);
}

/* matmulCpu (kernels.ts:3384-3392) in the GPU's weight layout (matmul_t, shaders.ts:28-43):
 * o[r][c] = f32(sum_i a[r][i] * w[c][i]) with the sum in double, w [n][k]. */
void brk_oracle_matmul_t(const float *a, const float *w, int m, int k, int n, float *o) {
    for (int r = 0; r < m; r++)
        for (int c = 0; c < n; c++) {
            double s = 0;
            const float *ar = a + (long long)r * k, *wr = w + (long long)c * k;
            for (int i = 0; i < k; i++) s += (double)ar[i] * (double)wr[i];
            o[(long long)r * n + c] = (float)s;
        }
}

/* quantize_kv shader (shaders.ts:1673-1705), in the shader's own f32 arithmetic:
 * amax over the head's D values, scale = amax == 0 ? 1e-8 : amax/127, inv = 1/scale,
 * code = clamp(round(x*inv), -127, 127) with WGSL round() = round-half-to-even (rintf). */
void brk_oracle_quantize_kv(const float *src, int rows, int n_kv_heads, int head_dim,
                            int row_offset, int8_t *codes, float *scales) {
    int kv_dim = n_kv_heads * head_dim;
    for (int row = 0; row < rows; row++)
        for (int head = 0; head < n_kv_heads; head++) {
            const float *s = src + (long long)row * kv_dim + head * head_dim;
            float amax = 0.0f;
            for (int d = 0; d < head_dim; d++) amax = fmaxf(amax, fabsf(s[d]));
            float scale = amax == 0.0f ? 1e-8f : amax / 127.0f;
            long long dst_row = (long long)row_offset + row;
            scales[dst_row * n_kv_heads + head] = scale;
            float inv = 1.0f / scale;
            for (int d = 0; d < head_dim; d++) {
                float prod = s[d] * inv;
                int qd = (int)rintf(prod);
                if (qd < -127) qd = -127;
                if (qd > 127) qd = 127;
                codes[dst_row * kv_dim + head * head_dim + d] = (int8_t)qd;
            }
        }
}

int brk_oracle_attention_batch(const float *q, const float *k, const float *v, int batch,
                               long long seq_stride, int n_tokens, int n_heads,
                               int n_kv_heads, int head_dim, const int *past_len,
                               double scale, double softcap, int window, int threads,
                               float *o) {
    scale = default_scale(scale, head_dim);
    double group = (double)n_heads / (double)n_kv_heads;
    int max_len = 0;
    for (int b = 0; b < batch; b++)
        if (past_len[b] + n_tokens > max_len) max_len = past_len[b] + n_tokens;
    int used = 1;
#ifdef _OPENMP
    if (threads <= 0) threads = omp_get_max_threads();
    used = threads;
#pragma omp parallel num_threads(threads)
#endif
    {
        double *scores = (double *)malloc(sizeof(double) * (size_t)(max_len + 1));
        long long n_items = (long long)batch * n_tokens * n_heads;
#ifdef _OPENMP
#pragma omp for schedule(dynamic, 1)
#endif
        for (long long it = 0; it < n_items; it++) {
            int b = (int)(it / ((long long)n_tokens * n_heads));
            int th = (int)(it % ((long long)n_tokens * n_heads));
            int t = th / n_heads, h = th % n_heads;
            int kvh = (int)floor((double)h / group);
            const float *qb = q + (long long)b * n_tokens * n_heads * head_dim;
            float *ob = o + (long long)b * n_tokens * n_heads * head_dim;
            long long row = (long long)t * n_heads + h;
            int last = past_len[b] + t;
            attend_row(qb + row * head_dim, k + b * seq_stride, v + b * seq_stride, kvh,
                       n_kv_heads, head_dim, window_lo(last, window), last, scale, softcap,
                       scores, ob + row * head_dim);
        }
        free(scores);
    }
    return used;
}
