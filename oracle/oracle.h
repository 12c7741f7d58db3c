/*
 * CPU oracle for the Brimkern attention path — TEST INFRASTRUCTURE ONLY.
 *
 * A plain-C restatement of the reference's module-private JavaScript CPU
 * functions in src/lib/webgpu/kernels.ts (RomainKH/Brimkern), kept with JS
 * `number` semantics: every intermediate is an IEEE double, and a value is
 * rounded to f32 only where the JS code stores it into a Float32Array.
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline legs may
 * load this library, and only as the checker / the timed CPU reference.  The
 * product (brimkern_b200/) never calls it.
 *
 * Parity status: the reference is TypeScript and no JavaScript engine exists
 * in this image, so the reference cannot be executed natively.  The oracle is
 * pinned against fixtures produced by interpreting the reference's own source
 * text for these functions (tests/golden/gen_golden.py); see that script.
 */
#ifndef BRK_ORACLE_H
#define BRK_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* rmsnormCpu — kernels.ts:3395-3404.  o[r,i] = f32(x * inv * g), inv = 1/sqrt(ss/dim + eps),
 * g = w[i] or 1 + w[i] (one_plus). */
void brk_oracle_rmsnorm(const float *x, const float *w, int rows, int dim, double eps,
                        int one_plus, float *o);

/* ropeCpu — kernels.ts:3445-3460.  NeoX rotate-half; pos = past_len + floor(r / n_heads). */
void brk_oracle_rope(const float *x, int rows, int head_dim, int n_heads, int past_len,
                     double base, float *o);

/* ropeFactorsCpu — kernels.ts:3428-3443.  As rope, with freq_i = pos / (base^(2i/D) * ff[i]). */
void brk_oracle_rope_factors(const float *x, const float *ff, int rows, int head_dim,
                             int n_heads, int past_len, double base, float *o);

/* attentionCpu — kernels.ts:3466-3495, extended with a sliding window.
 *   q: [n_tokens, n_heads, D]; k, v: [kv_len, n_kv_heads, D] with kv_len = past_len + n_tokens.
 *   scale: NaN selects the reference default 1/sqrt(D).  softcap <= 0 disables the tanh cap.
 *   window <= 0 reproduces the reference exactly (keys 0..past_len+t); window W > 0 keeps
 *   keys j >= past_len + t - W + 1 (extension; degenerate case W >= kv_len == reference).
 * o: [n_tokens, n_heads, D], overwritten. */
void brk_oracle_attention(const float *q, const float *k, const float *v, int n_tokens,
                          int n_heads, int n_kv_heads, int head_dim, int past_len,
                          double scale, double softcap, int window, float *o);

/* Split-KV partial (extension, no reference counterpart): the same scores as
 * brk_oracle_attention restricted to keys [key_lo, key_hi) (intersected with the causal /
 * window range), returned as (max m, sum l, unnormalised o = sum exp(s-m) v) in double.
 * Rows with no valid key get m = -inf, l = 0, o = 0.
 *   m, l: [n_tokens, n_heads]; o: [n_tokens, n_heads, D]. */
void brk_oracle_attention_partial(const float *q, const float *k, const float *v,
                                  int n_tokens, int n_heads, int n_kv_heads, int head_dim,
                                  int past_len, double scale, double softcap, int window,
                                  int key_lo, int key_hi, double *m, double *l, double *o);

/* Log-sum-exp combine of n_parts partials (extension): out = sum_s e^{m_s-M} o_s / sum_s e^{m_s-M} l_s.
 *   m, l: [n_parts, rows]; o: [n_parts, rows, D]; out: [rows, D] f32. */
void brk_oracle_combine(const double *m, const double *l, const double *o, int n_parts,
                        int rows, int head_dim, float *out);

/* matmulCpu (kernels.ts:3384) with [n][k] weights (matmul_t): o = a w^T, double sums. */
void brk_oracle_matmul_t(const float *a, const float *w, int m, int k, int n, float *o);

/* Non-causal attention as the attention_full gate computes it (kernels.ts:3168-3177). */
void brk_oracle_attention_full(const float *q, const float *k, const float *v, int n_tokens,
                               int n_heads, int n_kv_heads, int head_dim, int kv_len,
                               double scale, double softcap, float *o);

/* int8 KV quantisation — quantize_kv shader, shaders.ts:1673-1705 (symmetric amax/127,
 * per-(row, head) f32 scale, WGSL round() = round-half-to-even, clamp +-127), in the
 * shader's f32 arithmetic, written at row offset row_offset.
 * codes: [*, n_kv_heads*D] int8; scales: [*, n_kv_heads]. */
void brk_oracle_quantize_kv(const float *src, int rows, int n_kv_heads, int head_dim,
                            int row_offset, int8_t *codes, float *scales);

/* Batched decode attention over B independent sequences, OpenMP over (seq, head) — the
 * multi-core CPU baseline.  Per sequence b: q_b = q + b*n_tokens*n_heads*D,
 * k_b/v_b = k/v + b*seq_stride elements, past_len[b]; each (b, h) runs the attentionCpu loop.
 * threads <= 0 uses all host threads.  Returns the thread count used. */
int brk_oracle_attention_batch(const float *q, const float *k, const float *v, int batch,
                               long long seq_stride, int n_tokens, int n_heads,
                               int n_kv_heads, int head_dim, const int *past_len,
                               double scale, double softcap, int window, int threads,
                               float *o);

#ifdef __cplusplus
}
#endif

#endif /* BRK_ORACLE_H */
