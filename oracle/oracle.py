"""ctypes wrapper around the C oracle (oracle/liboracle.so) — TEST INFRASTRUCTURE ONLY.

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline legs import this module,
as the checker or as the timed CPU reference.  The product package never does.

Every function takes and returns numpy arrays in the reference's layouts
(src/lib/webgpu/kernels.ts:608-609): q/out ``[n_tokens, n_heads, D]``, k/v
``[kv_len, n_kv_heads, D]``, all float32.
"""
from __future__ import annotations

import ctypes
import math
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")
_lib = None

_f32p = ctypes.POINTER(ctypes.c_float)
_f64p = ctypes.POINTER(ctypes.c_double)
_i32p = ctypes.POINTER(ctypes.c_int)
_i8p = ctypes.POINTER(ctypes.c_int8)


def build() -> str:
    """Compile liboracle.so from oracle.c with the committed Makefile."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = ctypes.CDLL(_LIB_PATH)
        L.brk_oracle_rmsnorm.argtypes = [_f32p, _f32p, ctypes.c_int, ctypes.c_int, ctypes.c_double, ctypes.c_int, _f32p]
        L.brk_oracle_rope.argtypes = [_f32p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_double, _f32p]
        L.brk_oracle_rope_factors.argtypes = [_f32p, _f32p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_double, _f32p]
        L.brk_oracle_attention.argtypes = [_f32p, _f32p, _f32p] + [ctypes.c_int] * 5 + [ctypes.c_double, ctypes.c_double, ctypes.c_int, _f32p]
        L.brk_oracle_attention_partial.argtypes = ([_f32p, _f32p, _f32p] + [ctypes.c_int] * 5 + [ctypes.c_double, ctypes.c_double]
                                                   + [ctypes.c_int] * 3 + [_f64p, _f64p, _f64p])
        L.brk_oracle_combine.argtypes = [_f64p, _f64p, _f64p, ctypes.c_int, ctypes.c_int, ctypes.c_int, _f32p]
        L.brk_oracle_matmul_t.argtypes = [_f32p, _f32p, ctypes.c_int, ctypes.c_int, ctypes.c_int, _f32p]
        L.brk_oracle_attention_full.argtypes = [_f32p, _f32p, _f32p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                                ctypes.c_int, ctypes.c_int, ctypes.c_double, ctypes.c_double, _f32p]
        L.brk_oracle_quantize_kv.argtypes = [_f32p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, _i8p, _f32p]
        L.brk_oracle_attention_batch.argtypes = ([_f32p, _f32p, _f32p, ctypes.c_int, ctypes.c_longlong] + [ctypes.c_int] * 4
                                                 + [_i32p, ctypes.c_double, ctypes.c_double, ctypes.c_int, ctypes.c_int, _f32p])
        L.brk_oracle_attention_batch.restype = ctypes.c_int
        _lib = L
    return _lib


def _f32(a):
    a = np.ascontiguousarray(a, dtype=np.float32)
    return a, a.ctypes.data_as(_f32p)


def _f64(a):
    a = np.ascontiguousarray(a, dtype=np.float64)
    return a, a.ctypes.data_as(_f64p)


def rmsnorm(x, w, rows, dim, eps=1e-5, one_plus=False):
    """rmsnormCpu — kernels.ts:3395."""
    x, xp = _f32(x)
    w, wp = _f32(w)
    o = np.zeros(rows * dim, np.float32)
    lib().brk_oracle_rmsnorm(xp, wp, rows, dim, float(eps), int(bool(one_plus)), o.ctypes.data_as(_f32p))
    return o


def rope(x, rows, head_dim, n_heads, past_len=0, base=10000.0):
    """ropeCpu — kernels.ts:3445."""
    x, xp = _f32(x)
    o = np.zeros(x.size, np.float32)
    lib().brk_oracle_rope(xp, rows, head_dim, n_heads, past_len, float(base), o.ctypes.data_as(_f32p))
    return o


def rope_factors(x, ff, rows, head_dim, n_heads, past_len=0, base=10000.0):
    """ropeFactorsCpu — kernels.ts:3428."""
    x, xp = _f32(x)
    ff, fp = _f32(ff)
    o = np.zeros(x.size, np.float32)
    lib().brk_oracle_rope_factors(xp, fp, rows, head_dim, n_heads, past_len, float(base), o.ctypes.data_as(_f32p))
    return o


def attention(q, k, v, n_tokens, n_heads, n_kv_heads, head_dim, past_len=0, scale=None, softcap=0.0, window=0):
    """attentionCpu — kernels.ts:3466 (+ sliding window when window > 0)."""
    q, qp = _f32(q)
    k, kp = _f32(k)
    v, vp = _f32(v)
    o = np.zeros(n_tokens * n_heads * head_dim, np.float32)
    lib().brk_oracle_attention(qp, kp, vp, n_tokens, n_heads, n_kv_heads, head_dim, past_len,
                               math.nan if scale is None else float(scale), float(softcap), int(window),
                               o.ctypes.data_as(_f32p))
    return o


def attention_partial(q, k, v, n_tokens, n_heads, n_kv_heads, head_dim, past_len, key_lo, key_hi,
                      scale=None, softcap=0.0, window=0):
    """Split-KV partial (m, l, unnormalised o) over keys [key_lo, key_hi) — extension."""
    q, qp = _f32(q)
    k, kp = _f32(k)
    v, vp = _f32(v)
    rows = n_tokens * n_heads
    m = np.zeros(rows, np.float64)
    l = np.zeros(rows, np.float64)
    o = np.zeros(rows * head_dim, np.float64)
    lib().brk_oracle_attention_partial(qp, kp, vp, n_tokens, n_heads, n_kv_heads, head_dim, past_len,
                                       math.nan if scale is None else float(scale), float(softcap), int(window),
                                       int(key_lo), int(key_hi), m.ctypes.data_as(_f64p), l.ctypes.data_as(_f64p),
                                       o.ctypes.data_as(_f64p))
    return m, l, o


def combine(m, l, o, n_parts, rows, head_dim):
    """LSE combine of partials — extension."""
    m, mp = _f64(m)
    l, lp = _f64(l)
    o, op = _f64(o)
    out = np.zeros(rows * head_dim, np.float32)
    lib().brk_oracle_combine(mp, lp, op, n_parts, rows, head_dim, out.ctypes.data_as(_f32p))
    return out


def matmul_t(a, w, m, k, n):
    """matmulCpu (kernels.ts:3384) with [n][k] weights: a [m][k] . w^T, double sums."""
    a, ap = _f32(a)
    w, wp = _f32(w)
    o = np.zeros(m * n, np.float32)
    lib().brk_oracle_matmul_t(ap, wp, m, k, n, o.ctypes.data_as(_f32p))
    return o


def attention_full(q, k, v, n_tokens, n_heads, n_kv_heads, head_dim, kv_len, scale=None, softcap=0.0):
    """Non-causal attention of the attention_full gate (kernels.ts:3168-3177)."""
    q, qp = _f32(q)
    k, kp = _f32(k)
    v, vp = _f32(v)
    o = np.zeros(n_tokens * n_heads * head_dim, np.float32)
    lib().brk_oracle_attention_full(qp, kp, vp, n_tokens, n_heads, n_kv_heads, head_dim, kv_len,
                                    math.nan if scale is None else float(scale), float(softcap or 0.0),
                                    o.ctypes.data_as(_f32p))
    return o


def quantize_kv(src, rows, n_kv_heads, head_dim, row_offset=0, cap_rows=None):
    """quantize_kv shader (shaders.ts:1673) restated on the CPU."""
    src, sp = _f32(src)
    cap_rows = rows + row_offset if cap_rows is None else cap_rows
    codes = np.zeros(cap_rows * n_kv_heads * head_dim, np.int8)
    scales = np.zeros(cap_rows * n_kv_heads, np.float32)
    lib().brk_oracle_quantize_kv(sp, rows, n_kv_heads, head_dim, row_offset,
                                 codes.ctypes.data_as(_i8p), scales.ctypes.data_as(_f32p))
    return codes, scales


def dequantize_kv(codes, scales, rows, n_kv_heads, head_dim):
    """The dequant closure of the reference's q8 gate (kernels.ts:2577-2588): f32(code * scale)
    per element, scale per (row, head) -- one rounding of the exact product, as numpy's f32
    multiply gives."""
    c = np.asarray(codes, np.int8).reshape(rows, n_kv_heads, head_dim).astype(np.float32)
    s = np.asarray(scales, np.float32).reshape(rows, n_kv_heads, 1)
    return (c * s).astype(np.float32).ravel()


def attention_batch(q, k, v, batch, seq_stride, n_tokens, n_heads, n_kv_heads, head_dim, past_len,
                    scale=None, softcap=0.0, window=0, threads=0):
    """Multi-core batched attentionCpu (OpenMP over (seq, head)).  Returns (out, threads_used)."""
    q, qp = _f32(q)
    k, kp = _f32(k)
    v, vp = _f32(v)
    pl = np.ascontiguousarray(past_len, dtype=np.int32)
    o = np.zeros(batch * n_tokens * n_heads * head_dim, np.float32)
    used = lib().brk_oracle_attention_batch(qp, kp, vp, batch, int(seq_stride), n_tokens, n_heads, n_kv_heads,
                                            head_dim, pl.ctypes.data_as(_i32p),
                                            math.nan if scale is None else float(scale), float(softcap),
                                            int(window), int(threads), o.ctypes.data_as(_f32p))
    return o, used


def llama3_rope_factors(head_dim, base, factor, low_freq_factor, high_freq_factor, original_context):
    """Frequency divisors ff[i] for Meta's published llama3 RoPE scaling (the values
    llama.cpp stores as rope_freqs.weight, consumed by rope_factors, shaders.ts:1387).
    Written from the published formula: wavelengths shorter than orig/high keep their
    frequency, longer than orig/low are divided by `factor`, and the band between is
    interpolated linearly in orig/wavelength."""
    half = head_dim // 2
    ff = np.zeros(half, np.float32)
    low_wavelen = original_context / low_freq_factor
    high_wavelen = original_context / high_freq_factor
    for i in range(half):
        freq = 1.0 / base ** ((2.0 * i) / head_dim)
        wavelen = 2.0 * math.pi / freq
        if wavelen < high_wavelen:
            new = freq
        elif wavelen > low_wavelen:
            new = freq / factor
        else:
            smooth = (original_context / wavelen - low_freq_factor) / (high_freq_factor - low_freq_factor)
            new = (1.0 - smooth) * freq / factor + smooth * freq
        ff[i] = freq / new
    return ff
