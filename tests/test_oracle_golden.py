"""Pin the C oracle to the reference: bit-exact against fixtures made by executing the
reference's own attentionCpu / ropeCpu / ropeFactorsCpu / rmsnormCpu source
(src/lib/webgpu/kernels.ts:3395-3495) and the attention_full gate's reference loop
(kernels.ts:3171-3177) with tests/golden/jsmini.py."""
import math

import numpy as np
import pytest

from oracle import oracle as O


def _run(c, a):
    fn = c["fn"]
    if fn == "ropeCpu":
        return O.rope(a["x"], c["rows"], c["head_dim"], c["n_heads"], c["past_len"], c["base"])
    if fn == "ropeFactorsCpu":
        return O.rope_factors(a["x"], a["ff"], c["rows"], c["head_dim"], c["n_heads"], c["past_len"], c["base"])
    if fn == "rmsnormCpu":
        eps = 1e-5 if c["eps"] is None else c["eps"]  # kernels.ts:3395 default eps
        return O.rmsnorm(a["x"], a["w"], c["rows"], c["dim"], eps, bool(c["one_plus"]))
    if fn == "attentionFullGate":
        return O.attention_full(a["q"], a["k"], a["v"], c["n_tokens"], c["n_heads"], c["n_heads"], c["head_dim"],
                                c["kv_len"])
    return O.attention(a["q"], a["k"], a["v"], c["n_tokens"], c["n_heads"], c["n_kv_heads"], c["head_dim"],
                       c["past_len"], c["scale"], c["softcap"] or 0.0)


def test_golden_cases_present(golden):
    assert len(golden) >= 23
    fns = {c["fn"] for c, _ in golden.values()}
    assert fns == {"ropeCpu", "ropeFactorsCpu", "rmsnormCpu", "attentionCpu", "attentionFullGate"}


@pytest.mark.parametrize("name", [
    "rope_small", "rope_ff_ones", "rope_ff_plain", "rope_ff_distinct", "rope_qwen3_pos4095",
    "rope_llama_pos131071", "rmsnorm_qk_small", "rmsnorm_qk_hd128", "rmsnorm_oneplus", "rmsnorm_default_eps",
    "att_gqa_plain", "att_gqa_softcap", "att_decode_qwen05_past300", "att_decode_qwen05_nt10_past173",
    "att_decode_softcap_hd8", "att_decode_hd128_past70", "att_decode_hd256_gemma", "att_prefill_past0",
    "att_config1_qwen05_past1024", "full_gate_cross", "full_sdturbo_self", "full_clip_cross", "full_sdxs_hd160",
])
def test_oracle_bit_exact_vs_reference(golden, name):
    c, a = golden[name]
    got = _run(c, a)
    ref = a["out"]
    assert got.shape == ref.shape
    mism = int((got.view(np.uint32) != ref.view(np.uint32)).sum())
    assert mism == 0, f"{name}: {mism} of {ref.size} f32 values differ from the reference"


def test_rope_factors_ones_equals_rope(golden):
    """The reference's own invariant (kernels.ts:2531-2532): ff == 1 everywhere is plain RoPE."""
    _, a = golden["rope_ff_ones"]
    _, b = golden["rope_ff_plain"]
    assert np.array_equal(a["out"].view(np.uint32), b["out"].view(np.uint32))


def test_window_infinite_is_reference(golden):
    """Sliding-window extension, degenerate case: W >= kv_len reproduces attentionCpu exactly."""
    c, a = golden["att_decode_qwen05_nt10_past173"]
    kv = c["past_len"] + c["n_tokens"]
    got = O.attention(a["q"], a["k"], a["v"], c["n_tokens"], c["n_heads"], c["n_kv_heads"], c["head_dim"],
                      c["past_len"], None, 0.0, window=kv)
    assert np.array_equal(got.view(np.uint32), a["out"].view(np.uint32))


def test_window_masks_old_keys():
    """W = 1 attends only to the token's own key, so the output is exactly that V row."""
    rng = np.random.default_rng(1)
    nT, nH, nKv, D, past = 3, 4, 2, 8, 5
    q = rng.standard_normal(nT * nH * D).astype(np.float32)
    k = rng.standard_normal((past + nT) * nKv * D).astype(np.float32)
    v = rng.standard_normal((past + nT) * nKv * D).astype(np.float32)
    out = O.attention(q, k, v, nT, nH, nKv, D, past, None, 0.0, window=1).reshape(nT, nH, D)
    vv = v.reshape(past + nT, nKv, D)
    for t in range(nT):
        for h in range(nH):
            np.testing.assert_array_equal(out[t, h], vv[past + t, h // (nH // nKv)])


def test_prefill_then_decode_equals_prefill(golden):
    """KV-cache equivalence (kernels.ts:2742-2759) restated on attention: the last row of a
    3-token prefill equals a 1-token decode at pastLen 2 over the same K/V."""
    rng = np.random.default_rng(7)
    nH, nKv, D = 4, 2, 4
    q = rng.random(3 * nH * D).astype(np.float32) * 2 - 1
    k = rng.random(3 * nKv * D).astype(np.float32) * 2 - 1
    v = rng.random(3 * nKv * D).astype(np.float32) * 2 - 1
    full = O.attention(q, k, v, 3, nH, nKv, D, 0)
    dec = O.attention(q[2 * nH * D:], k, v, 1, nH, nKv, D, 2)
    np.testing.assert_array_equal(full[2 * nH * D:], dec)


@pytest.mark.parametrize("splits", [1, 2, 3, 7])
def test_partials_combine_equals_attention(golden, splits):
    """Split-KV extension: LSE-combining per-range partials reproduces attentionCpu."""
    c, a = golden["att_decode_qwen05_past300"]
    nT, nH, nKv, D, past = c["n_tokens"], c["n_heads"], c["n_kv_heads"], c["head_dim"], c["past_len"]
    kv = past + nT
    bounds = np.linspace(0, kv, splits + 1).astype(int)
    ms, ls, os_ = [], [], []
    for s in range(splits):
        m, l, o = O.attention_partial(a["q"], a["k"], a["v"], nT, nH, nKv, D, past, bounds[s], bounds[s + 1])
        ms.append(m), ls.append(l), os_.append(o)
    out = O.combine(np.concatenate(ms), np.concatenate(ls), np.concatenate(os_), splits, nT * nH, D)
    np.testing.assert_allclose(out, a["out"], rtol=1e-5, atol=1e-6)


def test_quantize_kv_roundtrip():
    """quantize_kv (shaders.ts:1673-1705): round-trip error bound of the reference's gate
    (kernels.ts:2592, max abs <= 0.05 for inputs in [-1, 1))."""
    rng = np.random.default_rng(3)
    rows, nKv, D = 9, 2, 16
    src = (rng.random(rows * nKv * D) * 2 - 1).astype(np.float32)
    codes, scales = O.quantize_kv(src, rows, nKv, D)
    deq = codes.reshape(rows, nKv, D).astype(np.float32) * scales.reshape(rows, nKv, 1)
    assert np.abs(deq.ravel() - src).max() <= 0.05
    assert codes.min() >= -127 and codes.max() <= 127


def test_llama3_factors_shape():
    ff = O.llama3_rope_factors(64, 500000.0, 32.0, 1.0, 4.0, 8192)
    assert ff.shape == (32,)
    assert ff[0] == 1.0 and math.isclose(float(ff[-1]), 32.0, rel_tol=1e-6)
    assert np.all(np.diff(ff) >= 0)


def test_batch_matches_single():
    rng = np.random.default_rng(5)
    B, nH, nKv, D, cap = 3, 4, 2, 16, 20
    past = np.array([5, 0, 12], np.int32)
    q = rng.standard_normal(B * nH * D).astype(np.float32)
    k = rng.standard_normal(B * cap * nKv * D).astype(np.float32)
    v = rng.standard_normal(B * cap * nKv * D).astype(np.float32)
    out, used = O.attention_batch(q, k, v, B, cap * nKv * D, 1, nH, nKv, D, past, threads=2)
    assert used >= 1
    for b in range(B):
        s = slice(b * cap * nKv * D, (b + 1) * cap * nKv * D)
        ref = O.attention(q[b * nH * D:(b + 1) * nH * D], k[s], v[s], 1, nH, nKv, D, int(past[b]))
        np.testing.assert_array_equal(out[b * nH * D:(b + 1) * nH * D], ref)
