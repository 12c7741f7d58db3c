"""int8 KV cache mode (setKvQuant, kernels.ts:1755-1760) on the GPU, through the C ABI.

- Quantisation (quantize_kv, shaders.ts:1673-1705): codes and scales bit-exact against the
  oracle's restatement, for the plain row store and for the fused append (QK-norm + RoPE in
  fp64, then the quantisation of the resulting f32 row, kernels.ts:1721-1725).
- Attention over the int8 cache (attention_q8kv / attention_decode_q8kv, shaders.ts:1711-1756,
  1856-1944): within the north-star tolerance of attentionCpu fed the dequantised K/V
  (f32(code * scale), kernels.ts:2577-2588) -- the reference's own q8 gate (kernels.ts:2570-2594)
  -- for the decode kernel (BASELINE shapes, windows, softcap, splits, partials) and the
  tensor-core prefill over dequantised staging.
"""
import os
import zlib

import numpy as np
import pytest

from oracle import oracle as O
from tests.util import assert_close, bits_equal, normal

pytestmark = pytest.mark.gpu


def _deq(kc, ks, rows, Hkv, D):
    return O.dequantize_kv(kc, ks, rows, Hkv, D)


@pytest.mark.parametrize("D,Hkv,rows", [(64, 2, 300), (128, 8, 129), (256, 4, 70), (4, 2, 5)])
def test_quantize_twin_bit_exact(eng, D, Hkv, rows):
    """quantizeKvReadback (kernels.ts:664) against the oracle, with all-zero rows (scale 1e-8),
    a row holding one large value, and values on exact code boundaries."""
    rng = np.random.default_rng(D * 1000 + rows)
    x = normal(rng, rows, Hkv, D) * rng.uniform(0.01, 30.0, (rows, Hkv, 1)).astype(np.float32)
    x[0] = 0.0
    x[1, 0] = 0.0
    x[1, 0, 0] = 1e4
    x[2, 0] = np.arange(D, dtype=np.float32) - D / 2  # integer grid: many half-way products
    codes, scales = eng.quantizeKvReadback(x.ravel(), rows, Hkv, D)
    rc, rs = O.quantize_kv(x.ravel(), rows, Hkv, D)
    assert bits_equal(scales, rs), "scales differ"
    assert bits_equal(codes, rc), f"{int((codes != rc).sum())} codes differ"
    # The reference gate's round-trip bound (kernels.ts:2593) on unit-scale inputs.
    y = normal(rng, rows, Hkv, D)
    c2, s2 = eng.quantizeKvReadback(y.ravel(), rows, Hkv, D)
    assert np.abs(_deq(c2, s2, rows, Hkv, D) - y.ravel()).max() <= 0.05


def _oracle_prologue(x, rows, D, n_heads, past, base, gain, eps):
    y = x
    if gain is not None:
        y = O.rmsnorm(y, gain, rows, D, eps, False)
    if base is not None:
        y = O.rope(y, rows, D, n_heads, past, base)
    return y


@pytest.mark.parametrize("name,Hq,Hkv,D,pasts,T", [
    ("qwen3", 32, 8, 128, [0, 100, 4093], 2),
    ("llama_d64", 32, 8, 64, [7, 65535], 1),
    ("gemma_d256", 8, 4, 256, [8191, 0], 1),
    ("prefill_rows", 32, 8, 128, [0, 1000], 300),
])
def test_append_q8_bit_exact(eng, name, Hq, Hkv, D, pasts, T):
    """Fused append into an int8 cache: rotated q bit-exact, K and V codes and scales equal to the
    oracle's quantize_kv of the oracle's f32 K (norm + RoPE) and of V."""
    import torch
    from brimkern_b200.engine import AttnConfig, KvCache, RopeTable
    rng = np.random.default_rng(zlib.crc32(name.encode()))
    B = len(pasts)
    base = 1e6
    kg = (1 + 0.02 * rng.standard_normal(D)).astype(np.float32)
    q_in, k_in, v_in = normal(rng, B, T, Hq, D), normal(rng, B, T, Hkv, D), normal(rng, B, T, Hkv, D)
    dev = eng.device
    rope = RopeTable(eng.ctx, D, base, None, max(pasts) + T)
    cfg = AttnConfig(Hq, Hkv, D, eps=1e-6, rope=rope, k_norm=torch.from_numpy(kg).to(dev))
    kv = KvCache(eng.ctx, 2, B, Hkv, D, max(pasts) + T, q8=True)
    q_out = torch.empty((B, T, Hq, D), dtype=torch.float32, device=dev)
    eng.appendKv(kv, 1, cfg, torch.from_numpy(q_in).to(dev), torch.from_numpy(k_in).to(dev),
                 torch.from_numpy(v_in).to(dev), q_out, pasts)
    eng.ctx.check()
    for b, past in enumerate(pasts):
        q_ref = _oracle_prologue(q_in[b].ravel(), T * Hq, D, Hq, past, base, None, 1e-6)
        assert bits_equal(q_out[b].cpu().numpy().ravel(), q_ref), f"{name}: rotated q differs"
        k_ref = _oracle_prologue(k_in[b].ravel(), T * Hkv, D, Hkv, past, base, kg, 1e-6)
        rkc, rks = O.quantize_kv(k_ref, T, Hkv, D)
        rvc, rvs = O.quantize_kv(v_in[b].ravel(), T, Hkv, D)
        kc, ks, vc, vs = kv.read_codes(1, b, past, T)
        assert bits_equal(kc.cpu().numpy().ravel(), rkc), f"{name}: K codes of sequence {b} differ"
        assert bits_equal(ks.cpu().numpy().ravel(), rks), f"{name}: K scales of sequence {b} differ"
        assert bits_equal(vc.cpu().numpy().ravel(), rvc), f"{name}: V codes of sequence {b} differ"
        assert bits_equal(vs.cpu().numpy().ravel(), rvs), f"{name}: V scales of sequence {b} differ"
        # Layer 0 is untouched (zero codes, zero scales).
        kc0, ks0, _, _ = kv.read_codes(0, b, past, T)
        assert not kc0.any().item() and not ks0.any().item()
    kv.close()
    rope.close()


ATT_GOLDEN = ["att_gqa_plain", "att_gqa_softcap", "att_decode_qwen05_past300", "att_decode_qwen05_nt10_past173",
              "att_decode_softcap_hd8", "att_decode_hd128_past70", "att_decode_hd256_gemma", "att_prefill_past0",
              "att_config1_qwen05_past1024"]


@pytest.mark.parametrize("name", ATT_GOLDEN)
@pytest.mark.parametrize("twin", ["attentionQ8Kv", "attentionQ8KvDecode"])
def test_q8_twins(eng, golden, name, twin):
    """The reference's q8 gate (kernels.ts:2570-2594) on the selfValidate shapes: quantise K/V,
    attend over the codes, compare with attentionCpu over the dequantised codes."""
    c, a = golden[name]
    T, Hq, Hkv, D, past = c["n_tokens"], c["n_heads"], c["n_kv_heads"], c["head_dim"], c["past_len"]
    L = past + T
    kc, ks = O.quantize_kv(a["k"], L, Hkv, D)
    vc, vs = O.quantize_kv(a["v"], L, Hkv, D)
    got = getattr(eng, twin)(a["q"], kc, ks, vc, vs, T, Hq, Hkv, D, past, c["scale"], c["softcap"] or 0.0)
    ref = O.attention(a["q"], _deq(kc, ks, L, Hkv, D), _deq(vc, vs, L, Hkv, D), T, Hq, Hkv, D, past, c["scale"],
                      c["softcap"] or 0.0)
    assert_close(got, ref, what=f"{twin}/{name}")
    # The packed Uint32 form of the codes (quantizeKvReadback's return type) is accepted as is.
    got32 = getattr(eng, twin)(a["q"], kc.view(np.uint32), ks, vc.view(np.uint32), vs, T, Hq, Hkv, D, past,
                               c["scale"], c["softcap"] or 0.0)
    assert np.array_equal(got32, got)


def _fill_q8(eng, kv, layer, rng, rows):
    """Quantised N(0,1) K/V rows for every sequence; returns the oracle's dequantised copies."""
    import torch
    ks, vs = [], []
    for b in range(kv.batch):
        k = normal(rng, rows, kv.n_kv_heads, kv.head_dim)
        v = normal(rng, rows, kv.n_kv_heads, kv.head_dim)
        kv.write_rows(layer, b, 0, torch.from_numpy(k).to(eng.device), torch.from_numpy(v).to(eng.device))
        kc, ksc = O.quantize_kv(k.ravel(), rows, kv.n_kv_heads, kv.head_dim)
        vc, vsc = O.quantize_kv(v.ravel(), rows, kv.n_kv_heads, kv.head_dim)
        ks.append(_deq(kc, ksc, rows, kv.n_kv_heads, kv.head_dim))
        vs.append(_deq(vc, vsc, rows, kv.n_kv_heads, kv.head_dim))
    return ks, vs


def _run_q8(eng, name, Hq, Hkv, D, pasts, T=1, scale=None, softcap=0.0, window=0, kernel="auto", splits=None,
            layers=2, layer=1):
    import torch
    from brimkern_b200.engine import AttnConfig, KvCache
    rng = np.random.default_rng(zlib.crc32(name.encode()))
    B = len(pasts)
    rows = max(pasts) + T
    kv = KvCache(eng.ctx, layers, B, Hkv, D, rows, q8=True)
    ks, vs = _fill_q8(eng, kv, layer, rng, rows)
    q = normal(rng, B, T, Hq, D)
    cfg = AttnConfig(Hq, Hkv, D, scale=scale, softcap=softcap, window=window)
    out = torch.full((B, T, Hq, D), float("nan"), dtype=torch.float32, device=eng.device)
    old = os.environ.get("BRK_DECODE_SPLITS")
    if splits is not None:
        os.environ["BRK_DECODE_SPLITS"] = str(splits)
    try:
        eng.recAttention(kv, layer, cfg, torch.from_numpy(q).to(eng.device), out, pasts, kernel=kernel)
        eng.ctx.check()
    finally:
        if splits is not None:
            if old is None:
                del os.environ["BRK_DECODE_SPLITS"]
            else:
                os.environ["BRK_DECODE_SPLITS"] = old
    got = out.cpu().numpy()
    kv.close()
    per_row = Hkv * D
    for b, past in enumerate(pasts):
        n = past + T
        ref = O.attention(q[b].ravel(), ks[b][:n * per_row], vs[b][:n * per_row], T, Hq, Hkv, D, past, scale,
                          softcap, window)
        assert_close(got[b].ravel(), ref, what=f"{name} seq {b} (past {past})")


def test_q8_decode_qwen3(eng):
    _run_q8(eng, "q8_qwen3", 32, 8, 128, [4095, 1000, 63, 0])


def test_q8_decode_gemma_window_softcap(eng):
    _run_q8(eng, "q8_gemma_win", 8, 4, 256, [8191, 5000, 100], scale=1 / 16, softcap=50.0, window=4096)
    _run_q8(eng, "q8_gemma_glob", 8, 4, 256, [8191, 70], scale=1 / 16, softcap=50.0)


def test_q8_decode_llama_long(eng):
    _run_q8(eng, "q8_llama_long", 32, 8, 64, [32767], layers=1, layer=0)


@pytest.mark.parametrize("past", [0, 1, 3, 62, 63, 64, 65, 129, 300])
def test_q8_ragged(eng, past):
    _run_q8(eng, f"q8_ragged{past}", 14, 2, 64, [past])


@pytest.mark.parametrize("splits", [1, 3, 4, 16])
def test_q8_forced_splits(eng, splits):
    _run_q8(eng, f"q8_split{splits}", 32, 8, 128, [2047, 999], splits=splits)


def test_q8_multi_token_and_window(eng):
    _run_q8(eng, "q8_multi_tok", 14, 2, 64, [173, 40], T=10)
    # Window starts that are not multiples of 4 (the kernel rounds the first key down and masks).
    _run_q8(eng, "q8_win_multi", 8, 2, 128, [301, 78, 999], T=5, window=65)
    _run_q8(eng, "q8_win_d256", 8, 4, 256, [1001], T=3, window=37, softcap=30.0)


@pytest.mark.parametrize("D", [64, 128])
def test_q8_prefill_kernel(eng, D):
    """Tensor-core prefill over the int8 cache (dequantised staging), causal with a chunk offset."""
    _run_q8(eng, f"q8_prefill{D}", 16, 4, D, [0, 300], T=200, kernel="prefill")
    _run_q8(eng, f"q8_prefill_win{D}", 8, 2, D, [513], T=130, kernel="prefill", window=200, softcap=20.0)


def test_q8_layer_step_and_prefill_step(eng):
    """attentionLayer (append + decode as one step) and prefillStep (append + fused-prologue
    prefill) on an int8 cache against the oracle chain norm -> rope -> quantise -> attention."""
    import torch
    from brimkern_b200.engine import AttnConfig, KvCache, RopeTable
    rng = np.random.default_rng(77)
    Hq, Hkv, D, base = 32, 8, 128, 1e6
    B, P, C = 2, 256, 1  # prompt of P tokens, then C decode token
    dev = eng.device
    qg = (1 + 0.02 * rng.standard_normal(D)).astype(np.float32)
    kg = (1 + 0.02 * rng.standard_normal(D)).astype(np.float32)
    rope = RopeTable(eng.ctx, D, base, None, P + C)
    cfg = AttnConfig(Hq, Hkv, D, eps=1e-6, rope=rope, q_norm=torch.from_numpy(qg).to(dev),
                     k_norm=torch.from_numpy(kg).to(dev))
    kv = KvCache(eng.ctx, 1, B, Hkv, D, P + C, q8=True)
    q_all, k_all, v_all = normal(rng, B, P + C, Hq, D), normal(rng, B, P + C, Hkv, D), normal(rng, B, P + C, Hkv, D)
    out_p = torch.empty((B, P, Hq, D), dtype=torch.float32, device=dev)
    eng.prefillStep(kv, 0, cfg, torch.from_numpy(q_all[:, :P].copy()).to(dev), torch.from_numpy(k_all[:, :P].copy()).to(dev),
                    torch.from_numpy(v_all[:, :P].copy()).to(dev), out_p, [0, 0])
    out_d = eng.attentionLayer(kv, 0, cfg, torch.from_numpy(q_all[:, P:].copy()).to(dev),
                               torch.from_numpy(k_all[:, P:].copy()).to(dev), torch.from_numpy(v_all[:, P:].copy()).to(dev),
                               [P, P])
    eng.ctx.check()
    got = np.concatenate([out_p.cpu().numpy(), out_d.cpu().numpy()], axis=1)
    L = P + C
    for b in range(B):
        qr = _oracle_prologue(q_all[b].ravel(), L * Hq, D, Hq, 0, base, qg, 1e-6)
        kr = _oracle_prologue(k_all[b].ravel(), L * Hkv, D, Hkv, 0, base, kg, 1e-6)
        kc, ks = O.quantize_kv(kr, L, Hkv, D)
        vc, vs = O.quantize_kv(v_all[b].ravel(), L, Hkv, D)
        ref = O.attention(qr, _deq(kc, ks, L, Hkv, D), _deq(vc, vs, L, Hkv, D), L, Hq, Hkv, D, 0)
        assert_close(got[b].ravel(), ref, what=f"q8 prefill+decode seq {b}")
    kv.close()
    rope.close()


def test_q8_partials_and_combine(eng):
    """Sequence-sharded partials over int8 shards, merged by the LSE combine."""
    import torch
    from brimkern_b200.engine import AttnConfig, KvCache
    rng = np.random.default_rng(21)
    Hq, Hkv, D, B, L, N = 32, 8, 64, 2, 4096, 4
    k, v, q = normal(rng, B, L, Hkv, D), normal(rng, B, L, Hkv, D), normal(rng, B, 1, Hq, D)
    rows = B * Hq
    parts_ml = torch.empty((N, rows, 2), dtype=torch.float32, device=eng.device)
    parts_o = torch.empty((N, rows, D), dtype=torch.float32, device=eng.device)
    shard = L // N
    for r in range(N):
        kv = KvCache(eng.ctx, 1, B, Hkv, D, shard, q8=True)
        for b in range(B):
            kv.write_rows(0, b, 0, torch.from_numpy(k[b, r * shard:(r + 1) * shard].copy()).to(eng.device),
                          torch.from_numpy(v[b, r * shard:(r + 1) * shard].copy()).to(eng.device))
        eng.decodePartial(kv, 0, AttnConfig(Hq, Hkv, D, kv_offset=r * shard), torch.from_numpy(q).to(eng.device),
                          parts_ml[r], parts_o[r], [L - 1] * B)
        eng.ctx.check()
        kv.close()
    out = torch.empty((rows, D), dtype=torch.float32, device=eng.device)
    eng.combine(N, rows, D, parts_ml, parts_o, out)
    eng.ctx.check()
    got = out.cpu().numpy().reshape(B, Hq, D)
    for b in range(B):
        kd, vd = [], []
        for r in range(N):  # each shard quantises its own rows (per-row scales: same as the whole)
            kc, ks = O.quantize_kv(k[b, r * shard:(r + 1) * shard].ravel(), shard, Hkv, D)
            vc, vs = O.quantize_kv(v[b, r * shard:(r + 1) * shard].ravel(), shard, Hkv, D)
            kd.append(_deq(kc, ks, shard, Hkv, D))
            vd.append(_deq(vc, vs, shard, Hkv, D))
        ref = O.attention(q[b].ravel(), np.concatenate(kd), np.concatenate(vd), 1, Hq, Hkv, D, L - 1)
        assert_close(got[b].ravel(), ref, what=f"q8 sharded seq {b}")


def test_q8_grow_keeps_rows_and_engine_mode(eng):
    """ensureKv growth copies codes and scales; setKvQuant switches the engine's cache type."""
    import torch
    from brimkern_b200.engine import KvCache
    rng = np.random.default_rng(3)
    kv = KvCache(eng.ctx, 2, 2, 2, 128, 1001, q8=True)
    k, v = normal(rng, 1001, 2, 128), normal(rng, 1001, 2, 128)
    kv.write_rows(1, 1, 0, torch.from_numpy(k).to(eng.device), torch.from_numpy(v).to(eng.device))
    before = [t.cpu().numpy() for t in kv.read_codes(1, 1, 0, 1001)]
    kv.grow(1500)
    assert kv.capacity == 2025
    after = [t.cpu().numpy() for t in kv.read_codes(1, 1, 0, 1001)]
    for x, y in zip(before, after):
        assert bits_equal(x, y)
    tail = kv.read_codes(1, 1, 1001, 1024)
    assert not any(t.any().item() for t in tail)
    kv.close()
    eng.setKvQuant(True)
    c = eng.ensureKv(1, 10, 1, 2, 64)
    assert c.q8 and c.capacity == 1024
    eng.setKvQuant(False)
    assert eng.kvGpu is None
    assert not eng.ensureKv(1, 10, 1, 2, 64).q8
    eng.resetKvGpu()


def test_q8_prefill_reserved_stage_allocates_nothing(eng):
    """With the staging buffer reserved by brk_ctx_reserve_stage's documented size (2 * batch *
    n_kv_heads * rows * head_dim * 2 bytes), int8-cache prefill calls of that size or smaller
    leave device free memory unchanged, and still match attentionCpu over the dequantised codes."""
    import ctypes

    import torch
    from brimkern_b200 import _lib as L
    from brimkern_b200.engine import AttnConfig, Context, KvCache
    rng = np.random.default_rng(4711)
    Hq, Hkv, D, T = 16, 4, 128, 256
    pasts = [768, 100]
    B, rows = len(pasts), max(pasts) + T
    ctx = Context(0)
    kv = KvCache(ctx, 1, B, Hkv, D, rows, q8=True)
    ks, vs = _fill_q8(eng, kv, 0, rng, rows)
    ctx.reserve_stage(2 * B * Hkv * rows * D * 2)
    cfg = AttnConfig(Hq, Hkv, D)
    q = torch.from_numpy(normal(rng, B, T, Hq, D)).to(eng.device)
    out = torch.full((B, T, Hq, D), float("nan"), dtype=torch.float32, device=eng.device)
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info(eng.device)[0]
    p = cfg.params()
    for call_pasts in (pasts, [pasts[0] - 64, pasts[1]], pasts):
        pos = (ctypes.c_int32 * B)(*call_pasts)
        rc = L.lib().brk_attn_prefill(ctx.handle, kv.handle, 0, ctypes.byref(p), B, T, pos, q.data_ptr(),
                                      out.data_ptr(), torch.cuda.current_stream().cuda_stream)
        assert rc == 0, L.lib().brk_last_error()
    ctx.check()
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info(eng.device)[0] == free0, "an int8 prefill call allocated device memory"
    got = out.cpu().numpy()
    per_row = Hkv * D
    qh = q.cpu().numpy()
    for b, past in enumerate(pasts):
        n = past + T
        ref = O.attention(qh[b].ravel(), ks[b][:n * per_row], vs[b][:n * per_row], T, Hq, Hkv, D, past)
        assert_close(got[b].ravel(), ref, what=f"reserved-stage int8 prefill seq {b}")
    kv.close()
    ctx.close()
