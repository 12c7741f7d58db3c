"""Decode attention parity (GPU), through the C ABI: outputs within the north-star tolerance
(|err| <= 2e-3 + 1e-2 |ref|) of the oracle (attentionCpu, kernels.ts:3466) fed the same
fp16-rounded K/V; the reference's own selfValidate shapes (kernels.ts:2556-2640) plus the
BASELINE config shapes, windows, softcap, split-KV and sequence-sharded partials."""
import os
import zlib

import numpy as np
import pytest

from oracle import oracle as O
from tests.util import assert_close, f16_round, normal

pytestmark = pytest.mark.gpu

ATT_GOLDEN = ["att_gqa_plain", "att_gqa_softcap", "att_decode_qwen05_past300", "att_decode_qwen05_nt10_past173",
              "att_decode_softcap_hd8", "att_decode_hd128_past70", "att_decode_hd256_gemma", "att_prefill_past0",
              "att_config1_qwen05_past1024"]


@pytest.mark.parametrize("name", ATT_GOLDEN)
@pytest.mark.parametrize("twin", ["attention", "attentionDecode"])
def test_attention_twins(eng, golden, name, twin):
    """Readback twins (kernels.ts:610, 624) on the selfValidate shapes."""
    c, a = golden[name]
    args = (c["n_tokens"], c["n_heads"], c["n_kv_heads"], c["head_dim"], c["past_len"])
    got = getattr(eng, twin)(a["q"], a["k"], a["v"], *args, c["scale"], c["softcap"] or 0.0)
    ref = O.attention(a["q"], f16_round(a["k"]), f16_round(a["v"]), *args, c["scale"], c["softcap"] or 0.0)
    assert_close(got, ref, what=f"{twin}/{name}")
    # Against the reference's own f32-KV output the only extra error is the fp16 storage of K/V.
    assert np.abs(got - a["out"]).max() < 2e-2


def _fill_cache(eng, kv, layer, rng, rows_per_seq):
    """Random N(0,1) K/V rows for every sequence; returns the fp16-rounded host copies."""
    import torch
    ks, vs = [], []
    for b in range(kv.batch):
        k = normal(rng, rows_per_seq, kv.n_kv_heads, kv.head_dim)
        v = normal(rng, rows_per_seq, kv.n_kv_heads, kv.head_dim)
        kv.write_rows(layer, b, 0, torch.from_numpy(k).to(eng.device), torch.from_numpy(v).to(eng.device))
        ks.append(f16_round(k))
        vs.append(f16_round(v))
    return ks, vs


def _run_decode(eng, name, Hq, Hkv, D, pasts, T=1, scale=None, softcap=0.0, window=0, kernel="auto", splits=None,
                layers=2, layer=1):
    import torch
    from brimkern_b200.engine import AttnConfig, KvCache
    rng = np.random.default_rng(zlib.crc32(name.encode()))
    B = len(pasts)
    rows = max(pasts) + T
    kv = KvCache(eng.ctx, layers, B, Hkv, D, rows)
    ks, vs = _fill_cache(eng, kv, layer, rng, rows)
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
    for b, past in enumerate(pasts):
        n = past + T
        ref = O.attention(q[b].ravel(), ks[b][:n].ravel(), vs[b][:n].ravel(), T, Hq, Hkv, D, past, scale, softcap,
                          window)
        assert_close(got[b].ravel(), ref, what=f"{name} seq {b} (past {past})")


def test_config2_qwen3_shape(eng):
    """Qwen3-4B decode: 32 q / 8 kv heads, D 128, KV length 4096 (and ragged shorter ones)."""
    _run_decode(eng, "qwen3", 32, 8, 128, [4095, 1000, 63, 0])


def test_config4_gemma_window_softcap(eng):
    """Gemma-2-2B decode: D 256, softcap 50, scale 1/16, sliding window 4096 and global."""
    _run_decode(eng, "gemma_win", 8, 4, 256, [8191, 5000, 100], scale=1 / 16, softcap=50.0, window=4096)
    _run_decode(eng, "gemma_glob", 8, 4, 256, [8191, 70], scale=1 / 16, softcap=50.0)


def test_config5_llama_long(eng):
    """Llama-3.2-1B long context on one GPU: D 64, KV length 32768 (split-KV exercised)."""
    _run_decode(eng, "llama_long", 32, 8, 64, [32767], layers=1, layer=0)


@pytest.mark.parametrize("past", [0, 1, 62, 63, 64, 65, 127, 129, 173, 300])
def test_ragged_lengths(eng, past):
    """Partial 64-key tiles and tiny caches (the reference's 'partial tile' gate, kernels.ts:2611)."""
    _run_decode(eng, f"ragged{past}", 14, 2, 64, [past])


@pytest.mark.parametrize("splits", [1, 2, 3, 4, 16])
def test_forced_splits(eng, splits):
    _run_decode(eng, f"split{splits}", 32, 8, 128, [2047, 999], splits=splits)


def test_multi_token_decode(eng):
    """nT = 10 with pastLen 173 at the Qwen2.5-0.5B shape (group 7 -> 70 rows, 5 row tiles)."""
    _run_decode(eng, "multi_tok", 14, 2, 64, [173, 40], T=10)


def test_window_multi_token(eng):
    _run_decode(eng, "win_multi", 8, 2, 128, [300, 77], T=5, window=64)


def test_prefill_then_decode_equals_prefill(eng):
    """KV-cache equivalence (kernels.ts:2742-2759): decoding token 3 after a 2-token prefill
    gives the last row of a 3-token prefill over the same cache."""
    import torch
    from brimkern_b200.engine import AttnConfig, KvCache
    rng = np.random.default_rng(11)
    Hq, Hkv, D = 4, 2, 64
    kv = KvCache(eng.ctx, 1, 1, Hkv, D, 3)
    _fill_cache(eng, kv, 0, rng, 3)
    q = torch.from_numpy(normal(rng, 1, 3, Hq, D)).to(eng.device)
    cfg = AttnConfig(Hq, Hkv, D)
    full = torch.empty_like(q)
    eng.recAttention(kv, 0, cfg, q, full, [0])
    last = torch.empty((1, 1, Hq, D), dtype=torch.float32, device=eng.device)
    eng.recAttention(kv, 0, cfg, q[:, 2:3].contiguous(), last, [2])
    eng.ctx.check()
    np.testing.assert_allclose(last.cpu().numpy()[0, 0], full.cpu().numpy()[0, 2], rtol=1e-5, atol=1e-6)
    kv.close()


def test_sequence_sharded_partials_combine(eng):
    """Config-5 sharding emulated on one GPU: each shard holds a contiguous range of positions
    (kv_offset), yields (m, l, o) partials; the LSE combine equals full attention."""
    import torch
    from brimkern_b200.engine import AttnConfig, KvCache
    rng = np.random.default_rng(5)
    Hq, Hkv, D, B, L, N = 32, 8, 64, 2, 8192, 4
    k = normal(rng, B, L, Hkv, D)
    v = normal(rng, B, L, Hkv, D)
    q = normal(rng, B, 1, Hq, D)
    past = [L - 1, L - 1]
    rows = B * Hq
    parts_ml = torch.empty((N, rows, 2), dtype=torch.float32, device=eng.device)
    parts_o = torch.empty((N, rows, D), dtype=torch.float32, device=eng.device)
    shard = L // N
    for r in range(N):
        kv = KvCache(eng.ctx, 1, B, Hkv, D, shard)
        for b in range(B):
            kv.write_rows(0, b, 0, torch.from_numpy(k[b, r * shard:(r + 1) * shard]).to(eng.device),
                          torch.from_numpy(v[b, r * shard:(r + 1) * shard]).to(eng.device))
        cfg = AttnConfig(Hq, Hkv, D, kv_offset=r * shard)
        eng.decodePartial(kv, 0, cfg, torch.from_numpy(q).to(eng.device), parts_ml[r], parts_o[r], past)
        eng.ctx.check()
        kv.close()
    out = torch.empty((rows, D), dtype=torch.float32, device=eng.device)
    eng.combine(N, rows, D, parts_ml, parts_o, out)
    eng.ctx.check()
    got = out.cpu().numpy().reshape(B, Hq, D)
    for b in range(B):
        ref = O.attention(q[b].ravel(), f16_round(k[b]).ravel(), f16_round(v[b]).ravel(), 1, Hq, Hkv, D, past[b])
        assert_close(got[b].ravel(), ref, what=f"sharded seq {b}")


def test_partial_matches_oracle_partial(eng):
    """The (m, l, o) partial itself against the oracle's partial over the same key range."""
    import torch
    from brimkern_b200.engine import AttnConfig, KvCache
    rng = np.random.default_rng(9)
    Hq, Hkv, D, L = 8, 2, 128, 1000
    kv = KvCache(eng.ctx, 1, 1, Hkv, D, L)
    ks, vs = _fill_cache(eng, kv, 0, rng, L)
    q = normal(rng, 1, 1, Hq, D)
    ml = torch.empty((Hq, 2), dtype=torch.float32, device=eng.device)
    o = torch.empty((Hq, D), dtype=torch.float32, device=eng.device)
    eng.decodePartial(kv, 0, AttnConfig(Hq, Hkv, D), torch.from_numpy(q).to(eng.device), ml, o, [L - 1])
    eng.ctx.check()
    m_ref, l_ref, o_ref = O.attention_partial(q.ravel(), ks[0].ravel(), vs[0].ravel(), 1, Hq, Hkv, D, L - 1, 0, L)
    ml = ml.cpu().numpy()
    # m may differ by the fp16 rounding of q; compare the normalised output and l * e^m.
    np.testing.assert_allclose(ml[:, 0], m_ref, atol=5e-3)
    np.testing.assert_allclose(ml[:, 1] * np.exp(ml[:, 0] - m_ref), l_ref, rtol=1e-2)
    assert_close(o.cpu().numpy() / ml[:, 1:2], (o_ref.reshape(Hq, D) / l_ref[:, None]).astype(np.float32))
    kv.close()


def test_errors(eng):
    import torch
    from brimkern_b200._lib import BRK_ERR_CAPACITY, BRK_ERR_INVALID, BRK_ERR_UNSUPPORTED, BrkError
    from brimkern_b200.engine import AttnConfig, KvCache
    with pytest.raises(BrkError) as ei:
        KvCache(eng.ctx, 1, 1, 2, 96, 16)
    assert ei.value.code == BRK_ERR_UNSUPPORTED
    kv = KvCache(eng.ctx, 1, 2, 2, 64, 16)
    q = torch.zeros((2, 1, 4, 64), dtype=torch.float32, device=eng.device)
    out = torch.empty_like(q)
    with pytest.raises(BrkError) as ei:  # position 16 needs 17 rows
        eng.recAttention(kv, 0, AttnConfig(4, 2, 64), q, out, [16, 0])
    assert ei.value.code == BRK_ERR_CAPACITY
    with pytest.raises(BrkError) as ei:  # 4 q heads over 3 kv heads
        eng.recAttention(kv, 0, AttnConfig(4, 3, 64), q, out, [1, 0])
    assert ei.value.code == BRK_ERR_INVALID
    with pytest.raises(BrkError) as ei:
        eng.recAttention(kv, 1, AttnConfig(4, 2, 64), q, out, [1, 0])
    assert ei.value.code == BRK_ERR_INVALID
    eng.ctx.check()
    kv.close()
