"""The one-token decode step (brk_attn_step with n_tokens = 1), whose append runs inside the
decode launch, against the oracle chain rmsnormCpu -> ropeCpu -> cache store -> attentionCpu
(kernels.ts:3395-3495) over the model variants the step has to cover: head dims 64 / 128 / 256,
GQA groups 1-8, QK-norm on and off (and the 1 + w gain convention), RoPE on and off, softcap,
sliding windows, a sequence-sharded cache (kv_offset), ragged positions, fp16 and int8 caches.

- The new K / V rows: bit for bit the oracle's (fp16 round to nearest even of the f32 rows, or
  quantize_kv's codes and scales for int8), and rows next to them untouched.
- The rotated q (q_work): within f32 rounding of the oracle's (the fused path rotates q in f32).
- The attention output: the north-star tolerance against attentionCpu fed the cache's rows.
"""
import zlib

import numpy as np
import pytest

from oracle import oracle as O
from tests.util import assert_close, bits_equal, f16_round, normal

pytestmark = pytest.mark.gpu

CASES = [
    # name, Hq, Hkv, D, pasts, qk_norm, one_plus, rope, softcap, window, kv_offset, q8
    ("qwen3", 32, 8, 128, [4095, 1000, 63, 0], True, False, True, 0.0, 0, 0, False),
    ("qwen3_q8", 32, 8, 128, [4095, 1000, 63, 0], True, False, True, 0.0, 0, 0, True),
    ("gemma_win", 8, 4, 256, [8191, 5000, 100], False, False, True, 50.0, 4096, 0, False),
    ("gemma_q8", 8, 4, 256, [8191, 70], False, False, True, 50.0, 0, 0, True),
    ("llama_d64", 32, 8, 64, [2047, 1500, 3], False, False, True, 0.0, 0, 0, False),
    ("mha_d64_onep", 8, 8, 64, [300, 0, 77], True, True, True, 0.0, 0, 0, False),
    ("qwen05_g7", 14, 2, 64, [1024, 999], False, False, True, 0.0, 0, 0, False),
    ("g8_norope", 16, 2, 128, [700, 129], True, False, False, 0.0, 0, 0, False),
    ("shard_offset", 32, 8, 64, [6143, 5000], False, False, True, 0.0, 0, 4096, False),
    ("q8_d64_win", 16, 4, 64, [999, 64], True, False, True, 20.0, 65, 0, True),
]


@pytest.mark.parametrize("name,Hq,Hkv,D,pasts,qk_norm,one_plus,rope,softcap,window,kv_offset,q8", CASES)
def test_fused_step_matches_oracle_chain(eng, name, Hq, Hkv, D, pasts, qk_norm, one_plus, rope, softcap, window,
                                         kv_offset, q8):
    import torch
    from brimkern_b200.engine import AttnConfig, KvCache, RopeTable
    rng = np.random.default_rng(zlib.crc32(name.encode()))
    dev = eng.device
    B = len(pasts)
    base = 1e6
    rows = max(pasts) + 1 - kv_offset
    kv = KvCache(eng.ctx, 2, B, Hkv, D, rows, q8=q8)
    hist_k, hist_v = [], []
    for b, past in enumerate(pasts):
        n = past - kv_offset
        k = normal(rng, rows, Hkv, D)
        v = normal(rng, rows, Hkv, D)
        kv.write_rows(1, b, 0, torch.from_numpy(k).to(dev), torch.from_numpy(v).to(dev))
        hist_k.append(k[:n])
        hist_v.append(v[:n])
    qg = (1 + 0.02 * rng.standard_normal(D)).astype(np.float32) if qk_norm else None
    kg = (1 + 0.02 * rng.standard_normal(D)).astype(np.float32) if qk_norm else None
    table = RopeTable(eng.ctx, D, base, None, max(pasts) + 1) if rope else None
    t = lambda a: None if a is None else torch.from_numpy(a).to(dev)  # noqa: E731
    scale = 1 / 16 if D == 256 else None
    cfg = AttnConfig(Hq, Hkv, D, scale=scale, softcap=softcap, window=window, eps=1e-6, one_plus=one_plus,
                     q_norm=t(qg), k_norm=t(kg), rope=table, kv_offset=kv_offset)
    q_in, k_in, v_in = normal(rng, B, 1, Hq, D), normal(rng, B, 1, Hkv, D), normal(rng, B, 1, Hkv, D)
    q_work = torch.full((B, 1, Hq, D), float("nan"), device=dev)
    out = torch.full((B, 1, Hq, D), float("nan"), device=dev)
    eng.attentionLayer(kv, 1, cfg, t(q_in), t(k_in), t(v_in), pasts, q_work, out)
    eng.ctx.check()
    got, qw = out.cpu().numpy(), q_work.cpu().numpy()

    def chain(x, rows_, heads, gain, past):
        y = x.ravel()
        if gain is not None:
            y = O.rmsnorm(y, gain, rows_, D, 1e-6, one_plus)
        if rope:
            y = O.rope(y, rows_, D, heads, past, base)
        return y

    for b, past in enumerate(pasts):
        r = past - kv_offset
        q_ref = chain(q_in[b], Hq, Hq, qg, past)
        k_ref = chain(k_in[b], Hkv, Hkv, kg, past)
        # q_work: the fused path rotates in f32.
        np.testing.assert_allclose(qw[b].ravel(), q_ref, rtol=2e-5, atol=2e-6, err_msg=f"{name}: q_work seq {b}")
        if q8:
            kc, ks, vc, vs = kv.read_codes(1, b, r, 1)
            rkc, rks = O.quantize_kv(k_ref, 1, Hkv, D)
            rvc, rvs = O.quantize_kv(v_in[b].ravel(), 1, Hkv, D)
            assert bits_equal(kc.cpu().numpy().ravel(), rkc) and bits_equal(ks.cpu().numpy().ravel(), rks), \
                f"{name}: K codes / scale of sequence {b} differ"
            assert bits_equal(vc.cpu().numpy().ravel(), rvc) and bits_equal(vs.cpu().numpy().ravel(), rvs), \
                f"{name}: V codes / scale of sequence {b} differ"
            hk = [O.dequantize_kv(*O.quantize_kv(hist_k[b].ravel(), r, Hkv, D), r, Hkv, D)] if r else []
            hv = [O.dequantize_kv(*O.quantize_kv(hist_v[b].ravel(), r, Hkv, D), r, Hkv, D)] if r else []
            kfull = np.concatenate(hk + [O.dequantize_kv(rkc, rks, 1, Hkv, D)])
            vfull = np.concatenate(hv + [O.dequantize_kv(rvc, rvs, 1, Hkv, D)])
        else:
            k_row, v_row = kv.read_rows(1, b, r, 1)
            assert bits_equal(k_row.cpu().numpy().ravel(), k_ref.astype(np.float16)), \
                f"{name}: K row of sequence {b} differs"
            assert bits_equal(v_row.cpu().numpy().ravel(), v_in[b].ravel().astype(np.float16)), \
                f"{name}: V row of sequence {b} differs"
            kfull = np.concatenate([f16_round(hist_k[b]).ravel(), f16_round(k_ref)])
            vfull = np.concatenate([f16_round(hist_v[b]).ravel(), f16_round(v_in[b].ravel())])
        # In cache-row coordinates the query sits at row r and attends rows [0, r] (a window
        # counts back from it the same way); rows below the shard's first position are absent.
        ref = O.attention(q_ref, kfull, vfull, 1, Hq, Hkv, D, r, scale, softcap, window)
        assert_close(got[b].ravel(), ref, what=f"{name} seq {b} (past {past})")
        # Layer 0 untouched.
        if not q8:
            k0, _ = kv.read_rows(0, b, r, 1)
            assert not k0.float().abs().sum().item()
    kv.close()
    if table:
        table.close()
