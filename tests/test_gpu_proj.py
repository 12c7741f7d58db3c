"""The projections either side of the attention operator (recordLayerKV, kernels.ts:1700-1736;
layerForwardCpu kernels.ts:3501-3522) on the GPU: RMSNorm + q / k / v projections (+ biases) and
the output projection with the residual (and Gemma-2's post-attention norm), against the oracle's
rmsnormCpu and matmulCpu (f32 activations, the same fp16 weights, double sums).  The GPU feeds
the tensor cores fp16 activations, so the tolerance is the north-star one on O(1) outputs; the
whole attention slice x -> h is checked end to end the same way."""
import zlib

import numpy as np
import pytest

from oracle import oracle as O
from tests.util import assert_close, f16_round, normal

pytestmark = pytest.mark.gpu


def _weights(rng, n, k):
    """fp16 weights ~ N(0, 1/k) (outputs O(1)); returned as the fp16 tensor and its f32 values."""
    w = (normal(rng, n, k) / np.sqrt(k)).astype(np.float16)
    return w, w.astype(np.float32)


@pytest.mark.parametrize("name,rows,d,qd,kvd,norm,bias,one_plus", [
    ("qwen3_decode", 64, 2560, 4096, 1024, True, False, False),
    ("qwen3_prefill", 512, 2560, 4096, 1024, True, False, False),
    ("qwen05_bias", 10, 896, 896, 128, True, True, False),
    ("gemma_oneplus", 33, 2304, 2048, 1024, True, False, True),
    ("no_norm", 7, 1024, 512, 256, False, False, False),
    # 48 feature tiles x 2 token tiles: one split, so the bias is added in the epilogue's TMA store.
    ("one_split_bias", 300, 1024, 4096, 1024, True, True, False),
])
def test_proj_qkv(eng, name, rows, d, qd, kvd, norm, bias, one_plus):
    import torch
    rng = np.random.default_rng(zlib.crc32(name.encode()))
    dev = eng.device
    x = normal(rng, rows, d)
    g = (0.1 * rng.standard_normal(d) if one_plus else 1 + 0.02 * rng.standard_normal(d)).astype(np.float32)
    ws = [_weights(rng, n, d) for n in (qd, kvd, kvd)]
    bs = [normal(rng, n) * 0.1 for n in (qd, kvd, kvd)] if bias else [None] * 3
    outs = [torch.full((rows, n), float("nan"), dtype=torch.float32, device=dev) for n in (qd, kvd, kvd)]
    t = lambda a: None if a is None else torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    eng.projQkv(t(x), t(ws[0][0]), t(ws[1][0]), t(ws[2][0]), *outs, attn_norm=t(g) if norm else None, eps=1e-6,
                one_plus=one_plus, bq=t(bs[0]), bk=t(bs[1]), bv=t(bs[2]))
    eng.ctx.check()
    n1 = O.rmsnorm(x.ravel(), g, rows, d, 1e-6, one_plus) if norm else x.ravel()
    for i, n in enumerate((qd, kvd, kvd)):
        ref = O.matmul_t(n1, ws[i][1], rows, d, n).reshape(rows, n)
        if bias:
            ref = ref + bs[i]
        assert_close(outs[i].cpu().numpy(), ref, what=f"{name} out {i}")


@pytest.mark.parametrize("name,rows,qd,d,post", [
    ("qwen3_decode", 64, 4096, 2560, False),
    ("qwen3_prefill", 300, 4096, 2560, False),
    ("gemma_post_norm", 17, 2048, 2304, True),
    # 32 feature tiles x 3 token tiles: one split, residual added in the epilogue's TMA store.
    ("one_split_residual", 600, 1024, 4096, False),
])
def test_proj_out(eng, name, rows, qd, d, post):
    import torch
    rng = np.random.default_rng(zlib.crc32(name.encode()))
    dev = eng.device
    attn, x = normal(rng, rows, qd), normal(rng, rows, d)
    w16, w32 = _weights(rng, d, qd)
    g = (0.1 * rng.standard_normal(d)).astype(np.float32)
    h = torch.full((rows, d), float("nan"), dtype=torch.float32, device=dev)
    eng.projOut(torch.from_numpy(attn).to(dev), torch.from_numpy(w16).to(dev), torch.from_numpy(x).to(dev), h,
                post_norm=torch.from_numpy(g).to(dev) if post else None, eps=1e-6, one_plus=post)
    eng.ctx.check()
    proj = O.matmul_t(attn.ravel(), w32, rows, qd, d)
    if post:
        proj = O.rmsnorm(proj, g, rows, d, 1e-6, True)
    assert_close(h.cpu().numpy(), x + proj.reshape(rows, d), what=name)


def test_attention_slice_end_to_end(eng):
    """x -> RMSNorm + q/k/v projections -> QK-norm + RoPE + append + decode attention -> output
    projection + residual, for a Qwen3-shaped layer at decode (the first half of layerForwardCpu)."""
    import torch
    from brimkern_b200.engine import AttnConfig, KvCache, RopeTable
    rng = np.random.default_rng(99)
    dev = eng.device
    B, d, Hq, Hkv, D, past = 4, 1024, 16, 4, 64, 200
    qd, kvd = Hq * D, Hkv * D
    g = (1 + 0.02 * rng.standard_normal(d)).astype(np.float32)
    qg = (1 + 0.02 * rng.standard_normal(D)).astype(np.float32)
    kg = (1 + 0.02 * rng.standard_normal(D)).astype(np.float32)
    (wq16, wq), (wk16, wk), (wv16, wv), (wo16, wo) = (_weights(rng, qd, d), _weights(rng, kvd, d),
                                                      _weights(rng, kvd, d), _weights(rng, d, qd))
    # Cached rows 0..past-1: arbitrary K/V already in the cache (fp16).
    kc, vc = normal(rng, B, past, Hkv, D), normal(rng, B, past, Hkv, D)
    x = normal(rng, B, d)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    rope = RopeTable(eng.ctx, D, 1e6, None, past + 1)
    cfg = AttnConfig(Hq, Hkv, D, eps=1e-6, rope=rope, q_norm=t(qg), k_norm=t(kg))
    kv = KvCache(eng.ctx, 1, B, Hkv, D, past + 1)
    for b in range(B):
        kv.write_rows(0, b, 0, t(kc[b]), t(vc[b]))
    q = torch.empty((B, qd), dtype=torch.float32, device=dev)
    k = torch.empty((B, kvd), dtype=torch.float32, device=dev)
    v = torch.empty_like(k)
    eng.projQkv(t(x), t(wq16), t(wk16), t(wv16), q, k, v, attn_norm=t(g), eps=1e-6)
    attn = eng.attentionLayer(kv, 0, cfg, q.view(B, 1, Hq, D), k.view(B, 1, Hkv, D), v.view(B, 1, Hkv, D), [past] * B)
    h = torch.empty((B, d), dtype=torch.float32, device=dev)
    eng.projOut(attn.view(B, qd), t(wo16), t(x), h)
    eng.ctx.check()
    got = h.cpu().numpy()
    for b in range(B):
        n1 = O.rmsnorm(x[b], g, 1, d, 1e-6)
        qp, kp, vp = O.matmul_t(n1, wq, 1, d, qd), O.matmul_t(n1, wk, 1, d, kvd), O.matmul_t(n1, wv, 1, d, kvd)
        qr = O.rope(O.rmsnorm(qp, qg, Hq, D, 1e-6), Hq, D, Hq, past, 1e6)
        kr = O.rope(O.rmsnorm(kp, kg, Hkv, D, 1e-6), Hkv, D, Hkv, past, 1e6)
        kall = np.concatenate([f16_round(kc[b]).ravel(), f16_round(kr)])
        vall = np.concatenate([f16_round(vc[b]).ravel(), f16_round(vp)])
        att = O.attention(qr, kall, vall, 1, Hq, Hkv, D, past)
        ref = x[b] + O.matmul_t(att, wo, 1, qd, d)
        assert_close(got[b], ref, what=f"slice seq {b}")
    kv.close()
    rope.close()
