"""Non-causal attention (attention_full / attention_full_wg, shaders.ts:1530-1667; recAttentionFull,
kernels.ts:1277-1290) on the GPU through brk_attn_full: the reference gate's own shapes
(kernels.ts:3168-3201, including head_dim 4 and 160) against the golden fixtures' oracle, UNet /
ViT-sized shapes, GQA, softcap, batches; within the north-star tolerance of the oracle fed the
same fp16-rounded K/V."""
import zlib

import numpy as np
import pytest

from oracle import oracle as O
from tests.util import assert_close, f16_round, normal

pytestmark = pytest.mark.gpu

GATES = ["full_gate_cross", "full_sdturbo_self", "full_clip_cross", "full_sdxs_hd160"]


@pytest.mark.parametrize("name", GATES)
@pytest.mark.parametrize("twin", ["attentionFull", "attentionFullWg"])
def test_full_twins_gate_shapes(eng, golden, name, twin):
    c, a = golden[name]
    T, kvL, H, D = c["n_tokens"], c["kv_len"], c["n_heads"], c["head_dim"]
    got = getattr(eng, twin)(a["q"], a["k"], a["v"], T, H, H, D, kvL)
    ref = O.attention_full(a["q"], f16_round(a["k"]), f16_round(a["v"]), T, H, H, D, kvL)
    assert_close(got, ref, what=f"{twin}/{name}")
    assert np.abs(got - a["out"]).max() < 2e-2  # the fp16 storage of K/V, against the f32 reference


@pytest.mark.parametrize("B,T,kvL,Hq,Hkv,D,softcap", [
    (1, 1024, 1024, 5, 5, 64, 0.0),    # UNet self-attention (32 x 32 latent), tensor-core path
    (2, 300, 77, 8, 8, 64, 0.0),       # cross-attention to a 77-token text, batch 2
    (1, 257, 257, 16, 16, 64, 0.0),    # ViT-L/14 at 224 px (256 patches + class token)
    (1, 500, 333, 8, 2, 128, 30.0),    # GQA + softcap (extension), head_dim 128
    (1, 40, 40, 4, 4, 80, 0.0),        # head_dim 80 (zero-padded to 128), decode-kernel path
    (2, 9, 9, 8, 8, 160, 0.0),         # head_dim 160 (SDXS 1280 ch), padded to 256
])
def test_full_shapes(eng, B, T, kvL, Hq, Hkv, D, softcap):
    import torch
    from brimkern_b200.engine import AttnConfig
    rng = np.random.default_rng(zlib.crc32(f"{B}{T}{kvL}{Hq}{Hkv}{D}".encode()))
    q, k, v = normal(rng, B, T, Hq, D), normal(rng, B, kvL, Hkv, D), normal(rng, B, kvL, Hkv, D)
    dev = eng.device
    out = torch.full((B, T, Hq, D), float("nan"), dtype=torch.float32, device=dev)
    eng.recAttentionFull(AttnConfig(Hq, Hkv, D, softcap=softcap), torch.from_numpy(q).to(dev),
                         torch.from_numpy(k).to(dev), torch.from_numpy(v).to(dev), out)
    eng.ctx.check()
    got = out.cpu().numpy()
    for b in range(B):
        ref = O.attention_full(q[b].ravel(), f16_round(k[b]).ravel(), f16_round(v[b]).ravel(), T, Hq, Hkv, D, kvL,
                               None, softcap)
        assert_close(got[b].ravel(), ref, what=f"B{B} T{T} kv{kvL} D{D} seq {b}")


def test_full_rejects_causal_options(eng):
    import torch
    from brimkern_b200._lib import BRK_ERR_INVALID, BRK_ERR_UNSUPPORTED, BrkError
    from brimkern_b200.engine import AttnConfig
    x = torch.zeros((1, 4, 2, 64), dtype=torch.float32, device=eng.device)
    with pytest.raises(BrkError) as ei:
        eng.recAttentionFull(AttnConfig(2, 2, 64, window=8), x, x, x, torch.empty_like(x))
    assert ei.value.code == BRK_ERR_INVALID
    y = torch.zeros((1, 4, 2, 300), dtype=torch.float32, device=eng.device)
    with pytest.raises(BrkError) as ei:
        eng.recAttentionFull(AttnConfig(2, 2, 300), y, y, y, torch.empty_like(y))
    assert ei.value.code == BRK_ERR_UNSUPPORTED
