"""Run-to-run determinism of the decode kernel: a race detector for its ring and split-merge
protocols.

The decode kernel's result does not depend on timing: every split's partial is merged in a
fixed order by the last CTA to arrive, so repeated launches over the same inputs must give the
same bits.  A race -- a TMA copy landing in a ring slot still being read, the merge reading a
split's partial before it is visible, an arrival counter out of step between launches -- shows
up as outputs that differ between launches.  Each case below queues many launches back to back
on one stream (no host synchronisation between them, so consecutive launches overlap their
tails), for every cache type and head dim and for the automatic and several forced split
counts, and requires identical bits from all of them plus the north-star tolerance against the
oracle (attentionCpu, kernels.ts:3466) for one sequence.  The fused append + decode chain of
several layers (programmatic dependent launches, decode -> next layer's append -> decode) is
repeated the same way.
"""
import contextlib
import ctypes
import os
import zlib

import numpy as np
import pytest

from oracle import oracle as O
from tests.util import assert_close, f16_round, normal

pytestmark = pytest.mark.gpu

REPEATS = 24


@contextlib.contextmanager
def _splits(n):
    old = os.environ.get("BRK_DECODE_SPLITS")
    if n is not None:
        os.environ["BRK_DECODE_SPLITS"] = str(n)
    try:
        yield
    finally:
        if n is not None:
            if old is None:
                del os.environ["BRK_DECODE_SPLITS"]
            else:
                os.environ["BRK_DECODE_SPLITS"] = old


CASES = [
    # (name, q8, Hq, Hkv, D, B, L)
    ("f16_d128", False, 32, 8, 128, 8, 4096),
    ("q8_d128", True, 32, 8, 128, 8, 4096),
    ("f16_d64", False, 32, 8, 64, 4, 8192),
    ("q8_d64", True, 32, 8, 64, 4, 8192),
    ("f16_d256", False, 8, 4, 256, 4, 8192),
    ("q8_d256", True, 8, 4, 256, 4, 8192),
]


@pytest.mark.parametrize("splits", [None, 4, 16])
@pytest.mark.parametrize("name,q8,Hq,Hkv,D,B,Lkv", CASES)
def test_decode_repeats_bit_identical(eng, name, q8, Hq, Hkv, D, B, Lkv, splits):
    import torch
    from brimkern_b200 import _lib as L
    from brimkern_b200.engine import AttnConfig, KvCache
    rng = np.random.default_rng(zlib.crc32(name.encode()))
    dev = eng.device
    kv = KvCache(eng.ctx, 1, B, Hkv, D, Lkv, q8=q8)
    k0 = v0 = None
    gen = torch.Generator(device=dev)
    gen.manual_seed(zlib.crc32(name.encode()))
    for b in range(B):
        if b == 0:
            k0, v0 = normal(rng, Lkv, Hkv, D), normal(rng, Lkv, Hkv, D)
            kv.write_rows(0, 0, 0, torch.from_numpy(k0).to(dev), torch.from_numpy(v0).to(dev))
        else:
            kv.write_rows(0, b, 0, torch.randn((Lkv, Hkv, D), generator=gen, device=dev),
                          torch.randn((Lkv, Hkv, D), generator=gen, device=dev))
    # Ragged lengths: full, and shorter ones that leave some splits with no keys.
    pasts = [Lkv - 1] + [max(0, (Lkv * (B - b)) // B - 37 * b) for b in range(1, B)]
    q = torch.from_numpy(normal(rng, B, 1, Hq, D)).to(dev)
    cfg = AttnConfig(Hq, Hkv, D, scale=1 / 16 if D == 256 else None, softcap=50.0 if D == 256 else 0.0)
    outs = [torch.full((B, 1, Hq, D), float("nan"), device=dev) for _ in range(REPEATS)]
    with _splits(splits):
        p = cfg.params()
        pos = (ctypes.c_int32 * B)(*pasts)
        n = L.lib().brk_attn_decode_splits(eng.ctx.handle, kv.handle, ctypes.byref(p), B, 1, pos)
        if splits is not None:
            assert n == splits
        for o in outs:
            eng.recAttention(kv, 0, cfg, q, o, pasts, kernel="decode")
        eng.ctx.check()
    first = outs[0]
    bad = [i for i, o in enumerate(outs) if not torch.equal(o, first)]
    assert not bad, f"{name} splits={splits}: launches {bad} differ from launch 0 (max diff " \
                    f"{max(float((outs[i] - first).abs().max()) for i in bad):.3g})"
    # Sequence 0 against the oracle.
    if q8:
        kc, ks = O.quantize_kv(k0.ravel(), Lkv, Hkv, D)
        vc, vs = O.quantize_kv(v0.ravel(), Lkv, Hkv, D)
        kref, vref = O.dequantize_kv(kc, ks, Lkv, Hkv, D), O.dequantize_kv(vc, vs, Lkv, Hkv, D)
    else:
        kref, vref = f16_round(k0).ravel(), f16_round(v0).ravel()
    ref = O.attention(q[0].cpu().numpy().ravel(), kref, vref, 1, Hq, Hkv, D, pasts[0], cfg.scale, cfg.softcap)
    assert_close(first[0].cpu().numpy().ravel(), ref, what=f"{name} splits={splits} seq 0")
    kv.close()


@pytest.mark.parametrize("q8", [False, True])
def test_step_chain_repeats_bit_identical(eng, q8):
    """append -> decode -> next layer's append -> ... as one stream of programmatic dependent
    launches (brk_attn_step per layer), the whole chain repeated; the appended row of each layer
    is rewritten with the same values every time, so every repeat must give the same bits."""
    import torch
    from brimkern_b200.engine import AttnConfig, KvCache, RopeTable
    dev = eng.device
    B, Hq, Hkv, D, Lkv, layers = 16, 32, 8, 128, 2048, 6
    gen = torch.Generator(device=dev)
    gen.manual_seed(4242 + q8)
    rope = RopeTable(eng.ctx, D, 1e6, None, Lkv)
    qn = (1 + 0.02 * torch.randn(D, generator=gen, device=dev)).float()
    cfg = AttnConfig(Hq, Hkv, D, q_norm=qn, k_norm=qn, rope=rope)
    kv = KvCache(eng.ctx, layers, B, Hkv, D, Lkv, q8=q8)
    for layer in range(layers):
        for b in range(B):
            kv.write_rows(layer, b, 0, torch.randn((Lkv, Hkv, D), generator=gen, device=dev),
                          torch.randn((Lkv, Hkv, D), generator=gen, device=dev))
    past = [Lkv - 1 - 3 * b for b in range(B)]
    q_in = torch.randn((layers, B, 1, Hq, D), generator=gen, device=dev)
    k_in = torch.randn((layers, B, 1, Hkv, D), generator=gen, device=dev)
    v_in = torch.randn((layers, B, 1, Hkv, D), generator=gen, device=dev)
    q_work = torch.empty_like(q_in)
    outs = [torch.full((layers, B, 1, Hq, D), float("nan"), device=dev) for _ in range(12)]
    eng.ctx.reserve(64 << 20)
    for o in outs:
        for layer in range(layers):
            eng.attentionLayer(kv, layer, cfg, q_in[layer], k_in[layer], v_in[layer], past, q_work[layer], o[layer])
    eng.ctx.check()
    bad = [i for i, o in enumerate(outs) if not torch.equal(o, outs[0])]
    assert not bad, f"q8={q8}: repeats {bad} of the layer chain differ from the first"
    assert torch.isfinite(outs[0]).all()
    kv.close()
    rope.close()


def test_split_counters_survive_shape_changes(eng):
    """Alternating launch shapes on one context: a split launch over few (sequence, kv head)
    tiles, then one over many, then the small one again.  The arrival counters of the large
    launch must not have been overwritten by the small launch's partials (they once shared one
    workspace, counters first: a small launch's partials landed on the counters of tiles only a
    larger launch uses, and that launch then merged too early or never)."""
    import torch
    from brimkern_b200.engine import AttnConfig, KvCache
    dev = eng.device
    Hq, Hkv, D, Lkv = 32, 8, 128, 2048
    gen = torch.Generator(device=dev)
    gen.manual_seed(31)
    rng = np.random.default_rng(31)
    cfg = AttnConfig(Hq, Hkv, D)
    caches, host, qs, outs = [], [], [], []
    for B in (1, 16):
        kv = KvCache(eng.ctx, 1, B, Hkv, D, Lkv)
        k0, v0 = normal(rng, Lkv, Hkv, D), normal(rng, Lkv, Hkv, D)
        for b in range(B):
            if b == B - 1:
                kv.write_rows(0, b, 0, torch.from_numpy(k0).to(dev), torch.from_numpy(v0).to(dev))
            else:
                kv.write_rows(0, b, 0, torch.randn((Lkv, Hkv, D), generator=gen, device=dev),
                              torch.randn((Lkv, Hkv, D), generator=gen, device=dev))
        caches.append(kv)
        host.append((k0, v0))
        qs.append(torch.from_numpy(normal(rng, B, 1, Hq, D)).to(dev))
    with _splits(8):
        for rep in range(3):
            for i, kv in enumerate(caches):
                o = torch.full_like(qs[i], float("nan"))
                eng.recAttention(kv, 0, cfg, qs[i], o, [Lkv - 1] * kv.batch, kernel="decode")
                outs.append((i, o))
        eng.ctx.check()
    for i, o in outs:
        k0, v0 = host[i]
        B = caches[i].batch
        ref = O.attention(qs[i][B - 1].cpu().numpy().ravel(), f16_round(k0).ravel(), f16_round(v0).ravel(), 1, Hq,
                          Hkv, D, Lkv - 1)
        assert torch.isfinite(o).all(), f"batch {B}: rows never written"
        assert_close(o[B - 1].cpu().numpy().ravel(), ref, what=f"batch {B} last sequence")
    for kv in caches:
        kv.close()


@pytest.mark.parametrize("splits,no_cluster", [(32, False), (16, True), (16, False)])
def test_q8_d256_full_residency_repeats(eng, splits, no_cluster):
    """int8 head_dim 256 with every SM holding several CTAs at once (4 sequences x 4 kv heads x
    16-32 splits), the configuration in which a ring slot's generic-proxy reads, not fenced
    against the next TMA write into the slot, let consumers see bytes of the following tile now
    and then: the outputs of 24 launches must agree bit for bit."""
    old = os.environ.get("BRK_DECODE_NO_CLUSTER")
    if no_cluster:
        os.environ["BRK_DECODE_NO_CLUSTER"] = "1"
    try:
        test_decode_repeats_bit_identical(eng, "q8_d256", True, 8, 4, 256, 4, 8192, splits)
    finally:
        if no_cluster:
            if old is None:
                del os.environ["BRK_DECODE_NO_CLUSTER"]
            else:
                os.environ["BRK_DECODE_NO_CLUSTER"] = old
