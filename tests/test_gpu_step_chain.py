"""Chains of decode steps queued back to back (no host synchronisation), against the oracle.

Every brk_attn_step is launched as a programmatic dependent of the kernel before it, so a step
starts while the previous one (the previous layer's, or the same layer's previous token's, whose
fused append wrote the row this step reads as history) is still finishing.  Checked over several
steps for layer after layer, one layer step after step, the append + decode pair (3 tokens) and
an int8 cache, and for a step directly after brk_attn_append of the rows it reads: every step's
output within the north-star tolerance of attentionCpu (kernels.ts:3466) over the cache rows, and
the appended rows bit for bit the oracle chain rmsnormCpu -> ropeCpu -> fp16
(kernels.ts:3395-3460).
"""
import numpy as np
import pytest

from oracle import oracle as O
from tests.util import assert_close, bits_equal

pytestmark = pytest.mark.gpu


def _oracle_rows(x, gain, n_tokens, heads, D, pos, base):
    """rmsnormCpu then ropeCpu over n_tokens tokens of `heads` heads starting at position pos."""
    rows = n_tokens * heads
    y = O.rmsnorm(x.ravel(), gain, rows, D, 1e-6) if gain is not None else x.ravel()
    return O.rope(y, rows, D, heads, pos, base)


@pytest.mark.parametrize("layers,n_tokens,q8", [(3, 1, False), (1, 1, False), (2, 3, False), (3, 1, True)])
def test_step_chain_against_oracle(eng, layers, n_tokens, q8):
    import torch
    from brimkern_b200.engine import AttnConfig, KvCache, RopeTable
    dev = eng.device
    B, Hq, Hkv, D, base, steps = 4, 32, 8, 128, 1e6, 6
    rng = np.random.default_rng(layers * 100 + n_tokens + 7 * q8)
    pasts0 = [900, 513, 64, 1]
    cap = max(pasts0) + steps * n_tokens
    gen = torch.Generator(device=dev)
    gen.manual_seed(layers + n_tokens)
    qn = (1 + 0.02 * rng.standard_normal(D)).astype(np.float32)
    kn = (1 + 0.02 * rng.standard_normal(D)).astype(np.float32)
    rope = RopeTable(eng.ctx, D, base, None, cap)
    cfg = AttnConfig(Hq, Hkv, D, q_norm=torch.from_numpy(qn).to(dev), k_norm=torch.from_numpy(kn).to(dev), rope=rope)
    kv = KvCache(eng.ctx, layers, B, Hkv, D, cap, q8=q8)
    for layer in range(layers):
        for b in range(B):
            kv.write_rows(layer, b, 0, torch.randn((cap, Hkv, D), generator=gen, device=dev),
                          torch.randn((cap, Hkv, D), generator=gen, device=dev))
    q_in = torch.from_numpy(rng.standard_normal((steps, layers, B, n_tokens, Hq, D)).astype(np.float32)).to(dev)
    k_in = torch.from_numpy(rng.standard_normal((steps, layers, B, n_tokens, Hkv, D)).astype(np.float32)).to(dev)
    v_in = torch.from_numpy(rng.standard_normal((steps, layers, B, n_tokens, Hkv, D)).astype(np.float32)).to(dev)
    q_work = torch.empty_like(q_in)
    out = torch.full_like(q_in, float("nan"))
    eng.ctx.reserve(64 << 20)
    for t in range(steps):
        past = [p + t * n_tokens for p in pasts0]
        for layer in range(layers):
            eng.attentionLayer(kv, layer, cfg, q_in[t, layer], k_in[t, layer], v_in[t, layer], past,
                               q_work[t, layer], out[t, layer])
    eng.ctx.check()
    got = out.cpu().numpy()
    qh, kh, vh = q_in.cpu().numpy(), k_in.cpu().numpy(), v_in.cpu().numpy()
    for layer in range(layers):
        for b in range(B):
            if q8:
                kc, ks, vc, vs = kv.read_codes(layer, b, 0, cap)
                n = cap
                krows = O.dequantize_kv(kc.cpu().numpy().ravel(), ks.cpu().numpy().ravel(), n, Hkv, D)
                vrows = O.dequantize_kv(vc.cpu().numpy().ravel(), vs.cpu().numpy().ravel(), n, Hkv, D)
            else:
                kr, vr = kv.read_rows(layer, b, 0, cap)
                krows, vrows = kr.float().cpu().numpy().ravel(), vr.float().cpu().numpy().ravel()
            for t in range(steps):
                p = pasts0[b] + t * n_tokens
                k_ref = _oracle_rows(kh[t, layer, b], kn, n_tokens, Hkv, D, p, base)
                if not q8:
                    new_k = krows[p * Hkv * D:(p + n_tokens) * Hkv * D]
                    assert bits_equal(new_k.astype(np.float16), k_ref.astype(np.float16)), \
                        f"layer {layer} seq {b} step {t}: appended K rows differ"
                    new_v = vrows[p * Hkv * D:(p + n_tokens) * Hkv * D]
                    assert bits_equal(new_v.astype(np.float16), vh[t, layer, b].ravel().astype(np.float16)), \
                        f"layer {layer} seq {b} step {t}: appended V rows differ"
                q_ref = _oracle_rows(qh[t, layer, b], qn, n_tokens, Hq, D, p, base)
                n = p + n_tokens
                ref = O.attention(q_ref, krows[:n * Hkv * D], vrows[:n * Hkv * D], n_tokens, Hq, Hkv, D, p)
                assert_close(got[t, layer, b].ravel(), ref, what=f"layer {layer} seq {b} step {t}")
    kv.close()
    rope.close()


def test_step_after_append_of_rows_it_reads(eng):
    """brk_attn_append of rows [p, p + 5), then brk_attn_step at position p + 5 of the same layer:
    the step reads the appended rows as history, written by the kernel directly before it."""
    import torch
    from brimkern_b200.engine import AttnConfig, KvCache
    dev = eng.device
    B, Hq, Hkv, D = 2, 16, 4, 64
    rng = np.random.default_rng(5)
    p0, n_app = 700, 5
    cap = p0 + n_app + 1
    kv = KvCache(eng.ctx, 2, B, Hkv, D, cap)
    gen = torch.Generator(device=dev)
    gen.manual_seed(5)
    for layer in range(2):
        for b in range(B):
            kv.write_rows(layer, b, 0, torch.randn((cap, Hkv, D), generator=gen, device=dev),
                          torch.randn((cap, Hkv, D), generator=gen, device=dev))
    cfg = AttnConfig(Hq, Hkv, D)
    for rep in range(4):
        # Inputs first: a host copy between the launches would end the dependent-launch chain.
        t = lambda *shape: torch.from_numpy(rng.standard_normal(shape).astype(np.float32)).to(dev)  # noqa: E731
        q0, k0, v0 = t(B, 1, Hq, D), t(B, 1, Hkv, D), t(B, 1, Hkv, D)
        ka, va = t(B, n_app, Hkv, D), t(B, n_app, Hkv, D)
        q1, k1, v1 = t(B, 1, Hq, D), t(B, 1, Hkv, D), t(B, 1, Hkv, D)
        w0, o0, w1, o1 = (torch.empty_like(x) for x in (q0, q0, q1, q1))
        # A step of layer 0, then the append of layer 1's rows and the step of layer 1 that reads
        # them, back to back.
        eng.attentionLayer(kv, 0, cfg, q0, k0, v0, [p0 + n_app] * B, w0, o0)
        eng.appendKv(kv, 1, cfg, None, ka, va, None, [p0] * B)
        eng.attentionLayer(kv, 1, cfg, q1, k1, v1, [p0 + n_app] * B, w1, o1)
        eng.ctx.check()
        kr, vr = kv.read_rows(1, 0, 0, cap)
        kr, vr = kr.float().cpu().numpy(), vr.float().cpu().numpy()
        assert bits_equal(kr[p0:p0 + n_app], ka[0].cpu().numpy().astype(np.float16).astype(np.float32))
        ref = O.attention(q1[0].cpu().numpy().ravel(), kr.ravel(), vr.ravel(), 1, Hq, Hkv, D, p0 + n_app)
        assert_close(o1[0].cpu().numpy().ravel(), ref, what=f"repeat {rep}")
    kv.close()
