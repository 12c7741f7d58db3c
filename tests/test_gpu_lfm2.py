"""LFM2 attention layers (kernels.ts:1990-2003, 2029-2111; lfm2Model.ts:320-333) on the GPU:
one cache per attention layer of a hybrid conv / attention stack, a prompt prefilled in 128-token
chunks, then decode tokens; per-layer outputs against the oracle chain rmsnormCpu -> ropeCpu ->
fp16 -> attentionCpu, and the batched prefill against the token-by-token
loop the reference keeps as its correctness reference (?lfm2batch=0)."""
import numpy as np
import pytest

from oracle import oracle as O
from tests.util import assert_close, f16_round, normal

pytestmark = pytest.mark.gpu

# LFM2-1.2B attention shape: 32 q / 8 kv heads of 64, theta 1e6, eps 1e-5, QK-norm; attention at
# a few layer indices of the hybrid stack (the others are short-conv layers with no K/V).
HQ, HKV, D, THETA, EPS = 32, 8, 64, 1e6, 1e-5
ATTN_LAYERS = [2, 5, 8, 10]


def _chain_ref(q, k, v, qg, kg, past, T):
    """Oracle over one sequence: q [T,Hq,D], k/v [past+T,Hkv,D] raw projections (all positions)."""
    L = past + T
    qn = O.rope(O.rmsnorm(q.ravel(), qg, T * HQ, D, EPS), T * HQ, D, HQ, past, THETA)
    kn = O.rope(O.rmsnorm(k.ravel(), kg, L * HKV, D, EPS), L * HKV, D, HKV, 0, THETA)
    return O.attention(qn, f16_round(kn), f16_round(v.ravel()), T, HQ, HKV, D, past)


def _run(eng, B, P, steps, chunk=None, token_by_token=False):
    import torch
    from brimkern_b200.engine import AttnConfig, RopeTable
    rng = np.random.default_rng(42)
    dev = eng.device
    total = P + steps
    rope = RopeTable(eng.ctx, D, THETA, None, total)
    inputs, outs = {}, {}
    for L in ATTN_LAYERS:
        qg = (1 + 0.02 * rng.standard_normal(D)).astype(np.float32)
        kg = (1 + 0.02 * rng.standard_normal(D)).astype(np.float32)
        q, k, v = normal(rng, B, total, HQ, D), normal(rng, B, total, HKV, D), normal(rng, B, total, HKV, D)
        inputs[L] = (qg, kg, q, k, v)
        cfg = AttnConfig(HQ, HKV, D, eps=EPS, rope=rope, q_norm=torch.from_numpy(qg).to(dev),
                         k_norm=torch.from_numpy(kg).to(dev))
        pieces = []
        spans = [(t, t + 1) for t in range(P)] if token_by_token else [(0, P)]
        spans += [(P + s, P + s + 1) for s in range(steps)]
        for t0, t1 in spans:
            o = eng.lfm2Attention(L, cfg, torch.from_numpy(q[:, t0:t1].copy()).to(dev),
                                  torch.from_numpy(k[:, t0:t1].copy()).to(dev),
                                  torch.from_numpy(v[:, t0:t1].copy()).to(dev), [t0] * B, chunk=chunk)
            pieces.append(o.cpu().numpy())
        outs[L] = np.concatenate(pieces, axis=1)
    eng.ctx.check()
    rope.close()
    return inputs, outs


def test_lfm2_chunked_prefill_then_decode(eng):
    B, P, steps = 2, 300, 2  # 128 + 128 + 44 prompt tokens, then 2 decode tokens
    inputs, outs = _run(eng, B, P, steps)
    assert sorted(eng.lfm2KvGpu) == ATTN_LAYERS  # one cache per attention layer, none for conv layers
    for L in ATTN_LAYERS:
        qg, kg, q, k, v = inputs[L]
        for b in range(B):
            ref = _chain_ref(q[b], k[b], v[b], qg, kg, 0, P + steps)
            assert_close(outs[L][b].ravel(), ref, what=f"layer {L} seq {b}")
    eng.resetKvGpu()
    assert not eng.lfm2KvGpu


def test_lfm2_batched_equals_token_by_token(eng):
    """The batched chunked prefill and the sequential loop give the same outputs (within the
    tolerance: different kernels, same math)."""
    _, batched = _run(eng, 1, 40, 1, chunk=16)
    eng.resetKvGpu()
    _, sequential = _run(eng, 1, 40, 1, token_by_token=True)
    eng.resetKvGpu()
    for L in ATTN_LAYERS:
        assert_close(batched[L], sequential[L], what=f"layer {L}")
