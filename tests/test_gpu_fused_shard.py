"""Sequence-sharded decode over peer memory (brk_attn_decode_push + brk_attn_combine_peers) on
one GPU: several ranks emulated in one process, each with its own cache shard and exchange area,
attached to one another.  All pushes are issued before any combine on one stream, so no kernel
waits for a kernel that has not already run.  Every rank's combined output must equal attention
over the whole context (oracle); a rank whose partials never arrive makes
the combine give up after its timeout and report a device error, and the context stays usable."""
import numpy as np
import pytest

from oracle import oracle as O
from tests.util import assert_close, f16_round, normal

pytestmark = pytest.mark.gpu


def _shards(eng, k, v, N, q8):
    import torch
    from brimkern_b200.engine import KvCache
    B, L, Hkv, D = k.shape
    shard = (L + N - 1) // N
    kvs = []
    for r in range(N):
        lo, hi = r * shard, min(L, (r + 1) * shard)
        kv = KvCache(eng.ctx, 1, B, Hkv, D, max(1, hi - lo), q8=q8)
        for b in range(B):
            kv.write_rows(0, b, 0, torch.from_numpy(k[b, lo:hi].copy()).to(eng.device),
                          torch.from_numpy(v[b, lo:hi].copy()).to(eng.device))
        kvs.append((kv, lo))
    return kvs


def _deq(x, q8):
    """What the cache holds for x [rows, Hkv, D]: fp16-rounded, or quantised and dequantised."""
    if not q8:
        return f16_round(x).ravel()
    rows, hkv, d = x.shape
    c, s = O.quantize_kv(x.ravel(), rows, hkv, d)
    return O.dequantize_kv(c, s, rows, hkv, d)


@pytest.mark.parametrize("N,q8", [(1, False), (2, False), (3, False), (4, True)])
def test_push_combine_emulated_ranks(eng, N, q8):
    import torch
    from brimkern_b200.engine import AttnConfig, PeerArea
    rng = np.random.default_rng(10 + N)
    Hq, Hkv, D, B, L = 32, 8, 64, 2, 5000
    k, v = normal(rng, B, L, Hkv, D), normal(rng, B, L, Hkv, D)
    kvs = _shards(eng, k, v, N, q8)
    rows = B * Hq
    areas = [PeerArea(eng.ctx, N, r, rows, D) for r in range(N)]
    for r in range(N):
        for p in range(N):
            if p != r:
                areas[r].attach(p, areas[p])
    past = [L - 1] * B
    shard = (L + N - 1) // N
    for epoch in (1, 2, 3):  # both parities, then the first one again
        q = normal(rng, B, 1, Hq, D)
        qd = torch.from_numpy(q).to(eng.device)
        for r, (kv, lo) in enumerate(kvs):
            eng.decodePush(kv, 0, AttnConfig(Hq, Hkv, D, kv_offset=lo), qd, areas[r], epoch, past)
        outs = []
        for r in range(N):
            out = torch.full((rows, D), float("nan"), dtype=torch.float32, device=eng.device)
            eng.combinePeers(areas[r], rows, epoch, out)
            outs.append(out)
        eng.ctx.check()
        got = [o.cpu().numpy() for o in outs]
        for r in range(1, N):
            assert np.array_equal(got[r], got[0]), f"rank {r} differs from rank 0"
        for b in range(B):
            kd = np.concatenate([_deq(k[b, r * shard:min(L, (r + 1) * shard)], q8) for r in range(N)])
            vd = np.concatenate([_deq(v[b, r * shard:min(L, (r + 1) * shard)], q8) for r in range(N)])
            ref = O.attention(q[b].ravel(), kd, vd, 1, Hq, Hkv, D, past[b])
            assert_close(got[0].reshape(B, Hq, D)[b].ravel(), ref, what=f"N={N} epoch {epoch} seq {b}")
    for a in areas:
        a.close()
    for kv, _ in kvs:
        kv.close()


def test_missing_rank_times_out(eng):
    """Rank 1 never pushes: rank 0's combine gives up after its timeout, writes nothing, and the
    context reports BRK_ERR_DEVICE once and then works again."""
    import torch
    from brimkern_b200._lib import BRK_ERR_DEVICE, BrkError
    from brimkern_b200.engine import AttnConfig, PeerArea
    rng = np.random.default_rng(5)
    Hq, Hkv, D, B, L = 8, 2, 64, 1, 300
    k, v = normal(rng, B, L, Hkv, D), normal(rng, B, L, Hkv, D)
    kvs = _shards(eng, k, v, 2, False)
    rows = B * Hq
    a0, a1 = PeerArea(eng.ctx, 2, 0, rows, D), PeerArea(eng.ctx, 2, 1, rows, D)
    a0.attach(1, a1)
    a1.attach(0, a0)
    q = torch.from_numpy(normal(rng, B, 1, Hq, D)).to(eng.device)
    eng.decodePush(kvs[0][0], 0, AttnConfig(Hq, Hkv, D, kv_offset=0), q, a0, 1, [L - 1])
    out = torch.full((rows, D), 7.0, dtype=torch.float32, device=eng.device)
    eng.combinePeers(a0, rows, 1, out, timeout_s=0.2)
    with pytest.raises(BrkError) as ei:
        eng.ctx.check()
    assert ei.value.code == BRK_ERR_DEVICE
    assert torch.all(out == 7.0).item(), "a combine that gave up must write nothing"
    # Rank 1 catches up: the same epoch now completes on both ranks.
    eng.decodePush(kvs[1][0], 0, AttnConfig(Hq, Hkv, D, kv_offset=kvs[1][1]), q, a1, 1, [L - 1])
    eng.combinePeers(a0, rows, 1, out)
    eng.ctx.check()
    kd = np.concatenate([f16_round(k[0, :kvs[1][1]]).ravel(), f16_round(k[0, kvs[1][1]:]).ravel()])
    vd = np.concatenate([f16_round(v[0, :kvs[1][1]]).ravel(), f16_round(v[0, kvs[1][1]:]).ravel()])
    ref = O.attention(q.cpu().numpy().ravel(), kd, vd, 1, Hq, Hkv, D, L - 1)
    assert_close(out.cpu().numpy().ravel(), ref, what="after recovery")
    a0.close()
    a1.close()
    for kv, _ in kvs:
        kv.close()


@pytest.mark.parametrize("N,q8", [(2, False), (4, True)])
def test_step_push_emulated_ranks(eng, N, q8):
    """brk_attn_step_push: the append fused into the push launch.  Every rank rotates the raw q
    (QK-norm + RoPE); the rank whose shard holds the new position stores its K / V row (the others
    pass none); the combine equals the oracle chain over the whole context plus the new token."""
    import torch
    from brimkern_b200.engine import AttnConfig, KvCache, PeerArea, RopeTable
    rng = np.random.default_rng(40 + N)
    Hq, Hkv, D, B, ctx_len = 32, 8, 64, 2, 3000
    base = 5e5
    k, v = normal(rng, B, ctx_len, Hkv, D), normal(rng, B, ctx_len, Hkv, D)
    shard = (ctx_len + N - 1) // N
    kvs = []
    for r in range(N):
        lo, hi = r * shard, min(ctx_len, (r + 1) * shard)
        kv = KvCache(eng.ctx, 1, B, Hkv, D, hi - lo + (1 if r == N - 1 else 0), q8=q8)
        for b in range(B):
            kv.write_rows(0, b, 0, torch.from_numpy(k[b, lo:hi].copy()).to(eng.device),
                          torch.from_numpy(v[b, lo:hi].copy()).to(eng.device))
        kvs.append((kv, lo))
    rows = B * Hq
    areas = [PeerArea(eng.ctx, N, r, rows, D) for r in range(N)]
    for r in range(N):
        for p in range(N):
            if p != r:
                areas[r].attach(p, areas[p])
    qg = (1 + 0.02 * rng.standard_normal(D)).astype(np.float32)
    kg = (1 + 0.02 * rng.standard_normal(D)).astype(np.float32)
    rope = RopeTable(eng.ctx, D, base, None, ctx_len + 1)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(eng.device)  # noqa: E731
    q_in, k_in, v_in = normal(rng, B, 1, Hq, D), normal(rng, B, 1, Hkv, D), normal(rng, B, 1, Hkv, D)
    past = [ctx_len] * B
    works = [torch.empty((B, 1, Hq, D), device=eng.device) for _ in range(N)]
    for r, (kv, lo) in enumerate(kvs):
        cfg = AttnConfig(Hq, Hkv, D, q_norm=t(qg), k_norm=t(kg), rope=rope, kv_offset=lo)
        owner = r == N - 1
        eng.stepPush(kv, 0, cfg, t(q_in), t(k_in) if owner else None, t(v_in) if owner else None, works[r],
                     areas[r], 1, past)
    outs = []
    for r in range(N):
        out = torch.full((rows, D), float("nan"), dtype=torch.float32, device=eng.device)
        eng.combinePeers(areas[r], rows, 1, out)
        outs.append(out)
    eng.ctx.check()
    got = [o.cpu().numpy() for o in outs]
    for r in range(1, N):
        assert np.array_equal(got[r], got[0]), f"rank {r} differs from rank 0"
    for b in range(B):
        q_ref = O.rope(O.rmsnorm(q_in[b].ravel(), qg, Hq, D, 1e-6), Hq, D, Hq, ctx_len, base)
        k_new = O.rope(O.rmsnorm(k_in[b].ravel(), kg, Hkv, D, 1e-6), Hkv, D, Hkv, ctx_len, base).reshape(1, Hkv, D)
        kd = np.concatenate([_deq(k[b, r * shard:min(ctx_len, (r + 1) * shard)], q8) for r in range(N)] +
                            [_deq(k_new, q8)])
        vd = np.concatenate([_deq(v[b, r * shard:min(ctx_len, (r + 1) * shard)], q8) for r in range(N)] +
                            [_deq(v_in[b], q8)])
        ref = O.attention(q_ref, kd, vd, 1, Hq, Hkv, D, ctx_len)
        assert_close(got[0].reshape(B, Hq, D)[b].ravel(), ref, what=f"step_push N={N} seq {b}")
    for a in areas:
        a.close()
    for kv, _ in kvs:
        kv.close()
    rope.close()
