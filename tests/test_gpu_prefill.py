"""Tensor-core prefill parity (GPU): brk_attn_prefill (tcgen05.mma, TMEM accumulators) against
the oracle (attentionCpu, kernels.ts:3466) fed the same fp16-rounded K/V, within the north-star
tolerance; causal chunks with a past offset (the reference's recAttention with pastLen), GQA,
partial tiles, window and softcap, and the chunked prefill loop end to end."""
import zlib

import numpy as np
import pytest

from oracle import oracle as O
from tests.util import assert_close, f16_round, normal

pytestmark = pytest.mark.gpu


def _run(eng, name, Hq, Hkv, D, pasts, T, scale=None, softcap=0.0, window=0, kernel="prefill"):
    import torch
    from brimkern_b200.engine import AttnConfig, KvCache
    rng = np.random.default_rng(zlib.crc32(name.encode()))
    B = len(pasts)
    rows = max(pasts) + T
    kv = KvCache(eng.ctx, 1, B, Hkv, D, rows)
    ks, vs = [], []
    for b in range(B):
        k = normal(rng, rows, Hkv, D)
        v = normal(rng, rows, Hkv, D)
        kv.write_rows(0, b, 0, torch.from_numpy(k).to(eng.device), torch.from_numpy(v).to(eng.device))
        ks.append(f16_round(k))
        vs.append(f16_round(v))
    q = normal(rng, B, T, Hq, D)
    out = torch.full((B, T, Hq, D), float("nan"), dtype=torch.float32, device=eng.device)
    cfg = AttnConfig(Hq, Hkv, D, scale=scale, softcap=softcap, window=window)
    eng.recAttention(kv, 0, cfg, torch.from_numpy(q).to(eng.device), out, pasts, kernel=kernel)
    eng.ctx.check()
    got = out.cpu().numpy()
    kv.close()
    refs, _ = O.attention_batch(q.ravel(), np.stack(ks).ravel(), np.stack(vs).ravel(), B, rows * Hkv * D, T, Hq, Hkv,
                                D, pasts, scale, softcap, window)
    assert_close(got.ravel(), refs, what=name)


@pytest.mark.parametrize("T,past", [(1, 0), (7, 0), (128, 0), (129, 0), (300, 173), (256, 1000)])
def test_prefill_shapes_d128(eng, T, past):
    _run(eng, f"pf128_{T}_{past}", 8, 2, 128, [past], T)


@pytest.mark.parametrize("T,past", [(5, 3), (200, 0), (130, 64)])
def test_prefill_gqa7_d64(eng, T, past):
    """The Qwen2.5-0.5B grouping (14 q / 2 kv heads, group 7) at head_dim 64."""
    _run(eng, f"pf64_{T}_{past}", 14, 2, 64, [past, past + 5], T)


def test_prefill_config3_chunk(eng):
    """BASELINE config 3 shape: Qwen3-4B 32 q / 8 kv, D 128, a 512-token chunk after 1536 cached
    tokens (the 4th chunk of a 2048 prompt) and a first chunk, batch 2."""
    _run(eng, "pf_cfg3", 32, 8, 128, [1536, 0], 512)


def test_prefill_window_softcap(eng):
    _run(eng, "pf_win_cap", 8, 4, 128, [700, 20], 200, scale=1 / 16, softcap=50.0, window=256)


def test_prefill_matches_decode_kernel(eng):
    """Both kernels on one multi-token shape agree through the dispatch paths."""
    _run(eng, "pf_vs_dec_p", 8, 2, 64, [77], 12, kernel="prefill")
    _run(eng, "pf_vs_dec_d", 8, 2, 64, [77], 12, kernel="decode")


def test_chunked_prefill_end_to_end(eng):
    """A 2048-token prompt in 512-token chunks through append + prefill (QK-norm + RoPE), checked
    against the oracle chain rmsnorm -> rope -> attentionCpu over the whole prompt."""
    import torch
    from brimkern_b200.engine import AttnConfig, KvCache, RopeTable
    rng = np.random.default_rng(31)
    Hq, Hkv, D, T, base = 8, 2, 128, 2048, 1e6
    qn = (1 + 0.02 * rng.standard_normal(D)).astype(np.float32)
    kn = (1 + 0.02 * rng.standard_normal(D)).astype(np.float32)
    q_in = normal(rng, 1, T, Hq, D)
    k_in = normal(rng, 1, T, Hkv, D)
    v_in = normal(rng, 1, T, Hkv, D)
    dev = eng.device
    rope = RopeTable(eng.ctx, D, base, None, T)
    cfg = AttnConfig(Hq, Hkv, D, q_norm=torch.from_numpy(qn).to(dev), k_norm=torch.from_numpy(kn).to(dev), rope=rope)
    kv = KvCache(eng.ctx, 1, 1, Hkv, D, T)
    out = eng.prefillChunked(kv, 0, cfg, torch.from_numpy(q_in).to(dev), torch.from_numpy(k_in).to(dev),
                             torch.from_numpy(v_in).to(dev), [0], chunk=512)
    eng.ctx.check()
    q = O.rope(O.rmsnorm(q_in.ravel(), qn, T * Hq, D, 1e-6), T * Hq, D, Hq, 0, base)
    k = O.rope(O.rmsnorm(k_in.ravel(), kn, T * Hkv, D, 1e-6), T * Hkv, D, Hkv, 0, base)
    ref, _ = O.attention_batch(q, f16_round(k), f16_round(v_in.ravel()), 1, T * Hkv * D, T, Hq, Hkv, D, [0])
    assert_close(out.cpu().numpy().ravel(), ref, what="chunked prefill")
    kv.close()
    rope.close()


@pytest.mark.parametrize("D,norm,one_plus", [(128, True, False), (64, False, False), (128, True, True)])
def test_prefill_step_fused_prologue_matches(eng, D, norm, one_plus):
    """brk_attn_prefill_step (q prologue fused into the prefill kernel, in f32) matches append +
    prefill on the append's fp64-rotated q within the north-star tolerance, and writes the same
    cache rows bit for bit."""
    import torch
    from brimkern_b200.engine import AttnConfig, KvCache, RopeTable
    rng = np.random.default_rng(D + 7 * norm + 13 * one_plus)
    Hq, Hkv, T, pasts, base = 8, 2, 300, [0, 100], 1e6
    dev = eng.device
    g = (0.1 if one_plus else 0.02)
    qn = torch.from_numpy(((0 if one_plus else 1) + g * rng.standard_normal(D)).astype(np.float32)).to(dev)
    kn = torch.from_numpy(((0 if one_plus else 1) + g * rng.standard_normal(D)).astype(np.float32)).to(dev)
    rope = RopeTable(eng.ctx, D, base, None, max(pasts) + T)
    cfg = AttnConfig(Hq, Hkv, D, q_norm=qn if norm else None, k_norm=kn if norm else None, one_plus=one_plus,
                     rope=rope)
    q = torch.from_numpy(normal(rng, 2, T, Hq, D)).to(dev)
    k = torch.from_numpy(normal(rng, 2, T, Hkv, D)).to(dev)
    v = torch.from_numpy(normal(rng, 2, T, Hkv, D)).to(dev)
    kv_a = KvCache(eng.ctx, 1, 2, Hkv, D, max(pasts) + T)
    kv_b = KvCache(eng.ctx, 1, 2, Hkv, D, max(pasts) + T)
    q_rot = torch.empty_like(q)
    out_a = torch.empty_like(q)
    out_b = torch.empty_like(q)
    eng.appendKv(kv_a, 0, cfg, q, k, v, q_rot, pasts)
    eng.recAttention(kv_a, 0, cfg, q_rot, out_a, pasts, kernel="prefill")
    eng.prefillStep(kv_b, 0, cfg, q, k, v, out_b, pasts)
    eng.ctx.check()
    assert_close(out_b.cpu().numpy(), out_a.cpu().numpy(), what="fused prologue")
    for b, p in enumerate(pasts):
        ka, va = kv_a.read_rows(0, b, p, T)
        kb, vb = kv_b.read_rows(0, b, p, T)
        assert torch.equal(ka.view(torch.int16), kb.view(torch.int16))
        assert torch.equal(va.view(torch.int16), vb.view(torch.int16))
    kv_a.close(), kv_b.close(), rope.close()


@pytest.mark.parametrize("name,Hq,Hkv,D,pasts,T,softcap,window", [
    ("h_d128", 32, 8, 128, [0, 1000, 37], 300, 0.0, 0),
    ("h_gqa7_d64", 14, 2, 64, [513, 0], 257, 0.0, 0),
    ("h_win_cap", 16, 4, 128, [700], 384, 30.0, 200),
])
def test_prefill_half_q_matches_oracle(eng, name, Hq, Hkv, D, pasts, T, softcap, window):
    """brk_attn_prefill_h: q given as fp16 rows and loaded by TMA (both streams' tiles, a lone
    stream at an odd GQA group's last tile, tiles past the chunk's end) against attentionCpu on the
    same fp16-rounded q and K/V."""
    import torch
    from brimkern_b200.engine import AttnConfig, KvCache
    rng = np.random.default_rng(zlib.crc32(name.encode()))
    B = len(pasts)
    rows = max(pasts) + T
    kv = KvCache(eng.ctx, 1, B, Hkv, D, rows)
    ks, vs = [], []
    for b in range(B):
        k = normal(rng, rows, Hkv, D)
        v = normal(rng, rows, Hkv, D)
        kv.write_rows(0, b, 0, torch.from_numpy(k).to(eng.device), torch.from_numpy(v).to(eng.device))
        ks.append(f16_round(k))
        vs.append(f16_round(v))
    q = f16_round(normal(rng, B, T, Hq, D))
    q16 = torch.from_numpy(q).to(eng.device).half()
    out = torch.full((B, T, Hq, D), float("nan"), dtype=torch.float32, device=eng.device)
    cfg = AttnConfig(Hq, Hkv, D, softcap=softcap, window=window)
    eng.prefillHalfQ(kv, 0, cfg, q16, out, pasts)
    eng.ctx.check()
    got = out.cpu().numpy()
    kv.close()
    refs, _ = O.attention_batch(q.ravel(), np.stack(ks).ravel(), np.stack(vs).ravel(), B, rows * Hkv * D, T, Hq, Hkv,
                                D, pasts, None, softcap, window)
    assert_close(got.ravel(), refs, what=name)


def test_prefill_step_short_chunk_uses_fused_prologue(eng):
    """brk_attn_prefill_step with fewer than 8 tokens (the q prologue inside the prefill kernel)
    against append + prefill on the append's rotated q."""
    import torch
    from brimkern_b200.engine import AttnConfig, KvCache, RopeTable
    rng = np.random.default_rng(5)
    Hq, Hkv, D, T, pasts = 8, 2, 128, 5, [40, 0]
    dev = eng.device
    qn = torch.from_numpy((1 + 0.02 * rng.standard_normal(D)).astype(np.float32)).to(dev)
    rope = RopeTable(eng.ctx, D, 1e6, None, max(pasts) + T)
    cfg = AttnConfig(Hq, Hkv, D, q_norm=qn, k_norm=qn, rope=rope)
    q = torch.from_numpy(normal(rng, 2, T, Hq, D)).to(dev)
    k = torch.from_numpy(normal(rng, 2, T, Hkv, D)).to(dev)
    v = torch.from_numpy(normal(rng, 2, T, Hkv, D)).to(dev)
    kv_a = KvCache(eng.ctx, 1, 2, Hkv, D, max(pasts) + T)
    kv_b = KvCache(eng.ctx, 1, 2, Hkv, D, max(pasts) + T)
    q_rot, out_a, out_b = torch.empty_like(q), torch.empty_like(q), torch.empty_like(q)
    eng.appendKv(kv_a, 0, cfg, q, k, v, q_rot, pasts)
    eng.recAttention(kv_a, 0, cfg, q_rot, out_a, pasts, kernel="prefill")
    eng.prefillStep(kv_b, 0, cfg, q, k, v, out_b, pasts)
    eng.ctx.check()
    assert_close(out_b.cpu().numpy(), out_a.cpu().numpy(), what="short chunk")
    kv_a.close(), kv_b.close(), rope.close()


def _mixed_rescale_warps(q, ks, pasts, Hq, Hkv, D, scale=None):
    """How many (sequence, head, warp of 32 query rows, 64-key tile) have rows that disagree on
    rescaling O at that tile, replaying the kernel's per-row rule on the CPU: a row's max (log2
    units) is raised when a tile's max exceeds it by more than 8, or on its first finite score,
    and O is rescaled on every raise but that first one.  Query tiles start at multiples of 128
    rows, so 32-row warps never straddle two tiles."""
    B, T = q.shape[0], q.shape[1]
    G = Hq // Hkv
    sc = (scale if scale is not None else 1.0 / np.sqrt(D)) * 1.4426950408889634
    mixed = 0
    for b in range(B):
        nkeys = pasts[b] + T
        ntiles = (nkeys + 63) // 64
        t = np.arange(T)
        keys = np.arange(ntiles * 64)
        valid = keys[None, :] <= pasts[b] + t[:, None]
        for h in range(Hq):
            s = q[b, :, h, :].astype(np.float64) @ ks[b][:nkeys, h // G, :].astype(np.float64).T * sc
            s = np.pad(s, ((0, 0), (0, ntiles * 64 - nkeys)), constant_values=-np.inf)
            s = np.where(valid, s, -np.inf).reshape(T, ntiles, 64).max(axis=2)
            m = np.full(T, -np.inf)
            for j in range(ntiles):
                mt = s[:, j]
                first = np.isneginf(m) & ~np.isneginf(mt)
                raise_ = (mt > m + 8) | first
                resc = raise_ & ~np.isneginf(m) & (j >= 1)
                m = np.where(raise_, mt, m)
                pad = (-T) % 32
                w = np.pad(resc, (0, pad)).reshape(-1, 32)
                mixed += int(np.sum(w.any(axis=1) & ~w.all(axis=1)))
    return mixed


@pytest.mark.parametrize("name,Hq,Hkv,D,pasts,T,qscale,half_q", [
    ("sharp_d128", 8, 2, 128, [0, 300], 256, 4.0, False),
    ("sharp_d128_h", 8, 2, 128, [0, 300], 256, 4.0, True),
    ("sharp_gqa7_d64", 14, 2, 64, [0, 129], 200, 4.0, False),
])
def test_prefill_sharp_scores_mixed_rescale(eng, name, Hq, Hkv, D, pasts, T, qscale, half_q):
    """Scores with a wide range (q four times N(0,1), no QK-norm): later key tiles raise some
    rows' running max by more than 2^8 but not their warp neighbours', so the rows of one warp
    disagree on rescaling O in TMEM.  The rescale pass uses warp-collective TMEM loads and stores,
    which the kernel must run with the whole warp (rows that need no rescale take factor 1).  The
    inputs are checked on the CPU to cause such mixed warps before the GPU result is compared with
    attentionCpu.  attentionCpu gets q rounded to fp16, the tensor core's operand: at these score
    ranges that rounding alone moves a few outputs by up to ~4e-3 (a CPU emulation of the kernel's
    arithmetic gives the same errors), which is not what this test is about."""
    import torch
    from brimkern_b200.engine import AttnConfig, KvCache
    rng = np.random.default_rng(zlib.crc32(name.encode()))
    B = len(pasts)
    rows = max(pasts) + T
    kv = KvCache(eng.ctx, 1, B, Hkv, D, rows)
    ks, vs = [], []
    for b in range(B):
        k = normal(rng, rows, Hkv, D)
        v = normal(rng, rows, Hkv, D)
        kv.write_rows(0, b, 0, torch.from_numpy(k).to(eng.device), torch.from_numpy(v).to(eng.device))
        ks.append(f16_round(k))
        vs.append(f16_round(v))
    q = normal(rng, B, T, Hq, D) * np.float32(qscale)
    if half_q:
        q = f16_round(q)
    q_ref = f16_round(q)
    assert _mixed_rescale_warps(q_ref, ks, pasts, Hq, Hkv, D) > 0, "inputs cause no mixed-rescale warp"
    out = torch.full((B, T, Hq, D), float("nan"), dtype=torch.float32, device=eng.device)
    cfg = AttnConfig(Hq, Hkv, D)
    if half_q:
        eng.prefillHalfQ(kv, 0, cfg, torch.from_numpy(q).to(eng.device).half(), out, pasts)
    else:
        eng.recAttention(kv, 0, cfg, torch.from_numpy(q).to(eng.device), out, pasts, kernel="prefill")
    eng.ctx.check()
    got = out.cpu().numpy()
    kv.close()
    refs, _ = O.attention_batch(q_ref.ravel(), np.stack(ks).ravel(), np.stack(vs).ravel(), B, rows * Hkv * D, T, Hq,
                                Hkv, D, pasts)
    assert_close(got.ravel(), refs, what=name)
