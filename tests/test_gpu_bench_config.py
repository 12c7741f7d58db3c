"""The exact configuration `bench.py` measures by default, checked against the oracle.

BASELINE config 2 at batch 64: Qwen3-4B shape (32 q / 8 kv heads, head_dim 128, per-head q/k
RMSNorm, NeoX RoPE theta 1e6), KV length 4096 including the token appended this step.  As in the
benchmark, every layer goes through brk_attn_step (one launch: the append fused into the decode
kernel, launched as a programmatic dependent of the previous layer's) with the automatic split
choice (one split per (sequence, kv head) on a 148-SM B200), and again with four splits merged
in-kernel by the last CTA; the step is replayed from a CUDA graph.  Two layers, so that layer 1
follows layer 0 in the chain.

Checked on a seeded sample of sequences: the appended K/V rows bit for bit against the oracle
chain rmsnormCpu -> ropeCpu -> fp16 (kernels.ts:3395-3460), and the attention output within the
north-star tolerance of attentionCpu (kernels.ts:3466) fed the cache's fp16 rows; every replay
gives the same bits.
"""
import ctypes

import numpy as np
import pytest

from oracle import oracle as O
from tests.util import assert_close, bits_equal

pytestmark = pytest.mark.gpu


@pytest.fixture(params=[None, 4], ids=["auto", "split4"])
def splits(request):
    import os
    old = os.environ.get("BRK_DECODE_SPLITS")
    if request.param is not None:
        os.environ["BRK_DECODE_SPLITS"] = str(request.param)
    yield request.param
    if request.param is not None:
        if old is None:
            del os.environ["BRK_DECODE_SPLITS"]
        else:
            os.environ["BRK_DECODE_SPLITS"] = old


def test_bench_config_step_graph_replay(eng, splits):
    import torch
    from brimkern_b200 import _lib as L
    from brimkern_b200.engine import AttnConfig, KvCache, RopeTable
    dev = eng.device
    B, Hq, Hkv, D, Lkv, layers, base = 64, 32, 8, 128, 4096, 2, 1e6
    past = [Lkv - 1] * B
    gen = torch.Generator(device=dev)
    gen.manual_seed(1000)
    qn = (1 + 0.02 * torch.randn(D, generator=gen, device=dev)).float()
    kn = (1 + 0.02 * torch.randn(D, generator=gen, device=dev)).float()
    rope = RopeTable(eng.ctx, D, base, None, Lkv)
    cfg = AttnConfig(Hq, Hkv, D, q_norm=qn, k_norm=kn, rope=rope)
    kv = KvCache(eng.ctx, layers, B, Hkv, D, Lkv)
    tmp_k = torch.empty((Lkv, Hkv, D), dtype=torch.float32, device=dev)
    tmp_v = torch.empty_like(tmp_k)
    for layer in range(layers):
        for b in range(B):
            tmp_k.normal_(generator=gen)
            tmp_v.normal_(generator=gen)
            kv.write_rows(layer, b, 0, tmp_k, tmp_v)
    q_in = torch.randn((layers, B, 1, Hq, D), generator=gen, device=dev)
    k_in = torch.randn((layers, B, 1, Hkv, D), generator=gen, device=dev)
    v_in = torch.randn((layers, B, 1, Hkv, D), generator=gen, device=dev)
    q_work = torch.empty_like(q_in)
    out = torch.full((layers, B, 1, Hq, D), float("nan"), device=dev)

    # The split count the benchmark's number comes from (one split -- two waves of 512 CTAs at
    # two per SM -- on a 148-SM B200), or a forced one.
    p = cfg.params()
    pos = (ctypes.c_int32 * B)(*past)
    nsplit = L.lib().brk_attn_decode_splits(eng.ctx.handle, kv.handle, ctypes.byref(p), B, 1, pos)
    if splits is None and torch.cuda.get_device_properties(dev).multi_processor_count == 148:
        assert nsplit == 1
    if splits is not None:
        assert nsplit == splits

    def step():
        for layer in range(layers):
            eng.attentionLayer(kv, layer, cfg, q_in[layer], k_in[layer], v_in[layer], past, q_work[layer], out[layer])

    eng.ctx.reserve(64 << 20)
    step()  # warm-up on the host, as the benchmark does before capturing
    torch.cuda.synchronize()
    eng.ctx.check()
    side = torch.cuda.Stream(device=dev)
    side.wait_stream(torch.cuda.current_stream())
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(side):
        with torch.cuda.graph(g, stream=side):
            step()
    torch.cuda.current_stream().wait_stream(side)
    replays = []
    for _ in range(3):
        out.fill_(float("nan"))
        g.replay()
        torch.cuda.synchronize()
        eng.ctx.check()
        replays.append(out.clone())
    for r in replays[1:]:
        assert torch.equal(r, replays[0]), "graph replays of the same step differ"

    got = replays[0].cpu().numpy()
    qn_h, kn_h = qn.cpu().numpy(), kn.cpu().numpy()
    qh, kh, vh = q_in.cpu().numpy(), k_in.cpu().numpy(), v_in.cpu().numpy()
    for layer in range(layers):
        for b in (0, 21, 42, 63):
            k_rows, v_rows = kv.read_rows(layer, b, 0, Lkv)
            k_rows = k_rows.float().cpu().numpy()
            v_rows = v_rows.float().cpu().numpy()
            # The appended row (position 4095): bit for bit.
            q_ref = O.rope(O.rmsnorm(qh[layer, b].ravel(), qn_h, Hq, D, 1e-6), Hq, D, Hq, past[b], base)
            k_ref = O.rope(O.rmsnorm(kh[layer, b].ravel(), kn_h, Hkv, D, 1e-6), Hkv, D, Hkv, past[b], base)
            assert bits_equal(k_rows[Lkv - 1].ravel().astype(np.float16), k_ref.astype(np.float16)), \
                f"layer {layer} seq {b}: appended K row differs"
            assert bits_equal(v_rows[Lkv - 1].ravel().astype(np.float16), vh[layer, b].ravel().astype(np.float16)), \
                f"layer {layer} seq {b}: appended V row differs"
            ref = O.attention(q_ref, k_rows.ravel(), v_rows.ravel(), 1, Hq, Hkv, D, past[b])
            assert_close(got[layer, b].ravel(), ref, what=f"bench config layer {layer} seq {b}")
    del g
    kv.close()
    rope.close()
