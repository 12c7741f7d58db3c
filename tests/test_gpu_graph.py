"""The decode step through the C ABI is capturable in a CUDA graph once the context workspace is
sized: a replay writes the same cache rows and outputs, bit for bit, as host-launched calls."""
import numpy as np
import pytest

from tests.util import normal

pytestmark = pytest.mark.gpu


def test_decode_step_graph_replay_matches_eager(eng):
    import torch
    from brimkern_b200.engine import AttnConfig, KvCache, RopeTable
    rng = np.random.default_rng(5)
    dev = eng.device
    B, Hq, Hkv, D, past, layers = 4, 32, 8, 128, 1500, 3
    rope = RopeTable(eng.ctx, D, 1e6, None, past + 2)
    qn = torch.from_numpy((1 + 0.02 * rng.standard_normal(D)).astype(np.float32)).to(dev)
    cfg = AttnConfig(Hq, Hkv, D, q_norm=qn, k_norm=qn, rope=rope)
    caches = []
    for _ in range(2):
        kv = KvCache(eng.ctx, layers, B, Hkv, D, past + 2)
        caches.append(kv)
    hist = [normal(rng, past, Hkv, D) for _ in range(2 * layers * B)]
    for kv in caches:
        i = 0
        for layer in range(layers):
            for b in range(B):
                kv.write_rows(layer, b, 0, torch.from_numpy(hist[i]).to(dev), torch.from_numpy(hist[i + 1]).to(dev))
                i += 2
    q = torch.from_numpy(normal(rng, layers, B, 1, Hq, D)).to(dev)
    k = torch.from_numpy(normal(rng, layers, B, 1, Hkv, D)).to(dev)
    v = torch.from_numpy(normal(rng, layers, B, 1, Hkv, D)).to(dev)
    outs = [torch.empty((layers, B, 1, Hq, D), device=dev) for _ in range(2)]
    work = [torch.empty((layers, B, 1, Hq, D), device=dev) for _ in range(2)]
    eng.ctx.reserve(64 << 20)

    def step(c):
        for layer in range(layers):
            eng.attentionLayer(caches[c], layer, cfg, q[layer], k[layer], v[layer], [past] * B, work[c][layer],
                               outs[c][layer])

    step(0)  # host launches
    torch.cuda.synchronize()
    side = torch.cuda.Stream(device=dev)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(side):
        with torch.cuda.graph(g, stream=side):
            step(1)
    g.replay()
    torch.cuda.synchronize()
    eng.ctx.check()
    assert torch.equal(outs[0], outs[1])
    for layer in range(layers):
        for b in range(B):
            k0, v0 = caches[0].read_rows(layer, b, past, 1)
            k1, v1 = caches[1].read_rows(layer, b, past, 1)
            assert torch.equal(k0.view(torch.int16), k1.view(torch.int16))
            assert torch.equal(v0.view(torch.int16), v1.view(torch.int16))
    for kv in caches:
        kv.close()
    rope.close()
