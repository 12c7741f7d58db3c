"""Per-sequence cache reset (brk_kv_reset with seq >= 0): the session restart of runDecodeGpu
(kernels.ts:1817-1825: a new session or pastLen 0 starts the cache over) for one sequence of a
batch, leaving every other sequence's rows -- in every layer -- untouched; seq -1 is
clearKvCache (kernels.ts:1777) for all of them.  fp16 and int8 caches."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("q8", [False, True])
def test_reset_one_sequence_keeps_the_others(eng, q8):
    import torch
    from brimkern_b200._lib import BRK_ERR_INVALID, BrkError
    from brimkern_b200.engine import KvCache
    dev = eng.device
    layers, B, Hkv, D, rows = 3, 4, 2, 64, 300
    kv = KvCache(eng.ctx, layers, B, Hkv, D, rows, q8=q8)
    gen = torch.Generator(device=dev)
    gen.manual_seed(3 + q8)
    for layer in range(layers):
        for b in range(B):
            kv.write_rows(layer, b, 0, torch.randn((rows, Hkv, D), generator=gen, device=dev),
                          torch.randn((rows, Hkv, D), generator=gen, device=dev))

    def snapshot():
        if q8:
            return {(l, b): [t.cpu().numpy() for t in kv.read_codes(l, b, 0, rows)]
                    for l in range(layers) for b in range(B)}
        return {(l, b): [t.cpu().numpy() for t in kv.read_rows(l, b, 0, rows)] for l in range(layers) for b in range(B)}

    before = snapshot()
    kv.reset(2)
    after = snapshot()
    for (l, b), arrs in after.items():
        if b == 2:
            assert all(not np.any(a) for a in arrs), f"layer {l}: sequence 2 not cleared"
        else:
            for x, y in zip(arrs, before[(l, b)]):
                assert np.array_equal(x.view(np.uint8), y.view(np.uint8)), f"layer {l} seq {b} changed"
    kv.reset(-1)
    assert all(not np.any(a) for arrs in snapshot().values() for a in arrs)
    with pytest.raises(BrkError) as ei:
        kv.reset(B)
    assert ei.value.code == BRK_ERR_INVALID
    eng.ctx.check()
    kv.close()


def test_engine_session_per_sequence(eng):
    """AttentionEngine.session with seq: one session per sequence of the batched cache."""
    import torch
    from brimkern_b200._lib import BrkError
    dev = eng.device
    kv = eng.ensureKv(1, 64, 2, 2, 64)
    eng.session("a", 0, seq=0)
    eng.session("b", 0, seq=1)
    rows = torch.randn((64, 2, 64), device=dev)
    for b in range(2):
        kv.write_rows(0, b, 0, rows, rows)
    eng.session("a", 10, seq=0)  # same session, later position: nothing happens
    eng.session("c", 0, seq=1)   # sequence 1 starts over; sequence 0 keeps its rows
    k0, _ = kv.read_rows(0, 0, 0, 64)
    k1, _ = kv.read_rows(0, 1, 0, 64)
    assert torch.equal(k0.float(), rows.half().float())
    assert not k1.float().abs().sum().item()
    with pytest.raises(BrkError):
        eng.session("unknown", 5, seq=0)  # cache lost for that sequence
    eng.ctx.check()
    eng.resetKvGpu()
