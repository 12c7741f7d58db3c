"""brk_attn_decode_static: the decode entry point for callers that cannot allocate device memory
while they run attention (hosts that give almost all of HBM to their own KV pool up front, or
whose decode loop must not stall on cudaMalloc's device-wide synchronisation).  It keeps its
split-KV partials in a fixed array inside the library instead of a growable workspace.

Checked through the C ABI against brk_attn_decode on two calls in a row (different inputs each
time, so stale contents of the shared array would show), with device free memory unchanged
across those calls, and the size limit reported as an error.  Kept in its own file so that it
is collected after every other test.
"""
import ctypes
import os

import numpy as np
import pytest

from tests.util import assert_close

pytestmark = pytest.mark.gpu


def _setup():
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from brimkern_b200 import _lib as L
    from brimkern_b200.engine import AttnConfig, Context, KvCache
    return torch, L, AttnConfig, Context, KvCache


def _call(L, fn, ctx, kv, cfg, pasts, q, out, stream):
    p = cfg.params()
    pos = (ctypes.c_int32 * len(pasts))(*pasts)
    return fn(ctx.handle, kv.handle, 0, ctypes.byref(p), len(pasts), 1, pos, q.data_ptr(), out.data_ptr(), stream)


def test_decode_static_matches_decode_twice():
    torch, L, AttnConfig, Context, KvCache = _setup()
    dev = torch.device("cuda", 0)
    Hq, Hkv, D, B, rows = 32, 8, 128, 8, 2048
    pasts = [rows - 1, 1500, 700, 63, rows - 1, 2000, 1, 1024]
    gen = torch.Generator(device=dev)
    gen.manual_seed(77)
    ref_ctx, ctx = Context(0), Context(0)
    kv_ref = KvCache(ref_ctx, 1, B, Hkv, D, rows)
    kv = KvCache(ctx, 1, B, Hkv, D, rows)
    for b in range(B):
        k = torch.randn((rows, Hkv, D), generator=gen, device=dev)
        v = torch.randn((rows, Hkv, D), generator=gen, device=dev)
        kv_ref.write_rows(0, b, 0, k, v)
        kv.write_rows(0, b, 0, k, v)
    cfg = AttnConfig(Hq, Hkv, D)
    qs = [torch.randn((B, 1, Hq, D), generator=gen, device=dev) for _ in range(3)]
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)

    # Reference outputs from the allocating entry point, on its own context.
    refs = []
    for q in qs[1:]:
        out = torch.empty_like(q)
        L.check(_call(L, L.lib().brk_attn_decode, ref_ctx, kv_ref, cfg, pasts, q, out, stream))
        refs.append(out)
    ref_ctx.check()

    outs = [torch.full_like(q, float("nan")) for q in qs]
    # First call on this device performs the one-time address lookup.
    L.check(_call(L, L.lib().brk_attn_decode_static, ctx, kv, cfg, pasts, qs[0], outs[0], stream))
    torch.cuda.synchronize()
    free_before, _ = torch.cuda.mem_get_info(dev)
    for i in (1, 2):
        L.check(_call(L, L.lib().brk_attn_decode_static, ctx, kv, cfg, pasts, qs[i], outs[i], stream))
    torch.cuda.synchronize()
    free_after, _ = torch.cuda.mem_get_info(dev)
    ctx.check()
    assert free_after == free_before, "the static entry point changed the device's free memory"
    for i in (1, 2):
        assert_close(outs[i].cpu().numpy(), refs[i - 1].cpu().numpy(), what=f"static call {i}")
    assert not torch.equal(outs[1], outs[2])  # different inputs, different outputs
    kv.close(), kv_ref.close(), ctx.close(), ref_ctx.close()


def test_decode_static_rejects_oversize_scratch():
    torch, L, AttnConfig, Context, KvCache = _setup()
    dev = torch.device("cuda", 0)
    Hq, Hkv, D, B, rows = 32, 8, 128, 64, 1024
    ctx = Context(0)
    kv = KvCache(ctx, 1, B, Hkv, D, rows)
    cfg = AttnConfig(Hq, Hkv, D)
    q = torch.zeros((B, 1, Hq, D), dtype=torch.float32, device=dev)
    out = torch.empty_like(q)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    old = os.environ.get("BRK_DECODE_SPLITS")
    os.environ["BRK_DECODE_SPLITS"] = "16"  # 16 x 2048 rows x 130 floats = 17 MB > 8 MiB
    try:
        rc = _call(L, L.lib().brk_attn_decode_static, ctx, kv, cfg, [rows - 1] * B, q, out, stream)
    finally:
        if old is None:
            del os.environ["BRK_DECODE_SPLITS"]
        else:
            os.environ["BRK_DECODE_SPLITS"] = old
    assert rc == L.BRK_ERR_CAPACITY
    assert b"static scratch" in L.lib().brk_last_error()
    ctx.check()
    kv.close(), ctx.close()
