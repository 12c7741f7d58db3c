"""brk_attn_decode_static: the decode entry point for callers that cannot allocate device memory
while they run attention (hosts that give almost all of HBM to their own KV pool up front, or
whose decode loop must not stall on cudaMalloc's device-wide synchronisation).  It keeps its
split-KV partials in a fixed array inside the library instead of a growable workspace.

Checked through the C ABI against brk_attn_decode on three calls in a row with the split-KV
path forced (different inputs each time, so stale contents of the shared array would show),
with device free memory unchanged from before the first static call to after the last (the
context creation takes what the calls need), and the size limit reported as an error.  Kept
in its own file so that it is collected after every other test.
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


def _with_splits(n):
    """Context manager setting BRK_DECODE_SPLITS for the calls inside it."""
    import contextlib

    @contextlib.contextmanager
    def cm():
        old = os.environ.get("BRK_DECODE_SPLITS")
        os.environ["BRK_DECODE_SPLITS"] = str(n)
        try:
            yield
        finally:
            if old is None:
                del os.environ["BRK_DECODE_SPLITS"]
            else:
                os.environ["BRK_DECODE_SPLITS"] = old
    return cm()


def test_decode_static_matches_decode_twice():
    torch, L, AttnConfig, Context, KvCache = _setup()
    dev = torch.device("cuda", 0)
    Hq, Hkv, D, B, rows = 32, 8, 128, 8, 2048
    pasts = [rows - 1, 1500, 700, 63, rows - 1, 2000, 1, 1024]
    torch.cuda.init()
    torch.cuda.synchronize()
    # The context takes what the static calls need (kernels loaded, the static array's module
    # loaded); in a fresh process that is where the array's memory goes.
    free_pre_ctx, _ = torch.cuda.mem_get_info(dev)
    ctx = Context(0)
    torch.cuda.synchronize()
    free_post_ctx, _ = torch.cuda.mem_get_info(dev)
    assert free_post_ctx <= free_pre_ctx
    gen = torch.Generator(device=dev)
    gen.manual_seed(77)
    ref_ctx = Context(0)
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
    pos = (ctypes.c_int32 * B)(*pasts)
    p = cfg.params()

    with _with_splits(4):
        # The split-KV path (partials in the static array, then the in-kernel merge) is used.
        assert L.lib().brk_attn_decode_splits(ctx.handle, kv.handle, ctypes.byref(p), B, 1, pos) == 4
        # Reference outputs from the allocating entry point, on its own context.
        refs = []
        for q in qs:
            out = torch.empty_like(q)
            L.check(_call(L, L.lib().brk_attn_decode, ref_ctx, kv_ref, cfg, pasts, q, out, stream))
            refs.append(out)
        ref_ctx.check()

        outs = [torch.full_like(q, float("nan")) for q in qs]
        torch.cuda.synchronize()
        free_before, _ = torch.cuda.mem_get_info(dev)
        # The very first static calls of the process (when run alone): no set-up left to do.
        for i in range(3):
            L.check(_call(L, L.lib().brk_attn_decode_static, ctx, kv, cfg, pasts, qs[i], outs[i], stream))
        torch.cuda.synchronize()
        free_after, _ = torch.cuda.mem_get_info(dev)
    ctx.check()
    assert free_after == free_before, "the static entry point changed the device's free memory"
    for i in range(3):
        assert_close(outs[i].cpu().numpy(), refs[i].cpu().numpy(), what=f"static call {i}")
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
    with _with_splits(16):  # 16 x 2048 rows x 130 floats = 17 MB > 8 MiB
        rc = _call(L, L.lib().brk_attn_decode_static, ctx, kv, cfg, [rows - 1] * B, q, out, stream)
    assert rc == L.BRK_ERR_CAPACITY
    assert b"static scratch" in L.lib().brk_last_error()
    ctx.check()
    kv.close(), ctx.close()
