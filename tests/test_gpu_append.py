"""KV append parity (GPU): the fused QK-norm + RoPE + fp16 store must reproduce the reference's
CPU chain rmsnormCpu -> ropeCpu/ropeFactorsCpu (kernels.ts:3395-3460) bit for bit, and place
every row at its position (kernels.ts:1727-1730)."""
import zlib

import numpy as np
import pytest

from oracle import oracle as O
from tests.util import bits_equal, normal

pytestmark = pytest.mark.gpu


def _oracle_prologue(x, rows, D, n_heads, past, base, ff, gain, eps, one_plus):
    y = x
    if gain is not None:
        y = O.rmsnorm(y, gain, rows, D, eps, one_plus)
    if base is not None:
        y = O.rope_factors(y, ff, rows, D, n_heads, past, base) if ff is not None else O.rope(y, rows, D, n_heads, past, base)
    return y


CASES = {
    # name: (Hq, Hkv, D, base, ff kind, qk-norm, one_plus, pasts, T, cap)
    "qwen3_norm_rope": (32, 8, 128, 1e6, None, True, False, [0, 100, 4093], 2, 4096),
    "llama_ff_pos131071": (32, 8, 64, 5e5, "llama3", False, False, [131070, 7, 65535], 1, 131072),
    "gemma_d256": (8, 4, 256, 1e4, None, False, False, [8191, 0], 1, 8192),
    "oneplus_norm_d64": (4, 2, 64, 1e4, "distinct", True, True, [5, 17], 3, 64),
    # Prefill-sized appends (>= 16384 head rows) take the 32-rows-per-warp kernel.
    "rows32_qwen3_d128": (32, 8, 128, 1e6, None, True, False, [0, 1000], 300, 1300),
    "rows32_llama_d64": (32, 8, 64, 5e5, "llama3", False, False, [100, 131000], 200, 131200),
    "rows32_oneplus_d256": (8, 4, 256, 1e4, None, True, True, [0, 50], 600, 700),
    # K rows spread over 10 decades (fp16 subnormals to overflow): the K store's f32 fast path and
    # its fallback to the fp64 chain near fp16 rounding midpoints.
    "rows32_wide_range_d128": (32, 8, 128, 1e6, None, False, False, [0, 700], 512, 1300, "wide"),
    "rows32_wide_range_norm_d64": (16, 4, 64, 1e4, None, True, True, [3, 0], 700, 710, "wide"),
}


@pytest.mark.parametrize("name", list(CASES))
def test_append_bit_exact(eng, name):
    import torch
    from brimkern_b200.engine import AttnConfig, KvCache, RopeTable, llama3_rope_factors

    Hq, Hkv, D, base, ffkind, norm, one_plus, pasts, T, cap = CASES[name][:10]
    spread = CASES[name][10] if len(CASES[name]) > 10 else None
    B = len(pasts)
    rng = np.random.default_rng(zlib.crc32(name.encode()))
    ff = None
    if ffkind == "llama3":
        ff = llama3_rope_factors(D, base, 32.0, 1.0, 4.0, 8192)
    elif ffkind == "distinct":
        ff = np.array([1 + (i % 5) * 0.7 for i in range(D // 2)], np.float32)
    qg = (1 + 0.02 * rng.standard_normal(D)).astype(np.float32) if norm else None
    kg = (1 + 0.02 * rng.standard_normal(D)).astype(np.float32) if norm else None
    if one_plus:
        qg = (0.1 * rng.standard_normal(D)).astype(np.float32)
        kg = (0.1 * rng.standard_normal(D)).astype(np.float32)
    q_in = normal(rng, B, T, Hq, D)
    k_in = normal(rng, B, T, Hkv, D)
    v_in = normal(rng, B, T, Hkv, D)
    if spread == "wide":
        k_in *= (10.0 ** rng.uniform(-6.0, 4.2, size=(B, T, Hkv, 1))).astype(np.float32)
        v_in *= (10.0 ** rng.uniform(-6.0, 4.2, size=(B, T, Hkv, 1))).astype(np.float32)

    dev = eng.device
    rope = RopeTable(eng.ctx, D, base, ff, max(pasts) + T)
    cfg = AttnConfig(Hq, Hkv, D, eps=1e-6, one_plus=one_plus, rope=rope,
                     q_norm=torch.from_numpy(qg).to(dev) if qg is not None else None,
                     k_norm=torch.from_numpy(kg).to(dev) if kg is not None else None)
    kv = KvCache(eng.ctx, 2, B, Hkv, D, cap)
    q_out = torch.empty((B, T, Hq, D), dtype=torch.float32, device=dev)
    eng.appendKv(kv, 1, cfg, torch.from_numpy(q_in).to(dev), torch.from_numpy(k_in).to(dev),
                 torch.from_numpy(v_in).to(dev), q_out, pasts)
    eng.ctx.check()
    q_got = q_out.cpu().numpy()
    for b, past in enumerate(pasts):
        q_ref = _oracle_prologue(q_in[b].ravel(), T * Hq, D, Hq, past, base, ff, qg, 1e-6, one_plus)
        assert bits_equal(q_got[b].ravel(), q_ref), f"{name}: rotated q of sequence {b} differs"
        k_ref = _oracle_prologue(k_in[b].ravel(), T * Hkv, D, Hkv, past, base, ff, kg, 1e-6, one_plus)
        k_ref16 = k_ref.astype(np.float16)
        kc, vc = kv.read_rows(1, b, past, T)
        assert bits_equal(kc.cpu().numpy().ravel(), k_ref16), f"{name}: K rows of sequence {b} differ"
        assert bits_equal(vc.cpu().numpy().ravel(), v_in[b].ravel().astype(np.float16)), f"{name}: V rows differ"
        # Rows around the appended ones, and layer 0, stay untouched (zero).
        if past > 0:
            kprev, _ = kv.read_rows(1, b, past - 1, 1)
            assert not kprev.cpu().numpy().any()
        k0, _ = kv.read_rows(0, b, past, T)
        assert not k0.cpu().numpy().any()
    kv.close()
    rope.close()


def test_rope_twins_match_golden(eng, golden):
    """rope / ropeFactors readback twins (kernels.ts:556, 568) equal the reference's own
    output (golden fixtures) bit for bit."""
    for name in ["rope_small", "rope_ff_ones", "rope_ff_plain", "rope_ff_distinct", "rope_qwen3_pos4095",
                 "rope_llama_pos131071"]:
        c, a = golden[name]
        if c["fn"] == "ropeCpu":
            got = eng.rope(a["x"], c["rows"], c["head_dim"], c["n_heads"], c["past_len"], c["base"])
        else:
            got = eng.ropeFactors(a["x"], a["ff"], c["rows"], c["head_dim"], c["n_heads"], c["past_len"], c["base"])
        assert bits_equal(got, a["out"]), name


def test_rmsnorm_twin_matches_golden(eng, golden):
    for name in ["rmsnorm_qk_small", "rmsnorm_qk_hd128", "rmsnorm_oneplus", "rmsnorm_default_eps"]:
        c, a = golden[name]
        eps = 1e-5 if c["eps"] is None else c["eps"]
        got = eng.rmsnorm(a["x"], a["w"], c["rows"], c["dim"], eps, bool(c["one_plus"]))
        assert bits_equal(got, a["out"]), name


def test_append_errors(eng):
    import torch
    from brimkern_b200._lib import BRK_ERR_CAPACITY, BrkError
    from brimkern_b200.engine import AttnConfig, KvCache, RopeTable

    kv = KvCache(eng.ctx, 1, 1, 2, 64, 16)
    rope = RopeTable(eng.ctx, 64, 1e4, None, 16)
    cfg = AttnConfig(4, 2, 64, rope=rope)
    z = lambda *s: torch.zeros(s, dtype=torch.float32, device=eng.device)  # noqa: E731
    with pytest.raises(BrkError) as ei:  # row 16 is beyond capacity 16
        eng.appendKv(kv, 0, cfg, z(1, 1, 4, 64), z(1, 1, 2, 64), z(1, 1, 2, 64), z(1, 1, 4, 64), [16])
    assert ei.value.code == BRK_ERR_CAPACITY
    kv.grow(17)
    assert kv.capacity == 1040  # ensureKv: max(rows, cap + 1024, 1024)
    with pytest.raises(BrkError) as ei:  # position 16 is beyond the 16-position rope table
        eng.appendKv(kv, 0, cfg, z(1, 1, 4, 64), z(1, 1, 2, 64), z(1, 1, 2, 64), z(1, 1, 4, 64), [16])
    assert ei.value.code == BRK_ERR_CAPACITY
    kv.close()
    rope.close()
