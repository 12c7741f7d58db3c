"""CPU checks of the drop-in boundary: the library loads without a GPU, exports every entry point
include/brk_attn.h declares, the Python binding types each of them, and host-only entry points
(llama3 factors, error reporting) behave as documented."""
import ctypes
import os
import re

import numpy as np
import pytest

from brimkern_b200 import _lib as L

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include", "brk_attn.h")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(brk_\w+)\s*\(", text)))


def test_header_declares_entry_points():
    names = declared_functions()
    assert "brk_attn_decode" in names and "brk_attn_append" in names and "brk_kv_grow" in names
    assert len(names) >= 20


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(L.LIB_PATH)
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, f"declared but not exported: {missing}"


def test_binding_types_every_entry_point():
    bound = {name for name, _, _ in L.SIGNATURES}
    assert bound == set(declared_functions())
    L.lib()  # applies every signature


def test_abi_version():
    assert L.lib().brk_abi_version() == 2


def test_llama3_factors_match_oracle():
    """Host-only entry point: Meta's llama3 RoPE scaling divisors, against the oracle's
    independent restatement."""
    from oracle import oracle as O
    ff = np.zeros(32, np.float32)
    rc = L.lib().brk_llama3_rope_factors(64, 500000.0, 32.0, 1.0, 4.0, 8192,
                                         ff.ctypes.data_as(ctypes.POINTER(ctypes.c_float)))
    assert rc == L.BRK_OK
    ref = O.llama3_rope_factors(64, 500000.0, 32.0, 1.0, 4.0, 8192)
    np.testing.assert_array_equal(ff, ref)


@pytest.mark.parametrize("D,base,factor,low,high,orig", [
    (64, 500000.0, 32.0, 1.0, 4.0, 8192),   # Llama-3.2-1B
    (128, 500000.0, 8.0, 1.0, 4.0, 8192),   # Llama-3.1-8B
])
def test_llama3_factors_match_transformers(D, base, factor, low, high, orig):
    """The llama3 divisors against an independent implementation: Hugging Face transformers'
    llama3 RoPE initialisation (modeling_rope_utils._compute_llama3_parameters), whose scaled
    inverse frequencies are plain / ff.  Agreement to f32 rounding (transformers computes in
    f32, this library in double rounded once)."""
    transformers = pytest.importorskip("transformers")
    torch = pytest.importorskip("torch")
    from transformers.modeling_rope_utils import _compute_llama3_parameters
    cfg = transformers.LlamaConfig(hidden_size=32 * D, num_attention_heads=32, head_dim=D,
                                   max_position_embeddings=131072,
                                   rope_parameters={"rope_type": "llama3", "rope_theta": base, "factor": factor,
                                                    "low_freq_factor": low, "high_freq_factor": high,
                                                    "original_max_position_embeddings": orig})
    inv_scaled, attention_scaling = _compute_llama3_parameters(cfg, device="cpu")
    assert attention_scaling == 1.0
    plain = 1.0 / (base ** (torch.arange(0, D, 2, dtype=torch.int64).float() / D))
    ref = (plain / inv_scaled).numpy()
    ff = np.zeros(D // 2, np.float32)
    rc = L.lib().brk_llama3_rope_factors(D, base, factor, low, high, orig,
                                         ff.ctypes.data_as(ctypes.POINTER(ctypes.c_float)))
    assert rc == L.BRK_OK
    assert ff[0] == 1.0 and ff[-1] == factor  # high frequencies untouched, low ones divided by factor
    assert np.any((ff > 1.0) & (ff < factor))  # the smoothed band is exercised
    np.testing.assert_allclose(ff, ref, rtol=1e-6, atol=0)


def test_errors_are_reported_not_raised():
    ff = np.zeros(4, np.float32)
    rc = L.lib().brk_llama3_rope_factors(7, 1e4, 8.0, 1.0, 4.0, 8192, ff.ctypes.data_as(ctypes.POINTER(ctypes.c_float)))
    assert rc == L.BRK_ERR_INVALID
    assert b"llama3" in L.lib().brk_last_error()
    # Null handles are rejected with a status, never dereferenced.
    assert L.lib().brk_attn_decode(None, None, 0, None, 1, 1, None, None, None, None) == L.BRK_ERR_INVALID
    assert L.lib().brk_kv_capacity(None) == 0
    assert L.lib().brk_ctx_destroy(None) == L.BRK_OK
