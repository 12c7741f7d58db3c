"""CPU checks of the drop-in boundary: the library loads without a GPU, exports every entry point
include/brk_attn.h declares, the Python binding types each of them, and host-only entry points
(llama3 factors, error reporting) behave as documented."""
import ctypes
import os
import re

import numpy as np

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
    assert L.lib().brk_abi_version() == 1


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


def test_errors_are_reported_not_raised():
    ff = np.zeros(4, np.float32)
    rc = L.lib().brk_llama3_rope_factors(7, 1e4, 8.0, 1.0, 4.0, 8192, ff.ctypes.data_as(ctypes.POINTER(ctypes.c_float)))
    assert rc == L.BRK_ERR_INVALID
    assert b"llama3" in L.lib().brk_last_error()
    # Null handles are rejected with a status, never dereferenced.
    assert L.lib().brk_attn_decode(None, None, 0, None, 1, 1, None, None, None, None) == L.BRK_ERR_INVALID
    assert L.lib().brk_kv_capacity(None) == 0
    assert L.lib().brk_ctx_destroy(None) == L.BRK_OK
