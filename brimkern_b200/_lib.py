"""ctypes binding of libbrk_attn.so (the C ABI in include/brk_attn.h).

The library is built in-tree (``brimkern_b200/libbrk_attn.so``, see ``build()``).  There is no
fallback: if the library cannot be loaded, importing the engine raises.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))
# The in-tree build; BRK_ATTN_LIB may name another build of the same sources (tuning variants).
LIB_PATH = os.environ.get("BRK_ATTN_LIB") or os.path.join(HERE, "libbrk_attn.so")
CSRC = os.path.join(HERE, "csrc")

BRK_OK = 0
BRK_ERR_INVALID = -1
BRK_ERR_CUDA = -2
BRK_ERR_CAPACITY = -3
BRK_ERR_UNSUPPORTED = -4
BRK_ERR_DEVICE = -5
BRK_MAX_BATCH = 512
BRK_KV_F16 = 0
BRK_KV_I8 = 1
BRK_DECODE_STATIC_SCRATCH_BYTES = 8 << 20
BRK_MAX_PEERS = 8
BRK_PEER_HANDLE_BYTES = 64

_ERR_NAMES = {BRK_ERR_INVALID: "INVALID", BRK_ERR_CUDA: "CUDA", BRK_ERR_CAPACITY: "CAPACITY",
              BRK_ERR_UNSUPPORTED: "UNSUPPORTED", BRK_ERR_DEVICE: "DEVICE"}


class BrkError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"brk error {_ERR_NAMES.get(code, code)}: {msg}")
        self.code = code


class KvDesc(ctypes.Structure):
    _fields_ = [("n_layers", ctypes.c_int), ("batch", ctypes.c_int), ("n_kv_heads", ctypes.c_int),
                ("head_dim", ctypes.c_int), ("capacity", ctypes.c_int), ("dtype", ctypes.c_int)]


class AttnParams(ctypes.Structure):
    _fields_ = [("n_heads", ctypes.c_int), ("n_kv_heads", ctypes.c_int), ("head_dim", ctypes.c_int),
                ("scale", ctypes.c_float), ("softcap", ctypes.c_float), ("window", ctypes.c_int),
                ("kv_offset", ctypes.c_int), ("norm_one_plus", ctypes.c_int), ("eps", ctypes.c_double),
                ("q_norm", ctypes.c_void_p), ("k_norm", ctypes.c_void_p), ("rope", ctypes.c_void_p)]


# (name, restype, argtypes) for every entry point of include/brk_attn.h.
_vp, _i, _f, _d, _sz = ctypes.c_void_p, ctypes.c_int, ctypes.c_float, ctypes.c_double, ctypes.c_size_t
_pp = ctypes.POINTER(ctypes.c_void_p)
_i32p = ctypes.POINTER(ctypes.c_int32)
_f32p = ctypes.POINTER(ctypes.c_float)
_PARAMS = ctypes.POINTER(AttnParams)
SIGNATURES = [
    ("brk_last_error", ctypes.c_char_p, []),
    ("brk_abi_version", _i, []),
    ("brk_ctx_create", _i, [_i, _pp]),
    ("brk_ctx_destroy", _i, [_vp]),
    ("brk_ctx_check", _i, [_vp, _vp]),
    ("brk_ctx_reserve", _i, [_vp, _sz]),
    ("brk_ctx_reserve_stage", _i, [_vp, _sz]),
    ("brk_ctx_launches", ctypes.c_uint64, [_vp]),
    ("brk_rope_create", _i, [_vp, _i, _d, _f32p, _i, _pp]),
    ("brk_rope_destroy", _i, [_vp]),
    ("brk_rope_max_positions", _i, [_vp]),
    ("brk_llama3_rope_factors", _i, [_i, _d, _d, _d, _d, _i, _f32p]),
    ("brk_kv_create", _i, [_vp, ctypes.POINTER(KvDesc), _pp]),
    ("brk_kv_destroy", _i, [_vp]),
    ("brk_kv_capacity", _i, [_vp]),
    ("brk_kv_grow", _i, [_vp, _i, _vp]),
    ("brk_kv_reset", _i, [_vp, _i, _vp]),
    ("brk_kv_write_rows", _i, [_vp, _i, _i, _i, _i, _vp, _vp, _vp]),
    ("brk_kv_read_rows", _i, [_vp, _i, _i, _i, _i, _vp, _vp, _vp]),
    ("brk_kv_write_codes", _i, [_vp, _i, _i, _i, _i, _vp, _vp, _vp, _vp, _vp]),
    ("brk_kv_read_codes", _i, [_vp, _i, _i, _i, _i, _vp, _vp, _vp, _vp, _vp]),
    ("brk_attn_append", _i, [_vp, _vp, _i, _PARAMS, _i, _i, _i32p, _vp, _vp, _vp, _vp, _vp]),
    ("brk_attn_step", _i, [_vp, _vp, _i, _PARAMS, _i, _i, _i32p, _vp, _vp, _vp, _vp, _vp, _vp]),
    ("brk_attn_forward", _i, [_vp, _vp, _i, _PARAMS, _i, _i, _i32p, _vp, _vp, _vp]),
    ("brk_attn_decode", _i, [_vp, _vp, _i, _PARAMS, _i, _i, _i32p, _vp, _vp, _vp]),
    ("brk_attn_decode_splits", _i, [_vp, _vp, _PARAMS, _i, _i, _i32p]),
    ("brk_attn_decode_static", _i, [_vp, _vp, _i, _PARAMS, _i, _i, _i32p, _vp, _vp, _vp]),
    ("brk_attn_prefill", _i, [_vp, _vp, _i, _PARAMS, _i, _i, _i32p, _vp, _vp, _vp]),
    ("brk_attn_prefill_h", _i, [_vp, _vp, _i, _PARAMS, _i, _i, _i32p, _vp, _vp, _vp]),
    ("brk_attn_prefill_step", _i, [_vp, _vp, _i, _PARAMS, _i, _i, _i32p, _vp, _vp, _vp, _vp, _vp]),
    ("brk_attn_full", _i, [_vp, _PARAMS, _i, _i, _i, _vp, _vp, _vp, _vp, _vp]),
    ("brk_attn_decode_partial", _i, [_vp, _vp, _i, _PARAMS, _i, _i, _i32p, _vp, _vp, _vp, _vp]),
    ("brk_attn_combine", _i, [_vp, _i, _i, _i, _vp, _vp, _sz, _vp, _vp]),
    ("brk_proj_qkv", _i, [_vp, _i, _i, _i, _i, _vp, _vp, _d, _i, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp]),
    ("brk_proj_out", _i, [_vp, _i, _i, _i, _vp, _vp, _vp, _d, _i, _vp, _vp, _vp]),
    ("brk_peer_create", _i, [_vp, _i, _i, _i, _i, _pp]),
    ("brk_peer_handle", _i, [_vp, _vp, _sz]),
    ("brk_peer_open", _i, [_vp, _i, _vp, _sz]),
    ("brk_peer_attach", _i, [_vp, _i, _vp]),
    ("brk_peer_destroy", _i, [_vp]),
    ("brk_attn_decode_push", _i, [_vp, _vp, _i, _PARAMS, _i, _i, _i32p, _vp, _vp, ctypes.c_uint32, _vp]),
    ("brk_attn_step_push", _i, [_vp, _vp, _i, _PARAMS, _i, _i32p, _vp, _vp, _vp, _vp, _vp, ctypes.c_uint32, _vp]),
    ("brk_attn_combine_peers", _i, [_vp, _vp, _i, ctypes.c_uint32, _d, _vp, _vp]),
]

_lib = None


def build(force: bool = False) -> str:
    """Compile libbrk_attn.so for sm_100a with the committed Makefile (nvcc cross-compiles
    without a GPU)."""
    if force and os.path.exists(LIB_PATH):
        os.remove(LIB_PATH)
    subprocess.run(["make", "-s", "-C", CSRC], check=True)
    return LIB_PATH


def lib():
    """The loaded library with typed entry points.  Raises if it is missing."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is not built; run brimkern_b200._lib.build() (there is no CPU fallback)")
        L = ctypes.CDLL(LIB_PATH)
        for name, res, args in SIGNATURES:
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def check(rc: int) -> None:
    if rc != BRK_OK:
        raise BrkError(rc, lib().brk_last_error().decode(errors="replace"))
