"""B200 (sm_100a) attention operator for the Brimkern engine: decode attention over a resident
fp16 KV cache, the fused KV append, chunked causal prefill on tensor cores, and split-KV
partials for sequence-sharded contexts.  CUDA kernels live in ``csrc/`` behind the C ABI of
``include/brk_attn.h``; ``engine`` mirrors the reference engine's host interface."""
from ._lib import BrkError, build, lib  # noqa: F401

__all__ = ["BrkError", "build", "lib"]
