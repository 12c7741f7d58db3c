"""Host side of the attention operator: a mirror of the reference engine's attention / KV-cache
surface (``WebGpuEngine`` in src/lib/webgpu/kernels.ts) over the C ABI of libbrk_attn.

The reference host is TypeScript; no JavaScript runtime exists in this image, so the host layer
is written in Python with the reference's method names and argument meanings:

* readback twins used by selfValidate -- ``attention`` (kernels.ts:610), ``attentionDecode``
  (:624), ``quantizeKvReadback`` (:664), ``attentionQ8Kv`` (:681), ``attentionQ8KvDecode``
  (:694), ``attentionFull`` (:639), ``attentionFullWg`` (:652), ``rope`` (:556), ``ropeFactors``
  (:568), ``rmsnorm`` (:428): numpy in, numpy out;
* the resident path -- ``ensureKv`` / ``setKvQuant`` / ``clearKvCache`` (:1760-1806), the
  session check of ``runDecodeGpu`` (:1817-1825), ``recAttention`` (:1626) and the attention
  slice of ``recordLayerKV`` (:1707-1731): device tensors in, device tensors out.

PyTorch only provides device memory and streams here; every computation runs in the library's
CUDA kernels.  Errors raise ``BrkError`` (the library has no fallback path).
"""
from __future__ import annotations

import ctypes
import math
import os
from dataclasses import dataclass
from typing import Optional, Sequence

import numpy as np
import torch

from . import _lib as L
from ._lib import BrkError, check

_SUPPORTED_DIMS = (64, 128, 256)


def _stream_ptr(stream: Optional[torch.cuda.Stream] = None) -> ctypes.c_void_p:
    s = stream if stream is not None else torch.cuda.current_stream()
    return ctypes.c_void_p(s.cuda_stream)


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _positions(past_len, batch: int):
    arr = (ctypes.c_int32 * batch)()
    vals = [int(past_len)] * batch if np.isscalar(past_len) else [int(x) for x in past_len]
    if len(vals) != batch:
        raise BrkError(L.BRK_ERR_INVALID, f"past_len has {len(vals)} entries for batch {batch}")
    for i, v in enumerate(vals):
        arr[i] = v
    return arr


class Context:
    """One library context per GPU (the engine instance of kernels.ts:100)."""

    def __init__(self, device: int = 0):
        self.device = int(device)
        h = ctypes.c_void_p()
        check(L.lib().brk_ctx_create(self.device, ctypes.byref(h)))
        self.handle = h

    def check(self, stream=None) -> None:
        """Synchronise and raise if a kernel gave up on a bounded wait."""
        check(L.lib().brk_ctx_check(self.handle, _stream_ptr(stream)))

    @property
    def launches(self) -> int:
        """Kernels launched through this context so far."""
        return int(L.lib().brk_ctx_launches(self.handle))

    def reserve(self, nbytes: int) -> None:
        check(L.lib().brk_ctx_reserve(self.handle, int(nbytes)))

    def reserve_stage(self, nbytes: int) -> None:
        """Pre-size the fp16 staging buffer (int8-cache prefill, non-causal attention)."""
        check(L.lib().brk_ctx_reserve_stage(self.handle, int(nbytes)))

    def close(self) -> None:
        if self.handle:
            L.lib().brk_ctx_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class RopeTable:
    """NeoX RoPE cos/sin table (rope / rope_factors, shaders.ts:1361-1408) for positions
    [0, max_positions), built on the host in double exactly like ropeCpu."""

    def __init__(self, ctx: Context, head_dim: int, base: float, ff: Optional[Sequence[float]] = None,
                 max_positions: int = 4096):
        self.ctx, self.head_dim, self.base = ctx, head_dim, float(base)
        h = ctypes.c_void_p()
        ffp = None
        if ff is not None:
            self._ff = np.ascontiguousarray(ff, dtype=np.float32)
            ffp = self._ff.ctypes.data_as(ctypes.POINTER(ctypes.c_float))
        check(L.lib().brk_rope_create(ctx.handle, head_dim, self.base, ffp, int(max_positions), ctypes.byref(h)))
        self.handle = h
        self.max_positions = int(max_positions)

    def close(self):
        if self.handle:
            L.lib().brk_rope_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def llama3_rope_factors(head_dim: int, base: float, factor: float, low_freq_factor: float,
                        high_freq_factor: float, original_context: int) -> np.ndarray:
    """Divisors ff[i] of the llama3 RoPE scaling (what rope_freqs.weight holds, model.ts:590)."""
    ff = np.zeros(head_dim // 2, np.float32)
    check(L.lib().brk_llama3_rope_factors(head_dim, float(base), float(factor), float(low_freq_factor),
                                          float(high_freq_factor), int(original_context),
                                          ff.ctypes.data_as(ctypes.POINTER(ctypes.c_float))))
    return ff


class KvCache:
    """Persistent KV cache of ``n_layers`` layers x ``batch`` sequences (KvEntry, kernels.ts:93),
    head-major in HBM: fp16, or int8 codes + per-(row, kv head) scales (``q8=True``, the
    reference's setKvQuant mode)."""

    def __init__(self, ctx: Context, n_layers: int, batch: int, n_kv_heads: int, head_dim: int, capacity: int,
                 q8: bool = False):
        self.ctx = ctx
        self.n_layers, self.batch, self.n_kv_heads, self.head_dim = n_layers, batch, n_kv_heads, head_dim
        self.q8 = bool(q8)
        desc = L.KvDesc(n_layers, batch, n_kv_heads, head_dim, int(capacity), L.BRK_KV_I8 if q8 else L.BRK_KV_F16)
        h = ctypes.c_void_p()
        check(L.lib().brk_kv_create(ctx.handle, ctypes.byref(desc), ctypes.byref(h)))
        self.handle = h

    @property
    def capacity(self) -> int:
        return L.lib().brk_kv_capacity(self.handle)

    def grow(self, rows: int, stream=None) -> None:
        """ensureKv growth rule: capacity -> max(rows, capacity + 1024, 1024) when rows > capacity."""
        check(L.lib().brk_kv_grow(self.handle, int(rows), _stream_ptr(stream)))

    def reset(self, seq: int = -1, stream=None) -> None:
        """Zero sequence `seq`'s rows in every layer (all sequences when seq == -1)."""
        check(L.lib().brk_kv_reset(self.handle, int(seq), _stream_ptr(stream)))

    def write_rows(self, layer: int, seq: int, row0: int, k: torch.Tensor, v: torch.Tensor, stream=None) -> None:
        """f32 rows [n, n_kv_heads, D] stored as fp16, or quantised (quantize_kv) in an int8 cache."""
        n = k.shape[0]
        check(L.lib().brk_kv_write_rows(self.handle, layer, seq, row0, n, _ptr(k.contiguous()), _ptr(v.contiguous()),
                                        _stream_ptr(stream)))

    def write_codes(self, layer: int, seq: int, row0: int, k_codes: torch.Tensor, k_scales: torch.Tensor,
                    v_codes: torch.Tensor, v_scales: torch.Tensor, stream=None) -> None:
        """int8 cache: given codes [n, n_kv_heads, D] int8 and scales [n, n_kv_heads] f32."""
        n = k_codes.shape[0]
        check(L.lib().brk_kv_write_codes(self.handle, layer, seq, row0, n, _ptr(k_codes.contiguous()),
                                         _ptr(k_scales.contiguous()), _ptr(v_codes.contiguous()),
                                         _ptr(v_scales.contiguous()), _stream_ptr(stream)))

    def read_codes(self, layer: int, seq: int, row0: int, n_rows: int, stream=None):
        """int8 cache: (k_codes, k_scales, v_codes, v_scales) in the reference's layout."""
        dev = torch.device("cuda", self.ctx.device)
        kc = torch.empty((n_rows, self.n_kv_heads, self.head_dim), dtype=torch.int8, device=dev)
        vc = torch.empty_like(kc)
        ks = torch.empty((n_rows, self.n_kv_heads), dtype=torch.float32, device=dev)
        vs = torch.empty_like(ks)
        check(L.lib().brk_kv_read_codes(self.handle, layer, seq, row0, n_rows, _ptr(kc), _ptr(ks), _ptr(vc), _ptr(vs),
                                        _stream_ptr(stream)))
        return kc, ks, vc, vs

    def read_rows(self, layer: int, seq: int, row0: int, n_rows: int, stream=None):
        """Rows in the reference's token-major layout [n_rows, n_kv_heads, D] as float16 tensors."""
        dev = torch.device("cuda", self.ctx.device)
        k = torch.empty((n_rows, self.n_kv_heads, self.head_dim), dtype=torch.int16, device=dev)
        v = torch.empty_like(k)
        check(L.lib().brk_kv_read_rows(self.handle, layer, seq, row0, n_rows, _ptr(k), _ptr(v), _stream_ptr(stream)))
        return k.view(torch.float16), v.view(torch.float16)

    def close(self):
        if self.handle:
            L.lib().brk_kv_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class PeerArea:
    """This rank's exchange area for sequence-sharded decode over peer memory (brk_peer): the
    other ranks' decode kernels store their partials here, and this rank's kernels store into
    theirs (mapped with CUDA IPC handles, or attached in-process)."""

    def __init__(self, ctx: Context, world: int, rank: int, max_rows: int, head_dim: int):
        self.ctx, self.world, self.rank = ctx, int(world), int(rank)
        h = ctypes.c_void_p()
        check(L.lib().brk_peer_create(ctx.handle, self.world, self.rank, int(max_rows), int(head_dim), ctypes.byref(h)))
        self.handle = h

    def ipc_handle(self) -> bytes:
        buf = (ctypes.c_char * L.BRK_PEER_HANDLE_BYTES)()
        check(L.lib().brk_peer_handle(self.handle, buf, L.BRK_PEER_HANDLE_BYTES))
        return bytes(buf)

    def open(self, peer_rank: int, handle: bytes) -> None:
        buf = (ctypes.c_char * len(handle)).from_buffer_copy(handle)
        check(L.lib().brk_peer_open(self.handle, int(peer_rank), buf, len(handle)))

    def attach(self, peer_rank: int, other: "PeerArea") -> None:
        check(L.lib().brk_peer_attach(self.handle, int(peer_rank), other.handle))

    def close(self):
        if self.handle:
            L.lib().brk_peer_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


@dataclass
class AttnConfig:
    """LayerCfg's attention fields (kernels.ts:24-56) plus the extensions of this build."""
    n_heads: int
    n_kv_heads: int
    head_dim: int
    scale: Optional[float] = None       # attnScale; None -> 1/sqrt(head_dim)
    softcap: float = 0.0                # attnLogitSoftcap
    window: int = 0                     # sliding window (0 = global)
    eps: float = 1e-6
    one_plus: bool = False              # rmsGainOnePlus
    q_norm: Optional[torch.Tensor] = None   # device [head_dim] f32
    k_norm: Optional[torch.Tensor] = None
    rope: Optional[RopeTable] = None
    kv_offset: int = 0

    def params(self) -> L.AttnParams:
        return L.AttnParams(self.n_heads, self.n_kv_heads, self.head_dim,
                            0.0 if self.scale is None else float(self.scale), float(self.softcap or 0.0),
                            int(self.window or 0), int(self.kv_offset), int(bool(self.one_plus)), float(self.eps),
                            _ptr(self.q_norm), _ptr(self.k_norm), self.rope.handle.value if self.rope else None)


class AttentionEngine:
    """Mirror of WebGpuEngine's attention / KV-cache methods (kernels.ts:556-704, 1626-1825)."""

    def __init__(self, device: int = 0):
        self.device = torch.device("cuda", device)
        self.ctx = Context(device)
        # ?attndecode=0 kill switch (kernels.ts:181-215) -> BRK_ATTN_DECODE=0.
        self.attnDecodeOk = os.environ.get("BRK_ATTN_DECODE", "1") != "0"
        self.kvGpu: Optional[KvCache] = None
        self.lfm2KvGpu: dict = {}  # LFM2 attention layer -> its own cache (kernels.ts:1990)
        self.kvSession = ""
        self.seqSessions: dict = {}  # sequence -> session id (batched caches, session(seq=...))
        self.kvQuant = False

    # ---- plumbing ---------------------------------------------------------------------
    def _dev(self, a) -> torch.Tensor:
        return torch.as_tensor(np.ascontiguousarray(a, dtype=np.float32)).to(self.device)

    @staticmethod
    def _host(t: torch.Tensor) -> np.ndarray:
        return t.detach().float().cpu().numpy().ravel()

    # ---- readback twins (selfValidate surface) ------------------------------------------
    def _attention_readback(self, q, k, v, nTokens, nHeads, nKvHeads, headDim, pastLen, scale, softcap, kernel,
                            window=0):
        kvLen = pastLen + nTokens
        D = self._padded_dim(headDim)
        sc = float(scale) if scale is not None else 1.0 / math.sqrt(headDim)

        def pad(a, rows, heads):
            a = np.asarray(a, np.float32).reshape(rows, heads, headDim)
            if D == headDim:
                return a
            out = np.zeros((rows, heads, D), np.float32)
            out[..., :headDim] = a  # zero lanes add nothing to q.k and produce unused outputs
            return out

        qd = self._dev(pad(q, nTokens, nHeads))
        kd = self._dev(pad(k, kvLen, nKvHeads))
        vd = self._dev(pad(v, kvLen, nKvHeads))
        kv = KvCache(self.ctx, 1, 1, nKvHeads, D, kvLen)
        kv.write_rows(0, 0, 0, kd, vd)
        cfg = AttnConfig(nHeads, nKvHeads, D, scale=sc, softcap=softcap, window=window)
        out = torch.empty((nTokens, nHeads, D), dtype=torch.float32, device=self.device)
        self.recAttention(kv, 0, cfg, qd, out, pastLen, kernel=kernel)
        self.ctx.check()
        kv.close()
        return out[..., :headDim].cpu().numpy().ravel()

    def attention(self, q, k, v, nTokens, nHeads, nKvHeads, headDim, pastLen=0, scale=None, softcap=0.0):
        """kernels.ts:610 — causal GQA attention; k/v [kvLen, nKvHeads, headDim] f32 (stored as fp16)."""
        return self._attention_readback(q, k, v, nTokens, nHeads, nKvHeads, headDim, pastLen, scale, softcap, "auto")

    def attentionDecode(self, q, k, v, nTokens, nHeads, nKvHeads, headDim, pastLen=0, scale=None, softcap=0.0):
        """kernels.ts:624 — the same through the decode kernel."""
        return self._attention_readback(q, k, v, nTokens, nHeads, nKvHeads, headDim, pastLen, scale, softcap,
                                        "decode")

    def quantizeKvReadback(self, src, rows, nKvHeads, headDim):
        """kernels.ts:664 — quantize_kv of src [rows, nKvHeads, headDim] f32 -> (codes int8
        [rows*nKvHeads*headDim] (the bytes of the reference's packed Uint32Array), scales f32
        [rows*nKvHeads])."""
        D = self._padded_dim(headDim)
        x = np.zeros((rows, nKvHeads, D), np.float32)
        x[..., :headDim] = np.asarray(src, np.float32).reshape(rows, nKvHeads, headDim)  # zeros leave amax as is
        xd = self._dev(x)
        kv = KvCache(self.ctx, 1, 1, nKvHeads, D, rows, q8=True)
        kv.write_rows(0, 0, 0, xd, xd)
        kc, ks, _, _ = kv.read_codes(0, 0, 0, rows)
        self.ctx.check()
        kv.close()
        return kc[..., :headDim].cpu().numpy().ravel(), ks.cpu().numpy().ravel()

    def attentionFull(self, q, k, v, nTokens, nHeads, nKvHeads, headDim, kvLen, scale=None, softcap=0.0):
        """kernels.ts:639 — non-causal attention: every query attends all kvLen keys
        (q [nTokens, nHeads, headDim], k / v [kvLen, nKvHeads, headDim] f32)."""
        qd = self._dev(np.asarray(q, np.float32).reshape(1, nTokens, nHeads, headDim))
        kd = self._dev(np.asarray(k, np.float32).reshape(1, kvLen, nKvHeads, headDim))
        vd = self._dev(np.asarray(v, np.float32).reshape(1, kvLen, nKvHeads, headDim))
        out = torch.empty_like(qd)
        cfg = AttnConfig(nHeads, nKvHeads, headDim, scale=scale, softcap=softcap)
        self.recAttentionFull(cfg, qd, kd, vd, out)
        self.ctx.check()
        return self._host(out)

    def attentionFullWg(self, q, k, v, nTokens, nHeads, nKvHeads, headDim, kvLen, scale=None, softcap=0.0):
        """kernels.ts:652 — the reference's workgroup-per-(token, head) variant of attentionFull;
        here the same operator (one kernel choice per shape)."""
        return self.attentionFull(q, k, v, nTokens, nHeads, nKvHeads, headDim, kvLen, scale, softcap)

    def recAttentionFull(self, cfg: "AttnConfig", q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, out: torch.Tensor,
                         stream=None) -> torch.Tensor:
        """recAttentionFull (kernels.ts:1277): q [B, T, Hq, D], k / v [B, kvLen, Hkv, D] f32 device
        tensors -> out [B, T, Hq, D]."""
        B, T = q.shape[0], q.shape[1]
        kv_len = k.shape[1]
        p = cfg.params()
        check(L.lib().brk_attn_full(self.ctx.handle, ctypes.byref(p), B, T, kv_len, _ptr(q.contiguous()),
                                    _ptr(k.contiguous()), _ptr(v.contiguous()), _ptr(out), _stream_ptr(stream)))
        return out

    def _attention_q8_readback(self, q, kc, ks, vc, vs, nTokens, nHeads, nKvHeads, headDim, pastLen, scale, softcap,
                               kernel):
        kvLen = pastLen + nTokens
        D = self._padded_dim(headDim)
        sc = float(scale) if scale is not None else 1.0 / math.sqrt(headDim)

        def codes(c):
            c = np.ascontiguousarray(c).view(np.int8).reshape(kvLen, nKvHeads, headDim)
            out = np.zeros((kvLen, nKvHeads, D), np.int8)
            out[..., :headDim] = c
            return torch.from_numpy(out).to(self.device)

        qp = np.zeros((nTokens, nHeads, D), np.float32)
        qp[..., :headDim] = np.asarray(q, np.float32).reshape(nTokens, nHeads, headDim)
        kv = KvCache(self.ctx, 1, 1, nKvHeads, D, kvLen, q8=True)
        kv.write_codes(0, 0, 0, codes(kc), self._dev(np.asarray(ks, np.float32).reshape(kvLen, nKvHeads)),
                       codes(vc), self._dev(np.asarray(vs, np.float32).reshape(kvLen, nKvHeads)))
        cfg = AttnConfig(nHeads, nKvHeads, D, scale=sc, softcap=softcap)
        out = torch.empty((nTokens, nHeads, D), dtype=torch.float32, device=self.device)
        self.recAttention(kv, 0, cfg, self._dev(qp), out, pastLen, kernel=kernel)
        self.ctx.check()
        kv.close()
        return out[..., :headDim].cpu().numpy().ravel()

    def attentionQ8Kv(self, q, kc, ks, vc, vs, nTokens, nHeads, nKvHeads, headDim, pastLen=0, scale=None, softcap=0.0):
        """kernels.ts:681 — attention over an int8 cache given as codes (int8, or the packed
        Uint32 words) and per-(row, head) f32 scales."""
        return self._attention_q8_readback(q, kc, ks, vc, vs, nTokens, nHeads, nKvHeads, headDim, pastLen, scale,
                                           softcap, "auto")

    def attentionQ8KvDecode(self, q, kc, ks, vc, vs, nTokens, nHeads, nKvHeads, headDim, pastLen=0, scale=None,
                            softcap=0.0):
        """kernels.ts:694 — the same through the decode kernel."""
        return self._attention_q8_readback(q, kc, ks, vc, vs, nTokens, nHeads, nKvHeads, headDim, pastLen, scale,
                                           softcap, "decode")

    @staticmethod
    def _padded_dim(headDim: int) -> int:
        D = next((d for d in _SUPPORTED_DIMS if d >= headDim), None)
        if D is None:
            raise BrkError(L.BRK_ERR_UNSUPPORTED, f"head_dim {headDim} > 256")
        return D

    def _q_prologue(self, x, rows, headDim, nHeads, pastLen, rope, gain, eps, onePlus):
        if rows % nHeads:
            raise BrkError(L.BRK_ERR_INVALID, "rows must be a multiple of nHeads")
        xd = self._dev(x)
        out = torch.empty_like(xd)
        cfg = AttnConfig(nHeads, 1, headDim, eps=eps, one_plus=onePlus, q_norm=gain, rope=rope)
        p = cfg.params()
        pos = _positions([pastLen], 1)
        check(L.lib().brk_attn_append(self.ctx.handle, None, 0, ctypes.byref(p), 1, rows // nHeads, pos, _ptr(xd),
                                      None, None, _ptr(out), _stream_ptr()))
        self.ctx.check()
        return self._host(out)

    def rope(self, x, rows, headDim, nHeads, pastLen=0, base=10000.0):
        """kernels.ts:556 — NeoX RoPE of x [rows = seq*nHeads, headDim] at pastLen + row/nHeads."""
        table = RopeTable(self.ctx, headDim, base, None, pastLen + rows // nHeads)
        return self._q_prologue(x, rows, headDim, nHeads, pastLen, table, None, 1e-6, False)

    def ropeFactors(self, x, ff, rows, headDim, nHeads, pastLen=0, base=10000.0):
        """kernels.ts:568 — RoPE with per-frequency divisors ff [headDim/2]."""
        table = RopeTable(self.ctx, headDim, base, ff, pastLen + rows // nHeads)
        return self._q_prologue(x, rows, headDim, nHeads, pastLen, table, None, 1e-6, False)

    def rmsnorm(self, x, w, rows, dim, eps=1e-5, onePlus=False):
        """kernels.ts:428 — RMSNorm of x [rows, dim] with gain w (per-head QK-norm when dim = headDim)."""
        return self._q_prologue(x, rows, dim, 1, 0, None, self._dev(w), eps, onePlus)

    # ---- KV manager (kernels.ts:1749-1806) ----------------------------------------------
    def setKvQuant(self, q8: bool) -> None:
        """kernels.ts:1760 — switch the cache between fp16 and int8 (resets it: layouts differ)."""
        q8 = bool(q8)
        if self.kvQuant != q8:
            self.kvQuant = q8
            self.resetKvGpu()

    def resetKvGpu(self) -> None:
        if self.kvGpu is not None:
            self.kvGpu.close()
        self.kvGpu = None
        for kv in self.lfm2KvGpu.values():
            kv.close()
        self.lfm2KvGpu = {}
        self.kvSession = ""
        self.seqSessions = {}

    def clearKvCache(self) -> None:
        self.resetKvGpu()

    def ensureKv(self, n_layers: int, rows: int, batch: int, n_kv_heads: int, head_dim: int) -> KvCache:
        """Cache holding >= rows rows for every layer; grows to max(rows, cap + 1024, 1024)."""
        kv = self.kvGpu
        if kv is not None and (kv.n_layers, kv.batch, kv.n_kv_heads, kv.head_dim, kv.q8) != (
                n_layers, batch, n_kv_heads, head_dim, self.kvQuant):
            self.resetKvGpu()
            kv = None
        if kv is None:
            kv = KvCache(self.ctx, n_layers, batch, n_kv_heads, head_dim, max(rows, 1024), q8=self.kvQuant)
            self.kvGpu = kv
        elif kv.capacity < rows:
            kv.grow(rows)
        return kv

    # ---- LFM2 attention layers (kernels.ts:1990-2003, 2029-2111; lfm2Model.ts:320-333) --------
    def ensureLfm2Kv(self, layer: int, rows: int, n_kv_heads: int, head_dim: int, batch: int = 1) -> KvCache:
        """ensureLfm2Kv (kernels.ts:1990): one cache per LFM2 attention layer (its conv layers
        keep no K/V), grown with ensureKv's rule max(rows, cap + 1024, 1024)."""
        kv = self.lfm2KvGpu.get(layer)
        if kv is not None and (kv.batch, kv.n_kv_heads, kv.head_dim, kv.q8) != (batch, n_kv_heads, head_dim,
                                                                              self.kvQuant):
            kv.close()
            kv = None
        if kv is None:
            kv = KvCache(self.ctx, 1, batch, n_kv_heads, head_dim, max(rows, 1024), q8=self.kvQuant)
            self.lfm2KvGpu[layer] = kv
        elif kv.capacity < rows:
            kv.grow(rows)
        return kv

    LFM2_PREFILL_CHUNK = 128  # lfm2Model.ts:320

    def lfm2Attention(self, layer: int, cfg: AttnConfig, q_in: torch.Tensor, k_in: torch.Tensor, v_in: torch.Tensor,
                      past_len, chunk: Optional[int] = None, stream=None) -> torch.Tensor:
        """The attention slice of an LFM2 attention layer in recordLfm2 (kernels.ts:2055-2067):
        per-head QK-norm and RoPE of the q / k projections, K/V appended to the layer's cache at
        pastLen, causal attention over it.  q_in [B, T, Hq, D], k_in / v_in [B, T, Hkv, D] f32;
        a prompt is prefilled in chunks of PREFILL_CHUNK tokens (lfm2Model.ts:320-333), a decode
        token goes through the fused append + decode step."""
        B, T = q_in.shape[0], q_in.shape[1]
        base = [int(past_len)] * B if np.isscalar(past_len) else [int(x) for x in past_len]
        kv = self.ensureLfm2Kv(layer, max(base) + T, cfg.n_kv_heads, cfg.head_dim, B)
        G = cfg.n_heads // cfg.n_kv_heads
        if T * G <= 64 and self.attnDecodeOk:
            return self.attentionLayer(kv, 0, cfg, q_in, k_in, v_in, base, stream=stream)
        return self.prefillChunked(kv, 0, cfg, q_in, k_in, v_in, base, chunk=chunk or self.LFM2_PREFILL_CHUNK,
                                   stream=stream)

    def session(self, session_id: str, past_len, seq: Optional[int] = None) -> None:
        """runDecodeGpu's session rule (kernels.ts:1817-1825): a new session id or pastLen 0
        resets the cache; pastLen > 0 on an unknown session means the cache is lost (raised).

        With ``seq`` the rule applies to one sequence of the batched cache (one session per
        sequence): only that sequence's rows are cleared (brk_kv_reset(kv, seq)), the others
        keep theirs."""
        first = int(past_len) if np.isscalar(past_len) else int(min(past_len))
        if seq is not None:
            seq = int(seq)
            if session_id != self.seqSessions.get(seq) or first == 0:
                if first > 0:
                    raise BrkError(L.BRK_ERR_INVALID, f'session "{session_id}" unknown on sequence {seq} with '
                                                      f'pastLen={first}: cache lost, restart at 0')
                if self.kvGpu is not None:
                    self.kvGpu.reset(seq)
                self.seqSessions[seq] = session_id
            return
        if session_id != self.kvSession or first == 0:
            if first > 0:
                raise BrkError(L.BRK_ERR_INVALID,
                               f'session "{session_id}" unknown with pastLen={first}: cache lost, restart at 0')
            self.resetKvGpu()
            self.kvSession = session_id

    # ---- resident path ------------------------------------------------------------------
    def recAttention(self, kv: KvCache, layer: int, cfg: AttnConfig, q: torch.Tensor, out: torch.Tensor, past_len,
                     kernel: str = "auto", stream=None) -> torch.Tensor:
        """recAttention (kernels.ts:1626): q [B, T, Hq, D] f32 (rotated) -> out [B, T, Hq, D] f32."""
        B = kv.batch
        T = q.numel() // (B * cfg.n_heads * cfg.head_dim)
        p = cfg.params()
        pos = _positions(past_len, B)
        if kernel == "auto" and not self.attnDecodeOk:
            kernel = "prefill"
        fn = {"auto": L.lib().brk_attn_forward, "decode": L.lib().brk_attn_decode,
              "prefill": L.lib().brk_attn_prefill}[kernel]
        check(fn(self.ctx.handle, kv.handle, layer, ctypes.byref(p), B, T, pos, _ptr(q), _ptr(out), _stream_ptr(stream)))
        return out

    def prefillHalfQ(self, kv: KvCache, layer: int, cfg: AttnConfig, q16: torch.Tensor, out: torch.Tensor, past_len,
                     stream=None) -> torch.Tensor:
        """The tensor-core prefill kernel on q already rotated, as fp16 [B, T, Hq, D] (loaded with
        TMA): the form brk_attn_prefill_step uses for fp16 caches."""
        if q16.dtype != torch.float16:
            raise BrkError(L.BRK_ERR_INVALID, "q16 must be float16")
        B = kv.batch
        T = q16.numel() // (B * cfg.n_heads * cfg.head_dim)
        p = cfg.params()
        pos = _positions(past_len, B)
        check(L.lib().brk_attn_prefill_h(self.ctx.handle, kv.handle, layer, ctypes.byref(p), B, T, pos, _ptr(q16),
                                         _ptr(out), _stream_ptr(stream)))
        return out

    def appendKv(self, kv: KvCache, layer: int, cfg: AttnConfig, q_in: torch.Tensor, k_in: torch.Tensor,
                 v_in: torch.Tensor, q_out: torch.Tensor, past_len, stream=None) -> torch.Tensor:
        """QK-norm + RoPE of q and the new k, fp16 store of k and v at row pastLen
        (kernels.ts:1707-1730)."""
        B = kv.batch
        T = (q_in.numel() // (B * cfg.n_heads * cfg.head_dim) if q_in is not None
             else k_in.numel() // (B * cfg.n_kv_heads * cfg.head_dim))
        p = cfg.params()
        pos = _positions(past_len, B)
        check(L.lib().brk_attn_append(self.ctx.handle, kv.handle, layer, ctypes.byref(p), B, T, pos, _ptr(q_in),
                                      _ptr(k_in), _ptr(v_in), _ptr(q_out), _stream_ptr(stream)))
        return q_out

    def attentionLayer(self, kv: KvCache, layer: int, cfg: AttnConfig, q_in, k_in, v_in, past_len,
                       q_work: Optional[torch.Tensor] = None, out: Optional[torch.Tensor] = None,
                       kernel: str = "auto", stream=None) -> torch.Tensor:
        """The attention slice of recordLayerKV (kernels.ts:1707-1731): q/k/v projections in,
        attention output out; K/V land in the cache."""
        q_work = torch.empty_like(q_in) if q_work is None else q_work
        out = torch.empty_like(q_in) if out is None else out
        B = kv.batch
        T = q_in.numel() // (B * cfg.n_heads * cfg.head_dim)
        if kernel == "auto" and self.attnDecodeOk and T * (cfg.n_heads // cfg.n_kv_heads) <= 64:
            # Decode: append and attention as one overlapped launch pair.
            p = cfg.params()
            pos = _positions(past_len, B)
            check(L.lib().brk_attn_step(self.ctx.handle, kv.handle, layer, ctypes.byref(p), B, T, pos, _ptr(q_in),
                                        _ptr(k_in), _ptr(v_in), _ptr(q_work), _ptr(out), _stream_ptr(stream)))
            return out
        self.appendKv(kv, layer, cfg, q_in, k_in, v_in, q_work, past_len, stream)
        return self.recAttention(kv, layer, cfg, q_work, out, past_len, kernel, stream)

    def prefillChunked(self, kv: KvCache, layer: int, cfg: AttnConfig, q_in: torch.Tensor, k_in: torch.Tensor,
                       v_in: torch.Tensor, past_len, chunk: int = 512, out: Optional[torch.Tensor] = None,
                       stream=None) -> torch.Tensor:
        """Chunked causal prefill of T new tokens per sequence ([B, T, H, D] inputs): per chunk,
        append its K/V at pastLen + offset, then attend over everything cached so far -- the
        reference's chunk loop (lfm2Model.ts:320-333, recAttention with pastLen) on the
        tensor-core kernel."""
        B = kv.batch
        T = q_in.shape[1]
        out = torch.empty_like(q_in) if out is None else out
        base = [int(past_len)] * B if np.isscalar(past_len) else [int(x) for x in past_len]
        q_work = torch.empty((B, min(chunk, T), cfg.n_heads, cfg.head_dim), dtype=torch.float32, device=q_in.device)
        G = cfg.n_heads // cfg.n_kv_heads
        for c0 in range(0, T, chunk):
            c1 = min(T, c0 + chunk)
            pos = [p + c0 for p in base]
            qc = q_in[:, c0:c1].contiguous()
            oc = torch.empty_like(qc)
            if (self.attnDecodeOk is False or (c1 - c0) * G > 128) and cfg.head_dim in (64, 128):
                # Tensor-core chunk with the q prologue fused into the kernel.
                self.prefillStep(kv, layer, cfg, qc, k_in[:, c0:c1].contiguous(), v_in[:, c0:c1].contiguous(), oc,
                                 pos, stream)
            else:
                qw = q_work[:, :c1 - c0]
                self.appendKv(kv, layer, cfg, qc, k_in[:, c0:c1].contiguous(), v_in[:, c0:c1].contiguous(), qw, pos,
                              stream)
                self.recAttention(kv, layer, cfg, qw, oc, pos, "auto", stream)
            out[:, c0:c1].copy_(oc)
        return out

    def prefillStep(self, kv: KvCache, layer: int, cfg: AttnConfig, q_in: torch.Tensor, k_in: torch.Tensor,
                    v_in: torch.Tensor, out: torch.Tensor, past_len, stream=None) -> torch.Tensor:
        """One prefill chunk: K/V append, then the tensor-core kernel with the q prologue fused."""
        B = kv.batch
        T = q_in.numel() // (B * cfg.n_heads * cfg.head_dim)
        p = cfg.params()
        pos = _positions(past_len, B)
        check(L.lib().brk_attn_prefill_step(self.ctx.handle, kv.handle, layer, ctypes.byref(p), B, T, pos,
                                            _ptr(q_in), _ptr(k_in), _ptr(v_in), _ptr(out), _stream_ptr(stream)))
        return out

    def decodePartial(self, kv: KvCache, layer: int, cfg: AttnConfig, q: torch.Tensor, part_ml: torch.Tensor,
                      part_o: torch.Tensor, past_len, stream=None):
        """Split-KV partial (m, l, o) of this cache's rows (sequence-sharded contexts)."""
        B = kv.batch
        T = q.numel() // (B * cfg.n_heads * cfg.head_dim)
        p = cfg.params()
        pos = _positions(past_len, B)
        check(L.lib().brk_attn_decode_partial(self.ctx.handle, kv.handle, layer, ctypes.byref(p), B, T, pos, _ptr(q),
                                              _ptr(part_ml), _ptr(part_o), _stream_ptr(stream)))

    # ---- the projections either side of the operator (recordLayerKV, kernels.ts:1700-1736) -----
    def projQkv(self, x: torch.Tensor, wq: torch.Tensor, wk: torch.Tensor, wv: torch.Tensor,
                q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, attn_norm: Optional[torch.Tensor] = None,
                eps: float = 1e-6, one_plus: bool = False, bq=None, bk=None, bv=None, stream=None):
        """n1 = rmsnorm(x, attn_norm); q / k / v = n1 W^T (+ bias).  x [rows, d] f32, weights
        [n, d] fp16, outputs [rows, n] f32."""
        rows, d = x.shape[0], x.shape[-1]
        check(L.lib().brk_proj_qkv(self.ctx.handle, rows, d, wq.shape[0], wk.shape[0], _ptr(x.contiguous()),
                                   _ptr(attn_norm), float(eps), int(bool(one_plus)), _ptr(wq.contiguous()),
                                   _ptr(wk.contiguous()), _ptr(wv.contiguous()), _ptr(bq), _ptr(bk), _ptr(bv), _ptr(q),
                                   _ptr(k), _ptr(v), _stream_ptr(stream)))
        return q, k, v

    def projOut(self, attn: torch.Tensor, wo: torch.Tensor, x: torch.Tensor, h: torch.Tensor,
                post_norm: Optional[torch.Tensor] = None, eps: float = 1e-6, one_plus: bool = False, stream=None):
        """h = x + attn Wo^T (Gemma-2: x + rmsnorm(attn Wo^T, post_norm)).  attn [rows, q_dim],
        wo [d, q_dim] fp16, x / h [rows, d] f32."""
        rows, q_dim = attn.shape[0], attn.shape[-1]
        check(L.lib().brk_proj_out(self.ctx.handle, rows, q_dim, wo.shape[0], _ptr(attn.contiguous()),
                                   _ptr(wo.contiguous()), _ptr(post_norm), float(eps), int(bool(one_plus)),
                                   _ptr(x.contiguous()), _ptr(h), _stream_ptr(stream)))
        return h

    def decodePush(self, kv: KvCache, layer: int, cfg: AttnConfig, q: torch.Tensor, peer: PeerArea, epoch: int,
                   past_len, stream=None) -> None:
        """Split-KV partial of this cache's rows, stored into every rank's exchange area."""
        B = kv.batch
        T = q.numel() // (B * cfg.n_heads * cfg.head_dim)
        p = cfg.params()
        pos = _positions(past_len, B)
        check(L.lib().brk_attn_decode_push(self.ctx.handle, kv.handle, layer, ctypes.byref(p), B, T, pos, _ptr(q),
                                           peer.handle, int(epoch), _stream_ptr(stream)))

    def stepPush(self, kv: KvCache, layer: int, cfg: AttnConfig, q_in: torch.Tensor, k_in: Optional[torch.Tensor],
                 v_in: Optional[torch.Tensor], q_work: torch.Tensor, peer: PeerArea, epoch: int, past_len,
                 stream=None) -> None:
        """decodePush for one token with the append fused into the launch: q_in raw (rotated into
        q_work), K / V stored by the rank whose cache holds the new position (others pass None)."""
        B = kv.batch
        p = cfg.params()
        pos = _positions(past_len, B)
        check(L.lib().brk_attn_step_push(self.ctx.handle, kv.handle, layer, ctypes.byref(p), B, pos, _ptr(q_in),
                                         _ptr(k_in), _ptr(v_in), _ptr(q_work), peer.handle, int(epoch),
                                         _stream_ptr(stream)))

    def combinePeers(self, peer: PeerArea, rows: int, epoch: int, out: torch.Tensor, timeout_s: float = 2.0,
                     stream=None) -> torch.Tensor:
        """Waits for every rank's partials of `epoch`, then their log-sum-exp combine -> out."""
        check(L.lib().brk_attn_combine_peers(self.ctx.handle, peer.handle, int(rows), int(epoch), float(timeout_s),
                                             _ptr(out), _stream_ptr(stream)))
        return out

    def combine(self, n_parts: int, rows: int, head_dim: int, part_ml: torch.Tensor, part_o: torch.Tensor,
                out: torch.Tensor, stream=None, part_stride: int = 0) -> torch.Tensor:
        """LSE combine of partials (dense [n_parts][rows] layouts, or a packed stride)."""
        check(L.lib().brk_attn_combine(self.ctx.handle, n_parts, rows, head_dim, _ptr(part_ml), _ptr(part_o),
                                       int(part_stride), _ptr(out), _stream_ptr(stream)))
        return out

    def close(self):
        self.resetKvGpu()
        self.ctx.close()
