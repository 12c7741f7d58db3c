"""Sequence-sharded long-context decode across GPUs (no reference counterpart: the reference
runs one GPU; this is the multi-GPU form of its decode over a very long KV cache).

Each rank owns a contiguous range of positions [lo, hi) of every (layer, sequence, kv head) and
keeps only those rows.  Per layer and step:
  1. every rank rotates q (replicated), and the rank owning the new position appends its K/V;
  2. every rank computes split-KV partials (max m, sum l, unnormalised o) over its rows;
  3. the partials [rows*2 | rows*D] reach every rank;
  4. every rank merges the N partials with the log-sum-exp combine.
The only communication is step 3 (B * Hq * (D + 2) * 4 bytes per rank per layer).  Two forms:
  - fused (``fused=True``, what bench.py runs): the decode kernel itself stores its partials into every rank's exchange
    area through NVLink (CUDA IPC mappings, brk_attn_decode_push) and publishes an epoch flag;
    the combine kernel waits for all flags (brk_attn_combine_peers).  No collective launch.
  - nccl: decode_partial, an NCCL all-gather, then the combine (the library-collective baseline).
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import torch
import torch.distributed as dist


@dataclass(frozen=True)
class ShardPlan:
    """Contiguous split of positions [0, context) over `world` ranks; the last rank also owns
    positions beyond `context` (new tokens appended at the end)."""
    context: int
    world: int
    rank: int

    @property
    def shard(self) -> int:
        return (self.context + self.world - 1) // self.world

    @property
    def lo(self) -> int:
        return min(self.context, self.rank * self.shard)

    @property
    def hi(self) -> int:
        return self.context if self.rank == self.world - 1 else min(self.context, (self.rank + 1) * self.shard)

    def owner(self, position: int) -> int:
        if position >= self.context:
            return self.world - 1
        return min(self.world - 1, position // self.shard)

    def capacity(self, extra: int = 0) -> int:
        """Rows this rank's cache needs (the last rank keeps room for `extra` appended tokens)."""
        return self.hi - self.lo + (extra if self.rank == self.world - 1 else 0)


def packed_partial_floats(rows: int, head_dim: int) -> int:
    return rows * (2 + head_dim)


def gather_partials(part: torch.Tensor, world: int, group=None, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """All-gather of one packed partial buffer per rank -> [world, numel] (rank order)."""
    if out is None:
        out = torch.empty((world, part.numel()), dtype=part.dtype, device=part.device)
    if world == 1:
        out[0].copy_(part.reshape(-1))
    else:
        dist.all_gather_into_tensor(out.view(-1), part.reshape(-1).contiguous(), group=group)
    return out


class ShardedDecoder:
    """One rank's part of a sequence-sharded decode over a context of `context` positions."""

    def __init__(self, engine, plan: ShardPlan, n_layers: int, batch: int, n_kv_heads: int, head_dim: int,
                 extra: int = 1, group=None, fused: bool = False, max_rows: int = 0):
        """fused=True needs max_rows (>= batch * n_tokens * n_heads of every step) and, with
        several ranks, an initialised process group: the ranks exchange IPC handles here (a
        collective) and must call close() together."""
        from .engine import KvCache, PeerArea
        self.engine, self.plan, self.group = engine, plan, group
        self.batch, self.head_dim = batch, head_dim
        self.kv = KvCache(engine.ctx, n_layers, batch, n_kv_heads, head_dim, max(1, plan.capacity(extra)))
        self._bufs = {}
        self.fused = bool(fused)
        self.peer = None
        self.epoch = 0
        if self.fused:
            if max_rows < 1:
                raise ValueError("fused sharded decode needs max_rows")
            self.peer = PeerArea(engine.ctx, plan.world, plan.rank, max_rows, head_dim)
            if plan.world > 1:
                handles = [None] * plan.world
                dist.all_gather_object(handles, self.peer.ipc_handle(), group=group)
                for r, h in enumerate(handles):
                    if r != plan.rank:
                        self.peer.open(r, h)

    def _buffers(self, rows: int, dev):
        key = rows
        if key not in self._bufs:
            n = packed_partial_floats(rows, self.head_dim)
            self._bufs[key] = (torch.empty(n, dtype=torch.float32, device=dev),
                               torch.empty((self.plan.world, n), dtype=torch.float32, device=dev))
        return self._bufs[key]

    def step(self, layer: int, cfg, q_in: torch.Tensor, k_in: torch.Tensor, v_in: torch.Tensor, position: int,
             q_work: torch.Tensor, out: torch.Tensor, stream=None) -> torch.Tensor:
        """One decode token per sequence at `position` (the same for every sequence)."""
        import dataclasses
        p = self.plan
        shard_cfg = dataclasses.replace(cfg, kv_offset=p.lo)
        owns = p.owner(position) == p.rank
        B = self.batch
        pos = [position] * B
        rows = B * cfg.n_heads
        q_tokens = q_in.numel() // (B * cfg.n_heads * cfg.head_dim)
        if self.fused and q_tokens == 1 and (cfg.head_dim != 256 or cfg.n_heads // cfg.n_kv_heads <= 4):
            # One launch: q rotation, the owner's K/V append and the partials pushed to every rank.
            self.epoch += 1
            self.engine.stepPush(self.kv, layer, shard_cfg, q_in, k_in if owns else None, v_in if owns else None,
                                 q_work, self.peer, self.epoch, pos, stream)
            return self.engine.combinePeers(self.peer, rows, self.epoch, out, stream=stream)
        # q rotation everywhere; K/V stored only by the owner of this position.
        self.engine.appendKv(self.kv, layer, shard_cfg, q_in, k_in if owns else None, v_in if owns else None, q_work,
                             pos, stream)
        if self.fused:
            self.epoch += 1
            self.engine.decodePush(self.kv, layer, shard_cfg, q_work, self.peer, self.epoch, pos, stream)
            return self.engine.combinePeers(self.peer, rows, self.epoch, out, stream=stream)
        part, gathered = self._buffers(rows, q_in.device)
        self.engine.decodePartial(self.kv, layer, shard_cfg, q_work, part[:rows * 2], part[rows * 2:], pos, stream)
        gather_partials(part, p.world, self.group, gathered)
        n = packed_partial_floats(rows, self.head_dim)
        self.engine.combine(p.world, rows, self.head_dim, gathered, gathered.reshape(-1)[rows * 2:], out, stream,
                            part_stride=n)
        return out

    def close(self):
        """Collective in fused mode: no rank unmaps its area while another may still store to it."""
        if self.peer is not None:
            torch.cuda.synchronize(self.kv.ctx.device)
            if self.plan.world > 1:
                dist.barrier(group=self.group)
            self.peer.close()
            self.peer = None
        self.kv.close()
