"""Multi-GPU partitioning of the DASH forward: one process per GPU.

Every (sequence, kv head) unit is independent once routed, and the router is a
single head per sequence, so the batch is split across ranks sequence-major;
when there are more ranks than sequences, a sequence's kv heads are split
across ranks and each of those ranks recomputes that sequence's (cheap) route.
Nothing crosses NVLink inside attention.  The one collective is the final
gather of the output shards: either fused into the attention kernel
(``run_sharded_fused``: each output row is stored into every rank's gathered
tensor over NVLink as soon as it is computed, then one stream-ordered NCCL
word marks completion) or an NCCL all-gather after it (``run_sharded``; gloo
on CPU in the tests).
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Callable, List, Optional

import torch
import torch.distributed as dist


@dataclass(frozen=True)
class Shard:
    b0: int
    b1: int      # sequences [b0, b1)
    h0: int
    h1: int      # kv heads [h0, h1)

    @property
    def empty(self) -> bool:
        return self.b1 <= self.b0 or self.h1 <= self.h0


def plan_shards(n_seq: int, n_kv_heads: int, world: int) -> List[Shard]:
    """Sequence-major partition of n_seq x n_kv_heads units over `world` ranks."""
    if world <= 0:
        raise ValueError("world must be positive")
    if world <= n_seq:
        base, rem = divmod(n_seq, world)
        out, b = [], 0
        for r in range(world):
            n = base + (1 if r < rem else 0)
            out.append(Shard(b, b + n, 0, n_kv_heads))
            b += n
        return out
    if world % n_seq != 0:
        raise ValueError(f"{world} ranks cannot split {n_seq} sequences evenly")
    per_seq = world // n_seq
    if n_kv_heads % per_seq != 0:
        raise ValueError(f"{n_kv_heads} kv heads not divisible over {per_seq} ranks per sequence")
    hs = n_kv_heads // per_seq
    return [Shard(r // per_seq, r // per_seq + 1, (r % per_seq) * hs, (r % per_seq + 1) * hs)
            for r in range(world)]


def run_sharded(attn: Callable, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                idx_q: torch.Tensor, idx_k: torch.Tensor, *, rank: int, world: int,
                group: Optional[dist.ProcessGroup] = None, gather: bool = True):
    """Run ``attn(q, k, v, idx_q, idx_k) -> out`` on this rank's shard of a
    [B, H, S, D] problem (router inputs [B, S, d]) and all-gather the output.

    Returns the full output [B, H, S, D] on every rank when ``gather`` (else the
    local shard and its Shard)."""
    B, H, S, D = q.shape
    Hkv = k.shape[1]
    G = H // Hkv
    plan = plan_shards(B, Hkv, world)
    sh = plan[rank]
    out_local = attn(q[sh.b0:sh.b1, sh.h0 * G:sh.h1 * G], k[sh.b0:sh.b1, sh.h0:sh.h1],
                     v[sh.b0:sh.b1, sh.h0:sh.h1], idx_q[sh.b0:sh.b1], idx_k[sh.b0:sh.b1])
    if not gather or world == 1:
        return (out_local, sh) if not gather else out_local
    # equal-sized buffers for the collective: pad every shard to the largest one
    max_units = max((s.b1 - s.b0) * (s.h1 - s.h0) for s in plan)
    per_unit = G * S * D
    send = out_local.new_zeros(max_units * per_unit)
    flat = out_local.permute(0, 1, 2, 3).reshape(-1)
    send[:flat.numel()] = flat
    recv = out_local.new_empty(world * max_units * per_unit)
    dist.all_gather_into_tensor(recv, send, group=group)
    full = q.new_empty(B, H, S, D, dtype=out_local.dtype)
    for r, s in enumerate(plan):
        n = (s.b1 - s.b0) * (s.h1 - s.h0) * per_unit
        chunk = recv[r * max_units * per_unit: r * max_units * per_unit + n]
        full[s.b0:s.b1, s.h0 * G:s.h1 * G] = chunk.view(s.b1 - s.b0, (s.h1 - s.h0) * G, S, D)
    return full


def run_sharded_fused(attn: Callable, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                      idx_q: torch.Tensor, idx_k: torch.Tensor, gather, *, rank: int,
                      world: int, complete: bool = True) -> torch.Tensor:
    """This rank's shard of a [B, H, S, D] problem with the gather fused into
    the attention: ``attn(q, k, v, idx_q, idx_k, out=, peers=)`` writes the
    shard's rows into ``out`` (this rank's slice of ``gather.full``, a
    ``peer.PeerGather`` over a [B, H, S, D] tensor every rank holds) and into
    the peers' copies.  Returns ``gather.full``, complete on every rank once
    the stream reaches the end of the call (``complete``)."""
    B, H, S, D = q.shape
    Hkv = k.shape[1]
    G = H // Hkv
    sh = plan_shards(B, Hkv, world)[rank]
    view = gather.full[sh.b0:sh.b1, sh.h0 * G:sh.h1 * G]
    attn(q[sh.b0:sh.b1, sh.h0 * G:sh.h1 * G], k[sh.b0:sh.b1, sh.h0:sh.h1],
         v[sh.b0:sh.b1, sh.h0:sh.h1], idx_q[sh.b0:sh.b1], idx_k[sh.b0:sh.b1],
         out=view, peers=gather.peers_for(view))
    if complete:
        gather.complete()
    return gather.full
