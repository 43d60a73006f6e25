"""Partitioning the routed sparse-attention path across the GPUs of one node.

Three layouts, one process per GPU, ``torch.distributed`` (NCCL over NVLink/NVSwitch) for the
exchanges. The reference runs one video per GPU in separate worker processes
(local_experiments/video_runtime_v1/batch.py:29-37) and has no cross-GPU split of one
attention call; its in-GPU split-K LSE merge (migration/unified_router/opt21/attention.py:7-15)
is the exchange used here for KV-block sharding.

* streams (replicas): every rank runs its own stream; no collective at all.
* heads: rank r owns a contiguous range of heads. Router and attention are per head, so the
  call itself needs no exchange; ``gather_heads`` assembles the full [Lq,H,D] output for the
  o-projection (one all_gather).
* KV blocks: rank r owns the blocks with ``id % world == r`` (block-cyclic, which spreads the
  always-kept sink and current-chunk blocks evenly). Every rank computes the same router
  selection (the exact-fp32 router is deterministic), attends over the blocks it owns, and the
  partial results are merged by log-sum-exp: all_gather of the per-rank LSE, then an all_reduce
  (sum) of the weighted fp32 partial outputs.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from . import ops


def head_range(H: int, rank: int, world: int) -> tuple[int, int]:
    """Contiguous head range [h0, h1) of ``rank`` (the first H % world ranks get one more)."""
    base, rem = divmod(H, world)
    h0 = rank * base + min(rank, rem)
    return h0, h0 + base + (1 if rank < rem else 0)


def head_shard(x: torch.Tensor, rank: int, world: int, dim: int = -2) -> torch.Tensor:
    """Contiguous copy of this rank's heads (dim -2 of [L,H,D] activations, dim 0 of [H,..] weights)."""
    H = x.shape[dim]
    h0, h1 = head_range(H, rank, world)
    return x.narrow(dim, h0, h1 - h0).contiguous()


def gather_heads(local: torch.Tensor, H: int, group=None) -> torch.Tensor:
    """[Lq, h1-h0, D] per rank -> [Lq, H, D] on every rank (one all_gather)."""
    world = dist.get_world_size(group)
    Lq, _, D = local.shape
    sizes = [head_range(H, r, world) for r in range(world)]
    width = max(h1 - h0 for h0, h1 in sizes)
    pad = local.new_zeros((Lq, width, D))
    pad[:, :local.shape[1]] = local
    bufs = [torch.empty_like(pad) for _ in range(world)]
    dist.all_gather(bufs, pad, group=group)
    return torch.cat([b[:, :h1 - h0] for b, (h0, h1) in zip(bufs, sizes)], dim=1)


def shard_ids(ids: torch.Tensor, rank: int, world: int) -> torch.Tensor:
    """Keep the block ids this rank owns (block-cyclic ``id % world == rank``); others become -1."""
    own = (ids >= 0) & (torch.remainder(ids, world) == rank)
    return torch.where(own, ids, torch.full_like(ids, -1))


def merge_partials(o_local: torch.Tensor, lse_local: torch.Tensor, group=None, out_dtype=torch.bfloat16):
    """LSE merge of per-rank partial attention results over a process group.

    o_local fp32 [Lq,H,D] (normalised over the rank's own blocks), lse_local fp32 [H,Lq]
    (natural log, -inf where the rank saw no block). Returns (merged [Lq,H,D], global LSE [H,Lq]).
    """
    world = dist.get_world_size(group)
    lses = [torch.empty_like(lse_local) for _ in range(world)]
    dist.all_gather(lses, lse_local.contiguous(), group=group)
    stacked = torch.stack(lses)                               # [W,H,Lq]
    total = torch.logsumexp(stacked, dim=0)                   # [H,Lq]
    safe = torch.where(torch.isfinite(total), total, torch.zeros_like(total))
    w = torch.exp(lse_local - safe)                           # [H,Lq], 0 for empty parts
    w = torch.where(torch.isfinite(total), w, torch.zeros_like(w))
    weighted = o_local.float() * w.transpose(0, 1)[:, :, None]
    dist.all_reduce(weighted, op=dist.ReduceOp.SUM, group=group)
    return weighted.to(out_dtype), total


class KVShardedAttention:
    """Routed sparse attention with the KV blocks split block-cyclically over a process group."""

    def __init__(self, sparse, group=None):
        self.sparse = sparse          # a plugin.SparseAttention (router weights + config)
        self.group = group

    def __call__(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
        rank, world = dist.get_rank(self.group), dist.get_world_size(self.group)
        ids = self.sparse.route(q, k)
        mine = shard_ids(ids, rank, world)
        o, lse = ops.sparse_attention(q, k, v, mine, block=self.sparse.config.block, out_dtype=torch.float32,
                                      return_lse=True)
        out, _ = merge_partials(o, lse, self.group)
        return out


class HeadShardedAttention:
    """Routed sparse attention over this rank's heads; ``gather`` returns all heads."""

    def __init__(self, sparse_local, H: int, group=None):
        self.sparse = sparse_local    # SparseAttention built with this rank's head slice of wq/wk
        self.H = H
        self.group = group

    def __call__(self, q_local, k_local, v_local, gather: bool = True):
        out = self.sparse.forward_one(q_local, k_local, v_local)
        return gather_heads(out, self.H, self.group) if gather else out
