"""Partitioning the routed sparse-attention path across the GPUs of one node.

Three layouts, one process per GPU, ``torch.distributed`` (NCCL) for set-up collectives. The
reference runs one video per GPU in separate worker processes
(local_experiments/video_runtime_v1/batch.py:29-37) and has no cross-GPU split of one attention
call; its in-GPU split merge (migration/unified_router/opt21/attention.py:7-15) is the combine
used here for KV-block sharding.

* streams (replicas): every rank runs its own stream; no collective at all.
* heads: rank r owns a contiguous range of heads. Router and attention are per head, so the
  call itself needs no exchange; the full [Lq,H,D] output for the o-projection is assembled
  either by ``gather_heads`` (one NCCL all_gather after the attention) or, fused, by the
  attention kernel itself: its epilogue stores every output row into all ranks' output buffers
  over NVLink (``ss_attention_heads``), and a flag barrier ends the call.
* KV blocks (``KVShardedAttention``): rank r stores only the window blocks j with
  ``j % world == r`` (block-cyclic, which spreads the always-kept sink and current-chunk blocks
  evenly), packed into a local window. The history's pooled key projections are computed by
  their owners and all-gathered once per commit; every rank then routes with the same exact-fp32
  router (bit-identical ids everywhere), pooling the current chunk itself from the window's tail.
  Exchange "push" (default): rank d owns query rows [d*rows, (d+1)*rows); each rank's attention
  epilogue stores every partial row (and its LSE) over NVLink into the owner's buffers
  (``ss_attention_kv_parts``, a reduce-scatter inside the attention); after a flag barrier each
  rank merges its own rows from its own memory and stores them into every rank's output
  (``ss_lse_merge_gather``, an all-gather inside the merge); a second barrier ends the call.
  Exchange "pull": each rank attends into buffers the other ranks have mapped (CUDA IPC), and one
  kernel per rank (``ss_lse_merge_peers``, after the flag barrier ``ss_peer_barrier``) reads all
  partials over NVLink and writes the merged rows.
"""
from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from . import ops
from ._lib import check, lib


# ----------------------------------------------------------------------------------------------
# heads
# ----------------------------------------------------------------------------------------------

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


class HeadShardedAttention:
    """Routed sparse attention over this rank's heads; ``gather`` returns all heads.

    Without ``Lq`` the heads are gathered with one NCCL all_gather after the attention. With
    ``Lq`` (the chunk length of every call) and ``device``, the gather is fused into the
    attention: each rank's [2, Lq, H, D] output buffer is mapped by every other rank (CUDA IPC),
    the attention kernel's epilogue stores each output row of this rank's heads into all ranks'
    buffers over NVLink (``ss_attention_heads``), and a flag barrier (``ss_peer_barrier``) ends the
    call. Calls alternate between the two slots; the returned view stays valid until the call
    after next (pass ``out`` for a copy). No host synchronisation: a call can be captured in a
    CUDA graph (capture calls in pairs). Every rank makes the same calls in the same order."""

    def __init__(self, sparse_local, H: int, group=None, Lq: int | None = None, device=None, slots: int = 2):
        self.sparse = sparse_local    # SparseAttention built with this rank's head slice of wq/wk
        self.H = H
        self.group = group
        self.peer = None
        if Lq is not None:
            self.rank, self.world = dist.get_rank(group), dist.get_world_size(group)
            if self.world > 8:
                raise ValueError("the fused head gather takes at most 8 ranks")
            self.h0, self.h1 = head_range(H, self.rank, self.world)
            self.Lq = Lq               # the most query rows of a call
            self.slots = slots
            self.device = torch.device(device)
            self.peer = PeerBuffers({"out": ((slots, Lq, H, ops.HEAD_DIM), torch.bfloat16),
                                     "flags": ((self.world,), torch.int32)}, self.device, group)
            self.epoch = torch.zeros(1, dtype=torch.int32, device=self.device)
            self.slot_bytes = Lq * H * ops.HEAD_DIM * 2
            self.ws = ops.Workspace()
            self.calls = 0

    def __call__(self, q_local, k_local, v_local, gather: bool = True, out: torch.Tensor | None = None):
        if self.peer is None or not gather:
            res = self.sparse.forward_one(q_local, k_local, v_local)
            res = gather_heads(res, self.H, self.group) if gather else res
            if out is not None:
                out.copy_(res)
                return out
            return res
        Lq, h, _ = q_local.shape
        assert Lq <= self.Lq and h == self.h1 - self.h0, "q_local must be this rank's heads of at most Lq rows"
        sp = self.sparse
        cache = sp.cache_of(k_local)
        ring = cache.ring if cache is not None and cache.ring_mode else None
        Lk = cache.window_rows() if ring is not None else k_local.shape[0]
        ids = sp._dense_ids(h, Lq, Lk, q_local.device) if sp.dense else sp.route(q_local, k_local, cache)
        sp.last_ids = ids
        sp.calls += 1
        slot = self.calls % self.slots
        ops.sparse_attention_heads(q_local, k_local, v_local, ids,
                                   [p + slot * self.slot_bytes for p in self.peer.ptrs["out"]], out_heads=self.H,
                                   h0=self.h0, block=sp.config.block, workspace=self.ws, ring=ring,
                                   Lk=Lk if ring is not None else None)
        stream = ops._stream(self.device)
        status = ops.DeviceStatus.word(self.device)
        check(lib().ss_peer_barrier(_ptr_array(self.peer.ptrs["flags"]), self.rank, self.world, ops._p(self.epoch),
                                    ops._p(status), stream), "ss_peer_barrier")
        self.calls += 1
        res = self.peer.local["out"][slot][:Lq]
        if out is not None:
            out.copy_(res)
            return out
        return res

    def close(self):
        if self.peer is not None:
            self.peer.close()
            self.peer = None


class HeadParallelAttention:
    """The attention a head-parallel model's plugin calls: every layer hands this rank's heads
    (q [1, n, h, D] and the layer's cache window of h heads) and gets all heads [1, n, H, D] back
    through that layer's fused head gather (``HeadShardedAttention``). Built from the full-model
    ``SparseAttention``: the router weights are sliced to this rank's heads.

    Each layer has one output buffer. Layer l's buffer is written again only in the next model
    call, after every rank has passed the barriers of the layers in between, and a rank posts
    each of those after the o-projection that read layer l's output -- so with two or more layers
    one buffer per layer is enough (one layer takes two, alternating). Attributes not set here
    (``config``, ``wq``, ``dense``, ``attach`` ...) are the local ``SparseAttention``'s."""

    def __init__(self, sparse_full, caches, Lq: int, device, group=None):
        from .plugin import SparseAttention
        rank, world = dist.get_rank(group), dist.get_world_size(group)
        H = sparse_full.wq.shape[0]
        local = SparseAttention(head_shard(sparse_full.wq, rank, world, 0), head_shard(sparse_full.wk, rank, world, 0),
                                sparse_full.config, validate=sparse_full.validate)
        object.__setattr__(self, "local", local)
        slots = 1 if len(caches) >= 2 else 2
        object.__setattr__(self, "layers", {id(c): HeadShardedAttention(local, H, group, Lq=Lq, device=device,
                                                                         slots=slots) for c in caches})

    def __getattr__(self, name):
        return getattr(self.local, name)

    def __setattr__(self, name, value):
        setattr(self.local, name, value)

    def __call__(self, q, k, v):
        cache = self.local.cache_of(k[0])
        if cache is None or id(cache) not in self.layers:
            raise ValueError("k is not the window of one of this model's caches")
        return self.layers[id(cache)](q[0], k[0], v[0])[None]

    def close(self):
        for hs in self.layers.values():
            hs.close()


# ----------------------------------------------------------------------------------------------
# KV blocks: ownership and the local window
# ----------------------------------------------------------------------------------------------

def owned_blocks(kb: int, rank: int, world: int) -> range:
    """Window blocks rank ``rank`` stores: j = rank, rank + world, ... (< kb)."""
    return range(rank, kb, world)


def local_len(Lk: int, block: int, rank: int, world: int) -> int:
    """Tokens of rank ``rank``'s local window: its blocks packed in order. Only the window's last
    block can be partial, and it is the last block of its owner, so every local block keeps the
    valid-token count of the window block it holds."""
    own = owned_blocks(ops.nblocks(Lk, block), rank, world)
    if len(own) == 0:
        return 0
    return (len(own) - 1) * block + min(block, Lk - own[-1] * block)


def local_rows(Lk: int, block: int, rank: int, world: int) -> torch.Tensor:
    """Window row of each local row (int64, ascending)."""
    own = torch.tensor(list(owned_blocks(ops.nblocks(Lk, block), rank, world)), dtype=torch.int64)
    rows = (own[:, None] * block + torch.arange(block)[None]).reshape(-1)
    return rows[rows < Lk]


def owner_rows(Lq: int, rank: int, world: int) -> tuple[int, int, int]:
    """Query rows [lo, hi) whose merged output rank ``rank`` owns under the push exchange, and
    the row count of every owner's buffers (ceil(Lq / world)); row t belongs to rank t // rows."""
    rows = -(-Lq // world)
    lo = min(Lq, rank * rows)
    return lo, min(Lq, lo + rows), rows


def shard_ids(ids: torch.Tensor, rank: int, world: int) -> torch.Tensor:
    """Keep the block ids this rank owns (window numbering); others become -1."""
    own = (ids >= 0) & (torch.remainder(ids, world) == rank)
    return torch.where(own, ids, torch.full_like(ids, -1))


def local_ids(ids: torch.Tensor, rank: int, world: int) -> torch.Tensor:
    """The block ids this rank owns, renumbered into its local window (j -> j // world); others -1."""
    own = (ids >= 0) & (torch.remainder(ids, world) == rank)
    return torch.where(own, torch.div(ids, world, rounding_mode="floor"), torch.full_like(ids, -1))


def assemble_keys(parts, world: int, n_blocks: int) -> torch.Tensor:
    """Window key table [H, n_blocks, R] from the ranks' tables of their own blocks
    (parts[r] [H, >= len(owned_blocks(n_blocks, r, world)), R]): window block j = jl*world + r is
    row jl of parts[r]."""
    H, _, R = parts[0].shape
    out = parts[0].new_empty((H, n_blocks, R))
    for r, part in enumerate(parts):
        n = len(owned_blocks(n_blocks, r, world))
        if n:
            out[:, r::world][:, :n] = part[:, :n]
    return out


# ----------------------------------------------------------------------------------------------
# buffers the ranks of a node read from each other (CUDA IPC through libssparse)
# ----------------------------------------------------------------------------------------------

class PeerBuffers:
    """Device buffers that every rank of a group can read: each rank allocates its own (one torch
    allocation, carved into the named buffers at 256-byte boundaries), exports it
    (``ss_ipc_handle``) and maps everyone else's (``ss_ipc_open``) once.
    ``ptrs[name][r]`` is rank r's buffer as a device address valid on this rank's GPU."""

    def __init__(self, specs: dict, device, group=None):
        self.group = group
        self.rank, self.world = dist.get_rank(group), dist.get_world_size(group)
        offsets, total = {}, 0
        for name, (shape, dtype) in specs.items():
            offsets[name] = total
            n = torch.Size(shape).numel() * torch.empty((), dtype=dtype).element_size()
            total += (n + 255) // 256 * 256
        self.storage = torch.zeros(total, dtype=torch.uint8, device=device)
        self.local = {name: self.storage[offsets[name]:].view(dtype)[:torch.Size(shape).numel()].view(shape)
                      for name, (shape, dtype) in specs.items()}
        torch.cuda.synchronize(device)
        handle = (ctypes.c_char * 64)()
        off = ctypes.c_size_t()
        check(lib().ss_ipc_handle(ctypes.c_void_p(self.storage.data_ptr()), handle, ctypes.byref(off)),
              "ss_ipc_handle")
        everyone = [None] * self.world
        dist.all_gather_object(everyone, (bytes(handle), off.value), group=group)
        bases, self._opened = [], []
        for r in range(self.world):
            if r == self.rank:
                bases.append(self.storage.data_ptr())
                continue
            h, o = everyone[r]
            p = ctypes.c_void_p()
            check(lib().ss_ipc_open((ctypes.c_char * 64).from_buffer_copy(h), o, ctypes.byref(p)), "ss_ipc_open")
            bases.append(p.value)
            self._opened.append((p.value, o))
        self.ptrs = {name: [b + offsets[name] for b in bases] for name in specs}
        dist.barrier(group=group)        # every mapping exists before anyone writes through it

    def close(self):
        """Unmap the peers' buffers (every rank calls it; the buffers stay alive until all did)."""
        for p, off in self._opened:
            lib().ss_ipc_close(ctypes.c_void_p(p), off)
        self._opened = []
        dist.barrier(group=self.group)


def _ptr_array(ptrs, offset: int = 0):
    arr = (ctypes.c_void_p * len(ptrs))()
    for i, p in enumerate(ptrs):
        arr[i] = p + offset
    return arr


class KVShardedAttention:
    """Routed sparse attention with the KV window split block-cyclically over a process group.

    One instance serves one layer's window geometry (chunk of ``Lq`` tokens at the end of an
    ``Lk``-token window). ``commit(k, v)`` takes a full window (post-RoPE K/V as the model's cache
    holds it), keeps this rank's blocks, pools the projections of its history blocks and
    all-gathers them (the commit-time pooling of the reference's streaming pipeline,
    migration/unified_router/opt23/pipeline.py:22-29). ``__call__(q, k_chunk, v_chunk)`` is one
    routed chunk-layer call: every rank passes the same chunk (its q/k/v come from the replicated
    activations) and gets the merged bf16 output [Lq, H, D]. A call has no host synchronisation
    and can be captured in a CUDA graph (capture calls in pairs: with ``exchange="pull"`` they
    alternate between two partial buffers); every rank makes the same calls in the same order.

    ``exchange="push"`` needs one buffer set: a rank's attention of call i+1 writes into a peer's
    partials only after the second barrier of call i, which the peer posts after its merge of
    call i has read them, and a peer's merge of call i+1 writes this rank's output only after the
    first barrier of call i+1, which this rank posts after the work it enqueued before the call.
    The returned output (a view of the mapped buffer) stays valid until the next call; pass
    ``out`` for a copy.
    """

    def __init__(self, sparse, Lq: int, Lk: int, device, group=None, part_dtype=torch.bfloat16,
                 exchange: str = "push"):
        self.sparse, self.group = sparse, group
        self.rank, self.world = dist.get_rank(group), dist.get_world_size(group)
        if self.world > 8:
            raise ValueError("the peer merge takes at most 8 ranks")
        if exchange not in ("push", "pull"):
            raise ValueError("exchange is 'push' or 'pull'")
        self.exchange = exchange
        c = sparse.config
        self.block, self.Lq, self.Lk = c.block, Lq, Lk
        self.H = sparse.wq.shape[0]
        self.R = sparse.wq.shape[2]
        self.extra = c.extra(Lq, Lk)
        self.kb = ops.nblocks(Lk, self.block)
        self.n_hist = ops.history_blocks(Lq, Lk, self.block)      # blocks wholly before the chunk
        self.row0 = self.n_hist * self.block                      # window row where the tail starts
        self.Lk_local = local_len(Lk, self.block, self.rank, self.world)
        rows = local_rows(Lk, self.block, self.rank, self.world)
        self.rows = rows.to(device)
        chunk0 = Lk - Lq
        in_chunk = rows >= chunk0
        self.chunk_src = (rows[in_chunk] - chunk0).to(device)     # chunk rows this rank stores
        self.chunk_dst = torch.nonzero(in_chunk).reshape(-1).to(device)
        D = ops.HEAD_DIM
        self.k_local = torch.zeros((max(self.Lk_local, 1), self.H, D), dtype=torch.bfloat16, device=device)
        self.v_local = torch.zeros_like(self.k_local)
        self.k_tail = torch.zeros((Lk - self.row0, self.H, D), dtype=torch.bfloat16, device=device)
        self.keys = ops.RouterKeys(self.H, Lk, block=self.block, R=self.R, device=device)
        self.ws = ops.Workspace()
        self.part_fp32 = part_dtype == torch.float32
        esz = 4 if self.part_fp32 else 2
        if exchange == "pull":
            self.peer = PeerBuffers({"o": ((2, Lq, self.H, D), part_dtype), "lse": ((2, self.H, Lq), torch.float32),
                                     "flags": ((self.world,), torch.int32)}, device, group)
            self.o_bytes = Lq * self.H * D * esz
            self.lse_bytes = self.H * Lq * 4
        else:
            # rank d owns output rows [d * rows, (d + 1) * rows): its "o" / "lse" hold every rank's
            # partial of those rows (slot = the writing rank), its "out" the merged output
            self.row_lo, self.row_hi, self.rows_per_rank = owner_rows(Lq, self.rank, self.world)
            self.peer = PeerBuffers({"o": ((self.world, self.rows_per_rank, self.H, D), part_dtype),
                                     "lse": ((self.world, self.H, self.rows_per_rank), torch.float32),
                                     "out": ((Lq, self.H, D), torch.bfloat16),
                                     "flags": ((self.world,), torch.int32)}, device, group)
            self.peer.local["lse"].fill_(float("-inf"))    # slots of ranks that store no block stay empty
            torch.cuda.synchronize(device)
            dist.barrier(group=group)
            self.o_slot_bytes = self.rows_per_rank * self.H * D * esz
            self.lse_slot_bytes = self.H * self.rows_per_rank * 4
            self.out_row_bytes = self.H * D * 2
        self.epoch = torch.zeros(1, dtype=torch.int32, device=device)   # advanced by the barrier kernels
        self.calls = 0
        self.device = device
        self.last_ids = None

    def commit(self, k: torch.Tensor, v: torch.Tensor) -> None:
        """Take the window [Lk, H, D] (the history rows matter; the chunk rows are rewritten by
        every call): keep this rank's blocks, pool the projections of its history blocks, and
        all-gather them into the window key table shared by every rank's router."""
        assert k.shape == (self.Lk, self.H, ops.HEAD_DIM) and v.shape == k.shape
        if self.Lk_local:
            self.k_local[:self.Lk_local] = k.index_select(0, self.rows)
            self.v_local[:self.Lk_local] = v.index_select(0, self.rows)
        self.k_tail.copy_(k[self.row0:])
        n_own = len(owned_blocks(self.n_hist, self.rank, self.world))
        n_max = len(owned_blocks(self.n_hist, 0, self.world))
        mine = torch.zeros((self.H, max(n_max, 1), self.R), dtype=torch.float32, device=self.device)
        if n_own:
            part = ops.RouterKeys(self.H, self.Lk_local, block=self.block, R=self.R, device=self.device)
            ops.pool_keys(self.k_local[:self.Lk_local], self.sparse.wk, part, j0=0, j1=n_own)
            mine[:, :n_own] = part.kh[:, :n_own]
        gathered = [torch.empty_like(mine) for _ in range(self.world)]
        dist.all_gather(gathered, mine, group=self.group)
        if self.n_hist:
            self.keys.kh[:, :self.n_hist] = assemble_keys(gathered, self.world, self.n_hist)
        self.keys.mark(("kv-shard", id(self)), self.n_hist)

    def route(self, q: torch.Tensor) -> torch.Tensor:
        c = self.sparse.config
        return ops.route(q, self.k_tail, self.sparse.wq, self.sparse.wk, block=self.block, extra=self.extra,
                         sink_tokens=c.sink_tokens, workspace=self.ws, keys=self.keys, n_cached=self.n_hist,
                         k_row0=self.row0, fast=c.fast)

    def write_chunk(self, k_chunk: torch.Tensor, v_chunk: torch.Tensor) -> None:
        """The chunk's k/v rows this rank stores into its local window, the whole chunk into the
        router's tail (the cache write of a denoising call, which a single-GPU cache makes in its
        append)."""
        assert k_chunk.shape == (self.Lq, self.H, ops.HEAD_DIM) and v_chunk.shape == k_chunk.shape
        if self.chunk_dst.numel():
            self.k_local.index_copy_(0, self.chunk_dst, k_chunk.index_select(0, self.chunk_src))
            self.v_local.index_copy_(0, self.chunk_dst, v_chunk.index_select(0, self.chunk_src))
        self.k_tail[self.Lk - self.Lq - self.row0:].copy_(k_chunk)

    def __call__(self, q: torch.Tensor, k_chunk: torch.Tensor, v_chunk: torch.Tensor,
                 out: torch.Tensor | None = None) -> torch.Tensor:
        """``write_chunk`` then ``attend``."""
        self.write_chunk(k_chunk, v_chunk)
        return self.attend(q, out)

    def attend(self, q: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        """Route and attend the chunk's queries over the window as last written, merged over the
        ranks."""
        Lq, H, D = q.shape
        assert Lq == self.Lq and H == self.H
        ids = self.route(q)                        # identical on every rank (exact-fp32 router)
        self.last_ids = ids
        if self.exchange == "push":
            return self._call_push(q, ids, out)
        slot = self.calls % 2
        o_part = self.peer.local["o"][slot]
        lse_part = self.peer.local["lse"][slot]
        if self.Lk_local:
            ops.sparse_attention(q, self.k_local[:self.Lk_local], self.v_local[:self.Lk_local],
                                 local_ids(ids, self.rank, self.world), block=self.block,
                                 out_dtype=torch.float32 if self.part_fp32 else torch.bfloat16, return_lse=True,
                                 out=o_part, lse=lse_part)
        else:
            o_part.zero_()
            lse_part.fill_(float("-inf"))
        # every rank's partial is written -> merged rows over peer memory
        stream = ops._stream(self.device)
        status = ops.DeviceStatus.word(self.device)
        check(lib().ss_peer_barrier(_ptr_array(self.peer.ptrs["flags"]), self.rank, self.world, ops._p(self.epoch),
                                    ops._p(status), stream), "ss_peer_barrier")
        if out is None:
            out = torch.empty((Lq, H, D), dtype=torch.bfloat16, device=self.device)
        check(lib().ss_lse_merge_peers(_ptr_array(self.peer.ptrs["o"], slot * self.o_bytes),
                                       _ptr_array(self.peer.ptrs["lse"], slot * self.lse_bytes), self.world,
                                       1 if self.part_fp32 else 0, H, Lq, 0, Lq, ops._p(out), 0, None, stream),
              "ss_lse_merge_peers")
        self.calls += 1
        return out

    def _call_push(self, q, ids, out):
        """Attention whose epilogue stores each partial row into its owner's slot for this rank
        (the reduce-scatter), a barrier, each rank's merge of its own rows from its own memory with
        the merged rows stored into every rank's output (the all-gather), a barrier."""
        Lq, H, D = q.shape
        stream = ops._stream(self.device)
        status = ops.DeviceStatus.word(self.device)
        dtype = 1 if self.part_fp32 else 0
        if self.Lk_local:
            # the window's ids: the kernel keeps the blocks this rank stores (j % world == rank)
            nws = ops.attention_workspace_bytes(H, Lq)
            ws = self.ws.tensor("attention_split", (max(nws, 256),), self.device, torch.uint8)
            check(lib().ss_attention_kv_parts(ops._p(q), ops._p(self.k_local), ops._p(self.v_local), ops._p(ids), H,
                                              Lq, self.Lk_local, self.block, ids.shape[2], 1.0 / D ** 0.5,
                                              _ptr_array(self.peer.ptrs["o"]), _ptr_array(self.peer.ptrs["lse"]),
                                              self.world, self.rows_per_rank, self.rank, dtype, ops._p(status),
                                              ops._p(ws) if nws else None, nws, stream), "ss_attention_kv_parts")
        # the first barrier is made by the merge kernel itself, before it reads the pushed partials
        flags = _ptr_array(self.peer.ptrs["flags"])
        o0, l0 = self.peer.ptrs["o"][self.rank], self.peer.ptrs["lse"][self.rank]
        o_parts = _ptr_array([o0 + p * self.o_slot_bytes for p in range(self.world)])
        lse_parts = _ptr_array([l0 + p * self.lse_slot_bytes for p in range(self.world)])
        check(lib().ss_lse_merge_gather(o_parts, lse_parts, self.world, dtype, H, self.rows_per_rank, 0,
                                        self.row_hi - self.row_lo,
                                        _ptr_array(self.peer.ptrs["out"], self.row_lo * self.out_row_bytes),
                                        self.world, 0, flags, self.rank, ops._p(self.epoch), ops._p(status), stream),
              "ss_lse_merge_gather")
        check(lib().ss_peer_barrier(flags, self.rank, self.world, ops._p(self.epoch), ops._p(status), stream),
              "ss_peer_barrier")
        self.calls += 1
        res = self.peer.local["out"]
        if out is not None:
            out.copy_(res)
            return out
        return res

    def close(self):
        self.peer.close()
