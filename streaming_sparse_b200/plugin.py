"""Drop-in plugin: routed block-sparse attention behind the reference's ``attention(q, k, v)``.

The reference swaps the module-level ``wan.modules.causal_model.attention`` symbol, which
CausalWanSelfAttention.forward calls with the RoPE'd queries of the current chunk and the
visible KV window (wan/modules/causal_model.py:247-251); ``SelfForcingAdapter.__enter__``
(streaming_sparse/integration/self_forcing_adapter.py:104-125) does the swap, rejects extra
positional/keyword options, refuses nested adapters and restores the symbol on exit.
``SparsePlugin`` does the same around ``SparseAttention``, a callable with that exact
signature: ``q [B,Lq,H,D]``, ``k, v [B,Lk,H,D]`` bf16 with the current chunk as the last
``Lq`` rows of ``k``/``v`` -> ``[B,Lq,H,D]`` bf16.
"""
from __future__ import annotations

import importlib
import math
import weakref
from dataclasses import dataclass

import torch

from . import ops

_PATCH_FLAG = "_streaming_sparse_b200_patch"


@dataclass(frozen=True)
class RouterConfig:
    """Block size and budget of the learned block router.

    Exactly one of ``topk`` (fixed count outside the forced set) or ``density`` is used;
    ``rule`` picks how ``density`` becomes a count (see ``ops.budget``). ``fast`` scores the blocks
    on the tensor cores (``ops.route(..., fast=True)``; same ids, proj_dim 32 or 64). ``int8`` runs
    the attention on the INT8-QK path (``ops.sparse_attention_i8``; the reference's
    ``attention(..., int8=True)``, migration/unified_router/opt23/attention.py:60-69), on plain
    windows and ring caches.
    """

    block: int = 64
    topk: int | None = None
    density: float | None = 0.25
    rule: str = "total"
    sink_tokens: int = 0
    proj_dim: int = 64
    fast: bool = False
    int8: bool = False

    def extra(self, Lq: int, Lk: int) -> int:
        kb = ops.nblocks(Lk, self.block)
        nf = ops.forced_count(Lq, Lk, self.block, self.sink_tokens)
        return ops.budget(kb, nf, topk=self.topk, density=self.density, rule=self.rule)


def init_router_weights(num_heads: int, head_dim: int = 128, proj_dim: int = 64, *, seed: int = 0,
                        device="cuda"):
    """W_q, W_k ~ N(0, 1/head_dim), [H, head_dim, proj_dim] fp32 (the benchmark's random init)."""
    g = torch.Generator(device="cpu").manual_seed(seed)
    std = 1.0 / math.sqrt(head_dim)
    wq = torch.randn((num_heads, head_dim, proj_dim), generator=g) * std
    wk = torch.randn((num_heads, head_dim, proj_dim), generator=g) * std
    return wq.to(device), wk.to(device)


class SparseAttention:
    """Router + block-sparse attention with the signature of the reference's ``attention``."""

    def __init__(self, wq: torch.Tensor, wk: torch.Tensor, config: RouterConfig = RouterConfig(),
                 workspace: ops.Workspace | None = None, validate: bool = False):
        self.wq = wq.float().contiguous()
        self.wk = wk.float().contiguous()
        self.config = config
        self.workspace = workspace if workspace is not None else ops.Workspace()
        self.validate = validate
        self.dense = False          # when True, every block is kept (the reference's context pass)
        self.last_ids = None
        self.calls = 0
        self._caches = {}           # k-cache storage address -> attached KVCache
        # KVCache -> [k_i8, ks, (history tag, Lk)] of the INT8-QK path, held weakly: a cache that is
        # gone takes its entry along, so a new cache at the same address starts from nothing
        self._i8 = weakref.WeakKeyDictionary()

    def attach(self, cache) -> None:
        """Let calls whose k is this ``KVCache``'s visible window reuse its history's pooled key
        projections (``KVCache.router_keys``): pooled once per commit, not once per call."""
        self._caches[cache.k.untyped_storage().data_ptr()] = cache

    def detach_all(self) -> None:
        self._caches.clear()

    def cache_of(self, k: torch.Tensor):
        """The attached cache whose current window is exactly ``k`` [Lk,H,D] (else None)."""
        cache = self._caches.get(k.untyped_storage().data_ptr()) if self._caches else None
        if cache is None:
            return None
        kw = cache.window()[0]
        return cache if (kw.data_ptr() == k.data_ptr() and kw.shape == k.shape) else None

    def route(self, q: torch.Tensor, k: torch.Tensor, cache=None) -> torch.Tensor:
        """Router ids for q against the window k. With ``cache`` (a ``KVCache`` whose window is k),
        the history's key projections come from the cache's key table when they are still valid
        for its rows, and the table is marked valid for this window's history afterwards."""
        Lq, Lk = q.shape[-3], k.shape[-3]
        c = self.config
        ring = cache.ring if cache is not None and cache.ring_mode else None
        if ring is not None:   # k is the ring cache's physical rows
            Lk = cache.window_rows()
        if cache is None:
            return ops.route(q, k, self.wq, self.wk, block=c.block, extra=c.extra(Lq, Lk), sink_tokens=c.sink_tokens,
                             workspace=self.workspace, validate=self.validate, fast=c.fast)
        keys = cache.router_keys(c.block, self.wq.shape[2])
        tag = cache.history_tag()
        ids = ops.route(q, k, self.wq, self.wk, block=c.block, extra=c.extra(Lq, Lk), sink_tokens=c.sink_tokens,
                        workspace=self.workspace, validate=self.validate, keys=keys, n_cached=keys.cached(tag),
                        fast=c.fast, ring=ring, Lk=Lk if ring is not None else None)
        keys.mark(tag, ops.history_blocks(Lq, Lk, c.block))
        return ids

    def int8_keys(self, q: torch.Tensor, k: torch.Tensor, cache=None):
        """int8 key pages and their scales for the window k (``ops.quant_k_pages``). With ``cache``
        (the ``KVCache`` whose window is k), pages wholly before the current chunk are quantised
        once per history tag and window length, as the reference's ``Quantized.history`` runs once
        per commit (migration/unified_router/opt23/pipeline.py); the current chunk's pages on every
        call."""
        ring = cache.ring if cache is not None and cache.ring_mode else None
        Lq, H = q.shape[0], k.shape[1]
        Lk = cache.window_rows() if ring is not None else k.shape[0]
        npg = ops.quant_pages(Lk)
        if cache is None:
            k_i8 = self.workspace.tensor("k_i8", tuple(k.shape), k.device, torch.int8)
            ks = self.workspace.tensor("k_i8_scales", (H, npg), k.device, torch.float32)
            return ops.quant_k_pages(k, k_i8=k_i8, ks=ks)
        key = (cache.history_tag(), Lk)
        ent = self._i8.get(cache)
        if ent is None or ent[0].shape != k.shape:
            ent = self._i8[cache] = [torch.empty(k.shape, dtype=torch.int8, device=k.device),
                                         torch.empty((H, npg), dtype=torch.float32, device=k.device), None]
        if ent[1].shape != (H, npg):
            ent[1] = torch.empty((H, npg), dtype=torch.float32, device=k.device)
            ent[2] = None
        p0 = (Lk - Lq) // ops.PAGE_TOKENS if ent[2] == key else 0
        ops.quant_k_pages(k, p0=p0, k_i8=ent[0], ks=ent[1], ring=ring, Lk=Lk if ring is not None else None)
        ent[2] = key
        return ent[0], ent[1]

    def _dense_ids(self, H: int, Lq: int, Lk: int, device) -> torch.Tensor:
        c = self.config
        qb, kb = ops.nblocks(Lq, c.block), ops.nblocks(Lk, c.block)
        ids = self.workspace.tensor("dense_ids", (H, qb, kb), device, torch.int32)
        ids.copy_(torch.arange(kb, device=device, dtype=torch.int32).expand(H, qb, kb))
        return ids

    def forward_one(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, out: torch.Tensor | None = None,
                    cache=None):
        """q [Lq,H,D], k/v [Lk,H,D] bf16 -> [Lq,H,D] bf16. ``cache``: the ``KVCache`` whose window
        k/v are (found among the attached caches when not given)."""
        Lq, H, _ = q.shape
        if cache is None:
            cache = self.cache_of(k)
        ring = cache.ring if cache is not None and cache.ring_mode else None
        Lk = cache.window_rows() if ring is not None else k.shape[0]
        if Lk < Lq:
            raise ValueError("the KV window must contain the current chunk (Lk >= Lq)")
        ids = self._dense_ids(H, Lq, Lk, q.device) if self.dense else self.route(q, k, cache)
        self.last_ids = ids
        self.calls += 1
        if self.config.int8:
            k_i8, ks = self.int8_keys(q, k, cache)
            return ops.sparse_attention_i8(q, k_i8, ks, v, ids, block=self.config.block, out=out,
                                           validate=self.validate, workspace=self.workspace, ring=ring,
                                           Lk=Lk if ring is not None else None)
        return ops.sparse_attention(q, k, v, ids, block=self.config.block, out=out, validate=self.validate, ring=ring,
                                    Lk=Lk if ring is not None else None)

    def __call__(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *args, **kwargs) -> torch.Tensor:
        if args or kwargs:
            raise ValueError("Unexpected attention options; audit upstream implementation")
        if q.dim() != 4 or k.dim() != 4 or v.dim() != 4:
            raise ValueError("expected q [B,Lq,H,D] and k, v [B,Lk,H,D]")
        q = q.to(torch.bfloat16).contiguous()
        k = k.to(torch.bfloat16).contiguous()
        v = v.to(torch.bfloat16).contiguous()
        out = torch.empty_like(q)
        for b in range(q.shape[0]):
            self.forward_one(q[b], k[b], v[b], out=out[b])
        return out


class SparsePlugin:
    """Context manager that routes ``<module>.attention`` through a ``SparseAttention``.

    ``target`` is a module object or its import path (default ``wan.modules.causal_model``).
    One plugin may be active per target; nested use raises, as in the reference adapter.
    """

    def __init__(self, sparse: SparseAttention, target="wan.modules.causal_model", attribute: str = "attention"):
        self.sparse = sparse
        self.target = target
        self.attribute = attribute
        self.module = None
        self.original = None

    def __enter__(self):
        module = importlib.import_module(self.target) if isinstance(self.target, str) else self.target
        current = getattr(module, self.attribute)
        if getattr(current, _PATCH_FLAG, False):
            raise RuntimeError("Nested/concurrent sparse plugins are unsupported")
        self.module, self.original = module, current
        sparse = self.sparse

        def wrapped(q, k, v, *args, **kwargs):
            return sparse(q, k, v, *args, **kwargs)

        setattr(wrapped, _PATCH_FLAG, True)
        wrapped.original = current
        setattr(module, self.attribute, wrapped)
        return self

    def __exit__(self, *exc):
        if self.module is not None:
            setattr(self.module, self.attribute, self.original)
        self.module = None
        return False
