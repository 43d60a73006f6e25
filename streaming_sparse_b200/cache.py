"""Streaming KV cache: append/evict on the GPU plus host-side index and position bookkeeping.

``KVCache`` holds one layer's K/V in the reference's layout (``{"k","v": [1,cap,H,128] bf16,
"global_end_index", "local_end_index"}``, pipeline/causal_inference.py:278-298) and applies a
chunk write with the rolling-window semantics of CausalWanSelfAttention.forward
(wan/modules/causal_model.py:216-253) through ``ss_cache_append``. The index state is mirrored
on the host, so no device->host read is needed per call (the reference calls ``.item()``).

Snapshots: ``snapshot``/``restore`` copy a layer's whole state (K/V rows and the index state) on
the device, so a stream can be forked or rewound. ``save_anchor``/``rebase_anchor`` keep a
canonical copy of the anchor (sink) frame's keys and rewrite the cache's anchor rows with their
temporal RoPE pairs rotated to a new frame position -- the reference's long-horizon "anchor
rebase" (``set_phase``, reproduction/vbench_current/phase.py:4-9, with ``shift_temporal_``,
local_experiments/anchor_rebase.py:8-18), through ``ss_cache_rope_shift``.

``PositionTracker`` restates the adapter's absolute-position bookkeeping
(streaming_sparse/integration/self_forcing_adapter.py:50-97): the absolute token index held in
every cache slot through roll/evict, and the positions of the visible window.
"""
from __future__ import annotations

import numpy as np
import torch

from .ops import Ring, cache_append, cache_append_ring, ring_refresh, rope_shift


def temporal_phase(offset: int, device, head_dim: int = 128) -> torch.Tensor:
    """(cos, sin) of offset * theta_p for the temporal RoPE pairs, float64 [P, 2] on `device`:
    row `offset` of the model's RoPE table (wan/modules/model.py:29-37, temporal part of the
    split in causal_model.py:500-505), built with torch.polar as the reference builds it."""
    n = head_dim - 4 * (head_dim // 6)
    theta = 1.0 / torch.pow(10000, torch.arange(0, n, 2, dtype=torch.float64).div(n))
    ang = float(offset) * theta
    z = torch.polar(torch.ones_like(ang), ang)
    return torch.view_as_real(z).contiguous().to(device)


class PositionTracker:
    """Absolute token position of every cache slot (-1 = empty)."""

    def __init__(self, size: int):
        self.flat = np.full(size, -1, dtype=np.int64)

    def update(self, *, start: int, n: int, old_global: int, old_local: int, local_attn: bool, sink_tokens: int,
               max_attention_size: int):
        """Apply one chunk write; return (visible positions, history token count)."""
        size = len(self.flat)
        end = start + n
        flat = self.flat
        evicted = 0
        if local_attn and end > old_global and n + old_local > size:
            evicted = n + old_local - size
            rolled = old_local - evicted - sink_tokens
            if rolled < 0:
                raise ValueError(f"a {n}-token chunk and a {sink_tokens}-token sink do not fit a {size}-slot cache")
            flat[sink_tokens:sink_tokens + rolled] = flat[sink_tokens + evicted:sink_tokens + evicted + rolled].copy()
        local_end = old_local + end - old_global - evicted
        local_start = local_end - n
        if local_start < 0 or local_end > size:
            raise ValueError(f"chunk rows [{local_start}, {local_end}) fall outside the {size}-slot cache")
        flat[local_start:local_end] = np.arange(start, end)
        visible_start = max(0, local_end - max_attention_size)
        if visible_start > local_start:
            raise ValueError(f"the {max_attention_size}-token visible window is shorter than the {n}-token chunk")
        visible = flat[visible_start:local_end].copy()
        if (visible < 0).any():
            raise ValueError("the visible window reaches cache slots that were never written")
        return visible, local_start - visible_start


class KVCache:
    """One layer's streaming K/V cache on the GPU.

    ``local_attn_size`` / ``sink_size`` are in frames as in CausalWanSelfAttention; a value of -1
    for ``local_attn_size`` means a global cache (no eviction, window of 32760 tokens).

    ``ring``: keep the rows after the sink in a ring buffer (``ops.Ring``): a roll then moves the
    ring's head instead of shifting the window's rows, and a write costs only the chunk's rows.
    ``k``/``v`` are then the physical rows [1, S + C + 64, H, D] (C = capacity - S + 64) and
    ``window()`` returns them with ``ring`` and ``window_rows()`` describing the window; the
    attention and router calls take them as they are (``ops.sparse_attention/route(..., ring=,
    Lk=)``), ``window_logical()`` gathers the window in order. The window must cover the whole
    cache. The index state, window contents and block grid are those of the shifting cache.
    """

    def __init__(self, capacity: int, num_heads: int = 12, head_dim: int = 128, *, frame_tokens: int = 1560,
                 local_attn_size: int = -1, sink_size: int = 0, device="cuda", dtype=torch.bfloat16,
                 track_positions: bool = True, ring: bool = False):
        self.capacity, self.H, self.D = capacity, num_heads, head_dim
        # first model head this cache holds (head-parallel models: a rank's caches hold the heads
        # head0 .. head0 + H - 1 of the model's)
        self.head0 = 0
        self.frame_tokens = frame_tokens
        self.local_attn_size, self.sink_size = local_attn_size, sink_size
        self.max_attention_size = 32760 if local_attn_size == -1 else local_attn_size * frame_tokens
        self.ring_mode = bool(ring)
        self.ring = None
        rows = capacity
        if self.ring_mode:
            if self.max_attention_size < capacity:
                raise ValueError("a ring cache needs a visible window that covers the whole cache")
            S = self.sink_tokens
            if S >= capacity:
                raise ValueError("the sink must leave room for the ring")
            # the head on the host (host checks, the window's order) and in device memory (what the
            # kernels follow, so that captured CUDA graphs see later rolls)
            self._ring_head_dev = torch.zeros(1, dtype=torch.int32, device=device)
            self.ring = Ring(S, capacity - S + 64, 0, self._ring_head_dev)
            rows = self.ring.phys_rows()
        self.k = torch.zeros((1, rows, num_heads, head_dim), device=device, dtype=dtype)
        self.v = torch.zeros_like(self.k)
        self.global_end = 0
        self.local_end = 0
        self.positions = PositionTracker(capacity) if track_positions else None
        self.commits = 0
        self.anchor = None
        # Bumped whenever rows that stay in the window change place or content outside the
        # current chunk (a roll, a restore, an anchor rebase): a router key table pooled from
        # the old rows is then stale.
        self.epoch = 0
        self._router_keys = None

    @property
    def sink_tokens(self) -> int:
        return self.sink_size * self.frame_tokens

    def as_reference_dict(self):
        """The reference's cache dict view (shares storage)."""
        dev = self.k.device
        return {"k": self.k, "v": self.v, "global_end_index": torch.tensor([self.global_end], device=dev),
                "local_end_index": torch.tensor([self.local_end], device=dev)}

    def _rolls(self, n: int, current_start: int) -> bool:
        end = current_start + n
        return self.local_attn_size != -1 and end > self.global_end and n + self.local_end > self.capacity

    def write_plan(self, n: int, current_start: int) -> tuple[bool, int, int]:
        """(rolls, evicted tokens, local end after) of writing n tokens at current_start."""
        end = current_start + n
        rolls = self._rolls(n, current_start)
        evicted = n + self.local_end - self.capacity if rolls else 0
        return rolls, evicted, self.local_end + end - self.global_end - evicted

    def advance(self, n: int, current_start: int):
        """Host-side index update of one chunk write (what ``append`` does besides the copy);
        for a caller whose write already happened on the device (a replayed CUDA graph).
        Returns (visible positions, history) when positions are tracked."""
        vis = None
        if self.positions is not None:
            vis = self.positions.update(start=current_start, n=n, old_global=self.global_end, old_local=self.local_end,
                                        local_attn=self.local_attn_size != -1, sink_tokens=self.sink_tokens,
                                        max_attention_size=self.max_attention_size)
        end = current_start + n
        rolls, evicted, local_end = self.write_plan(n, current_start)
        if local_end - n < 0 or local_end > self.capacity:
            raise ValueError(f"chunk rows [{local_end - n}, {local_end}) fall outside the {self.capacity}-slot cache")
        self.local_end, self.global_end = local_end, end
        self.commits += 1
        if rolls:
            self.epoch += 1
            if self.ring_mode:   # the device head moves in the append's own kernels
                self.ring = self.ring.with_head((self.ring.head + evicted) % self.ring.cap)
        return vis

    def window_start(self, local_end: int | None = None) -> int:
        """First cache row of the visible window (for the given local end, default the current)."""
        end = self.local_end if local_end is None else local_end
        return max(0, end - self.max_attention_size)

    def history_tag(self):
        """Names the rows of the current window for a router key table (``ops.RouterKeys``): two
        calls with the same tag see the same history rows at the same block alignment."""
        return (id(self), self.epoch, self.window_start())

    def tag_after(self, n: int, current_start: int):
        """``history_tag`` as it will be once a write of n tokens at current_start is applied."""
        rolls, _, local_end = self.write_plan(n, current_start)
        return (id(self), self.epoch + (1 if rolls else 0), self.window_start(local_end))

    def router_keys(self, block: int = 64, R: int = 64):
        """This layer's router key table (created on first use, sized for the whole cache)."""
        from .ops import RouterKeys
        rk = self._router_keys
        if rk is None or rk.block != block or rk.R != R:
            rk = self._router_keys = RouterKeys(self.H, self.capacity, block=block, R=R, device=self.k.device)
        return rk

    def append(self, k_new: torch.Tensor, v_new: torch.Tensor, current_start: int):
        """Write a chunk (post-RoPE K, V: [n,H,D] or [1,n,H,D]); returns (visible positions, history)."""
        n = k_new.shape[-3]
        old_global, old_local, old_ring = self.global_end, self.local_end, self.ring
        vis = self.advance(n, current_start)
        if self.ring_mode:
            new_end, head = cache_append_ring(self.k, self.v, k_new, v_new, cap=self.capacity,
                                              local_attn=self.local_attn_size != -1, global_end=old_global,
                                              local_end=old_local, current_start=current_start,
                                              sink_tokens=self.sink_tokens, ring=old_ring)
            assert head == self.ring.head
        else:
            new_end = cache_append(self.k, self.v, k_new, v_new, local_attn=self.local_attn_size != -1,
                                   global_end=old_global, local_end=old_local, current_start=current_start,
                                   sink_tokens=self.sink_tokens)
        assert new_end == self.local_end
        return vis

    def write_qkv(self, qkv, norm_q, norm_k, eps: float, cos, sin, q_out, current_start: int,
                  model_heads: int | None = None):
        """A ring cache's counterpart of ``reserve`` + the fused projection: q/k RMSNorm + RoPE from
        ``qkv`` with k and v written straight into the ring rows of this write, placed by the
        device head (so a captured CUDA graph stays right after later rolls), then the sink's copy
        and the head updated when the write rolled; advances the index state like ``append``.
        ``model_heads``: qkv holds that many heads, of which this cache stores head0 .. head0 + H - 1."""
        from .ops import qkv_norm_rope_ring, ring_commit
        if not self.ring_mode:
            raise RuntimeError("write_qkv is for ring caches; use reserve() on a shifting cache")
        n = q_out.shape[0]
        rolls, evicted, local_end = self.write_plan(n, current_start)
        start = local_end - n
        old_ring = self.ring
        self.advance(n, current_start)
        ev = evicted if rolls else 0
        qkv_norm_rope_ring(qkv, norm_q, norm_k, eps, cos, sin, q_out, self.k, self.v, ring=old_ring, t0=start,
                           evicted=ev, model_heads=model_heads, h0=self.head0)
        ring_commit(self.k, self.v, old_ring, evicted=ev, refresh=start < self.sink_tokens)

    def reserve(self, n: int, current_start: int):
        """Claim the rows a chunk of n tokens occupies, for a producer that writes them itself.

        Returns (k rows, v rows) as [n,H,D] views of the cache and advances the index state as
        ``append`` would, when the write needs no roll of the window; returns None (state
        unchanged) when it does, in which case the caller writes through ``append``.
        """
        if self.ring_mode or self._rolls(n, current_start):
            return None
        self.advance(n, current_start)
        return self.k[0, self.local_end - n:self.local_end], self.v[0, self.local_end - n:self.local_end]

    def snapshot(self) -> dict:
        """Device copy of the K/V rows in use and the index state (see ``restore``)."""
        n = self.k.shape[1] if self.ring_mode else self.local_end
        return {"k": self.k[0, :n].clone(), "v": self.v[0, :n].clone(), "global_end": self.global_end,
                "local_end": self.local_end, "commits": self.commits,
                "ring": self.ring.head if self.ring_mode else None,
                "positions": None if self.positions is None else self.positions.flat.copy()}

    def restore(self, snap: dict) -> None:
        """Put back a ``snapshot`` of this cache (same capacity and heads)."""
        le = snap["local_end"]
        n = self.k.shape[1] if self.ring_mode else le
        if not (0 <= le <= self.capacity and tuple(snap["k"].shape) == (n, self.H, self.D) and
                snap["v"].shape == snap["k"].shape and (snap.get("ring") is None) != self.ring_mode):
            raise ValueError("snapshot does not match this cache's geometry")
        self.k[0, :n].copy_(snap["k"])
        self.v[0, :n].copy_(snap["v"])
        if self.ring_mode:
            self.ring = self.ring.with_head(snap["ring"])
            self._ring_head_dev.fill_(snap["ring"])
        self.global_end, self.local_end, self.commits = snap["global_end"], le, snap["commits"]
        self.epoch += 1
        if self.positions is not None and snap["positions"] is not None:
            self.positions.flat[:] = snap["positions"]

    def save_anchor(self, tokens: int | None = None) -> None:
        """Keep the canonical (unshifted) keys of the first `tokens` rows (default: the sink
        frames, else one frame)."""
        t = tokens if tokens is not None else (self.sink_tokens or self.frame_tokens)
        if t <= 0 or t > self.local_end:
            raise ValueError("the anchor rows must be written before they are saved")
        if self.ring_mode and t > self.sink_tokens:
            raise ValueError("a ring cache keeps only its sink rows in place: the anchor must lie in the sink")
        self.anchor = self.k[0, :t].clone()

    def rebase_anchor(self, offset: int) -> None:
        """Rewrite the anchor rows from the saved canonical keys with their temporal RoPE pairs
        rotated by `offset` frames (offset 0 restores them as saved)."""
        if getattr(self, "anchor", None) is None:
            raise RuntimeError("save_anchor() first")
        t = self.anchor.shape[0]
        rope_shift(self.anchor, self.k[0, :t], temporal_phase(offset, self.k.device, self.D))
        if self.ring_mode:
            ring_refresh(self.k, self.v, self.ring)   # the sink's copy before the ring's head
        self.epoch += 1

    def reset(self) -> None:
        """Empty the cache (index state only; rows are overwritten by the next writes)."""
        self.global_end = self.local_end = 0
        if self.ring_mode:
            self.ring = self.ring.with_head(0)
            self._ring_head_dev.zero_()
        self.epoch += 1
        if self.positions is not None:
            self.positions.flat[:] = -1

    def window(self):
        """Visible K/V window [Lk,H,D] (views into the cache): the last tokens are the current chunk.
        A ring cache returns its physical rows (see ``ring``, ``window_rows``)."""
        if self.ring_mode:
            return self.k[0], self.v[0]
        a = max(0, self.local_end - self.max_attention_size)
        return self.k[0, a:self.local_end], self.v[0, a:self.local_end]

    def window_rows(self) -> int:
        """Rows of the visible window."""
        return self.local_end - self.window_start()

    def physical_rows(self, n: int | None = None) -> torch.Tensor:
        """Physical cache row of each of the window's first n rows (default: all), int64 on the device."""
        n = self.window_rows() if n is None else n
        t = torch.arange(n, device=self.k.device)
        if not self.ring_mode:
            return t + self.window_start()
        S, C, head = self.ring
        return torch.where(t < S, t, S + torch.remainder(t - S + head, C))

    def window_logical(self):
        """The visible window gathered in order (a copy; a plain cache returns its views)."""
        if not self.ring_mode:
            return self.window()
        rows = self.physical_rows()
        return self.k[0].index_select(0, rows), self.v[0].index_select(0, rows)
