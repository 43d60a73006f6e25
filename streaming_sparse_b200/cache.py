"""Streaming KV cache: append/evict on the GPU plus host-side index and position bookkeeping.

``KVCache`` holds one layer's K/V in the reference's layout (``{"k","v": [1,cap,H,128] bf16,
"global_end_index", "local_end_index"}``, pipeline/causal_inference.py:278-298) and applies a
chunk write with the rolling-window semantics of CausalWanSelfAttention.forward
(wan/modules/causal_model.py:216-253) through ``ss_cache_append``. The index state is mirrored
on the host, so no device->host read is needed per call (the reference calls ``.item()``).

``PositionTracker`` restates the adapter's absolute-position bookkeeping
(streaming_sparse/integration/self_forcing_adapter.py:50-97): the absolute token index held in
every cache slot through roll/evict, and the positions of the visible window.
"""
from __future__ import annotations

import numpy as np
import torch

from .ops import cache_append


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
                raise ValueError("Cache too small for sink and current chunk")
            flat[sink_tokens:sink_tokens + rolled] = flat[sink_tokens + evicted:sink_tokens + evicted + rolled].copy()
        local_end = old_local + end - old_global - evicted
        local_start = local_end - n
        if local_start < 0 or local_end > size:
            raise ValueError("Invalid KV cache bounds; reduce length or use local attention")
        flat[local_start:local_end] = np.arange(start, end)
        visible_start = max(0, local_end - max_attention_size)
        if visible_start > local_start:
            raise ValueError("Attention window must contain the entire current chunk")
        visible = flat[visible_start:local_end].copy()
        if (visible < 0).any():
            raise ValueError("Uninitialized visible cache positions")
        return visible, local_start - visible_start


class KVCache:
    """One layer's streaming K/V cache on the GPU.

    ``local_attn_size`` / ``sink_size`` are in frames as in CausalWanSelfAttention; a value of -1
    for ``local_attn_size`` means a global cache (no eviction, window of 32760 tokens).
    """

    def __init__(self, capacity: int, num_heads: int = 12, head_dim: int = 128, *, frame_tokens: int = 1560,
                 local_attn_size: int = -1, sink_size: int = 0, device="cuda", dtype=torch.bfloat16,
                 track_positions: bool = True):
        self.capacity, self.H, self.D = capacity, num_heads, head_dim
        self.frame_tokens = frame_tokens
        self.local_attn_size, self.sink_size = local_attn_size, sink_size
        self.max_attention_size = 32760 if local_attn_size == -1 else local_attn_size * frame_tokens
        self.k = torch.zeros((1, capacity, num_heads, head_dim), device=device, dtype=dtype)
        self.v = torch.zeros_like(self.k)
        self.global_end = 0
        self.local_end = 0
        self.positions = PositionTracker(capacity) if track_positions else None
        self.commits = 0

    @property
    def sink_tokens(self) -> int:
        return self.sink_size * self.frame_tokens

    def as_reference_dict(self):
        """The reference's cache dict view (shares storage)."""
        dev = self.k.device
        return {"k": self.k, "v": self.v, "global_end_index": torch.tensor([self.global_end], device=dev),
                "local_end_index": torch.tensor([self.local_end], device=dev)}

    def append(self, k_new: torch.Tensor, v_new: torch.Tensor, current_start: int):
        """Write a chunk (post-RoPE K, V: [n,H,D] or [1,n,H,D]); returns (visible positions, history)."""
        n = k_new.shape[-3]
        local_attn = self.local_attn_size != -1
        vis = None
        if self.positions is not None:
            vis = self.positions.update(start=current_start, n=n, old_global=self.global_end, old_local=self.local_end,
                                        local_attn=local_attn, sink_tokens=self.sink_tokens,
                                        max_attention_size=self.max_attention_size)
        new_end = cache_append(self.k, self.v, k_new, v_new, local_attn=local_attn, global_end=self.global_end,
                               local_end=self.local_end, current_start=current_start, sink_tokens=self.sink_tokens)
        self.local_end = new_end
        self.global_end = current_start + n
        self.commits += 1
        return vis

    def reserve(self, n: int, current_start: int):
        """Claim the rows a chunk of n tokens occupies, for a producer that writes them itself.

        Returns (k rows, v rows) as [n,H,D] views of the cache and advances the index state as
        ``append`` would, when the write needs no roll of the window; returns None (state
        unchanged) when it does, in which case the caller writes through ``append``.
        """
        end = current_start + n
        if self.local_attn_size != -1 and end > self.global_end and n + self.local_end > self.capacity:
            return None
        if self.positions is not None:
            self.positions.update(start=current_start, n=n, old_global=self.global_end, old_local=self.local_end,
                                  local_attn=self.local_attn_size != -1, sink_tokens=self.sink_tokens,
                                  max_attention_size=self.max_attention_size)
        local_end = self.local_end + end - self.global_end
        start = local_end - n
        if start < 0 or local_end > self.capacity:
            raise ValueError("Invalid KV cache bounds; reduce length or use local attention")
        self.local_end, self.global_end = local_end, end
        self.commits += 1
        return self.k[0, start:local_end], self.v[0, start:local_end]

    def window(self):
        """Visible K/V window [Lk,H,D] (views into the cache): the last tokens are the current chunk."""
        a = max(0, self.local_end - self.max_attention_size)
        return self.k[0, a:self.local_end], self.v[0, a:self.local_end]
