"""Ring-buffer KV cache on the GPU: ss_cache_append_ring writes exactly the rows of the numpy
model (tests/ring_model.py) and keeps the oracle's shifted window; the router (exact and fast,
with a cached key table) and the attention read a ring cache with the same results, bit for bit,
as on the shifted window; the plugin streams through a ring cache as through a shifting one."""
import math

import numpy as np
import pytest
import torch

from helpers import router_weights
from ring_model import RingModel

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")


def _stream(cap, sink, chunk, H, chunks, steps=2, seed=0):
    """Yield (shift cache, ring cache, model, q, chunk index) after every write of a stream: a
    window of the whole cache, `sink` rows kept, chunks of `chunk` rows (frames of their gcd)."""
    from streaming_sparse_b200.cache import KVCache
    ftok = math.gcd(math.gcd(cap, sink), chunk)
    kw = dict(frame_tokens=ftok, local_attn_size=cap // ftok, sink_size=sink // ftok, device=DEV,
              track_positions=False)
    shift = KVCache(cap, H, 128, **kw)
    ring = KVCache(cap, H, 128, ring=True, **kw)
    model = RingModel(cap, H, sink)
    g = torch.Generator().manual_seed(seed)
    for c in range(chunks):
        for _ in range(steps):
            kn = torch.randn((chunk, H, 128), generator=g).bfloat16()
            vn = torch.randn((chunk, H, 128), generator=g).bfloat16()
            q = torch.randn((chunk, H, 128), generator=g).bfloat16().to(DEV)
            ge, le = ring.global_end, ring.local_end
            shift.append(kn.to(DEV), vn.to(DEV), c * chunk)
            ring.append(kn.to(DEV), vn.to(DEV), c * chunk)
            model.append(kn.float().numpy(), vn.float().numpy(), local_attn=True, global_end=ge, local_end=le,
                         current_start=c * chunk)
            yield shift, ring, model, q, c


@pytest.mark.parametrize("cap,sink,chunk", [(34320, 1560, 4680), (1000, 100, 150), (900, 40, 300)])
def test_ring_append_rows_and_window(cap, sink, chunk):
    for shift, ring, model, _, c in _stream(cap, sink, chunk, 2, 3 * cap // chunk + 1):
        assert ring.ring.head == model.head and ring.local_end == shift.local_end
        np.testing.assert_array_equal(ring.k[0].float().cpu().numpy(), model.k)
        np.testing.assert_array_equal(ring.v[0].float().cpu().numpy(), model.v)
        kl, vl = ring.window_logical()
        ks, vs = shift.window()
        assert torch.equal(kl, ks) and torch.equal(vl, vs)
    assert ring.ring.head != 0


@pytest.mark.parametrize("fast", [False, True])
def test_router_and_attention_on_ring_equal_shifted(fast):
    from streaming_sparse_b200 import ops
    from streaming_sparse_b200.plugin import RouterConfig
    cap, sink, chunk, H, block = 34320, 1560, 4680, 3, 128
    cfg = RouterConfig(block=block, density=0.1, rule="rest", sink_tokens=sink)
    wq, wk = (w.to(DEV) for w in router_weights(4, H))
    checked = 0
    for shift, ring, _, q, c in _stream(cap, sink, chunk, H, 12, steps=1):
        if c < 7:
            continue                                  # after the window has rolled a few times
        Lk = ring.window_rows()
        extra = cfg.extra(chunk, Lk)
        ks, vs = shift.window()
        kp, vp = ring.window()
        want = ops.route(q, ks, wq, wk, block=block, extra=extra, sink_tokens=sink, return_mask=True)
        got = ops.route(q, kp, wq, wk, block=block, extra=extra, sink_tokens=sink, return_mask=True, fast=fast,
                        ring=ring.ring, Lk=Lk)
        assert torch.equal(got[0], want[0]) and torch.equal(got[1], want[1])
        # the cached key table pooled from the ring at commit, then the chunk's call
        keys = ops.RouterKeys(H, cap, block=block, device=DEV)
        nh = ops.history_blocks(chunk, Lk, block)
        ops.pool_keys(kp, wk, keys, j0=0, j1=nh, ring=ring.ring, Lk=Lk)
        got2 = ops.route(q, kp, wq, wk, block=block, extra=extra, sink_tokens=sink, keys=keys, n_cached=nh, fast=fast,
                         ring=ring.ring, Lk=Lk)
        assert torch.equal(got2, want[0])
        o_want, l_want = ops.sparse_attention(q, ks, vs, want[0], block=block, return_lse=True)
        o_got, l_got = ops.sparse_attention(q, kp, vp, want[0], block=block, return_lse=True, ring=ring.ring, Lk=Lk)
        assert torch.equal(o_got, o_want) and torch.equal(l_got, l_want)
        checked += 1
    assert checked >= 3


def test_plugin_streams_through_ring_cache():
    from streaming_sparse_b200.cache import KVCache
    from streaming_sparse_b200.plugin import RouterConfig, SparseAttention
    H, ftok, local, sink = 2, 300, 5, 1
    cfg = RouterConfig(block=64, density=0.3, rule="rest", sink_tokens=sink * ftok, fast=True)
    wq, wk = (w.to(DEV) for w in router_weights(6, H))
    caches = [KVCache(local * ftok, H, 128, frame_tokens=ftok, local_attn_size=local, sink_size=sink, device=DEV,
                      ring=r) for r in (False, True)]
    sps = [SparseAttention(wq, wk, cfg) for _ in caches]
    for sp, cache in zip(sps, caches):
        sp.attach(cache)
    g = torch.Generator().manual_seed(1)
    n = 2 * ftok
    for c in range(8):
        for _ in range(2):
            kn = torch.randn((n, H, 128), generator=g).bfloat16().to(DEV)
            vn = torch.randn((n, H, 128), generator=g).bfloat16().to(DEV)
            q = torch.randn((n, H, 128), generator=g).bfloat16().to(DEV)
            outs = []
            for sp, cache in zip(sps, caches):
                cache.append(kn, vn, c * n)
                kw, vw = cache.window()
                outs.append(sp(q[None], kw[None], vw[None]))
            assert torch.equal(outs[0], outs[1])
            assert torch.equal(sps[0].last_ids, sps[1].last_ids)
    assert caches[1].ring.head != 0
