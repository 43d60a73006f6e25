"""The router with the history's key projections pooled once per commit (ss_router_pool_keys +
ss_router_cached, the refresh_history / current split of migration/unified_router/opt23/
pipeline.py:22-34) gives the uncached router's ids, masks and scores bit for bit."""
import numpy as np
import pytest
import torch

from helpers import np32, qkv, router_weights

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")


def _cpu(*ts):
    return tuple(t.cpu().numpy() for t in ts)


@pytest.mark.parametrize("Lq,Lk,H,block,sink,extra", [
    (4680, 32760, 12, 64, 0, 54),        # config 2: history blocks 0..437, block 438 straddles the chunk
    (4680, 34320, 4, 128, 1560, 21),     # config 4 shape
    (100, 333, 2, 64, 0, 2),             # ragged
    (64, 64, 1, 64, 0, 0),               # no history at all
])
def test_pool_keys_then_cached_route_is_bit_exact(oracle, Lq, Lk, H, block, sink, extra):
    from streaming_sparse_b200 import ops
    q, k, _ = qkv(21, Lq, Lk, H)
    wq, wk = router_weights(21, H)
    q, k, wq, wk = (t.to(DEV) for t in (q, k, wq, wk))
    keys = ops.RouterKeys(H, Lk, block=block, device=DEV)
    n_hist = ops.history_blocks(Lq, Lk, block)
    ops.pool_keys(k, wk, keys, j0=0, j1=n_hist)                      # at commit
    want = ops.route(q, k, wq, wk, block=block, extra=extra, sink_tokens=sink, return_mask=True,
                     return_scores=True, validate=True)
    for step in range(3):                                            # the chunk's denoising calls
        got = ops.route(q, k, wq, wk, block=block, extra=extra, sink_tokens=sink, return_mask=True,
                        return_scores=True, validate=True, keys=keys, n_cached=n_hist)
        torch.cuda.synchronize()
        g, w = _cpu(*got), _cpu(*want)
        np.testing.assert_array_equal(g[0], w[0])
        np.testing.assert_array_equal(g[1], w[1])
        np.testing.assert_array_equal(g[2].view(np.uint32), w[2].view(np.uint32))
        # the next call rewrites the current chunk (new keys and queries); the history stays
        q = torch.randn_like(q.float()).bfloat16()
        k[Lk - Lq:] = torch.randn_like(k[Lk - Lq:].float()).bfloat16()
        want = ops.route(q, k, wq, wk, block=block, extra=extra, sink_tokens=sink, return_mask=True,
                         return_scores=True, validate=True)
    # and the cached path equals the CPU oracle too
    r = oracle.route(np32(q), np32(k), wq.cpu().numpy(), wk.cpu().numpy(), block, extra, sink_tokens=sink)
    got = ops.route(q, k, wq, wk, block=block, extra=extra, sink_tokens=sink, keys=keys, n_cached=n_hist)
    np.testing.assert_array_equal(got.cpu().numpy(), r["ids"])


@pytest.mark.parametrize("local,sink,block,chunks", [(-1, 0, 64, 4), (5, 1, 128, 7), (4, 0, 64, 6)])
def test_streaming_cache_reuses_history_keys(local, sink, block, chunks):
    """A stream through a KVCache (three routed calls per chunk, each rewriting the chunk's rows):
    every call's ids equal the uncached router's; calls after a chunk's first reuse the history's
    projections, and a roll of the window (or an anchor rebase) makes the next call pool afresh."""
    from streaming_sparse_b200 import ops
    from streaming_sparse_b200.cache import KVCache
    from streaming_sparse_b200.plugin import RouterConfig, SparseAttention
    H, ftok, fpc = 2, 300, 2                   # 600-token chunks: neither block size divides them
    cap = (local if local != -1 else fpc * chunks) * ftok
    cache = KVCache(cap, num_heads=H, frame_tokens=ftok, local_attn_size=local, sink_size=sink, device=DEV)
    wq, wk = router_weights(9, H)
    cfg = RouterConfig(block=block, density=0.3, rule="rest" if sink else "total", sink_tokens=sink * ftok)
    sp = SparseAttention(wq.to(DEV), wk.to(DEV), cfg)
    ref = SparseAttention(wq.to(DEV), wk.to(DEV), cfg)      # never attached: pools everything per call
    sp.attach(cache)
    g = torch.Generator().manual_seed(3)
    n = fpc * ftok
    reused = 0
    for c in range(chunks):
        for step in range(3):
            kn = torch.randn((n, H, 128), generator=g).bfloat16().to(DEV)
            vn = torch.randn((n, H, 128), generator=g).bfloat16().to(DEV)
            q = torch.randn((n, H, 128), generator=g).bfloat16().to(DEV)
            cache.append(kn, vn, c * n)
            if c == 2 and step == 1 and sink:
                cache.save_anchor()
                cache.rebase_anchor(1)                       # sink rows rewritten: keys stale
            kw, vw = cache.window()
            keys = cache.router_keys(block)
            before = keys.cached(cache.history_tag())
            got = sp.forward_one(q, kw, vw)
            ids_got = sp.last_ids.clone()
            ref.forward_one(q, kw, vw)
            torch.cuda.synchronize()
            np.testing.assert_array_equal(ids_got.cpu().numpy(), ref.last_ids.cpu().numpy())
            if step > 0 and not (c == 2 and step == 1 and sink):
                assert before == ops.history_blocks(n, kw.shape[0], block)
                reused += before > 0
            if c == 2 and step == 1 and sink:
                assert before == 0
    assert reused > 0
    ops.DeviceStatus.check(DEV)
