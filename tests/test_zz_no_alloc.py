"""ss_router_noalloc: the router for callers that cannot allocate device memory.

Such callers -- a host whose device memory is handed out by its own fixed pool, or a host binding
the library from a language without a device allocator -- cannot supply the workspace ss_router
takes. This entry point keeps the router's intermediates in a static device array instead. The
test calls it through the C ABI twice in a row (the array keeps the first call's contents when
the second runs) and checks each result against ss_router with a caller workspace: the router is
exact, so ids, masks and scores must be identical. It also checks that a problem larger than the
array is refused on the host. This file is collected last so a failure here comes after every
other test has run; it also passes on its own in a fresh process.
"""
import ctypes
import math

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _inputs(seed, Lq, Lk, H, dev):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn((Lq, H, 128), generator=g).bfloat16().to(dev)
    k = torch.randn((Lk, H, 128), generator=g).bfloat16().to(dev)
    wq = (torch.randn((H, 128, 64), generator=g) / math.sqrt(128)).to(dev)
    wk = (torch.randn((H, 128, 64), generator=g) / math.sqrt(128)).to(dev)
    return q, k, wq, wk


def _p(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _call(lib, noalloc, q, k, wq, wk, block, sink, extra, n_ids, workspace, status, dev):
    Lq, H, _ = q.shape
    Lk = k.shape[0]
    qb, kb = -(-Lq // block), -(-Lk // block)
    ids = torch.full((H, qb, n_ids), -7, dtype=torch.int32, device=dev)
    mask = torch.zeros((H, qb, kb), dtype=torch.uint8, device=dev)
    scores = torch.zeros((H, qb, kb), dtype=torch.float32, device=dev)
    stream = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
    if noalloc:
        rc = lib.ss_router_noalloc(_p(q), _p(k), _p(wq), _p(wk), H, Lq, Lk, 64, block, sink, extra, _p(ids), n_ids,
                                   _p(mask), _p(scores), _p(status), stream)
    else:
        rc = lib.ss_router(_p(q), _p(k), _p(wq), _p(wk), H, Lq, Lk, 64, block, sink, extra, _p(ids), n_ids, _p(mask),
                           _p(scores), _p(workspace), workspace.numel(), _p(status), stream)
    assert rc == 0, rc
    torch.cuda.synchronize(dev)
    return ids.cpu().numpy(), mask.cpu().numpy(), scores.cpu().numpy()


def test_router_noalloc_matches_router_twice():
    from streaming_sparse_b200 import build, ops
    build.build()
    from streaming_sparse_b200._lib import lib as load
    lib = load()
    dev = torch.device("cuda:0")
    torch.cuda.set_device(dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    # two different problems back to back: config 2, then a sink/128-token-block case
    cases = [(4680, 32760, 12, 64, 0, 54, 0), (1000, 5000, 4, 128, 300, 9, 1)]
    for Lq, Lk, H, block, sink, extra, seed in cases:
        q, k, wq, wk = _inputs(seed, Lq, Lk, H, dev)
        n_ids = ops.forced_count(Lq, Lk, block, sink) + extra
        ws = torch.empty(ops.router_workspace_bytes(H, Lq, Lk, 64, block), dtype=torch.uint8, device=dev)
        ref = _call(lib, False, q, k, wq, wk, block, sink, extra, n_ids, ws, status, dev)
        got = _call(lib, True, q, k, wq, wk, block, sink, extra, n_ids, None, status, dev)
        np.testing.assert_array_equal(got[0], ref[0])
        np.testing.assert_array_equal(got[1], ref[1])
        np.testing.assert_array_equal(got[2].view(np.uint32), ref[2].view(np.uint32))
        assert (got[0] >= 0).all() and (np.diff(got[0], axis=-1) > 0).all()
    assert int(status.item()) == 0


def test_router_noalloc_refuses_oversized_problem():
    from streaming_sparse_b200 import build, ops
    build.build()
    from streaming_sparse_b200._lib import lib as load
    lib = load()
    H, Lq, Lk, block = 64, 4680, 32760, 64               # 64 heads: ~9.6 MB of intermediates
    assert ops.router_workspace_bytes(H, Lq, Lk, 64, block) > (8 << 20)
    fake = ctypes.c_void_p(0x100000)                     # never dereferenced: refused on the host
    n_ids = ops.forced_count(Lq, Lk, block) + 1
    rc = lib.ss_router_noalloc(fake, fake, fake, fake, H, Lq, Lk, 64, block, 0, 1, fake, n_ids, None, None, None,
                               None)
    assert rc == 1003  # SS_ERR_WORKSPACE


def test_router_noalloc_near_the_array_limit():
    """A problem whose intermediates fill ~98 % of the static array (98 280-token window, 20
    heads, 64-token blocks) gives ss_router's results bit for bit; one more head no longer fits
    and is refused on the host before anything is launched."""
    from streaming_sparse_b200 import build, ops
    build.build()
    from streaming_sparse_b200._lib import lib as load
    lib = load()
    dev = torch.device("cuda:0")
    torch.cuda.set_device(dev)
    Lq, Lk, block, extra = 4680, 98280, 64, 3
    limit = 8 << 20
    assert 0.95 * limit < ops.router_workspace_bytes(20, Lq, Lk, 64, block) <= limit
    assert ops.router_workspace_bytes(21, Lq, Lk, 64, block) > limit
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    q, k, wq, wk = _inputs(5, Lq, Lk, 20, dev)
    n_ids = ops.forced_count(Lq, Lk, block) + extra
    ws = torch.empty(ops.router_workspace_bytes(20, Lq, Lk, 64, block), dtype=torch.uint8, device=dev)
    ref = _call(lib, False, q, k, wq, wk, block, 0, extra, n_ids, ws, status, dev)
    got = _call(lib, True, q, k, wq, wk, block, 0, extra, n_ids, None, status, dev)
    np.testing.assert_array_equal(got[0], ref[0])
    np.testing.assert_array_equal(got[1], ref[1])
    np.testing.assert_array_equal(got[2].view(np.uint32), ref[2].view(np.uint32))
    assert int(status.item()) == 0
    del q, k, ws
    fake = ctypes.c_void_p(0x100000)                     # never dereferenced: refused on the host
    rc = lib.ss_router_noalloc(fake, fake, fake, fake, 21, Lq, Lk, 64, block, 0, extra, fake, n_ids, None, None,
                               None, None)
    assert rc == 1003  # SS_ERR_WORKSPACE
