"""Router on the GPU == the exact-fp32 CPU oracle, bit for bit (scores, ids, masks)."""
import numpy as np
import pytest
import torch

from helpers import np32, qkv, router_weights

pytestmark = pytest.mark.gpu

CASES = [
    # Lq, Lk, H, block, sink, extra
    (1560, 6240, 12, 64, 0, 24),        # config 1
    (4680, 32760, 12, 64, 0, 54),       # config 2 (25% of 512 blocks in total)
    (4680, 34320, 4, 128, 1560, 21),    # config 4 shape: sink frame, 128-token blocks
    (100, 333, 2, 64, 0, 2),            # ragged: partial query and key blocks
    (64, 64, 1, 64, 0, 0),              # single block, everything forced
    (130, 4000, 3, 128, 200, 5),        # sink not block-aligned
    (64, 26240, 2, 64, 0, 102),         # 410 key blocks, own block forced: 103 kept (review_v1/test_ops.py:39-47)
]


def _route(q, k, wq, wk, block, sink, extra):
    from streaming_sparse_b200 import ops
    dev = torch.device("cuda:0")
    ids, mask, scores = ops.route(q.to(dev), k.to(dev), wq.to(dev), wk.to(dev), block=block, extra=extra,
                                  sink_tokens=sink, return_mask=True, return_scores=True, validate=True)
    torch.cuda.synchronize()
    return ids.cpu().numpy(), mask.cpu().numpy(), scores.cpu().numpy()


@pytest.mark.parametrize("Lq,Lk,H,block,sink,extra", CASES)
def test_router_bit_exact(oracle, Lq, Lk, H, block, sink, extra):
    q, k, _ = qkv(7, Lq, Lk, H)
    wq, wk = router_weights(7, H)
    ids, mask, scores = _route(q, k, wq, wk, block, sink, extra)
    r = oracle.route(np32(q), np32(k), wq.numpy(), wk.numpy(), block, extra, sink_tokens=sink)
    np.testing.assert_array_equal(scores.view(np.uint32), r["scores"].view(np.uint32))
    np.testing.assert_array_equal(ids, r["ids"])
    np.testing.assert_array_equal(mask, r["mask"])
    assert (np.diff(ids, axis=-1) > 0).all()


def test_router_ties_go_to_lower_index(oracle):
    """Identical key blocks give identical scores: the lower block index must win every tie."""
    Lq, Lk, H, block, extra = 128, 1024, 2, 64, 5
    q, k, _ = qkv(3, Lq, Lk, H)
    k = k.clone()
    pattern = k[:64].clone()
    for b in range(0, Lk // 64 - 2):       # every history block identical -> all history scores tie
        k[b * 64:(b + 1) * 64] = pattern
    wq, wk = router_weights(3, H)
    ids, mask, scores = _route(q, k, wq, wk, block, 0, extra)
    r = oracle.route(np32(q), np32(k), wq.numpy(), wk.numpy(), block, extra)
    np.testing.assert_array_equal(ids, r["ids"])
    # forced current blocks are 14, 15; the five lowest history blocks win the tie
    np.testing.assert_array_equal(ids[0, 0], [0, 1, 2, 3, 4, 14, 15])


def test_router_zero_scores_are_canonical(oracle):
    """A zero query gives +0 / -0 scores everywhere; -0 == +0 so ties resolve by index."""
    Lq, Lk, H, block, extra = 64, 640, 1, 64, 3
    q, k, _ = qkv(4, Lq, Lk, H)
    q = torch.zeros_like(q)
    wq, wk = router_weights(4, H)
    ids, _, scores = _route(q, k, wq, wk, block, 0, extra)
    assert (scores.view(np.uint32) == 0).all()
    np.testing.assert_array_equal(ids[0, 0], [0, 1, 2, 9])


def test_router_nonfinite_is_reported():
    from streaming_sparse_b200 import ops
    Lq, Lk, H = 64, 256, 1
    q, k, _ = qkv(5, Lq, Lk, H)
    q[3, 0, 7] = float("inf")
    wq, wk = router_weights(5, H)
    dev = torch.device("cuda:0")
    with pytest.raises(FloatingPointError):
        ops.route(q.to(dev), k.to(dev), wq.to(dev), wk.to(dev), block=64, extra=1, validate=True)
