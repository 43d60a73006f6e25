"""The router's fast mode (ss_router_fast): block scores on tcgen05 (3xTF32), query blocks whose
selection the error bound cannot settle scored again in exact fp32. Its ids and masks must equal
the exact mode's bit for bit: on random inputs, on inputs built with exact ties and near-ties at
the threshold (which must be re-scored), at every shape class the kernels branch on, and through
the cached-key path. The measured tensor-core error must stay well inside the bound the
selection relies on."""
import math

import numpy as np
import pytest
import torch

from helpers import np32, qkv, router_weights

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")
FAST_BOUND = 2.0 ** -13     # |fast - exact| <= FAST_BOUND * |qh_i| * |kh_j| (router.cu)


def _both(q, k, wq, wk, block, extra, sink, **kw):
    from streaming_sparse_b200 import ops
    exact = ops.route(q, k, wq, wk, block=block, extra=extra, sink_tokens=sink, return_mask=True, validate=True,
                      **kw)
    n = torch.zeros(1, dtype=torch.int32, device=DEV)
    fast = ops.route(q, k, wq, wk, block=block, extra=extra, sink_tokens=sink, return_mask=True, validate=True,
                     fast=True, rescored=n, **kw)
    torch.cuda.synchronize()
    return exact, fast, int(n.item())


def _assert_same(exact, fast):
    np.testing.assert_array_equal(fast[0].cpu().numpy(), exact[0].cpu().numpy())
    np.testing.assert_array_equal(fast[1].cpu().numpy(), exact[1].cpu().numpy())


@pytest.mark.parametrize("Lq,Lk,H,block,sink,extra,R", [
    (4680, 32760, 12, 64, 0, 54, 64),      # config 2
    (4680, 34320, 6, 128, 1560, 21, 64),   # config 4 shape (block 128, sink frame)
    (4680, 98280, 4, 64, 0, 307, 64),      # config 5, Lk 98280: 1536 key blocks (keys in shared memory)
    (9360, 20000, 2, 64, 0, 40, 64),       # 147 query blocks: two query tiles of the score GEMM
    (1560, 6240, 12, 64, 0, 24, 32),       # config 1, R = 32
    (100, 333, 2, 64, 0, 2, 64),           # ragged, a partial key tile
    (64, 64, 1, 64, 0, 0, 64),             # nothing to choose
])
def test_fast_ids_equal_exact(Lq, Lk, H, block, sink, extra, R):
    for seed in (1, 2):
        q, k, _ = qkv(40 + seed, Lq, Lk, H)
        wq, wk = router_weights(40 + seed, H, R=R)
        q, k, wq, wk = (t.to(DEV) for t in (q, k, wq, wk))
        exact, fast, n = _both(q, k, wq, wk, block, extra, sink)
        _assert_same(exact, fast)
        print(f"Lq={Lq} Lk={Lk} H={H} R={R}: {n} of {H * exact[0].shape[1]} query blocks scored again")


def test_fast_equals_oracle_small(oracle):
    from streaming_sparse_b200 import ops
    q, k, _ = qkv(5, 640, 2000, 3)
    wq, wk = router_weights(5, 3)
    r = oracle.route(np32(q), np32(k), wq.numpy(), wk.numpy(), 64, 9, sink_tokens=100)
    got = ops.route(q.to(DEV), k.to(DEV), wq.to(DEV), wk.to(DEV), block=64, extra=9, sink_tokens=100, fast=True)
    np.testing.assert_array_equal(got.cpu().numpy(), r["ids"])


def test_tensor_core_error_inside_bound():
    """|fast - S| and |exact - S| against an fp64 S from the same fp32 projections, in units of
    |qh_i| |kh_j|: their sum must be far inside FAST_BOUND (the bound the selection trusts)."""
    from streaming_sparse_b200 import ops
    Lq, Lk, H, block = 4680, 32760, 12, 64
    q, k, _ = qkv(77, Lq, Lk, H)
    wq, wk = router_weights(77, H)
    q, k, wq, wk = (t.to(DEV) for t in (q, k, wq, wk))
    qb, kb = ops.nblocks(Lq, block), ops.nblocks(Lk, block)
    kt = ops.RouterKeys(H, Lk, block=block, device=DEV)
    ops.pool_keys(k, wk, kt, j0=0, j1=kb)
    qt = ops.RouterKeys(H, Lq, block=block, device=DEV)
    ops.pool_keys(q, wq, qt, j0=0, j1=qb)          # the query projections, by the same arithmetic
    qh, kh = qt.kh[:, :qb].double(), kt.kh[:, :kb].double()
    s64 = torch.einsum("hir,hjr->hij", qh, kh)
    norm = qh.norm(dim=2)[:, :, None] * kh.norm(dim=2)[:, None, :]
    _, se = ops.route(q, k, wq, wk, block=block, extra=54, return_scores=True)
    _, sf = ops.route(q, k, wq, wk, block=block, extra=54, return_scores=True, fast=True)
    ef = float(((sf.double() - s64).abs() / norm).max())
    ee = float(((se.double() - s64).abs() / norm).max())
    print(f"max |fast - S| = {ef:.3e}, max |exact - S| = {ee:.3e} (x |q||k|); bound {FAST_BOUND:.3e}")
    assert ef + ee < FAST_BOUND / 8


def test_exact_ties_are_rescored():
    """Key blocks in identical pairs give every score twice: thresholds fall on ties, the fast
    mode must score those query blocks again and keep the lower block of a tie, as the exact mode."""
    Lq, Lk, H, block = 1024, 16384, 4, 64
    q, k, _ = qkv(8, Lq, Lk, H)
    hist = (Lk - Lq) // block
    kb = k.view(-1, block, H, 128)
    kb[1:hist:2] = kb[0:hist - 1:2]
    wq, wk = router_weights(8, H)
    q, k, wq, wk = (t.to(DEV) for t in (q, k, wq, wk))
    exact, fast, n = _both(q, k, wq, wk, block, 31, 0)
    _assert_same(exact, fast)
    assert n > 0, "tied thresholds must be scored again"
    print(f"ties: {n} of {H * exact[0].shape[1]} query blocks scored again")


def test_near_ties_are_rescored():
    """Pairs of key blocks one bf16 step apart in a single value: their scores differ by far less
    than the bound, so every threshold between a pair must be settled by the exact scores."""
    Lq, Lk, H, block = 1024, 16384, 4, 64
    q, k, _ = qkv(9, Lq, Lk, H)
    hist = (Lk - Lq) // block
    kb = k.view(-1, block, H, 128)
    kb[1:hist:2] = kb[0:hist - 1:2]
    kb[1:hist:2, 0, :, 0] = (kb[1:hist:2, 0, :, 0].float() * (1 + 2.0 ** -7)).bfloat16()
    wq, wk = router_weights(9, H)
    q, k, wq, wk = (t.to(DEV) for t in (q, k, wq, wk))
    exact, fast, n = _both(q, k, wq, wk, block, 31, 0)
    _assert_same(exact, fast)
    assert n > 0
    print(f"near ties: {n} of {H * exact[0].shape[1]} query blocks scored again")


@pytest.mark.parametrize("Lq,Lk,H,block,sink,extra", [
    (4680, 32760, 12, 64, 0, 54),
    (4680, 34320, 4, 128, 1560, 21),
])
def test_fast_with_cached_keys(Lq, Lk, H, block, sink, extra):
    from streaming_sparse_b200 import ops
    q, k, _ = qkv(31, Lq, Lk, H)
    wq, wk = router_weights(31, H)
    q, k, wq, wk = (t.to(DEV) for t in (q, k, wq, wk))
    keys = ops.RouterKeys(H, Lk, block=block, device=DEV)
    n_hist = ops.history_blocks(Lq, Lk, block)
    ops.pool_keys(k, wk, keys, j0=0, j1=n_hist)
    exact, fast, _ = _both(q, k, wq, wk, block, extra, sink, keys=keys, n_cached=n_hist)
    _assert_same(exact, fast)
    # and a KV-sharded rank's call: k holds only the window's tail
    k_row0 = n_hist * block - (n_hist * block) % 256
    exact2, fast2, _ = _both(q, k[k_row0:], wq, wk, block, extra, sink, keys=keys, n_cached=n_hist, k_row0=k_row0)
    _assert_same(exact, exact2)
    _assert_same(exact2, fast2)
