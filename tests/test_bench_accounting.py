"""The bench's FLOP accounting against an independent count, on the oracle router's selections.

``bench.effective_flops`` turns block ids into 4*D*sum(valid selected tokens) per query row. Here
the oracle selects blocks for configs 1 and 2 (seeded inputs, as the bench makes them), every
query row's attended tokens are counted from a token mask, and the totals are checked against
the closed forms: config 1 = 24 routed blocks + the current frame's 25 blocks (1568 tokens),
3104 tokens per row, 29.75 GFLOP; config 2 = 54 routed blocks + the 74 current blocks (4728
tokens), 8184 tokens per row, 235.32 GFLOP.
"""
import math

import numpy as np
import pytest

import bench
from oracle import oracle as o

H, D, B = 12, 128, 64


def _tokens_per_row(ids: np.ndarray, Lq: int, Lk: int) -> np.ndarray:
    """[H, Lq] attended tokens, from a [Lk] token mask per (head, query block)."""
    out = np.zeros((ids.shape[0], Lq), dtype=np.int64)
    for h in range(ids.shape[0]):
        for i in range(ids.shape[1]):
            mask = np.zeros(Lk, dtype=bool)
            for j in ids[h, i]:
                if j >= 0:
                    mask[j * B:(j + 1) * B] = True
            out[h, i * B:min(Lq, (i + 1) * B)] = mask.sum()
    return out


@pytest.mark.parametrize("Lq,Lk,extra,per_row", [(1560, 6240, 24, 3104), (4680, 32760, None, 8184)])
def test_effective_flops_match_token_count(Lq, Lk, extra, per_row):
    g = np.random.default_rng(0)
    q = g.standard_normal((Lq, H, D), dtype=np.float32)
    k = g.standard_normal((Lk, H, D), dtype=np.float32)
    wq = (g.standard_normal((H, D, 64)) / math.sqrt(D)).astype(np.float32)
    wk = (g.standard_normal((H, D, 64)) / math.sqrt(D)).astype(np.float32)
    kb, qb = math.ceil(Lk / B), math.ceil(Lq / B)
    if extra is None:    # "top-k at 25 % density": ceil(0.25 kb) blocks in all, the forced current blocks first
        extra = o.budget(kb, kb - (Lk - Lq) // B, density=0.25)
    ids = o.route(q, k, wq, wk, B, extra)["ids"]
    assert ids.shape[:2] == (H, qb)
    tok = _tokens_per_row(ids, Lq, Lk)
    assert (tok == per_row).all()
    assert bench.effective_flops(ids, Lq, Lk, B) == 4 * D * tok.sum() == 4 * D * H * Lq * per_row


def test_config_points_have_unique_short_names():
    pts = bench.config_points()
    assert len({p[0] for p in pts}) == len(pts) == 17
    assert all(p[2] <= p[3] for p in pts)          # Lq <= Lk everywhere
