"""tcgen05 block-sparse attention == the float64 gather-softmax oracle."""
import math

import numpy as np
import pytest
import torch

from helpers import assert_attention_close, np32, qkv, router_weights

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")


def _attend(q, k, v, ids, block, out_dtype=torch.bfloat16):
    from streaming_sparse_b200 import ops
    out, lse = ops.sparse_attention(q.to(DEV), k.to(DEV), v.to(DEV), torch.as_tensor(ids).to(DEV), block=block,
                                    out_dtype=out_dtype, return_lse=True, validate=True)
    torch.cuda.synchronize()
    return out.float().cpu().numpy(), lse.cpu().numpy()


def _random_ids(rng, H, qb, kb, n, pad=0, forced=()):
    ids = np.full((H, qb, n + pad), -1, np.int32)
    for h in range(H):
        for i in range(qb):
            rest = [j for j in range(kb) if j not in forced]
            pick = sorted(set(forced) | set(rng.choice(rest, n - len(forced), replace=False).tolist()))
            ids[h, i, :n] = pick
    return ids


@pytest.mark.parametrize("Lq,Lk,H,block,n,pad", [
    (100, 333, 2, 64, 3, 2),       # partial query tile, partial last key block, -1 padding
    (256, 1024, 3, 64, 7, 0),      # two full tiles
    (300, 1000, 2, 128, 4, 1),     # 128-token router blocks
    (64, 4096, 1, 64, 64, 0),      # one tile, all 64 blocks listed
    (1, 65, 1, 64, 2, 0),          # a single query row, a 1-token last block
])
def test_attention_random_lists(oracle, Lq, Lk, H, block, n, pad):
    q, k, v = qkv(11, Lq, Lk, H)
    rng = np.random.default_rng(11)
    qb, kb = math.ceil(Lq / block), math.ceil(Lk / block)
    ids = _random_ids(rng, H, qb, kb, min(n, kb), pad, forced=(kb - 1,))
    out, lse = _attend(q, k, v, ids, block)
    ref, ref_lse = oracle.attention(np32(q), np32(k), np32(v), ids, block)
    assert_attention_close(out, ref)
    np.testing.assert_allclose(lse, ref_lse, rtol=0, atol=2e-3)


def test_attention_fp32_output_and_lse(oracle):
    Lq, Lk, H, block = 200, 2000, 2, 64
    q, k, v = qkv(12, Lq, Lk, H)
    rng = np.random.default_rng(12)
    ids = _random_ids(rng, H, math.ceil(Lq / 64), math.ceil(Lk / 64), 9, forced=(31,))
    out, lse = _attend(q, k, v, ids, block, torch.float32)
    ref, ref_lse = oracle.attention(np32(q), np32(k), np32(v), ids, block)
    err = np.abs(out - ref)
    assert err.max() < 5e-3 and err.mean() < 5e-4
    np.testing.assert_allclose(lse, ref_lse, rtol=0, atol=2e-3)


def test_attention_config1_routed(oracle):
    """Config 1 end to end: router ids from the GPU (bit-exact to the oracle), attention vs oracle."""
    from streaming_sparse_b200 import ops
    Lq, Lk, H = 1560, 6240, 12
    q, k, v = qkv(1, Lq, Lk, H)
    wq, wk = router_weights(1, H)
    ids = ops.route(q.to(DEV), k.to(DEV), wq.to(DEV), wk.to(DEV), block=64, extra=24, validate=True)
    ids_np = ids.cpu().numpy()
    r = oracle.route(np32(q), np32(k), wq.numpy(), wk.numpy(), 64, 24)
    np.testing.assert_array_equal(ids_np, r["ids"])
    out, lse = _attend(q, k, v, ids_np, 64)
    ref, ref_lse = oracle.attention(np32(q), np32(k), np32(v), ids_np, 64)
    assert_attention_close(out, ref)
    np.testing.assert_allclose(lse, ref_lse, rtol=0, atol=2e-3)


@pytest.mark.parametrize("rho", [0.0, 0.1, 0.3, 1.0])
def test_attention_history_budgets(oracle, rho):
    """History budgets floor(rho * pages) from the GPU router, budget 0 (the current chunk alone)
    and the whole history included, against the oracle (streaming_sparse/v07/tests.py:24-37)."""
    from streaming_sparse_b200 import ops
    H, Lq, hist_blocks = 3, 256, 16
    Lk = hist_blocks * 64 + Lq
    q, k, v = qkv(11, Lq, Lk, H)
    wq, wk = router_weights(11, H)
    extra = math.floor(rho * hist_blocks)
    ids = ops.route(q.to(DEV), k.to(DEV), wq.to(DEV), wk.to(DEV), block=64, extra=extra, validate=True)
    ids_np = ids.cpu().numpy()
    r = oracle.route(np32(q), np32(k), wq.numpy(), wk.numpy(), 64, extra)
    np.testing.assert_array_equal(ids_np, r["ids"])
    assert ((ids_np < hist_blocks).sum(-1) == extra).all()
    out, lse = _attend(q, k, v, ids_np, 64)
    ref, ref_lse = oracle.attention(np32(q), np32(k), np32(v), ids_np, 64)
    assert_attention_close(out, ref)
    np.testing.assert_allclose(lse, ref_lse, rtol=0, atol=2e-3)


def test_attention_config2_sampled(oracle):
    """Config 2 at full size; the float64 oracle checks every head on 16 query blocks (both ends,
    the partial last block, and every sixth block between): 192 of the 888 (head, query-block)
    pairs."""
    from streaming_sparse_b200 import ops
    Lq, Lk, H = 4680, 32760, 12
    q, k, v = qkv(2, Lq, Lk, H)
    wq, wk = router_weights(2, H)
    ids = ops.route(q.to(DEV), k.to(DEV), wq.to(DEV), wk.to(DEV), block=64, extra=54, validate=True)
    ids_np = ids.cpu().numpy()
    assert ids_np.shape == (12, 74, 128)
    out, lse = _attend(q, k, v, ids_np, 64)
    heads, qblocks = list(range(12)), sorted({0, 1, 72, 73} | set(range(3, 72, 6)))
    assert len(qblocks) >= 16
    ref, ref_lse = oracle.attention(np32(q), np32(k), np32(v), ids_np, 64, heads=heads, qblocks=qblocks)
    assert_attention_close(out, ref)
    m = np.isfinite(ref_lse)
    np.testing.assert_allclose(lse[m], ref_lse[m], rtol=0, atol=2e-3)
    assert np.isfinite(out).all()


def test_attention_config4_routed_sampled(oracle):
    """Config 4 shape: 128-token router blocks, a one-frame sink, 10 % of the unforced blocks;
    router bit-exact to the oracle, attention checked on sampled query blocks."""
    from streaming_sparse_b200 import ops
    Lq, Lk, H, block, sink = 4680, 34320, 4, 128, 1560
    kb = ops.nblocks(Lk, block)
    nf = ops.forced_count(Lq, Lk, block, sink)
    extra = (kb - nf) // 10
    assert (kb, nf, extra) == (269, 51, 21)
    q, k, v = qkv(4, Lq, Lk, H)
    wq, wk = router_weights(4, H)
    ids = ops.route(q.to(DEV), k.to(DEV), wq.to(DEV), wk.to(DEV), block=block, extra=extra, sink_tokens=sink,
                    validate=True)
    ids_np = ids.cpu().numpy()
    r = oracle.route(np32(q), np32(k), wq.numpy(), wk.numpy(), block, extra, sink_tokens=sink)
    np.testing.assert_array_equal(ids_np, r["ids"])
    out, lse = _attend(q, k, v, ids_np, block)
    ref, ref_lse = oracle.attention(np32(q), np32(k), np32(v), ids_np, block, heads=[0, 3], qblocks=[0, 17, 36])
    assert_attention_close(out, ref)
    m = np.isfinite(ref_lse)
    np.testing.assert_allclose(lse[m], ref_lse[m], rtol=0, atol=2e-3)


@pytest.mark.parametrize("block,density", [(64, 0.5), (128, 0.05)])
def test_attention_config5_longest_window_sampled(oracle, block, density):
    """Config 5's longest window (63 latent frames, 98280 tokens) at the sweep's densest and
    sparsest points; routed lists from the GPU router, attention on sampled query blocks."""
    from streaming_sparse_b200 import ops
    Lq, Lk, H = 4680, 98280, 2
    kb = ops.nblocks(Lk, block)
    nf = ops.forced_count(Lq, Lk, block)
    extra = ops.budget(kb, nf, density=density)
    q, k, v = qkv(5, Lq, Lk, H)
    wq, wk = router_weights(5, H)
    ids = ops.route(q.to(DEV), k.to(DEV), wq.to(DEV), wk.to(DEV), block=block, extra=extra, validate=True)
    ids_np = ids.cpu().numpy()
    assert ids_np.shape[-1] == nf + extra
    out, lse = _attend(q, k, v, ids_np, block)
    qbs = ops.nblocks(Lq, block)
    ref, ref_lse = oracle.attention(np32(q), np32(k), np32(v), ids_np, block, heads=[0, 1],
                                    qblocks=[0, qbs // 2, qbs - 1])
    assert_attention_close(out, ref)
    m = np.isfinite(ref_lse)
    np.testing.assert_allclose(lse[m], ref_lse[m], rtol=0, atol=2e-3)


CONFIG5_GRID = [(4680, 64, 0.25)] + [(lk, 64, d) for lk in (9360, 65520, 98280) for d in (0.05, 0.10, 0.25, 0.5)] + \
    [(98280, 128, 0.05), (98280, 128, 0.5)]


@pytest.mark.parametrize("Lk,block,density", CONFIG5_GRID)
def test_config5_grid_point(oracle, Lk, block, density):
    """Every config-5 point the bench times (4680 queries, windows of 1, 2, 14 and 21 chunks,
    densities 5-50 %, blocks 64 and 128), 2 heads: the router -- full, and with the history keys
    pooled at commit -- bit for bit against the oracle, then the attention on the router's ids
    against the float64 oracle on a sample of query blocks of both heads."""
    from streaming_sparse_b200 import ops
    Lq, H = 4680, 2
    q, k, v = qkv(55, Lq, Lk, H)
    wq, wk = router_weights(55, H)
    kb = ops.nblocks(Lk, block)
    nf = ops.forced_count(Lq, Lk, block)
    extra = ops.budget(kb, nf, density=density)
    qd, kd, vd, wqd, wkd = (t.to(DEV) for t in (q, k, v, wq, wk))
    ids = ops.route(qd, kd, wqd, wkd, block=block, extra=extra, validate=True)
    keys = ops.RouterKeys(H, Lk, block=block, device=DEV)
    n_hist = ops.history_blocks(Lq, Lk, block)
    ops.pool_keys(kd, wkd, keys, j0=0, j1=n_hist)
    cached = ops.route(qd, kd, wqd, wkd, block=block, extra=extra, validate=True, keys=keys, n_cached=n_hist)
    r = oracle.route(np32(q), np32(k), wq.numpy(), wk.numpy(), block, extra)
    ids_np = ids.cpu().numpy()
    np.testing.assert_array_equal(ids_np, r["ids"])
    np.testing.assert_array_equal(cached.cpu().numpy(), r["ids"])
    out, lse = _attend(q, k, v, ids_np, block)
    qbs = ops.nblocks(Lq, block)
    ref, ref_lse = oracle.attention(np32(q), np32(k), np32(v), ids_np, block, heads=[0, 1],
                                    qblocks=[0, qbs // 3, qbs // 2, qbs - 1])
    assert_attention_close(out, ref)
    m = np.isfinite(ref_lse)
    np.testing.assert_allclose(lse[m], ref_lse[m], rtol=0, atol=2e-3)


def test_all_selected_equals_sdpa():
    """Every block listed == dense attention (local_experiments/review_v1/test_ops.py:19-23)."""
    Lq, Lk, H = 192, 700, 2
    q, k, v = qkv(13, Lq, Lk, H)
    kb = math.ceil(Lk / 64)
    ids = np.tile(np.arange(kb, dtype=np.int32), (H, math.ceil(Lq / 64), 1))
    out, _ = _attend(q, k, v, ids, 64)
    dense = torch.nn.functional.scaled_dot_product_attention(
        q.float().permute(1, 0, 2), k.float().permute(1, 0, 2), v.float().permute(1, 0, 2)).permute(1, 0, 2)
    assert_attention_close(out, dense.numpy())


def test_golden_reference_gather(golden):
    """Inputs and output of streaming_sparse/v08/attention.py:115-123 (bf16-valued inputs)."""
    g = golden("attention_v08.npz")
    for c in ("c0", "c1"):
        f = lambda key: torch.from_numpy(g[f"{c}_{key}"].view(np.int16)).view(torch.bfloat16)
        q, kh, vh, kc, vc = (f(x) for x in ("q", "kh", "vh", "kc", "vc"))
        bm = g[f"{c}_block_mask"]
        nh = kh.shape[0]
        k = torch.cat([kh, kc])[:, None, :].contiguous()
        v = torch.cat([vh, vc])[:, None, :].contiguous()
        kb = math.ceil(k.shape[0] / 64)
        ids = np.full((1, bm.shape[0], kb), -1, np.int32)
        for i in range(bm.shape[0]):
            sel = [j for j in range(nh // 64) if bm[i, j]] + list(range(nh // 64, kb))
            ids[0, i, :len(sel)] = sel
        out, _ = _attend(q[:, None, :].contiguous(), k, v, ids, 64)
        assert_attention_close(out[:, 0, :], g[f"{c}_out"])


def test_padded_reference_ids_are_ignored(oracle, golden):
    """RouteOps.select LUTs pad with -1 (local_experiments/review_v1/ops.py:115-135): never read."""
    g = golden("padded_ids.npz")
    ids = g["ids"].astype(np.int32)              # [2, 3, 128] over 410 pages of 64 tokens
    H, qb, _ = ids.shape
    Lq, Lk = qb * 64, 410 * 64
    q, k, v = qkv(14, Lq, Lk, H)
    out, lse = _attend(q, k, v, ids, 64)
    ref, ref_lse = oracle.attention(np32(q), np32(k), np32(v), ids, 64)
    assert_attention_close(out, ref)


def test_empty_list_gives_zero_and_neg_inf():
    Lq, Lk, H = 128, 256, 1
    q, k, v = qkv(15, Lq, Lk, H)
    ids = np.full((1, 2, 2), -1, np.int32)
    ids[0, 0] = [0, 3]                          # second query block has no blocks at all
    out, lse = _attend(q, k, v, ids, 64)
    assert (out[64:] == 0).all() and np.isneginf(lse[0, 64:]).all()
    assert np.isfinite(out[:64]).all()


def test_bad_block_id_is_reported():
    from streaming_sparse_b200 import ops
    q, k, v = qkv(16, 64, 128, 1)
    ids = torch.tensor([[[0, 5]]], dtype=torch.int32, device=DEV)   # kb = 2
    with pytest.raises(IndexError):
        ops.sparse_attention(q.to(DEV), k.to(DEV), v.to(DEV), ids, block=64, validate=True)


@pytest.mark.parametrize("Lq,Lk,H,n", [
    (6400, 2048, 4, 12),     # 200 tiles: CTAs of one and two tiles (split / pair jobs)
    (25600, 4096, 4, 16),    # 800 tiles: CTAs of five and six tiles (pair, pair, split)
])
def test_attention_many_tiles_per_cta(oracle, Lq, Lk, H, n):
    """A persistent CTA that runs several tiles in turn (each tile's Q reloaded into TMEM while the
    previous tile's output is written, tile ranges that cross heads, per-CTA step lists that fill
    most of the shared-memory budget) against the oracle on sampled query blocks."""
    q, k, v = qkv(17, Lq, Lk, H)
    rng = np.random.default_rng(17)
    qb, kb = math.ceil(Lq / 64), math.ceil(Lk / 64)
    ids = np.zeros((H, qb, n), np.int32)
    forced = list(range(kb - 4, kb)) + [0]
    for h in range(H):
        for i in range(qb):
            rest = rng.choice(np.arange(1, kb - 4), n - len(forced), replace=False)
            ids[h, i] = np.sort(np.concatenate([forced, rest]))
    out, lse = _attend(q, k, v, ids, 64)
    qblocks = sorted(set([0, 1, 2, 3, qb // 2, qb // 2 + 1, qb - 2, qb - 1] + rng.choice(qb, 8).tolist()))
    heads = list(range(H))
    ref, ref_lse = oracle.attention(np32(q), np32(k), np32(v), ids, 64, heads=heads, qblocks=qblocks)
    assert_attention_close(out, ref)
    m = np.isfinite(ref_lse)
    np.testing.assert_allclose(lse[m], ref_lse[m], rtol=0, atol=2e-3)
    assert np.isfinite(out).all()


@pytest.mark.parametrize("Lq,Lk,H,block,n", [
    (1560, 6240, 12, 64, 49),       # config 1's shape: 156 tiles on 148 SMs
    (4680, 34320, 6, 128, 72),      # config 4 with 6 heads (a 2-way head shard): 222 tiles
    (4680, 34320, 2, 128, 72),      # config 4 with 2 heads (8-way head shard): 74 tiles, two CTAs each
    (4680, 34320, 1, 128, 72),      # 1 head: 37 tiles, four CTAs each
    (3600, 6000, 10, 64, 2),        # 290 tiles with two-step lists: pieces without steps
    (3650, 3000, 10, 128, 3),       # partial last tile of every head, 128-token blocks
])
def test_split_tiles_match_unsplit_and_oracle(oracle, Lq, Lk, H, block, n):
    """ss_attention_ws on problems of one to two tiles per SM or half a tile per SM or less (tiles cut across CTAs,
    pieces merged by log-sum-exp) against ss_attention (whole tiles) and, with the north-star
    tolerance, against the float64 oracle; fp32 output and LSE too, twice in a row (the
    workspace keeps nothing between calls)."""
    from streaming_sparse_b200 import ops
    q, k, v = qkv(61, Lq, Lk, H)
    rng = np.random.default_rng(61)
    qb, kb = math.ceil(Lq / block), math.ceil(Lk / block)
    ids = _random_ids(rng, H, qb, kb, min(n, kb), 1, forced=(kb - 1,))
    assert ops.attention_workspace_bytes(H, Lq) > 0
    qd, kd, vd, idd = q.to(DEV), k.to(DEV), v.to(DEV), torch.from_numpy(ids).to(DEV)
    whole, whole_lse = ops.sparse_attention(qd, kd, vd, idd, block=block, out_dtype=torch.float32, return_lse=True,
                                            split=False, validate=True)
    for rep in range(2):
        split, split_lse = ops.sparse_attention(qd, kd, vd, idd, block=block, out_dtype=torch.float32, return_lse=True,
                                                validate=True)
        torch.cuda.synchronize()
        # each piece exponentiates against its own running max, so P's bf16 rounding differs
        # from the whole tile's: agreement at that level (relative 2^-9 of P), not fp32 rounding
        d = (split - whole).abs()
        assert d.max().item() < 2e-3 and d.mean().item() < 2 ** -8 * whole.abs().mean().item()
        assert (split_lse - whole_lse).abs().max().item() < 1e-4
    ref, ref_lse = oracle.attention(np32(q), np32(k), np32(v), ids, block)
    out, lse = _attend(q, k, v, ids, block)
    assert_attention_close(out, ref)
    m = np.isfinite(ref_lse)
    np.testing.assert_allclose(lse[m], ref_lse[m], rtol=0, atol=2e-3)
