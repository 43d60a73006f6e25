"""Pin the CPU oracle against vectors produced by the reference's own code (tests/golden/)."""
import math

import numpy as np
import pytest


def test_select_matches_reference_stable_select(oracle, golden):
    """v05 select (streaming_sparse/v05/primitives.py:35-56): score desc, lower id on ties, -0 == +0."""
    g = golden("select_v05.npz")
    forced = g["forced"]
    names = sorted({k.rsplit("_", 1)[0] for k in g.files if k.endswith("_scores")})
    assert len(names) >= 40
    for name in names:
        scores = g[name + "_scores"][None]           # [1,Q,B]
        extra = int(g[name + "_extra"])
        ids, mask = oracle.select(scores, forced, extra)
        np.testing.assert_array_equal(mask[0].astype(np.uint8), g[name + "_mask"], err_msg=name)
        assert (np.diff(ids, axis=-1) > 0).all()


def test_attention_matches_reference_gather(oracle, golden):
    """v08 reference (streaming_sparse/v08/attention.py:115-123) == global-block gather over [history|current]."""
    g = golden("attention_v08.npz")
    for c in ("c0", "c1"):
        f = lambda key: g[f"{c}_{key}"].astype(np.uint32) << 16
        q, kh, vh, kc, vc = (f(k).view(np.float32) for k in ("q", "kh", "vh", "kc", "vc"))
        bm = g[f"{c}_block_mask"]
        nh, nc = len(kh), len(kc)
        assert nh % 64 == 0
        k = np.concatenate([kh, kc])[:, None, :]
        v = np.concatenate([vh, vc])[:, None, :]
        kb = math.ceil((nh + nc) / 64)
        qb = bm.shape[0]
        ids = np.full((1, qb, kb), -1, np.int32)
        for i in range(qb):
            sel = [j for j in range(nh // 64) if bm[i, j]] + list(range(nh // 64, kb))
            ids[0, i, :len(sel)] = sel
        out, lse = oracle.attention(q[:, None, :], k, v, ids, 64)
        np.testing.assert_allclose(out[:, 0, :], g[f"{c}_out"], rtol=1e-5, atol=1e-6)
        assert np.isfinite(lse).all()


def test_all_selected_equals_dense(oracle):
    """all-selected == dense softmax (local_experiments/review_v1/test_ops.py:19-23)."""
    rng = np.random.default_rng(3)
    q = oracle.bf16_round(rng.standard_normal((100, 2, 128)).astype(np.float32))
    k = oracle.bf16_round(rng.standard_normal((300, 2, 128)).astype(np.float32))
    v = oracle.bf16_round(rng.standard_normal((300, 2, 128)).astype(np.float32))
    kb = math.ceil(300 / 64)
    ids = np.tile(np.arange(kb, dtype=np.int32), (2, 2, 1))
    out, lse = oracle.attention(q, k, v, ids, 64)
    for h in range(2):
        z = q[:, h].astype(np.float64) @ k[:, h].T.astype(np.float64) / math.sqrt(128)
        p = np.exp(z - z.max(1, keepdims=True))
        dense = (p / p.sum(1, keepdims=True)) @ v[:, h]
        np.testing.assert_allclose(out[:, h], dense, rtol=1e-10, atol=1e-12)
        ref_lse = np.log(np.exp(z - z.max(1, keepdims=True)).sum(1)) + z.max(1)
        np.testing.assert_allclose(lse[h], ref_lse, rtol=1e-12)


def test_merge_matches_reference(oracle, golden):
    """merge (local_experiments/video_runtime_v1/attention.py:40-45); its output is bf16."""
    g = golden("merge_vr1.npz")
    parts = np.stack([g["exact"][0], g["approx"].transpose(1, 0, 2)])
    lses = np.stack([g["exact_lse"], g["approx_lse"]])
    out, _ = oracle.lse_merge(parts, lses)
    np.testing.assert_allclose(oracle.bf16_round(out.astype(np.float32)), g["out"][0], rtol=0, atol=1e-2)
    np.testing.assert_allclose(out, g["out"][0], rtol=8e-3, atol=1e-5)


def test_positions_match_reference_adapter(golden):
    """PositionTracker == SelfForcingAdapter._pre (streaming_sparse/integration/self_forcing_adapter.py:50-97)."""
    from streaming_sparse_b200.cache import PositionTracker
    g = golden("positions_adapter.npz")
    for name in ("validate", "long", "global"):
        ftok, local, sink, cache, n, chunks, steps, frame = (int(x) for x in g[f"{name}_meta"])
        calls = g[f"{name}_calls"]
        flat_all = g[f"{name}_positions"]
        tr = PositionTracker(cache)
        max_att = 32760 if local == -1 else local * frame
        ge = le = off = 0
        for start, nn, hist, count in calls:
            vis, h = tr.update(start=int(start), n=int(nn), old_global=ge, old_local=le, local_attn=local != -1,
                               sink_tokens=sink * ftok, max_attention_size=max_att)
            np.testing.assert_array_equal(vis, flat_all[off:off + count], err_msg=f"{name} start={start}")
            assert h == hist
            off += count
            end = int(start) + int(nn)
            if local != -1 and end > ge and nn + le > cache:
                le = le + end - ge - (nn + le - cache)
            else:
                le = le + end - ge
            ge = end


def test_cache_known_answer(oracle):
    """evaluation/validate.py:57-88: after 3 chunks the visible positions are [0..3] + [16..35]."""
    cap, n = 24, 12
    kc = np.full((cap, 1, 2), -1.0)
    vc = np.full((cap, 1, 2), -1.0)
    ge = le = 0
    for chunk in range(3):
        for _ in range(3):
            start = chunk * n
            tok = np.arange(start, start + n, dtype=np.float64)[:, None, None].repeat(2, 2)
            le = oracle.cache_append(kc, vc, tok, tok, local_attn=True, global_end=ge, local_end=le,
                                     current_start=start, sink_tokens=4)
            ge = start + n
    np.testing.assert_array_equal(kc[:le, 0, 0], list(range(4)) + list(range(16, 36)))


def test_budget_sizes_per_config(oracle):
    # config 1: Lq 1560, Lk 6240, block 64 -> current-frame blocks 73..97 forced, extra 24
    f = oracle.forced_blocks(1560, 6240, 64)
    assert f.sum() == 25 and f[73:].all() and not f[:73].any()
    # config 2: 74 forced current blocks (438..511), total ceil(.25*512)=128 -> extra 54
    f = oracle.forced_blocks(4680, 32760, 64)
    assert f.sum() == 74 and f[438:].all() and not f[:438].any()
    assert oracle.budget(512, 74, density=0.25, rule="total") == 54
    # config 4: window 34320 with one sink frame, block 128: 13 sink + 37/38 current blocks
    f = oracle.forced_blocks(4680, 34320, 128, sink_tokens=1560)
    kb = len(f)
    assert kb == 269 and f[:13].all()
    assert oracle.budget(kb, int(f.sum()), density=0.1, rule="rest") == math.floor(0.1 * (kb - f.sum()))


def test_count_rule_known_answer(oracle):
    """The count known answer of local_experiments/review_v1/test_ops.py:39-47: 410 pages at the
    25 % "total" rule keep ceil(0.25 * 410) = 103 blocks, the forced own page included, and drop
    the other 307; the kept mask has exactly that many entries and contains the own page."""
    rng = np.random.default_rng(410)
    kb, own = 410, 339
    S = rng.random((2, 3, kb)).astype(np.float32)
    forced = np.zeros(kb, np.uint8)
    forced[own] = 1
    extra = oracle.budget(kb, 1, density=0.25, rule="total")
    assert extra + 1 == 103
    ids, mask = oracle.select(S, forced, extra)
    assert ids.shape == (2, 3, 103) and (mask.sum(-1) == 103).all() and ((~mask).sum(-1) == 307).all()
    assert mask[..., own].all() and (np.diff(ids, axis=-1) > 0).all()
    # the 102 others are the best-scoring unforced pages
    for h in range(2):
        for i in range(3):
            rest = np.delete(S[h, i], own)
            assert S[h, i][mask[h, i]].sum() - S[h, i, own] == pytest.approx(np.sort(rest)[-102:].sum(), rel=1e-6)


@pytest.mark.parametrize("rho", [0.0, 0.1, 0.2, 0.3, 1.0])
def test_budgets_match_direct_gather(oracle, rho):
    """streaming_sparse/v07/tests.py:24-37 restated: for history budgets floor(rho * pages), the
    routed output of a query row equals exact softmax attention over the directly gathered tokens
    (the selected history blocks, then the current chunk), budget 0 (current chunk only) and the
    whole history (dense) included."""
    rng = np.random.default_rng(7)
    H, Lq, hist_blocks, block = 2, 128, 16, 64
    Lk = hist_blocks * block + Lq
    q = oracle.bf16_round(rng.standard_normal((Lq, H, 128)).astype(np.float32))
    k = oracle.bf16_round(rng.standard_normal((Lk, H, 128)).astype(np.float32))
    v = oracle.bf16_round(rng.standard_normal((Lk, H, 128)).astype(np.float32))
    wq = (rng.standard_normal((H, 128, 64)) / math.sqrt(128)).astype(np.float32)
    wk = (rng.standard_normal((H, 128, 64)) / math.sqrt(128)).astype(np.float32)
    extra = math.floor(rho * hist_blocks)
    ids = oracle.route(q, k, wq, wk, block, extra)["ids"]
    out, _ = oracle.attention(q, k, v, ids, block)
    for h in range(H):
        for row in (0, 63, 64, Lq - 1):
            i = row // block
            hist = [j for j in ids[h, i] if j < hist_blocks]
            assert len(hist) == extra
            tokens = [t for j in hist for t in range(j * block, (j + 1) * block)] + list(range(Lk - Lq, Lk))
            kk = k[tokens, h].astype(np.float64)
            vv = v[tokens, h].astype(np.float64)
            s = kk @ q[row, h].astype(np.float64) / math.sqrt(128)
            p = np.exp(s - s.max())
            direct = (p / p.sum()) @ vv
            np.testing.assert_allclose(out[row, h], direct, rtol=1e-5, atol=1e-6)


def test_router_invariants(oracle):
    """ids in range and strictly increasing (migration/unified_router/opt28/validate_selection.py:30);
    forced blocks present; no unselected unforced block outranks a selected one."""
    rng = np.random.default_rng(0)
    Lq, Lk, H = 300, 1000, 3
    q = oracle.bf16_round(rng.standard_normal((Lq, H, 128)).astype(np.float32))
    k = oracle.bf16_round(rng.standard_normal((Lk, H, 128)).astype(np.float32))
    wq = (rng.standard_normal((H, 128, 64)) / math.sqrt(128)).astype(np.float32)
    wk = (rng.standard_normal((H, 128, 64)) / math.sqrt(128)).astype(np.float32)
    r = oracle.route(q, k, wq, wk, 64, extra=4)
    ids, mask, S, f = r["ids"], r["mask"], r["scores"], r["forced"].astype(bool)
    kb = len(f)
    assert ((ids >= 0) & (ids < kb)).all() and (np.diff(ids, axis=-1) > 0).all()
    assert mask[..., f].all()
    for h in range(H):
        for i in range(ids.shape[1]):
            sel = mask[h, i] & ~f
            rest = ~mask[h, i] & ~f
            assert sel.sum() == 4
            assert S[h, i][sel].min() >= S[h, i][rest].max()


def test_router_pooling_is_exact_fp32_order(oracle):
    """The block mean is a sequential fp32 sum and one divide; projection is ascending fmaf."""
    rng = np.random.default_rng(1)
    x = oracle.bf16_round(rng.standard_normal((70, 1, 128)).astype(np.float32))
    w = rng.standard_normal((1, 128, 64)).astype(np.float32)
    pooled, proj = oracle.pool_project(x, w, 64)
    for b, (t0, t1) in enumerate([(0, 64), (64, 70)]):
        s = np.float32(0)
        for t in range(t0, t1):
            s = np.float32(s + x[t, 0])
        np.testing.assert_array_equal(pooled[0, b], s / np.float32(t1 - t0))
    # fma order: compare with float64 accumulation loosely, exact equality is checked on the GPU
    np.testing.assert_allclose(proj[0], pooled[0].astype(np.float64) @ w[0], rtol=1e-4, atol=1e-5)


def _bf16_bits_to_f32(a):
    return (a.astype(np.uint16).astype(np.uint32) << 16).view(np.float32)


def test_rope_shift_matches_reference_anchor_rebase(oracle, golden):
    """local_experiments/anchor_rebase.py:8-18 shift_temporal_: bit for bit, every case."""
    g = golden("anchor_rebase.npz")
    keys = _bf16_bits_to_f32(g["keys"])
    for name in g.files:
        if not name.startswith("out_"):
            continue
        _, offset, tokens = name.split("_")
        got = oracle.rope_shift(keys, int(tokens), oracle.rope_phase(int(offset)))
        np.testing.assert_array_equal(got.view(np.uint32), _bf16_bits_to_f32(g[name]).view(np.uint32), err_msg=name)


def test_temporal_phase_table_matches_oracle(oracle):
    from streaming_sparse_b200.cache import temporal_phase
    for off in (0, 1, 15, 1023):
        np.testing.assert_allclose(temporal_phase(off, "cpu").numpy(), oracle.rope_phase(off), rtol=0, atol=1e-15)


def test_cache_index_plan_matches_oracle_roll(oracle):
    """KVCache.write_plan/advance (host-only index arithmetic, which keys the rollout's graphs)
    against the oracle's restatement of the cache roll + write, over random chunk sequences with
    rewrites of the same chunk and rolling windows with sink frames."""
    import numpy as np
    from streaming_sparse_b200.cache import KVCache
    rng = np.random.default_rng(5)
    for local, sink, ft in [(-1, 0, 8), (6, 1, 8), (5, 2, 4), (4, 0, 16)]:
        cap = (local if local > 0 else 12) * ft
        c = KVCache(cap, 1, 128, frame_tokens=ft, local_attn_size=local, sink_size=sink, device="cpu",
                    track_positions=False)
        kc = np.zeros((cap, 1, 1), np.float32)
        vc = np.zeros((cap, 1, 1), np.float32)
        g_end, l_end, start = 0, 0, 0
        total = 0
        while total < (3 * cap if local > 0 else cap - 3 * ft):
            n = int(rng.integers(1, 3)) * ft
            for rep in range(int(rng.integers(1, 4))):          # the same chunk written 1-3 times
                new = np.full((n, 1, 1), start + rep, np.float32)
                rolls, evicted, end_after = c.write_plan(n, start)
                l_ref = oracle.cache_append(kc, vc, new, new, local_attn=local != -1, global_end=g_end,
                                            local_end=l_end, current_start=start, sink_tokens=sink * ft)
                assert end_after == l_ref
                assert rolls == (evicted > 0) and (rolls == (local != -1 and start + n > g_end and n + l_end > cap))
                c.advance(n, start)
                g_end, l_end = start + n, l_ref
                assert (c.global_end, c.local_end) == (g_end, l_end)
            start += n
            total += n


def test_window_retention_matches_reference_first_chunk_policy():
    """The retention known answers of local_experiments/test_kv_history.py:11-24 for the policy
    that keeps the first chunk and the latest frames ("A_first_chunk": 3-frame chunks, 15 frames
    kept), which is the rolling window with sink frames: a KVCache with a 3-frame sink and a
    15-frame window, one token per frame, so visible positions are frame indices. After every
    chunk the visible frames are min(15, 3 * chunks) sorted distinct frames drawn from the
    previous set and the new chunk; after 20 chunks they are 0..2 and 48..59."""
    from streaming_sparse_b200.cache import KVCache
    c = KVCache(15, 1, 128, frame_tokens=1, local_attn_size=15, sink_size=3, device="cpu")
    old = []
    for completed in range(1, 43):
        for _ in range(2):                       # a chunk's denoising passes rewrite it in place
            vis, _ = c.advance(3, (completed - 1) * 3)
        chosen = vis.tolist()
        assert len(chosen) == min(15, completed * 3)
        assert chosen == sorted(set(chosen))
        assert set(chosen) <= set(old + list(range((completed - 1) * 3, completed * 3)))
        old = chosen
        if completed == 20:
            assert chosen == list(range(3)) + list(range(48, 60))


def test_router_scores_match_reference_score_cached(oracle, golden):
    """The exact-fp32 router scores against the reference's own block scores
    (migration/unified_router/fast_route.py:25-34 ``score_cached`` with one mean prototype per key
    block, golden from tests/golden/make_golden.py): with W_q = W_k = the reference's basis,
    score_ref = score / sqrt(128) + log(count). The ids agree wherever the selection margin (the
    extra-th against the next unforced score) is wider than the arithmetic tolerance."""
    g = golden("score_cached.npz")
    bits = lambda a: (a.astype(np.int32) << 16).view(np.float32)   # bf16 bit patterns -> float32
    q, k = bits(g["q_bf16"].astype(np.uint16)), bits(g["k_bf16"].astype(np.uint16))
    basis, block = g["basis"], int(g["block"])
    Lq, Lk = q.shape[0], k.shape[0]
    extra = 6
    r = oracle.route(q, k, basis, basis, block, extra)
    ours = r["scores"].astype(np.float64) / np.sqrt(128.0) + g["logcount"][:, None, :]
    tol = 2e-6                               # measured difference: 2.4e-7 on scores of magnitude ~4
    np.testing.assert_allclose(ours, g["score"], rtol=0, atol=tol)
    # selection on the reference's scores: forced current blocks, then the extra best unforced
    forced = oracle.forced_blocks(Lq, Lk, block)
    ref = g["score"]
    checked = 0
    for h in range(ref.shape[0]):
        for i in range(ref.shape[1]):
            cand = [j for j in range(ref.shape[2]) if not forced[j]]
            order = sorted(cand, key=lambda j: (-ref[h, i, j], j))
            if extra < len(order) and ref[h, i, order[extra - 1]] - ref[h, i, order[extra]] <= 2 * tol:
                continue
            want = sorted(order[:extra] + [j for j in range(ref.shape[2]) if forced[j]])
            np.testing.assert_array_equal(r["ids"][h, i], want)
            checked += 1
    assert checked == ref.shape[0] * ref.shape[1]
