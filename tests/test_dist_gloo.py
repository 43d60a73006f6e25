"""Multi-rank host logic on CPU (gloo, world sizes 2 and 3): LSE merge of KV-block shards (every
partial to every rank, and the push exchange: partial rows to their owners, merged rows to
everyone) and the head all_gather, with the per-rank partial attention computed by the CPU oracle
in the test."""
import math
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, fn, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        q.put((rank, fn(rank, world)))
    except Exception as e:  # report to the parent instead of hanging it
        q.put((rank, e))
    finally:
        dist.destroy_process_group()


def _run(fn, world=2):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, fn, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    for r, v in res.items():
        if isinstance(v, Exception):
            raise v
    return res


def _inputs():
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    from oracle import oracle as o
    rng = np.random.default_rng(5)
    Lq, Lk, H = 130, 900, 3
    q = o.bf16_round(rng.standard_normal((Lq, H, 128)).astype(np.float32))
    k = o.bf16_round(rng.standard_normal((Lk, H, 128)).astype(np.float32))
    v = o.bf16_round(rng.standard_normal((Lk, H, 128)).astype(np.float32))
    kb = math.ceil(Lk / 64)
    ids = np.stack([np.stack([np.sort(rng.choice(kb, 6, replace=False)) for _ in range(3)]) for _ in range(H)])
    return o, q, k, v, ids.astype(np.int32)


def kv_shard_rank(rank, world):
    """This rank's partial over its local window (its own blocks, packed) with the ids renumbered
    into it -- the layout KVShardedAttention gives the attention kernel -- gathered to every rank
    and combined by the LSE merge."""
    from streaming_sparse_b200.distributed import local_ids, local_len, local_rows
    o, q, k, v, ids = _inputs()
    Lk = k.shape[0]
    rows = local_rows(Lk, 64, rank, world).numpy()
    assert len(rows) == local_len(Lk, 64, rank, world)
    mine = local_ids(torch.from_numpy(ids), rank, world).numpy()
    part, lse = o.attention(q, k[rows], v[rows], mine, 64)
    lse = np.where(np.isnan(lse), -np.inf, lse)
    part = np.where(np.isneginf(lse).T[:, :, None], 0.0, part)
    parts = [torch.empty(0)] * world
    dist.all_gather_object(parts, (part.astype(np.float32), lse.astype(np.float32)))
    return o.lse_merge(np.stack([p_[0] for p_ in parts]), np.stack([p_[1] for p_ in parts]))


def kv_push_rank(rank, world):
    """The push exchange of KVShardedAttention restated: this rank's partial (as kv_shard_rank)
    goes to the owners of its rows, slot = this rank (the attention epilogue's stores into the
    owners' [world][rows][H][D] and [world][H][rows] buffers); each owner merges its rows from its
    slots and every rank gathers the merged rows (the merge's stores into every rank's output)."""
    from streaming_sparse_b200.distributed import local_ids, local_rows, owner_rows
    o, q, k, v, ids = _inputs()
    Lq, H = q.shape[0], q.shape[1]
    rows = local_rows(k.shape[0], 64, rank, world).numpy()
    part, lse = o.attention(q, k[rows], v[rows], local_ids(torch.from_numpy(ids), rank, world).numpy(), 64)
    lse = np.where(np.isnan(lse), -np.inf, lse)
    part = np.where(np.isneginf(lse).T[:, :, None], 0.0, part)
    _, _, n = owner_rows(Lq, rank, world)
    # what this rank pushes to each owner d: rows [lo_d, hi_d) at local rows 0 .. hi_d - lo_d
    pushes = []
    for d in range(world):
        lo, hi, _ = owner_rows(Lq, d, world)
        o_buf = np.zeros((n, H, 128), np.float32)
        l_buf = np.full((H, n), -np.inf, np.float32)
        o_buf[:hi - lo] = part[lo:hi]
        l_buf[:, :hi - lo] = lse[:, lo:hi]
        pushes.append((o_buf, l_buf))
    everyone = [None] * world
    dist.all_gather_object(everyone, pushes)
    lo, hi, _ = owner_rows(Lq, rank, world)
    o_slots = np.stack([everyone[src][rank][0] for src in range(world)])      # [world][rows][H][D]
    l_slots = np.stack([everyone[src][rank][1] for src in range(world)])      # [world][H][rows]
    merged, merged_lse = o.lse_merge(o_slots[:, :hi - lo], l_slots[:, :, :hi - lo])
    gathered = [None] * world
    dist.all_gather_object(gathered, (merged, merged_lse))
    return np.concatenate([g_[0] for g_ in gathered]), np.concatenate([g_[1] for g_ in gathered], axis=1)


def kv_keys_rank(rank, world):
    """Every rank pools the history blocks it owns from its local window; the all-gathered tables
    assembled into window order must equal the projections of the whole window's blocks."""
    from streaming_sparse_b200.distributed import assemble_keys, local_len, local_rows, owned_blocks
    o, q, k, v, ids = _inputs()
    Lk = k.shape[0]
    wk = np.random.default_rng(8).standard_normal((k.shape[1], 128, 64)).astype(np.float32) / math.sqrt(128)
    n_hist = (Lk - q.shape[0]) // 64
    rows = local_rows(Lk, 64, rank, world).numpy()
    n_own = len(owned_blocks(n_hist, rank, world))
    n_max = len(owned_blocks(n_hist, 0, world))
    mine = np.zeros((k.shape[1], max(n_max, 1), 64), np.float32)
    if n_own:
        _, kh = o.pool_project(k[rows][:n_own * 64], wk, 64)
        mine[:, :n_own] = kh
    parts = [None] * world
    dist.all_gather_object(parts, mine)
    table = assemble_keys([torch.from_numpy(p_) for p_ in parts], world, n_hist).numpy()
    _, whole = o.pool_project(k, wk, 64)
    return table, whole[:, :n_hist], local_len(Lk, 64, rank, world)


def head_shard_rank(rank, world):
    from streaming_sparse_b200.distributed import gather_heads, head_range
    o, q, k, v, ids = _inputs()
    h0, h1 = head_range(q.shape[1], rank, world)
    part, _ = o.attention(q[:, h0:h1], k[:, h0:h1], v[:, h0:h1], ids[h0:h1], 64)
    return gather_heads(torch.from_numpy(part).float(), q.shape[1]).numpy()


@pytest.mark.parametrize("world", [2, 3])
def test_kv_sharded_lse_merge_equals_full(world):
    """World 3: block-cyclic ownership leaves some ranks without blocks for some rows (LSE -inf);
    the window's partial last block (900 = 14 x 64 + 4 tokens) is the last local block of its
    owner."""
    res = _run(kv_shard_rank, world)
    o, q, k, v, ids = _inputs()
    ref, ref_lse = o.attention(q, k, v, ids, 64)
    for r in range(world):
        np.testing.assert_allclose(res[r][0], ref, rtol=1e-5, atol=1e-6)
        np.testing.assert_allclose(res[r][1], ref_lse, rtol=1e-6, atol=1e-6)


@pytest.mark.parametrize("world", [2, 3])
def test_kv_sharded_push_exchange_equals_full(world):
    """130 query rows over 3 owners: 44 + 44 + 42 (the last owner's buffers partly unused)."""
    res = _run(kv_push_rank, world)
    o, q, k, v, ids = _inputs()
    ref, ref_lse = o.attention(q, k, v, ids, 64)
    for r in range(world):
        np.testing.assert_allclose(res[r][0], ref, rtol=1e-5, atol=1e-6)
        np.testing.assert_allclose(res[r][1], ref_lse, rtol=1e-6, atol=1e-6)


def test_owner_rows():
    from streaming_sparse_b200.distributed import owner_rows
    assert [owner_rows(130, r, 3) for r in range(3)] == [(0, 44, 44), (44, 88, 44), (88, 130, 44)]
    assert [owner_rows(4680, r, 8)[:2] for r in range(8)][-1] == (4095, 4680)
    assert owner_rows(3, 3, 4) == (3, 3, 1)          # more owners than rows: an empty range
    for world in (1, 2, 3, 4, 8):
        spans = [owner_rows(4680, r, world) for r in range(world)]
        assert spans[0][0] == 0 and spans[-1][1] == 4680
        assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))


@pytest.mark.parametrize("world", [2, 3, 8])
def test_kv_sharded_history_keys_gather(world):
    """The history's key projections pooled by their owners and all-gathered are the whole
    window's, bit for bit (the router then runs identically on every rank)."""
    res = _run(kv_keys_rank, world)
    lens = []
    for r in range(world):
        table, whole, n = res[r]
        np.testing.assert_array_equal(table.view(np.uint32), whole.view(np.uint32))
        lens.append(n)
    assert sum(lens) == 900


@pytest.mark.parametrize("world", [2, 3])
def test_head_sharded_gather_equals_full(world):
    res = _run(head_shard_rank, world)
    o, q, k, v, ids = _inputs()
    ref, _ = o.attention(q, k, v, ids, 64)
    for r in range(world):
        np.testing.assert_allclose(res[r], ref, rtol=1e-6, atol=1e-7)


def test_local_window_geometry():
    from streaming_sparse_b200.distributed import local_ids, local_len, local_rows, owned_blocks
    # config 4 at 8 ranks: 34320 tokens in 128-token blocks -> 269 blocks, the last one 16 tokens
    Lk, block = 34320, 128
    assert sum(local_len(Lk, block, r, 8) for r in range(8)) == Lk
    last_owner = (268) % 8
    assert local_len(Lk, block, last_owner, 8) == (len(owned_blocks(269, last_owner, 8)) - 1) * 128 + 16
    rows = [local_rows(Lk, block, r, 8) for r in range(8)]
    assert torch.equal(torch.sort(torch.cat(rows)).values, torch.arange(Lk))
    ids = torch.tensor([[[0, 5, 8, 13, -1]]], dtype=torch.int32)
    assert local_ids(ids, 0, 8).tolist() == [[[0, -1, 1, -1, -1]]]
    assert local_ids(ids, 5, 8).tolist() == [[[-1, 0, -1, 1, -1]]]


def test_head_range_and_shard_ids():
    from streaming_sparse_b200.distributed import head_range, shard_ids
    assert [head_range(12, r, 4) for r in range(4)] == [(0, 3), (3, 6), (6, 9), (9, 12)]
    assert [head_range(12, r, 5) for r in range(5)] == [(0, 3), (3, 6), (6, 8), (8, 10), (10, 12)]
    ids = torch.tensor([[[0, 1, 2, 3, 4, 5, 6, -1]]], dtype=torch.int32)
    parts = [shard_ids(ids, r, 3) for r in range(3)]
    assert parts[0].tolist() == [[[0, -1, -1, 3, -1, -1, 6, -1]]]
    union = torch.stack(parts).max(0).values
    assert union.tolist() == ids.tolist()
