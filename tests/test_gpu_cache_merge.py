"""KV-cache append/evict and the LSE merge on the GPU against the oracle and reference fixtures."""
import numpy as np
import pytest
import torch

from helpers import np32

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")


def test_cache_known_answer_on_gpu():
    """evaluation/validate.py:57-88 schedule: visible positions [0..3] + [16..35] after 3 chunks."""
    from streaming_sparse_b200.cache import KVCache
    c = KVCache(24, num_heads=1, frame_tokens=4, local_attn_size=6, sink_size=1, device=DEV)
    for chunk in range(3):
        for _ in range(3):
            start = chunk * 12
            tok = torch.arange(start, start + 12, device=DEV, dtype=torch.float32)
            kv = tok[:, None, None].expand(12, 1, 128).to(torch.bfloat16).contiguous()
            vis, hist = c.append(kv, kv, start)
    k, v = c.window()
    expected = list(range(4)) + list(range(16, 36))
    np.testing.assert_array_equal(k[:, 0, 0].float().cpu().numpy(), expected)
    np.testing.assert_array_equal(vis, expected)
    assert hist == 12


@pytest.mark.parametrize("local,sink,frames_per_chunk,chunks,strided",
                         [(5, 1, 2, 9, False), (-1, 0, 3, 3, False), (4, 0, 1, 10, False), (5, 1, 2, 9, True)])
def test_cache_matches_oracle(oracle, local, sink, frames_per_chunk, chunks, strided):
    """Append/evict against the oracle's roll. `strided`: the chunk's k/v are row-strided views
    (slices of a fused [n, 3, H, 128] projection output), so the chunk write takes the strided copy
    while the window shifts take the contiguous one."""
    from streaming_sparse_b200.cache import KVCache
    H, ftok = 3, 70                      # 70-token frames: rows never align with 16-byte vector groups of rows
    cap = (local if local != -1 else frames_per_chunk * chunks) * ftok
    c = KVCache(cap, num_heads=H, frame_tokens=ftok, local_attn_size=local, sink_size=sink, device=DEV)
    ok, ov = np.zeros((cap, H, 128), np.float32), np.zeros((cap, H, 128), np.float32)
    ge = le = 0
    g = torch.Generator().manual_seed(0)
    n = frames_per_chunk * ftok
    for chunk in range(chunks):
        for step in range(2):
            start = chunk * n
            kn = torch.randn((n, H, 128), generator=g).bfloat16()
            vn = torch.randn((n, H, 128), generator=g).bfloat16()
            if strided:
                fused = torch.zeros((n, 3, H, 128), dtype=torch.bfloat16, device=DEV)
                fused[:, 1], fused[:, 2] = kn.to(DEV), vn.to(DEV)
                c.append(fused[:, 1], fused[:, 2], start)
            else:
                c.append(kn.to(DEV), vn.to(DEV), start)
            le = oracle.cache_append(ok, ov, np32(kn), np32(vn), local_attn=local != -1, global_end=ge,
                                     local_end=le, current_start=start, sink_tokens=sink * ftok)
            ge = start + n
            assert c.local_end == le and c.global_end == ge
            np.testing.assert_array_equal(c.k[0].float().cpu().numpy()[:le], ok[:le])
            np.testing.assert_array_equal(c.v[0].float().cpu().numpy()[:le], ov[:le])


def test_merge_matches_reference_fixture(golden):
    from streaming_sparse_b200 import ops
    g = golden("merge_vr1.npz")
    eo, el = torch.from_numpy(g["exact"]).to(DEV), torch.from_numpy(g["exact_lse"]).to(DEV)
    ap, al = torch.from_numpy(g["approx"]).to(DEV), torch.from_numpy(g["approx_lse"]).to(DEV)
    out = ops.merge(eo, el, ap, al).float().cpu().numpy()
    np.testing.assert_allclose(out, g["out"], rtol=0, atol=1.6e-2)
    assert np.abs(out - g["out"]).mean() < 1e-3


def test_lse_merge_many_parts(oracle):
    from streaming_sparse_b200 import ops
    g = torch.Generator().manual_seed(2)
    P, Lq, H = 5, 77, 3
    o = torch.randn((P, Lq, H, 128), generator=g)
    l = torch.randn((P, H, Lq), generator=g) * 4
    l[2, 1, :10] = -float("inf")
    l[:, 0, 5] = -float("inf")           # a row with every part empty
    out, lse = ops.lse_merge(o.to(DEV), l.to(DEV), out_dtype=torch.float32, return_lse=True)
    ref, ref_lse = oracle.lse_merge(o.numpy(), l.numpy())
    ref[5, 0] = 0.0
    np.testing.assert_allclose(out.cpu().numpy(), ref, rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(lse.cpu().numpy(), ref_lse, rtol=1e-5, atol=1e-5)


def test_split_blocks_then_merge_equals_whole(oracle):
    """Attention over a block list == LSE merge of attention over a partition of that list
    (the exchange step of KV-block sharding)."""
    from helpers import qkv
    from streaming_sparse_b200 import ops
    from streaming_sparse_b200.distributed import shard_ids
    Lq, Lk, H = 256, 4096, 2
    q, k, v = qkv(21, Lq, Lk, H)
    rng = np.random.default_rng(21)
    ids = np.stack([np.stack([np.sort(rng.choice(64, 20, replace=False)) for _ in range(4)]) for _ in range(H)])
    ids = torch.from_numpy(ids.astype(np.int32)).to(DEV)
    qd, kd, vd = q.to(DEV), k.to(DEV), v.to(DEV)
    whole = ops.sparse_attention(qd, kd, vd, ids, out_dtype=torch.float32)
    parts, lses = [], []
    for r in range(3):
        o, l = ops.sparse_attention(qd, kd, vd, shard_ids(ids, r, 3), out_dtype=torch.float32, return_lse=True)
        parts.append(o)
        lses.append(l)
    merged = ops.lse_merge(torch.stack(parts), torch.stack(lses), out_dtype=torch.float32)
    torch.testing.assert_close(merged, whole, rtol=2e-3, atol=2e-3)


def _bf16_bits(a):
    return torch.from_numpy(a.astype(np.int16)).view(torch.bfloat16)


def test_rope_shift_matches_reference_fixture(golden):
    """ss_cache_rope_shift == the reference's shift_temporal_ (anchor_rebase.npz), bit for bit."""
    from streaming_sparse_b200 import ops
    from streaming_sparse_b200.cache import temporal_phase
    g = golden("anchor_rebase.npz")
    keys = _bf16_bits(g["keys"]).cuda()                       # [2, 64, 2, 128]
    for name in g.files:
        if not name.startswith("out_"):
            continue
        _, offset, tokens = name.split("_")
        t = int(tokens)
        out = keys.clone()
        for layer in range(keys.shape[0]):
            if t:
                ops.rope_shift(keys[layer, :t], out[layer, :t], temporal_phase(int(offset), "cuda"))
        exp = _bf16_bits(g[name])
        assert torch.equal(out.cpu().view(torch.int16), exp.view(torch.int16)), name


def test_anchor_rebase_and_snapshot_restore():
    from streaming_sparse_b200.cache import KVCache
    dev = torch.device("cuda:0")
    g = torch.Generator(device=dev).manual_seed(5)
    c = KVCache(64 * 8, 2, 128, frame_tokens=64, local_attn_size=6, sink_size=1, device=dev)
    for start in range(0, 64 * 6, 64):
        k = torch.randn(64, 2, 128, device=dev, generator=g).bfloat16()
        c.append(k, k.neg(), start)
    snap = c.snapshot()
    c.save_anchor()
    canonical = c.anchor.clone()
    assert canonical.shape[0] == 64                      # the sink frame
    c.rebase_anchor(9)
    moved = c.k[0, :64].clone()
    assert not torch.equal(moved, canonical)
    assert torch.equal(moved[..., 44:], canonical[..., 44:])   # spatial pairs untouched
    c.rebase_anchor(0)
    assert torch.equal(c.k[0, :64], canonical)
    # one more chunk, then restore brings back the rows and the index state
    k = torch.randn(64, 2, 128, device=dev, generator=g).bfloat16()
    c.append(k, k, 64 * 6)
    assert c.global_end == 64 * 7
    c.restore(snap)
    assert (c.global_end, c.local_end) == (snap["global_end"], snap["local_end"])
    assert torch.equal(c.k[0, :c.local_end], snap["k"]) and torch.equal(c.v[0, :c.local_end], snap["v"])


@pytest.mark.parametrize("P,part_dtype,rows", [(3, torch.float32, (0, 700)), (2, torch.bfloat16, (100, 333)),
                                               (8, torch.bfloat16, (0, 700))])
def test_lse_merge_peers_equals_lse_merge(P, part_dtype, rows):
    """ss_lse_merge_peers with every part local (the pointers a rank passes for its own part): the
    values of ss_lse_merge bit for bit, for the rows asked and nothing else; empty parts (-inf)
    and a row with every part empty included."""
    import ctypes
    from streaming_sparse_b200 import ops
    from streaming_sparse_b200._lib import lib
    Lq, H = 700, 3
    g = torch.Generator(device=DEV).manual_seed(9)
    o = torch.randn((P, Lq, H, 128), generator=g, device=DEV).to(part_dtype)
    lse = 3 * torch.randn((P, H, Lq), generator=g, device=DEV)
    lse[0, :, 5] = float("-inf")
    lse[:, 1, 7] = float("-inf")
    want, want_lse = ops.lse_merge(o.float(), lse, out_dtype=torch.float32, return_lse=True)
    out = torch.full((Lq, H, 128), 7.0, device=DEV)
    lse_out = torch.full((H, Lq), 7.0, device=DEV)
    optr = (ctypes.c_void_p * P)(*[o[p].data_ptr() for p in range(P)])
    lptr = (ctypes.c_void_p * P)(*[lse[p].data_ptr() for p in range(P)])
    r0, r1 = rows
    rc = lib().ss_lse_merge_peers(optr, lptr, P, 1 if part_dtype == torch.float32 else 0, H, Lq, r0, r1,
                                  ctypes.c_void_p(out.data_ptr()), 1, ctypes.c_void_p(lse_out.data_ptr()),
                                  ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 0
    torch.cuda.synchronize()
    assert torch.equal(out[r0:r1], want[r0:r1])
    assert torch.equal(lse_out[:, r0:r1], want_lse[:, r0:r1])
    assert (out[:r0] == 7).all() and (out[r1:] == 7).all()


def test_peer_barrier_single_rank_advances_epoch():
    """A one-rank barrier posts into its own flags only (no wait on another launch): the device
    epoch counter advances by one per call and the status word stays clear."""
    import ctypes
    from streaming_sparse_b200._lib import lib
    flags = torch.zeros(1, dtype=torch.int32, device=DEV)
    epoch = torch.zeros(1, dtype=torch.int32, device=DEV)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    ptrs = (ctypes.c_void_p * 1)(flags.data_ptr())
    for _ in range(3):
        assert lib().ss_peer_barrier(ptrs, 0, 1, ctypes.c_void_p(epoch.data_ptr()), ctypes.c_void_p(status.data_ptr()),
                                     ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)) == 0
    torch.cuda.synchronize()
    assert int(epoch.item()) == 3 and int(flags.item()) == 3 and int(status.item()) == 0
