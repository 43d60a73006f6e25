"""INT8-QK path on the GPU: ss_quant_k_pages bit-exact to the oracle's page quantiser (and to the
reference kernel's golden int8 keys and scales); ss_attention_i8 against the oracle's INT8-QK
attention (exact int32 logits, float64 softmax) at the north-star tolerance, and against the
reference kernel's golden output (its P is fp16 where this kernel's is bf16)."""
import os

import numpy as np
import pytest
import torch

from helpers import assert_attention_close, np32, qkv, router_weights
from oracle import oracle

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")
GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "int8_qk.npz")


def _quant(k):
    from streaming_sparse_b200 import ops
    k_i8, ks = ops.quant_k_pages(k.to(DEV))
    torch.cuda.synchronize()
    return k_i8.cpu().numpy(), ks.cpu().numpy()


def _attend_i8(q, k, v, ids, block, out_dtype=torch.bfloat16, split=True):
    from streaming_sparse_b200 import ops
    k_i8, ks = ops.quant_k_pages(k.to(DEV))
    out, lse = ops.sparse_attention_i8(q.to(DEV), k_i8, ks, v.to(DEV), torch.as_tensor(ids).to(DEV), block=block,
                                       out_dtype=out_dtype, return_lse=True, validate=True, split=split)
    torch.cuda.synchronize()
    return out.float().cpu().numpy(), lse.cpu().numpy(), k_i8.cpu().numpy(), ks.cpu().numpy()


def _random_ids(rng, H, qb, kb, n, pad=0):
    ids = np.full((H, qb, n + pad), -1, np.int32)
    for h in range(H):
        for i in range(qb):
            ids[h, i, :n] = np.sort(np.concatenate([rng.choice(kb - 1, n - 1, replace=False), [kb - 1]]))
    return ids


@pytest.mark.parametrize("Lk,H", [(64, 1), (333, 2), (4680, 12), (32760, 3)])
def test_quant_k_pages_bit_exact(Lk, H):
    _, k, _ = qkv(5, 1, Lk, H)
    k[:64, 0] = 0                                   # an all-zero page
    k[min(70, Lk - 1), -1, 3] = 200.0                # an outlier sets its page's scale
    ki, ks = _quant(k)
    ri, rs = oracle.quant_rows(np32(k), oracle.QUANT_PAGE)
    assert np.array_equal(ki, ri)
    assert np.array_equal(ks.view(np.uint32), rs.view(np.uint32))


def test_quant_k_pages_ranges_equal_whole():
    from streaming_sparse_b200 import ops
    _, k, _ = qkv(6, 1, 4680 * 3, 2)
    kd = k.to(DEV)
    whole = ops.quant_k_pages(kd)
    npg = ops.quant_pages(kd.shape[0])
    hist = (kd.shape[0] - 4680) // 64
    part = ops.quant_k_pages(kd, p0=0, p1=hist)
    part = ops.quant_k_pages(kd, p0=hist, p1=npg, k_i8=part[0], ks=part[1])
    torch.cuda.synchronize()
    assert torch.equal(whole[0], part[0]) and torch.equal(whole[1], part[1])


def test_golden_reference_kernel():
    g = np.load(GOLD)
    k = torch.from_numpy(g["k"].transpose(1, 0, 2).copy()).bfloat16()
    q = torch.from_numpy(g["q"].transpose(1, 0, 2).copy()).bfloat16()
    v = torch.from_numpy(g["v"].transpose(1, 0, 2).copy()).bfloat16()   # bf16-exact values
    assert np.array_equal(np32(v), g["v"].transpose(1, 0, 2))
    out, lse, ki, ks = _attend_i8(q, k, v, g["page_lists"], 64, torch.float32)
    assert np.array_equal(ki, g["k_i8"].transpose(1, 0, 2))
    assert np.array_equal(ks.view(np.uint32), g["ks"].view(np.uint32))
    ref = g["out"].transpose(1, 0, 2)
    err = np.abs(out - ref)
    assert err.max() <= 1e-2 and err.mean() <= 1e-3, (err.max(), err.mean())


def test_golden_reference_kernel_128_token_blocks():
    """The reference kernel's output with 128-token routing blocks (int8_qk_b128.npz)."""
    g, g2 = np.load(GOLD), np.load(GOLD.replace("int8_qk.npz", "int8_qk_b128.npz"))
    k = torch.from_numpy(g["k"].transpose(1, 0, 2).copy()).bfloat16()
    v = torch.from_numpy(g["v"].transpose(1, 0, 2).copy()).bfloat16()
    q = torch.from_numpy(g2["q"].transpose(1, 0, 2).copy()).bfloat16()
    out, _, ki, ks = _attend_i8(q, k, v, g2["block_lists"], 128, torch.float32)
    assert np.array_equal(ki, g["k_i8"].transpose(1, 0, 2))
    err = np.abs(out - g2["out"].transpose(1, 0, 2))
    assert err.max() <= 1e-2 and err.mean() <= 1e-3, (err.max(), err.mean())


@pytest.mark.parametrize("Lq,Lk,H,block,n,pad,out_dtype", [
    (100, 333, 2, 64, 3, 2, torch.bfloat16),      # partial tile, partial last page, -1 padding
    (256, 1024, 3, 64, 7, 0, torch.float32),      # two full tiles, fp32 out
    (300, 1000, 2, 128, 4, 1, torch.bfloat16),    # 128-token router blocks (two pages per id)
    (64, 4096, 1, 64, 64, 0, torch.float32),      # every block listed: 64 steps
    (1, 65, 1, 64, 2, 0, torch.float32),          # one query row, a 1-token last page
])
@pytest.mark.parametrize("split", [True, False])
def test_attention_i8_random_lists(Lq, Lk, H, block, n, pad, out_dtype, split):
    """split: these small problems cut every tile into pieces (some of them empty) merged by LSE;
    without it each tile is one CTA."""
    q, k, v = qkv(13, Lq, Lk, H)
    rng = np.random.default_rng(Lq + Lk)
    ids = _random_ids(rng, H, oracle.nblocks(Lq, block), oracle.nblocks(Lk, block), n, pad)
    out, lse, ki, ks = _attend_i8(q, k, v, ids, block, out_dtype, split)
    ref, ref_lse = oracle.attention_i8(np32(q), ki, ks, np32(v), ids, block)
    assert_attention_close(out, ref)
    assert np.abs(lse - ref_lse).max() <= 2e-3


def test_attention_i8_routed_and_empty_lists():
    """Router ids over a two-chunk window, one query block with an empty list (zeros, LSE -inf)."""
    from streaming_sparse_b200 import ops
    Lq, Lk, H = 300, 1200, 2
    q, k, v = qkv(17, Lq, Lk, H)
    wq, wk = router_weights(17, H)
    ids = ops.route(q.to(DEV), k.to(DEV), wq.to(DEV), wk.to(DEV), block=64, extra=3, validate=True).cpu().numpy()
    ids[1, 2] = -1
    for split in (True, False):
        out, lse, ki, ks = _attend_i8(q, k, v, ids, 64, torch.float32, split)
        ref, ref_lse = oracle.attention_i8(np32(q), ki, ks, np32(v), ids, 64)
        assert np.all(out[128:192, 1] == 0) and np.all(np.isneginf(lse[1, 128:192]))
        assert_attention_close(out, ref)


def test_attention_i8_config2_sampled():
    """Config 2's chunk-layer (4680 queries, 32760-token window, 12 heads, block 64, 25 % of the
    blocks): every head, 8 query blocks each, against the oracle; the whole output against the
    bf16 kernel (int8 quantisation error only)."""
    from streaming_sparse_b200 import ops
    Lq, Lk, H = 4680, 32760, 12
    q, k, v = qkv(21, Lq, Lk, H)
    wq, wk = router_weights(21, H)
    qd, kd, vd = q.to(DEV), k.to(DEV), v.to(DEV)
    kb = oracle.nblocks(Lk, 64)
    extra = ops.budget(kb, ops.forced_count(Lq, Lk, 64), density=0.25)
    ids = ops.route(qd, kd, wq.to(DEV), wk.to(DEV), block=64, extra=extra, validate=True)
    k_i8, ks = ops.quant_k_pages(kd)
    out = ops.sparse_attention_i8(qd, k_i8, ks, vd, ids, block=64, out_dtype=torch.float32, validate=True)
    dense = ops.sparse_attention(qd, kd, vd, ids, block=64, out_dtype=torch.float32, validate=True)
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    qblocks = [0, 9, 18, 36, 45, 54, 63, 73]
    ref, _ = oracle.attention_i8(np32(q), k_i8.cpu().numpy(), ks.cpu().numpy(), np32(v), ids.cpu().numpy(), 64,
                                 qblocks=qblocks)
    assert_attention_close(got, ref)
    d = (out - dense).abs()
    assert float(d.mean()) < 5e-3, float(d.mean())
    # 444 tiles: the default call cuts them in pieces (each piece rounds P against its own running
    # maximum); the whole-tile call meets the same bound
    whole = ops.sparse_attention_i8(qd, k_i8, ks, vd, ids, block=64, out_dtype=torch.float32, split=False)
    assert ops.attention_i8_workspace_bytes(H, Lq) > 0
    assert_attention_close(whole.cpu().numpy(), ref)


@pytest.mark.parametrize("local,sink,block", [(-1, 0, 64), (5, 1, 128)])
def test_plugin_int8_stream_reuses_history_pages(local, sink, block):
    """RouterConfig(int8=True) through a KVCache stream (three calls per chunk, each rewriting the
    chunk's rows; a roll of the window; an anchor rebase): the attached plugin quantises the
    history's pages once per window and equals, bit for bit, a plugin that quantises every page on
    every call; both stay within the int8 rounding of the bf16 path."""
    from streaming_sparse_b200 import ops
    from streaming_sparse_b200.cache import KVCache
    from streaming_sparse_b200.plugin import RouterConfig, SparseAttention
    H, ftok, fpc, chunks = 2, 300, 2, 5
    cap = (local if local != -1 else fpc * chunks) * ftok
    cache = KVCache(cap, num_heads=H, frame_tokens=ftok, local_attn_size=local, sink_size=sink, device=DEV)
    wq, wk = router_weights(12, H)
    cfg = RouterConfig(block=block, density=0.3, rule="rest" if sink else "total", sink_tokens=sink * ftok, int8=True)
    sp = SparseAttention(wq.to(DEV), wk.to(DEV), cfg)
    ref = SparseAttention(wq.to(DEV), wk.to(DEV), cfg)      # never attached: quantises every page per call
    bf = SparseAttention(wq.to(DEV), wk.to(DEV), RouterConfig(block=block, density=0.3, rule=cfg.rule,
                                                             sink_tokens=cfg.sink_tokens))
    sp.attach(cache)
    g = torch.Generator().manual_seed(4)
    n = fpc * ftok
    for c in range(chunks):
        for step in range(3):
            kn = torch.randn((n, H, 128), generator=g).bfloat16().to(DEV)
            vn = torch.randn((n, H, 128), generator=g).bfloat16().to(DEV)
            q = torch.randn((n, H, 128), generator=g).bfloat16().to(DEV)
            cache.append(kn, vn, c * n)
            if c == 3 and step == 1 and sink:
                cache.save_anchor()
                cache.rebase_anchor(1)
            kw, vw = cache.window()
            got = sp.forward_one(q, kw, vw).clone()
            want = ref.forward_one(q, kw, vw)
            dense = bf.forward_one(q, kw, vw)
            torch.cuda.synchronize()
            assert torch.equal(got, want), (c, step)
            d = (got.float() - dense.float())
            assert float((d * d).sum() / (dense.float() ** 2).sum()) < 2e-3
    ops.DeviceStatus.check(DEV)


@pytest.mark.parametrize("block,density", [(64, 0.05), (128, 0.5)])
def test_attention_i8_config5_long_window(block, density):
    """Config 5's longest window (98280 tokens = 1536 pages, 4680 queries): the largest page lists
    the benched shapes give a tile, two heads, sampled query blocks against the oracle."""
    from streaming_sparse_b200 import ops
    Lq, Lk, H = 4680, 98280, 2
    q, k, v = qkv(31, Lq, Lk, H)
    wq, wk = router_weights(31, H)
    qd, kd, vd = q.to(DEV), k.to(DEV), v.to(DEV)
    kb = oracle.nblocks(Lk, block)
    extra = ops.budget(kb, ops.forced_count(Lq, Lk, block), density=density)
    ids = ops.route(qd, kd, wq.to(DEV), wk.to(DEV), block=block, extra=extra, validate=True)
    k_i8, ks = ops.quant_k_pages(kd)
    out = ops.sparse_attention_i8(qd, k_i8, ks, vd, ids, block=block, out_dtype=torch.float32, validate=True)
    torch.cuda.synchronize()
    nqb = oracle.nblocks(Lq, block)
    qblocks = sorted({0, nqb // 3, nqb // 2, nqb - 1})
    ref, _ = oracle.attention_i8(np32(q), k_i8.cpu().numpy(), ks.cpu().numpy(), np32(v), ids.cpu().numpy(), block,
                                 qblocks=qblocks)
    assert_attention_close(out.cpu().numpy(), ref)


@pytest.mark.parametrize("block", [64, 128])
def test_plugin_int8_ring_cache_equals_shifting_cache(block):
    """RouterConfig(int8=True) streaming through a ring-buffer KVCache (a roll moves the head) and
    through the shifting cache: the int8 keys, scales and outputs are the same, bit for bit, at
    every call, over rolls of the window."""
    from streaming_sparse_b200 import ops
    from streaming_sparse_b200.cache import KVCache
    from streaming_sparse_b200.plugin import RouterConfig, SparseAttention
    H, ftok, local, sink = 2, 300, 5, 1
    cfg = RouterConfig(block=block, density=0.3, rule="rest", sink_tokens=sink * ftok, int8=True)
    wq, wk = (w.to(DEV) for w in router_weights(16, H))
    caches = [KVCache(local * ftok, H, 128, frame_tokens=ftok, local_attn_size=local, sink_size=sink, device=DEV,
                      ring=r) for r in (False, True)]
    sps = [SparseAttention(wq, wk, cfg) for _ in caches]
    for sp, cache in zip(sps, caches):
        sp.attach(cache)
    g = torch.Generator().manual_seed(2)
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
            torch.cuda.synchronize()
            assert torch.equal(sps[0].last_ids, sps[1].last_ids)
            assert torch.equal(outs[0], outs[1]), c
            assert torch.equal(sps[0]._i8[caches[0]][1], sps[1]._i8[caches[1]][1])   # page scales
    assert caches[1].ring.head != 0
    ops.DeviceStatus.check(DEV)
