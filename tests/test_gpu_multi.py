"""The multi-GPU layouts on real GPUs: NCCL ranks (one process per GPU, spawned), KV-block sharding
(each rank stores its own blocks, the history keys all-gathered at commit, the partials pushed
to their rows' owners by the attention epilogue and merged there, or pulled and merged over peer
memory) and head sharding with the all_gather, each against the single-GPU result; the
fused head gather (the attention epilogue storing every rank's heads into all ranks' buffers over
NVLink) against the all_gather, bit for bit, through both output slots, in the split mode and
with an uneven head split.
Skipped where fewer than two GPUs are visible."""
import datetime
import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

LQ, LK, H = 1024, 8192, 4


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _inputs():
    from helpers import qkv, router_weights
    q, k, v = qkv(31, LQ, LK, H)
    wq, wk = router_weights(31, H)
    return q, k, v, wq, wk


def _worker(rank, world, port, q_out):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    try:
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                                device_id=dev)
        from streaming_sparse_b200 import ops
        from streaming_sparse_b200.distributed import HeadShardedAttention, KVShardedAttention, head_shard
        from streaming_sparse_b200.plugin import RouterConfig, SparseAttention
        q, k, v, wq, wk = (t.to(dev) for t in _inputs())
        cfg = RouterConfig(density=0.25)
        c0 = LK - LQ
        outs_by = {}
        for exchange in ("push", "pull"):
            shard = KVShardedAttention(SparseAttention(wq, wk, cfg), LQ, LK, dev, exchange=exchange)
            shard.commit(k, v)
            # three calls: with "pull" both partial slots, then the first again
            outs_by[exchange] = [shard(q, k[c0:], v[c0:]).clone() for _ in range(3)]
            ids = shard.last_ids.cpu().numpy()
            torch.cuda.synchronize()
            dist.barrier()
            shard.close()
        outs = outs_by["push"]
        push_eq_pull = all(torch.equal(a, b) for a, b in zip(outs_by["push"], outs_by["pull"]))
        hs = HeadShardedAttention(SparseAttention(head_shard(wq, rank, world, 0), head_shard(wk, rank, world, 0), cfg),
                                  H)(head_shard(q, rank, world), head_shard(k, rank, world), head_shard(v, rank, world))
        fused_ok = []
        # (Lq, Lk, heads): 16 tiles per rank; 150 (the split mode, one to two tiles per SM); and
        # 3 heads, split 2 + 1 (uneven ranks, as 12 heads over 8 GPUs)
        for lq, lk, nh in ((LQ, LK, H), (9600, 12800, H), (LQ, LK, 3)):
            g = torch.Generator().manual_seed(lq + nh)
            fq, fk, fv = (torch.randn((n, nh, 128), generator=g).bfloat16().to(dev) for n in (lq, lk, lk))
            hwq, hwk = wq[:nh].contiguous(), wk[:nh].contiguous()
            sps = [SparseAttention(head_shard(hwq, rank, world, 0), head_shard(hwk, rank, world, 0), cfg)
                   for _ in range(2)]
            args = (head_shard(fq, rank, world), head_shard(fk, rank, world), head_shard(fv, rank, world))
            want = HeadShardedAttention(sps[0], nh)(*args)
            fused = HeadShardedAttention(sps[1], nh, Lq=lq, device=dev)
            got = [fused(*args).clone() for _ in range(3)]       # both output slots, then the first again
            torch.cuda.synchronize()
            fused_ok.append(all(torch.equal(x, want) for x in got))
            dist.barrier()
            fused.close()
        torch.cuda.synchronize()
        ops.DeviceStatus.check(dev)
        same = all(torch.equal(outs[0], o_) for o_ in outs[1:])
        q_out.put((rank, (outs[0].float().cpu().numpy(), ids, same and push_eq_pull, fused_ok),
                   hs.float().cpu().numpy()))
        dist.barrier()
        dist.destroy_process_group()
    except Exception as e:   # report to the parent instead of hanging it
        q_out.put((rank, repr(e), None))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_kv_and_head_sharding_on_two_gpus_match_one_gpu():
    import torch.multiprocessing as mp
    from streaming_sparse_b200.plugin import RouterConfig, SparseAttention
    from helpers import assert_attention_close

    ctx = mp.get_context("spawn")
    q_out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q_out)) for r in range(2)]
    for p in procs:
        p.start()
    results = {}
    try:
        for _ in procs:
            rank, kv, hs = q_out.get(timeout=240)
            results[rank] = (kv, hs)
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():      # a rank that never reported: end it rather than leave it running
                p.terminate()
                p.join(timeout=30)
    assert len(results) == 2
    for rank, (kv, hs) in results.items():
        assert not isinstance(kv, str), f"rank {rank}: {kv}"
    # the single-GPU path, same inputs
    dev = torch.device("cuda:0")
    q, k, v, wq, wk = (t.to(dev) for t in _inputs())
    sp = SparseAttention(wq, wk, RouterConfig(density=0.25))
    whole = sp(q[None], k[None], v[None])[0].float().cpu().numpy()
    whole_ids = sp.last_ids.cpu().numpy()
    for rank, ((kv, ids, same, fused_ok), hs) in results.items():
        assert fused_ok == [True, True, True], f"rank {rank}: fused head gather differs from the all_gather"
        np.testing.assert_array_equal(ids, whole_ids)          # the sharded router: same ids, bit for bit
        assert same                                            # repeated calls; push == pull, bit for bit
        assert_attention_close(kv, whole)                       # KV-block shards merged by LSE
        np.testing.assert_array_equal(hs, whole)               # heads are independent: identical bits


def _rollout_cfg(ring: bool):
    from streaming_sparse_b200 import rollout as R
    return R.WanConfig(dim=512, ffn_dim=1024, num_heads=4, num_layers=2, text_dim=64, text_len=16, latent_h=16,
                       latent_w=12, frames=12, cache_frames=7, local_attn_frames=7, sink_frames=1, ring_cache=ring)


def _rollout_inputs(cfg, dev):
    g = torch.Generator(device=dev)
    noise = torch.randn(cfg.frames, 16, cfg.latent_h, cfg.latent_w, device=dev, generator=g.manual_seed(3))
    text = torch.randn(10, cfg.text_dim, device=dev, generator=g.manual_seed(4))
    return noise, text, g


def _run_rollout(cfg, dev, head_parallel: bool):
    """Eager run, then capture, then replay; returns (eager, replayed) latents on the CPU."""
    from streaming_sparse_b200 import rollout as R
    from streaming_sparse_b200.plugin import RouterConfig, SparseAttention, init_router_weights
    m = R.build_model(cfg, device=dev)
    wq, wk = init_router_weights(cfg.num_heads, device=dev)
    sp = SparseAttention(wq, wk, RouterConfig(density=0.5, sink_tokens=cfg.frame_tokens))
    ro = R.Rollout(m, sparse=sp, graphs=True, head_parallel=head_parallel)
    noise, text, g = _rollout_inputs(cfg, dev)
    eager = ro.run(noise, text, generator=g.manual_seed(5))
    ro.run(noise, text, generator=g.manual_seed(5))            # captures
    replayed = ro.run(noise, text, generator=g.manual_seed(5))
    torch.cuda.synchronize()
    res = (eager.float().cpu(), replayed.float().cpu())
    ro.close()
    return res


def _rollout_worker(rank, world, port, q_out):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    try:
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                                device_id=dev)
        from streaming_sparse_b200 import ops
        runs = {}
        for ring in (False, True):
            runs[ring] = _run_rollout(_rollout_cfg(ring), dev, head_parallel=True)
            dist.barrier()
        ops.DeviceStatus.check(dev)
        q_out.put((rank, runs))
        dist.barrier()
        dist.destroy_process_group()
    except Exception as e:   # report to the parent instead of hanging it
        q_out.put((rank, repr(e)))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_head_parallel_rollout_on_two_gpus_matches_one_gpu():
    """Config 4's stream shape in miniature (rolling window with a sink frame, shifting and ring
    caches) with the attention split by heads over two GPUs: each rank's caches hold its two of
    the four heads, the fused kernel writes only those, and every layer's attention output
    reaches both ranks through the fused head gather. No tile is split at this size, so every
    head's arithmetic is the single GPU's: the latents are equal bit for bit, eager and replayed
    from CUDA graphs."""
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q_out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rollout_worker, args=(r, 2, port, q_out)) for r in range(2)]
    for p in procs:
        p.start()
    results = {}
    try:
        for _ in procs:
            rank, runs = q_out.get(timeout=300)
            results[rank] = runs
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.terminate()
                p.join(timeout=30)
    assert len(results) == 2
    for rank, runs in results.items():
        assert not isinstance(runs, str), f"rank {rank}: {runs}"
    dev = torch.device("cuda:0")
    for ring in (False, True):
        eager, replayed = _run_rollout(_rollout_cfg(ring), dev, head_parallel=False)
        for rank in (0, 1):
            hp_eager, hp_replayed = results[rank][ring]
            assert torch.isfinite(hp_eager).all()
            assert torch.equal(hp_eager, eager), f"ring={ring} rank {rank}: eager latents differ"
            assert torch.equal(hp_replayed, replayed), f"ring={ring} rank {rank}: replayed latents differ"
