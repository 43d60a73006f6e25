"""Rollout harness: the model pieces against restatements of the reference's formulas (CPU), and a
small streaming rollout on the GPU (sparse plugin with every block kept == dense model; a routed
rollout stays finite and routes every denoising layer call)."""
import math

import pytest
import torch

from streaming_sparse_b200 import ops
from streaming_sparse_b200 import rollout as R

TINY = R.WanConfig(dim=256, ffn_dim=512, num_heads=2, num_layers=2, text_dim=64, text_len=16, latent_h=16,
                   latent_w=16, frames=6, cache_frames=6)


def _complex_rope(x, f, h, w, angles, start_frame):
    """wan/modules/causal_model.py:27-55 restated: complex multiply in float64."""
    n, H, D = x.shape
    c = D // 2
    parts = torch.polar(torch.ones_like(angles), angles).split([c - 2 * (c // 3), c // 3, c // 3], dim=1)
    fr = torch.cat([parts[0][start_frame:start_frame + f].view(f, 1, 1, -1).expand(f, h, w, -1),
                    parts[1][:h].view(1, h, 1, -1).expand(f, h, w, -1),
                    parts[2][:w].view(1, 1, w, -1).expand(f, h, w, -1)], dim=-1).reshape(n, 1, -1)
    xc = torch.view_as_complex(x.double().reshape(n, H, -1, 2))
    return torch.view_as_real(xc * fr).flatten(2)


def test_rope_matches_complex_form():
    g = torch.Generator().manual_seed(0)
    f, h, w, H = 3, 4, 5, 2
    x = torch.randn(f * h * w, H, 128, generator=g)
    ang = R.rope_angles()
    for start in (0, 6, 18):
        cos, sin = R.rope_tables(ang, start, f, h, w, "cpu")
        got = R.apply_rope(x, cos, sin)
        ref = _complex_rope(x, f, h, w, ang, start)
        assert (got.double() - ref).abs().max() < 1e-5


def test_rope_split_is_22_21_21():
    ang = R.rope_angles()
    assert ang.shape == (1024, 64)
    # frame part: theta^(-2i/44); height/width parts: theta^(-2i/42)
    assert torch.allclose(ang[1, :22], 1.0 / torch.pow(10000, torch.arange(0, 44, 2, dtype=torch.float64) / 44))
    assert torch.allclose(ang[1, 22:43], 1.0 / torch.pow(10000, torch.arange(0, 42, 2, dtype=torch.float64) / 42))


def test_patchify_is_the_strided_conv_and_unpatchify_inverts_the_layout():
    m = R.build_model(TINY, device="cpu").float()
    g = torch.Generator().manual_seed(1)
    x = torch.randn(16, 3, 16, 16, generator=g)
    tok = m.patchify(x)
    conv = torch.nn.functional.conv3d(x[None], m.patch, m.patch_b, stride=(1, 2, 2))[0].flatten(1).t()
    assert (tok - conv).abs().max() < 1e-4
    # unpatchify: u.view(f,h,w,1,2,2,c) -> einsum('fhwpqrc->cfphqwr') (causal_model.py:1045-1050)
    u = torch.randn(3 * 8 * 8, 64, generator=g)
    out = m.unpatchify(u, 3)
    ref = torch.einsum("fhwpqrc->cfphqwr", u.view(3, 8, 8, 1, 2, 2, 16)).reshape(16, 3, 16, 16)
    assert torch.equal(out, ref)


def test_flow_schedule_and_warped_steps():
    fm = R.FlowMatch()
    assert fm.denoising == [1000.0, 937.5, 833.3333333333334, 625.0]
    assert fm.sigma(1000.0) == 1.0 and abs(fm.sigma(625.0) - 0.625) < 1e-12
    x0, eps = torch.randn(4, dtype=torch.float64), torch.randn(4, dtype=torch.float64)
    xt = fm.add_noise(x0, eps, 937.5)
    s = 0.9375
    assert torch.allclose(xt, (1 - s) * x0 + s * eps)
    assert torch.allclose(fm.to_x0(eps - x0, xt, 937.5), x0)   # flow target = noise - x0


def test_sinusoidal_embedding():
    t = torch.tensor([0.0, 625.0])
    e = R.sinusoidal_embedding(256, t)
    k = torch.arange(128, dtype=torch.float64)
    ang = 625.0 * torch.pow(10000, -k / 128)
    assert torch.allclose(e[1], torch.cat([torch.cos(ang), torch.sin(ang)]))
    assert torch.equal(e[0, :128], torch.ones(128, dtype=torch.float64))


@pytest.mark.gpu
def test_rollout_dense_plugin_matches_dense_model():
    from streaming_sparse_b200.plugin import RouterConfig, SparseAttention, init_router_weights

    dev = torch.device("cuda:0")
    m = R.build_model(TINY, device=dev)
    g = torch.Generator(device=dev)
    noise = torch.randn(TINY.frames, 16, 16, 16, device=dev, generator=g.manual_seed(3))
    text = torch.randn(10, TINY.text_dim, device=dev, generator=g.manual_seed(4))
    dense = R.Rollout(m).run(noise, text, generator=g.manual_seed(5))
    wq, wk = init_router_weights(TINY.num_heads, device=dev)
    sp = SparseAttention(wq, wk, RouterConfig(density=1.0))
    routed = R.Rollout(m, sparse=sp).run(noise, text, generator=g.manual_seed(5))
    assert torch.isfinite(routed).all()
    err = (routed - dense).abs()
    # bf16 model: the two attention paths differ only by rounding
    assert err.max() < 0.15 and err.mean() < 5e-3, (err.max().item(), err.mean().item())


@pytest.mark.gpu
def test_rollout_routes_every_denoising_call():
    from streaming_sparse_b200.plugin import RouterConfig, SparseAttention, init_router_weights

    dev = torch.device("cuda:0")
    m = R.build_model(TINY, device=dev)
    g = torch.Generator(device=dev)
    noise = torch.randn(TINY.frames, 16, 16, 16, device=dev, generator=g.manual_seed(3))
    text = torch.randn(10, TINY.text_dim, device=dev, generator=g.manual_seed(4))
    wq, wk = init_router_weights(TINY.num_heads, device=dev)
    sp = SparseAttention(wq, wk, RouterConfig(density=0.25))
    ro = R.Rollout(m, sparse=sp)
    out = ro.run(noise, text, generator=g.manual_seed(5))
    assert torch.isfinite(out).all()
    chunks = math.ceil(TINY.frames / TINY.frames_per_chunk)
    assert sp.calls == chunks * 5 * TINY.num_layers       # 4 denoising + 1 context pass per chunk
    # the plugin is removed after the rollout
    assert R.attention.__name__ == "attention"
    # the cache holds every frame: the last window covers the whole rollout
    assert ro.caches[0].local_end == TINY.frames * TINY.frame_tokens


@pytest.mark.gpu
def test_rollout_graph_replay_matches_eager():
    from streaming_sparse_b200.plugin import RouterConfig, SparseAttention, init_router_weights

    dev = torch.device("cuda:0")
    m = R.build_model(TINY, device=dev)
    g = torch.Generator(device=dev)
    noise = torch.randn(TINY.frames, 16, 16, 16, device=dev, generator=g.manual_seed(3))
    text = torch.randn(10, TINY.text_dim, device=dev, generator=g.manual_seed(4))
    wq, wk = init_router_weights(TINY.num_heads, device=dev)
    sp = SparseAttention(wq, wk, RouterConfig(density=0.25))
    ro = R.Rollout(m, sparse=sp, graphs=True)
    eager = ro.run(noise, text, generator=g.manual_seed(5))          # first run: eager
    captured = ro.run(noise, text, generator=g.manual_seed(5))       # captures, then replays
    replayed = ro.run(noise, text, generator=g.manual_seed(5))       # replays only
    # per chunk: the clean pass, and the denoising calls -- one graph if the chunk's first call
    # finds every history key block already pooled, else two (the first call pools the blocks the
    # previous chunk turned into history, the later ones reuse them)
    n = TINY.frames_per_chunk * TINY.frame_tokens
    chunks = math.ceil(TINY.frames / TINY.frames_per_chunk)
    want, prev = 0, 0
    for c in range(chunks):
        now = ops.history_blocks(n, (c + 1) * n, 64)
        want += 1 + (1 if now == prev else 2)
        prev = now
    assert len(ro._graph) == want
    assert torch.equal(captured, replayed)
    assert (captured - eager).abs().max() < 1e-2
    ro.release_graphs()


@pytest.mark.gpu
def test_rollout_fused_kernels_match_torch_layer():
    from streaming_sparse_b200.plugin import RouterConfig, SparseAttention, init_router_weights

    dev = torch.device("cuda:0")
    m = R.build_model(TINY, device=dev)
    g = torch.Generator(device=dev)
    noise = torch.randn(TINY.frames, 16, 16, 16, device=dev, generator=g.manual_seed(3))
    text = torch.randn(10, TINY.text_dim, device=dev, generator=g.manual_seed(4))
    wq, wk = init_router_weights(TINY.num_heads, device=dev)
    outs = []
    for fused in (False, True):
        sp = SparseAttention(wq, wk, RouterConfig(density=1.0))
        outs.append(R.Rollout(m, sparse=sp, fused=fused).run(noise, text, generator=g.manual_seed(5)))
    err = (outs[0] - outs[1]).abs()
    assert err.max() < 0.15 and err.mean() < 5e-3, (err.max().item(), err.mean().item())


TINY_WINDOW = R.WanConfig(dim=256, ffn_dim=512, num_heads=2, num_layers=2, text_dim=64, text_len=16, latent_h=16,
                          latent_w=16, frames=15, cache_frames=7, local_attn_frames=7, sink_frames=1)


@pytest.mark.gpu
def test_rolling_window_rollout_graphs_match_eager():
    """A rolling window with a sink frame (config 4's cache policy, small): chunks from the third
    on roll the window; graphs keyed by the write plan replay every roll and write exactly."""
    from streaming_sparse_b200.plugin import RouterConfig, SparseAttention, init_router_weights

    dev = torch.device("cuda:0")
    cfg = TINY_WINDOW
    m = R.build_model(cfg, device=dev)
    g = torch.Generator(device=dev)
    noise = torch.randn(cfg.frames, 16, 16, 16, device=dev, generator=g.manual_seed(3))
    text = torch.randn(10, cfg.text_dim, device=dev, generator=g.manual_seed(4))
    wq, wk = init_router_weights(cfg.num_heads, device=dev)
    sp = SparseAttention(wq, wk, RouterConfig(density=0.5, sink_tokens=cfg.frame_tokens))
    ro = R.Rollout(m, sparse=sp, graphs=True)
    eager = ro.run(noise, text, generator=g.manual_seed(5))
    state = [(c.global_end, c.local_end) for c in ro.caches]
    k_eager = ro.caches[1].k.clone()
    captured = ro.run(noise, text, generator=g.manual_seed(5))
    replayed = ro.run(noise, text, generator=g.manual_seed(5))
    assert [(c.global_end, c.local_end) for c in ro.caches] == state == [(cfg.frames * 64, 7 * 64)] * 2
    assert torch.equal(captured, replayed)
    assert (captured - eager).abs().max() < 1e-2
    assert (ro.caches[1].k - k_eager).abs().max() < 1e-2
    # chunks 0 and 1 fill the window, chunk 2 rolls from a partial window, chunks 3-4 share the
    # steady-state graphs: (roll, rewrite, clean) x 1 + per-chunk (first, clean) x 2 + 3 + ...
    assert len(ro._graph) < 3 * math.ceil(cfg.frames / cfg.frames_per_chunk)
    ro.release_graphs()


@pytest.mark.gpu
def test_rollout_with_a_short_last_chunk():
    """7 frames in chunks of 3: the last chunk has one frame (its own RoPE table, graphs and a
    64-token query chunk); graph replay equals the eager run."""
    from streaming_sparse_b200.plugin import RouterConfig, SparseAttention, init_router_weights

    dev = torch.device("cuda:0")
    cfg = R.WanConfig(dim=256, ffn_dim=512, num_heads=2, num_layers=2, text_dim=64, text_len=16, latent_h=16,
                      latent_w=16, frames=7, cache_frames=7)
    m = R.build_model(cfg, device=dev)
    g = torch.Generator(device=dev)
    noise = torch.randn(cfg.frames, 16, 16, 16, device=dev, generator=g.manual_seed(3))
    text = torch.randn(10, cfg.text_dim, device=dev, generator=g.manual_seed(4))
    wq, wk = init_router_weights(cfg.num_heads, device=dev)
    ro = R.Rollout(m, sparse=SparseAttention(wq, wk, RouterConfig(density=0.5)), graphs=True)
    eager = ro.run(noise, text, generator=g.manual_seed(5))
    ro.run(noise, text, generator=g.manual_seed(5))
    replayed = ro.run(noise, text, generator=g.manual_seed(5))
    assert torch.isfinite(eager).all() and ro.caches[0].local_end == 7 * 64
    assert (replayed - eager).abs().max() < 1e-2
    ro.release_graphs()


@pytest.mark.gpu
def test_ring_cache_rollout_equals_shifting_cache():
    """The rolling-window rollout with ring-buffer caches (heads in device memory, so replayed
    graphs follow every roll) gives the shifting caches' latents bit for bit, eager and replayed.
    48-token frames: the sink frame ends inside a 64-row sub-block, so its copy before the head is
    exercised too."""
    import dataclasses

    from streaming_sparse_b200.plugin import RouterConfig, SparseAttention, init_router_weights

    dev = torch.device("cuda:0")
    base = R.WanConfig(dim=256, ffn_dim=512, num_heads=2, num_layers=2, text_dim=64, text_len=16, latent_h=16,
                       latent_w=12, frames=15, cache_frames=7, local_attn_frames=7, sink_frames=1)
    g = torch.Generator(device=dev)
    noise = torch.randn(base.frames, 16, 16, 12, device=dev, generator=g.manual_seed(3))
    text = torch.randn(10, base.text_dim, device=dev, generator=g.manual_seed(4))
    runs = {}
    for ring in (False, True):
        cfg = dataclasses.replace(base, ring_cache=ring)
        m = R.build_model(cfg, device=dev)
        wq, wk = init_router_weights(cfg.num_heads, device=dev)
        sp = SparseAttention(wq, wk, RouterConfig(density=0.5, sink_tokens=cfg.frame_tokens))
        ro = R.Rollout(m, sparse=sp, graphs=True)
        eager = ro.run(noise, text, generator=g.manual_seed(5))
        ro.run(noise, text, generator=g.manual_seed(5))                 # captures
        replayed = ro.run(noise, text, generator=g.manual_seed(5))
        runs[ring] = (eager, replayed)
        if ring:
            c = ro.caches[0]
            assert c.ring.head != 0 and int(c.ring.head_dev.item()) == c.ring.head
        ro.release_graphs()
    assert torch.equal(runs[True][0], runs[False][0])
    assert torch.equal(runs[True][1], runs[False][1])
