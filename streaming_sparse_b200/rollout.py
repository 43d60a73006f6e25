"""Streaming rollout harness: a random-init causal Wan DiT with the sparse plugin in every layer.

This is the workload the "latent frames/s" figure is quoted on: Self-Forcing-style chunked
generation, where every self-attention layer reads a growing KV cache and the sparse plugin
replaces its ``attention(q, k, v)`` call. The model and loop restate, in plain PyTorch with the
library's cache and attention kernels, the reference's

* causal Wan DiT (wan/modules/causal_model.py:58-353 blocks and head, :387-518 embeddings and
  parameters, :730-857 inference forward, :1029-1052 unpatchify, :1054-1076 init) and the
  shared pieces of wan/modules/model.py (sinusoidal_embedding_1d :15-26, rope_params :29-37,
  WanRMSNorm :70-86, WanLayerNorm :89-99, WanT2VCrossAttention :159-202);
* the causal RoPE with a frame offset (wan/modules/causal_model.py:27-55);
* the flow-matching scheduler (utils/scheduler.py:106-170 with shift 5, sigma_min 0 and
  extra_one_step, utils/wan_wrapper.py:169-193 for x0 = x_t - sigma_t * flow);
* the rollout (pipeline/causal_inference.py:176-244): per chunk of frames, the warped denoising
  steps [1000, 750, 500, 250] with re-noising between them, then one clean pass at timestep 0
  that leaves the chunk's K/V in the cache.

As in the reference adapter (streaming_sparse/integration/self_forcing_adapter.py:110-122) only
the denoising passes are routed; the clean context pass attends densely (here through the same
attention kernel with every block listed).

Layout and kernels: the model runs in bf16 with fp32 norms; q, k and v come from one fused
[3*dim, dim] GEMM; RMSNorm and RoPE run in fp32 before the chunk is written into the cache by
``ss_cache_append``; self-attention goes through the module-level ``attention`` symbol, which
``plugin.SparsePlugin(target=this module)`` replaces. The unpatched ``attention`` is dense
scaled-dot-product attention (the reference's flash-attention call). Cross-attention over the
512 text tokens is dense (its K/V are computed once per rollout, as the reference's
cross-attention cache does). Weights are random (there is no checkpoint here): linear layers
Xavier-uniform with zero bias, text/time embeddings N(0, 0.02), as init_weights; the output
head is Xavier-uniform too (the reference zero-initialises it for training from a
checkpoint, which would make a random model's output ignore its blocks).
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import ops
from .cache import KVCache
from .plugin import _PATCH_FLAG as _PLUGIN_FLAG

HEAD_DIM = 128


@dataclass(frozen=True)
class WanConfig:
    """Wan2.1-T2V-1.3B (wan/configs/wan_t2v_1_3B.py) and the Self-Forcing rollout shape."""

    dim: int = 1536
    ffn_dim: int = 8960
    num_heads: int = 12
    num_layers: int = 30
    in_dim: int = 16
    out_dim: int = 16
    text_dim: int = 4096
    text_len: int = 512
    freq_dim: int = 256
    eps: float = 1e-6
    latent_h: int = 60            # latent height / width (patch 1x2x2 -> 30 x 52 tokens per frame)
    latent_w: int = 104
    frames: int = 21              # latent frames generated per rollout
    frames_per_chunk: int = 3
    cache_frames: int = 21        # KV cache capacity in frames
    local_attn_frames: int = -1   # rolling window in frames (-1: global cache, no eviction)
    sink_frames: int = 0          # frames kept at the front when the window rolls
    ring_cache: bool = False      # KV caches as ring buffers (a roll moves a head, not the window)

    @property
    def frame_tokens(self) -> int:
        return (self.latent_h // 2) * (self.latent_w // 2)

    @property
    def chunk_tokens(self) -> int:
        return self.frames_per_chunk * self.frame_tokens


# ---------------------------------------------------------------------------------------------
# scheduler (flow matching, shift 5, 1000 training steps, warped 4-step list)
# ---------------------------------------------------------------------------------------------
class FlowMatch:
    """sigma(t) and the warped denoising timesteps of the Self-Forcing config."""

    def __init__(self, shift: float = 5.0, steps: int = 1000, denoising_steps=(1000, 750, 500, 250)):
        s = torch.linspace(1.0, 0.0, steps + 1, dtype=torch.float64)[:-1]
        self.sigmas = shift * s / (1 + (shift - 1) * s)
        self.timesteps = self.sigmas * steps
        ext = torch.cat([self.timesteps, torch.zeros(1, dtype=torch.float64)])
        self.denoising = [float(ext[steps - t]) for t in denoising_steps]

    def sigma(self, t: float) -> float:
        return float(self.sigmas[torch.argmin((self.timesteps - t).abs())])

    def to_x0(self, flow: torch.Tensor, xt: torch.Tensor, t: float) -> torch.Tensor:
        return (xt.double() - self.sigma(t) * flow.double()).to(flow.dtype)

    def add_noise(self, x0: torch.Tensor, noise: torch.Tensor, t: float) -> torch.Tensor:
        s = self.sigma(t)
        return ((1 - s) * x0.double() + s * noise.double()).to(x0.dtype)


# ---------------------------------------------------------------------------------------------
# embeddings and RoPE tables
# ---------------------------------------------------------------------------------------------
def sinusoidal_embedding(dim: int, t: torch.Tensor) -> torch.Tensor:
    half = dim // 2
    t = t.double()
    ang = torch.outer(t, torch.pow(10000, -torch.arange(half, dtype=torch.float64, device=t.device).div(half)))
    return torch.cat([torch.cos(ang), torch.sin(ang)], dim=1)


def rope_angles(max_len: int = 1024, head_dim: int = HEAD_DIM) -> torch.Tensor:
    """[max_len, head_dim/2] float64 angles: frame, height and width parts (22 + 21 + 21 at 128)."""
    d = head_dim

    def part(n):
        return torch.outer(torch.arange(max_len, dtype=torch.float64),
                           1.0 / torch.pow(10000, torch.arange(0, n, 2, dtype=torch.float64).div(n)))

    return torch.cat([part(d - 4 * (d // 6)), part(2 * (d // 6)), part(2 * (d // 6))], dim=1)


def rope_tables(angles: torch.Tensor, start_frame: int, frames: int, hp: int, wp: int, device):
    """cos/sin [frames*hp*wp, 64] fp32 for tokens (f, h, w) of a chunk starting at start_frame."""
    c = angles.shape[1]
    cf, ch = c - 2 * (c // 3), c // 3
    fa = angles[start_frame:start_frame + frames, :cf]
    ha = angles[:hp, cf:cf + ch]
    wa = angles[:wp, cf + ch:]
    a = torch.cat([fa.view(frames, 1, 1, -1).expand(frames, hp, wp, -1),
                   ha.view(1, hp, 1, -1).expand(frames, hp, wp, -1),
                   wa.view(1, 1, wp, -1).expand(frames, hp, wp, -1)], dim=-1).reshape(frames * hp * wp, c)
    return torch.cos(a).float().to(device), torch.sin(a).float().to(device)


def apply_rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """x [n, H, 128] (pairs (2i, 2i+1) are complex numbers) rotated by the table; fp32 math."""
    n, H, D = x.shape
    xf = x.float().view(n, H, D // 2, 2)
    xr, xi = xf[..., 0], xf[..., 1]
    c, s = cos[:, None, :], sin[:, None, :]
    return torch.stack([xr * c - xi * s, xr * s + xi * c], dim=-1).view(n, H, D).to(x.dtype)


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    xf = x.float()
    return (xf * torch.rsqrt(xf.pow(2).mean(dim=-1, keepdim=True) + eps)).type_as(x) * weight


def layer_norm(x: torch.Tensor, eps: float, weight=None, bias=None) -> torch.Tensor:
    w = None if weight is None else weight.float()
    b = None if bias is None else bias.float()
    return F.layer_norm(x.float(), (x.shape[-1],), w, b, eps).type_as(x)


# ---------------------------------------------------------------------------------------------
# the patchable attention symbol (wan/modules/causal_model.py:247-251 calls attention(q, k, v))
# ---------------------------------------------------------------------------------------------
def dense_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
    """Dense attention: q [B,Lq,H,D], k/v [B,Lk,H,D] -> [B,Lq,H,D] (scale 1/sqrt(D))."""
    o = F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2))
    return o.transpose(1, 2)


def attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
    """Self-attention over the cached window; the symbol a plugin replaces (dense when unpatched)."""
    return dense_attention(q, k, v)


# ---------------------------------------------------------------------------------------------
# model
# ---------------------------------------------------------------------------------------------
class Block(nn.Module):
    def __init__(self, cfg: WanConfig):
        super().__init__()
        d = cfg.dim
        self.cfg = cfg
        self.qkv = nn.Linear(d, 3 * d)          # the reference's q, k, v linears stacked
        self.o = nn.Linear(d, d)
        self.norm_q = nn.Parameter(torch.ones(d))
        self.norm_k = nn.Parameter(torch.ones(d))
        self.norm3_w = nn.Parameter(torch.ones(d))
        self.norm3_b = nn.Parameter(torch.zeros(d))
        self.cq = nn.Linear(d, d)
        self.ck = nn.Linear(d, d)
        self.cv = nn.Linear(d, d)
        self.co = nn.Linear(d, d)
        self.cnorm_q = nn.Parameter(torch.ones(d))
        self.cnorm_k = nn.Parameter(torch.ones(d))
        self.ffn1 = nn.Linear(d, cfg.ffn_dim)
        self.ffn2 = nn.Linear(cfg.ffn_dim, d)
        self.modulation = nn.Parameter(torch.randn(1, 6, d) / d ** 0.5)

    def cross_kv(self, context: torch.Tensor):
        H = self.cfg.num_heads
        k = rms_norm(self.ck(context), self.cnorm_k, self.cfg.eps).view(1, -1, H, HEAD_DIM)
        v = self.cv(context).view(1, -1, H, HEAD_DIM)
        return k, v

    def forward(self, x, e0, rope, cache: KVCache, cross, current_start: int, fused: bool = True):
        """x [n, dim] bf16 (n = frames * frame_tokens), e0 [frames, 6, dim] fp32 -> new x.

        ``fused`` (CUDA only): the per-token work between the GEMMs runs in the library's
        kernels (AdaLN, q/k RMSNorm + RoPE with k/v written into the cache rows, RMSNorm, gated
        residual adds, in place on x); otherwise as the PyTorch expressions below, which state
        the same arithmetic.
        """
        if fused and x.is_cuda:
            return self._forward_fused(x, e0, rope, cache, cross, current_start)
        return self._forward_torch(x, e0, rope, cache, cross, current_start)

    def _forward_fused(self, x, e0, rope, cache: KVCache, cross, current_start: int):
        cfg, H = self.cfg, self.cfg.num_heads
        n, d = x.shape
        ft = n // e0.shape[0]
        em = self.modulation.float() + e0                                 # [frames, 6, dim]
        x = x.contiguous()

        h = ops.adaln(x, eps=cfg.eps, shift=em[:, 0], scale=em[:, 1], frame_tokens=ft)
        qkv = self.qkv(h)
        # a head-parallel rank's cache holds heads head0 .. head0 + cache.H - 1: q, k and v of
        # those heads only (the q/k RMSNorm still over the whole width)
        nh = cache.H
        part = dict(model_heads=H, h0=cache.head0) if nh != H else {}
        q = torch.empty((n, nh, HEAD_DIM), device=x.device, dtype=x.dtype)
        rows = cache.reserve(n, current_start)
        if rows is not None:
            ops.qkv_norm_rope(qkv, self.norm_q, self.norm_k, cfg.eps, rope[0], rope[1], q, rows[0], rows[1], **part)
        elif cache.ring_mode:   # straight into the ring rows, placed by the head in device memory
            cache.write_qkv(qkv, self.norm_q, self.norm_k, cfg.eps, rope[0], rope[1], q, current_start,
                            model_heads=H if part else None)
        else:   # the write rolls the window: stage k/v, then the cache kernel rolls and writes
            k = torch.empty_like(q)
            v = torch.empty_like(q)
            ops.qkv_norm_rope(qkv, self.norm_q, self.norm_k, cfg.eps, rope[0], rope[1], q, k, v, **part)
            cache.append(k, v, current_start)
        kw, vw = _window_for(cache)
        y = _module_attention()(q[None], kw[None], vw[None])[0]
        ops.gate_residual(x, self.o(y.reshape(n, d)), gate=em[:, 2], frame_tokens=ft)

        hq = ops.rms_norm(self.cq(ops.adaln(x, eps=cfg.eps, weight=self.norm3_w, bias=self.norm3_b)), self.cnorm_q,
                          cfg.eps)
        ck, cv = cross
        y = dense_attention(hq.view(1, n, H, HEAD_DIM), ck, cv)[0]
        ops.gate_residual(x, self.co(y.reshape(n, d)))

        h = ops.adaln(x, eps=cfg.eps, shift=em[:, 3], scale=em[:, 4], frame_tokens=ft)
        # bias + tanh-GELU in the GEMM's epilogue (cuBLASLt GELU_BIAS; checked against
        # F.gelu(approximate="tanh") in tests/test_gpu_dit.py)
        f1 = torch._addmm_activation(self.ffn1.bias, h, self.ffn1.weight.t(), use_gelu=True)
        ops.gate_residual(x, self.ffn2(f1), gate=em[:, 5], frame_tokens=ft)
        return x

    def _forward_torch(self, x, e0, rope, cache: KVCache, cross, current_start: int):
        cfg, H = self.cfg, self.cfg.num_heads
        n, d = x.shape
        fr = e0.shape[0]
        e = (self.modulation.float() + e0).unsqueeze(2).chunk(6, dim=1)   # 6 x [frames, 1, 1, dim]
        e = [t.squeeze(1) for t in e]                                     # [frames, 1, dim]

        def modulate(y, shift, scale):
            return (y.view(fr, -1, d).float() * (1 + scale) + shift).to(x.dtype).view(n, d)

        def gate(y, g):
            return (y.view(fr, -1, d).float() * g).to(x.dtype).view(n, d)

        # self-attention: fused q/k/v GEMM, RMSNorm, RoPE, cache write, attention over the window
        h = modulate(layer_norm(x, cfg.eps), e[0], e[1])
        q, k, v = self.qkv(h).split(d, dim=1)
        q = apply_rope(rms_norm(q, self.norm_q, cfg.eps).view(n, H, HEAD_DIM), *rope)
        k = apply_rope(rms_norm(k, self.norm_k, cfg.eps).view(n, H, HEAD_DIM), *rope)
        v = v.contiguous().view(n, H, HEAD_DIM)
        cache.append(k, v, current_start)
        kw, vw = _window_for(cache)
        y = _module_attention()(q[None], kw[None], vw[None])[0]
        x = x + gate(self.o(y.reshape(n, d)), e[2])

        # cross-attention over the text tokens (K/V cached per rollout)
        hq = rms_norm(self.cq(layer_norm(x, cfg.eps, self.norm3_w, self.norm3_b)), self.cnorm_q, cfg.eps)
        ck, cv = cross
        y = dense_attention(hq.view(1, n, H, HEAD_DIM), ck, cv)[0]
        x = x + self.co(y.reshape(n, d))

        # feed-forward
        h = modulate(layer_norm(x, cfg.eps), e[3], e[4])
        x = x + gate(self.ffn2(F.gelu(self.ffn1(h), approximate="tanh")), e[5])
        return x


def _module_attention():
    # looked up at call time so that a plugin that swapped the module symbol is seen
    return globals()["attention"]


def _window_for(cache: KVCache):
    """The K/V window handed to the module's attention: a ring cache's physical rows go only to the
    sparse plugin (which follows the ring); any other attention gets the window in order."""
    if cache.ring_mode and not getattr(_module_attention(), _PLUGIN_FLAG, False):
        return cache.window_logical()
    return cache.window()


class CausalWanDiT(nn.Module):
    """Random-init causal Wan DiT (bf16) for chunked streaming inference."""

    def __init__(self, cfg: WanConfig = WanConfig()):
        super().__init__()
        d = cfg.dim
        self.cfg = cfg
        self.patch = nn.Parameter(torch.empty(d, cfg.in_dim, 1, 2, 2))   # Conv3d layout
        self.patch_b = nn.Parameter(torch.zeros(d))
        self.text1 = nn.Linear(cfg.text_dim, d)
        self.text2 = nn.Linear(d, d)
        self.time1 = nn.Linear(cfg.freq_dim, d)
        self.time2 = nn.Linear(d, d)
        self.time_proj = nn.Linear(d, 6 * d)
        self.blocks = nn.ModuleList([Block(cfg) for _ in range(cfg.num_layers)])
        self.head = nn.Linear(d, cfg.out_dim * 4)
        self.head_modulation = nn.Parameter(torch.randn(1, 2, d) / d ** 0.5)
        self.angles = rope_angles()

    @torch.no_grad()
    def init_weights(self, seed: int = 0):
        dev = self.patch.device
        g = torch.Generator(device=dev).manual_seed(seed)

        def uniform(t, a):
            t.copy_(torch.rand(t.shape, generator=g, device=dev) * 2 * a - a)

        for m in self.modules():
            if isinstance(m, nn.Linear):
                uniform(m.weight, math.sqrt(6.0 / (m.weight.shape[1] + m.weight.shape[0])))
                m.bias.zero_()
        uniform(self.patch, math.sqrt(6.0 / (self.patch[0].numel() + self.patch.shape[0])))
        for m in (self.text1, self.text2, self.time1, self.time2):
            m.weight.copy_(torch.randn(m.weight.shape, generator=g, device=dev) * 0.02)
        for b in self.blocks:
            b.modulation.copy_(torch.randn(b.modulation.shape, generator=g, device=dev) / self.cfg.dim ** 0.5)
        self.head_modulation.copy_(torch.randn(self.head_modulation.shape, generator=g, device=dev) /
                                   self.cfg.dim ** 0.5)
        return self

    def embed_text(self, text: torch.Tensor) -> torch.Tensor:
        """text [L<=text_len, text_dim] -> [text_len, dim] (zero-padded as the reference)."""
        L = self.cfg.text_len
        if text.shape[0] < L:
            text = torch.cat([text, text.new_zeros(L - text.shape[0], text.shape[1])])
        return self.text2(F.gelu(self.text1(text), approximate="tanh"))

    def embed_time(self, t, frames: int, device):
        """t: a number, or a one-element device tensor (read at run time, as inside a CUDA graph)."""
        tt = t.reshape(1).expand(frames) if torch.is_tensor(t) else torch.full((frames,), float(t), device=device)
        e = self.time2(F.silu(self.time1(sinusoidal_embedding(self.cfg.freq_dim, tt).to(self.time1.weight.dtype))))
        e0 = self.time_proj(F.silu(e)).float().view(frames, 6, self.cfg.dim)
        return e.float(), e0

    def patchify(self, x: torch.Tensor) -> torch.Tensor:
        """x [C, F, Hl, Wl] -> tokens [F*(Hl/2)*(Wl/2), dim] (the stride-(1,2,2) Conv3d as a GEMM)."""
        C, Fr, Hl, Wl = x.shape
        p = x.reshape(C, Fr, Hl // 2, 2, Wl // 2, 2).permute(1, 2, 4, 0, 3, 5).reshape(-1, C * 4)
        return F.linear(p.to(self.patch.dtype), self.patch.view(self.patch.shape[0], -1), self.patch_b)

    def unpatchify(self, y: torch.Tensor, Fr: int) -> torch.Tensor:
        cfg = self.cfg
        hp, wp = cfg.latent_h // 2, cfg.latent_w // 2
        u = y.view(Fr, hp, wp, 1, 2, 2, cfg.out_dim)
        u = torch.einsum("fhwpqrc->cfphqwr", u)
        return u.reshape(cfg.out_dim, Fr, cfg.latent_h, cfg.latent_w)

    def forward_chunk(self, x: torch.Tensor, t, caches, cross, start_frame: int, rope,
                      fused: bool = True) -> torch.Tensor:
        """x [C, F, Hl, Wl] latents of one chunk -> flow prediction [C, F, Hl, Wl]."""
        cfg = self.cfg
        Fr = x.shape[1]
        e, e0 = self.embed_time(t, Fr, x.device)
        h = self.patchify(x)
        current_start = start_frame * cfg.frame_tokens
        for blk, cache, cr in zip(self.blocks, caches, cross):
            h = blk(h, e0, rope, cache, cr, current_start, fused=fused)
        m = self.head_modulation.float() + e.unsqueeze(1)                     # [F, 2, dim]
        d = cfg.dim
        if fused and h.is_cuda:
            hn = ops.adaln(h, eps=cfg.eps, shift=m[:, 0], scale=m[:, 1], frame_tokens=h.shape[0] // Fr)
        else:
            hn = (layer_norm(h, cfg.eps).view(Fr, -1, d).float() * (1 + m[:, 1:2]) + m[:, 0:1]).to(h.dtype)
        out = self.head(hn.view(-1, d))
        return self.unpatchify(out, Fr)


# ---------------------------------------------------------------------------------------------
# rollout
# ---------------------------------------------------------------------------------------------
class Rollout:
    """One generation stream: per-layer KV caches, cross-attention K/V and the chunk loop.

    ``sparse`` (a ``plugin.SparseAttention``) is used through ``plugin.SparsePlugin`` on this
    module for the denoising passes; its ``dense`` switch lists every block for the clean
    context pass. ``sparse=None`` runs the dense model (the unpatched ``attention``).

    ``fused`` selects the library's per-token kernels between the GEMMs (see ``Block.forward``).

    ``graphs=True``: the first ``run`` executes eagerly (it also warms up the libraries); from
    the second on, every model call (one chunk, one phase: 30 layers of GEMMs, norms, cache
    writes, routing and attention) is captured once into a CUDA graph and replayed, so the host
    enqueues one launch per call instead of ~1500. A call's device work is fixed by its shape,
    phase and cache write plan (whether the window rolls, by how much, where the chunk ends), so
    graphs are keyed by those: the calls of a chunk that rewrite the same rows share a graph, and
    with a rolling window (``local_attn_frames``) every steady-state chunk reuses the same three
    (rolling first call, later calls, clean pass). The cross-attention K/V, the inputs and the
    RoPE tables live in static buffers.
    """

    def __init__(self, model: CausalWanDiT, sparse=None, scheduler: FlowMatch | None = None, graphs: bool = False,
                 fused: bool = True, head_parallel: bool = False, group=None):
        self.model = model
        self.cfg = model.cfg
        self.sparse = sparse
        self.sched = scheduler or FlowMatch()
        dev = next(model.parameters()).device
        cfg = self.cfg
        h0, nh = 0, cfg.num_heads
        if head_parallel:
            import torch.distributed as dist

            from .distributed import head_range
            if sparse is None or not fused:
                raise ValueError("a head-parallel rollout runs the sparse plugin with the fused kernels")
            h0, h1 = head_range(cfg.num_heads, dist.get_rank(group), dist.get_world_size(group))
            nh = h1 - h0
        self.caches = [KVCache(cfg.cache_frames * cfg.frame_tokens, nh, HEAD_DIM,
                               frame_tokens=cfg.frame_tokens, local_attn_size=cfg.local_attn_frames,
                               sink_size=cfg.sink_frames, device=dev, track_positions=False, ring=cfg.ring_cache)
                       for _ in range(cfg.num_layers)]
        for c in self.caches:
            c.head0 = h0
        self.head_parallel = head_parallel
        if head_parallel:
            from .distributed import HeadParallelAttention
            self.sparse = HeadParallelAttention(sparse, self.caches, cfg.chunk_tokens, dev, group)
        self.device = dev
        self._rope = {}
        self.graphs = graphs
        self.fused = fused
        self._runs = 0
        self._graph = {}          # (start_frame, frames, phase) -> (graph, x_in, t_in, flow_out)
        self._pool = None
        self._cross = None        # static cross-attention K/V per layer
        self._rope_in = {}        # frames -> static (cos, sin) buffers read by the graphs

    def reset(self):
        for c in self.caches:
            c.reset()

    def rope(self, start_frame: int, frames: int):
        key = (start_frame, frames)
        if key not in self._rope:
            cfg = self.cfg
            self._rope[key] = rope_tables(self.model.angles, start_frame, frames, cfg.latent_h // 2,
                                          cfg.latent_w // 2, self.device)
        return self._rope[key]

    @torch.no_grad()
    def run(self, noise: torch.Tensor, text: torch.Tensor, generator: torch.Generator | None = None) -> torch.Tensor:
        """noise [frames, C, Hl, Wl] and text [L, text_dim] on the device -> latents [frames, C, Hl, Wl]."""
        from .plugin import SparsePlugin
        import sys

        cfg, sched, model = self.cfg, self.sched, self.model
        self.reset()
        ctx = model.embed_text(text.to(model.text1.weight.dtype))
        cross = [blk.cross_kv(ctx) for blk in model.blocks]
        if self._cross is None:
            self._cross = [(k.clone(), v.clone()) for k, v in cross]
        else:
            for (sk, sv), (k, v) in zip(self._cross, cross):
                sk.copy_(k)
                sv.copy_(v)
        cross = self._cross
        use_graphs = self.graphs and self._runs > 0
        out = torch.empty_like(noise)
        plugin = SparsePlugin(self.sparse, target=sys.modules[__name__]) if self.sparse is not None else None
        if plugin is not None:
            for c in self.caches:     # routed calls reuse each layer's pooled history keys
                self.sparse.attach(c)
            plugin.__enter__()
        try:
            for c0 in range(0, cfg.frames, cfg.frames_per_chunk):
                nf = min(cfg.frames_per_chunk, cfg.frames - c0)
                rope = self.rope(c0, nf)
                xt = noise[c0:c0 + nf].transpose(0, 1)          # [C, F, Hl, Wl]
                if self.sparse is not None:
                    self.sparse.dense = False
                steps = sched.denoising
                for i, t in enumerate(steps):
                    flow = self._call(xt, t, cross, c0, nf, rope, "denoise", use_graphs)
                    x0 = sched.to_x0(flow.float(), xt.float(), t)
                    if i + 1 < len(steps):
                        eps = torch.randn(x0.shape, device=x0.device, generator=generator, dtype=x0.dtype)
                        xt = sched.add_noise(x0, eps, steps[i + 1])
                out[c0:c0 + nf] = x0.transpose(0, 1).to(out.dtype)
                # clean pass at timestep 0: rewrites the chunk's K/V in the cache (dense attention)
                if self.sparse is not None:
                    self.sparse.dense = True
                self._call(x0, 0.0, cross, c0, nf, rope, "context", use_graphs)
        finally:
            if plugin is not None:
                plugin.__exit__(None, None, None)
                self.sparse.dense = False
        self._runs += 1
        return out

    def _call(self, x, t: float, cross, c0: int, nf: int, rope, phase: str, use_graphs: bool):
        """One model call on latents x [C, F, Hl, Wl] (any float dtype) -> flow prediction."""
        model = self.model
        if not use_graphs:
            return model.forward_chunk(x.to(torch.bfloat16), t, self.caches, cross, c0, rope, fused=self.fused)
        # A call's device work is fixed by its shape, phase and the caches' index state (where
        # the chunk lands, whether the window rolls); the RoPE table comes through a static
        # buffer. So one graph serves every call with the same key -- with a rolling window, every
        # steady-state chunk -- and the host index mirrors are advanced after each replay.
        start = c0 * self.cfg.frame_tokens
        n = x.shape[1] * self.cfg.frame_tokens
        # a routed call also depends on how many history key blocks the layers' router tables
        # hold for the window this write leaves (pooled at the chunk's first call, reused after)
        routed = self.sparse is not None and phase == "denoise"
        cached = None
        if routed:
            c = self.sparse.config
            cached = self.caches[0].router_keys(c.block, self.sparse.wq.shape[2]).cached(self.caches[0].tag_after(n, start))
        key = (nf, phase, cached) + self.caches[0].write_plan(n, start)
        ent = self._graph.get(key)
        if nf not in self._rope_in:
            self._rope_in[nf] = (torch.empty_like(rope[0]), torch.empty_like(rope[1]))
        rope_in = self._rope_in[nf]
        rope_in[0].copy_(rope[0])
        rope_in[1].copy_(rope[1])
        if ent is None:
            x_in = torch.empty(x.shape, device=self.device, dtype=torch.bfloat16)
            t_in = torch.zeros(1, device=self.device, dtype=torch.float64)
            x_in.copy_(x)
            t_in.fill_(t)
            if self._pool is None:
                self._pool = torch.cuda.graph_pool_handle()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, pool=self._pool):   # the host mirrors advance here, once
                flow = model.forward_chunk(x_in, t_in, self.caches, cross, c0, rope_in, fused=self.fused)
            ent = self._graph[key] = (g, x_in, t_in, flow)
            advance = False
        else:
            advance = True
        g, x_in, t_in, flow = ent
        x_in.copy_(x)
        t_in.fill_(t)
        g.replay()
        if advance:
            for cache in self.caches:
                cache.advance(n, start)
                if routed:   # what the captured route marked in each layer's key table
                    c = self.sparse.config
                    lk = cache.local_end - cache.window_start()
                    cache.router_keys(c.block, self.sparse.wq.shape[2]).mark(cache.history_tag(),
                                                                             ops.history_blocks(n, lk, c.block))
        return flow

    def release_graphs(self):
        self._graph.clear()
        self._pool = None
        self._rope_in.clear()

    def close(self):
        """Release the graphs and, for a head-parallel rollout, the peer mappings (every rank)."""
        self.release_graphs()
        if self.head_parallel:
            self.sparse.close()


def build_model(cfg: WanConfig = WanConfig(), device="cuda", seed: int = 0) -> CausalWanDiT:
    """Random-init model in bf16, created and initialised on ``device`` (fp32, then cast)."""
    with torch.device(device):
        m = CausalWanDiT(cfg)
    m.init_weights(seed)
    return m.to(dtype=torch.bfloat16).eval()


def model_flops_per_call(cfg: WanConfig, Lk: int, attended_per_query: float | None = None) -> float:
    """GEMM + attention FLOPs of one forward_chunk (attention at `attended_per_query` keys)."""
    n, d, T = cfg.chunk_tokens, cfg.dim, cfg.text_len
    gemm = 2 * n * d * (3 * d + d + d + d + 2 * cfg.ffn_dim) * cfg.num_layers
    att = attended_per_query if attended_per_query is not None else Lk
    attn = 4 * n * att * d * cfg.num_layers + 4 * n * T * d * cfg.num_layers
    return float(gemm + attn)


__all__ = ["WanConfig", "FlowMatch", "CausalWanDiT", "Rollout", "build_model", "attention", "dense_attention",
           "apply_rope",
           "rope_angles", "rope_tables", "sinusoidal_embedding", "model_flops_per_call"]


def main(argv=None):
    """python -m streaming_sparse_b200.rollout [--density D | --dense] [--profile] ...

    Times full rollouts of one stream on cuda:0 (CUDA-graph replay after a warm-up), or with
    --profile prints the per-kernel GPU time (torch profiler) of one denoising and one clean call
    of the last chunk, after a rollout has filled the cache.
    """
    import argparse
    import time

    from .plugin import RouterConfig, SparseAttention, SparsePlugin, init_router_weights

    ap = argparse.ArgumentParser(prog="python -m streaming_sparse_b200.rollout")
    ap.add_argument("--config4", action="store_true",
                    help="config 4's long-horizon stream: 120 frames, 21-frame window + 1 sink frame, "
                         "128-token router blocks at 10%% of the unforced blocks")
    ap.add_argument("--density", type=float, default=0.25)
    ap.add_argument("--dense", action="store_true", help="no plugin: dense attention everywhere")
    ap.add_argument("--unfused", action="store_true", help="PyTorch per-token ops instead of csrc/dit.cu")
    ap.add_argument("--layers", type=int, default=30)
    ap.add_argument("--frames", type=int, default=21)
    ap.add_argument("--runs", type=int, default=2)
    ap.add_argument("--profile", action="store_true")
    a = ap.parse_args(argv)
    dev = torch.device("cuda:0")
    if a.config4:
        cfg = WanConfig(num_layers=a.layers, frames=120, cache_frames=22, local_attn_frames=22, sink_frames=1)
        rcfg = RouterConfig(block=128, density=0.10, rule="rest", sink_tokens=cfg.frame_tokens)
    else:
        cfg = WanConfig(num_layers=a.layers, frames=a.frames, cache_frames=a.frames)
        rcfg = RouterConfig(density=a.density)
    model = build_model(cfg, device=dev)
    g = torch.Generator(device=dev)
    noise = torch.randn(cfg.frames, cfg.in_dim, cfg.latent_h, cfg.latent_w, device=dev, generator=g.manual_seed(0))
    text = torch.randn(cfg.text_len, cfg.text_dim, device=dev, generator=g.manual_seed(1))
    sparse = None
    if not a.dense:
        wq, wk = init_router_weights(cfg.num_heads, device=dev)
        sparse = SparseAttention(wq, wk, rcfg)
    fused = not a.unfused
    if a.profile:
        from torch.profiler import ProfilerActivity, profile

        ro = Rollout(model, sparse=sparse, fused=fused)
        ro.run(noise, text, generator=g.manual_seed(2))
        c0 = cfg.frames - cfg.frames_per_chunk
        ctx = model.embed_text(text.bfloat16())
        cross = [b.cross_kv(ctx) for b in model.blocks]
        x = noise[c0:].transpose(0, 1).bfloat16()
        rope = ro.rope(c0, cfg.frames_per_chunk)
        import sys
        plugin = SparsePlugin(sparse, target=sys.modules[__name__]) if sparse is not None else None
        if plugin is not None:
            plugin.__enter__()
        try:
            with torch.no_grad():
                for phase in ("denoise", "clean"):
                    if sparse is not None:
                        sparse.dense = phase == "clean"
                    t = 0.0 if phase == "clean" else ro.sched.denoising[1]
                    model.forward_chunk(x, t, ro.caches, cross, c0, rope, fused=fused)
                    torch.cuda.synchronize()
                    with profile(activities=[ProfilerActivity.CUDA]) as prof:
                        model.forward_chunk(x, t, ro.caches, cross, c0, rope, fused=fused)
                        torch.cuda.synchronize()
                    print(f"== {phase} call, chunk at frame {c0}, window {ro.caches[0].local_end} tokens")
                    print(prof.key_averages().table(sort_by="cuda_time_total", row_limit=16,
                                                    max_name_column_width=60))
        finally:
            if plugin is not None:
                plugin.__exit__(None, None, None)
        return
    ro = Rollout(model, sparse=sparse, graphs=True, fused=fused)
    for _ in range(2):
        ro.run(noise, text, generator=g.manual_seed(2))
    torch.cuda.synchronize()
    for _ in range(a.runs):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        w0 = time.perf_counter()
        e0.record()
        out = ro.run(noise, text, generator=g.manual_seed(2))
        e1.record()
        w1 = time.perf_counter()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1)
        print(f"rollout {cfg.frames} frames: {ms:.1f} ms GPU, {1e3 * (w1 - w0):.1f} ms host enqueue, "
              f"{cfg.frames / (ms * 1e-3):.2f} latent frames/s, finite={bool(torch.isfinite(out).all())}")


if __name__ == "__main__":
    main()
