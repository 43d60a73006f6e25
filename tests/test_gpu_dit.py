"""Per-token DiT-layer kernels (csrc/dit.cu) against the PyTorch expressions they replace."""
import pytest
import torch

from streaming_sparse_b200 import ops
from streaming_sparse_b200 import rollout as R
from streaming_sparse_b200.cache import KVCache

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")


def _gen(seed):
    return torch.Generator(device=DEV).manual_seed(seed)


def _ulp_close(a, b, frac=1e-3):
    """bf16 results that differ only where a one-ulp rounding flip can happen."""
    d = (a.float() - b.float()).abs()
    tol = b.float().abs() * 2 ** -7 + 1e-6
    bad = (d > tol).float().mean().item()
    assert bad <= frac, bad


@pytest.mark.parametrize("H,n", [(12, 4680), (2, 100), (3, 17)])
def test_qkv_norm_rope_matches_torch(H, n):
    d = H * 128
    g = _gen(H)
    qkv = torch.randn(n, 3 * d, device=DEV, generator=g).bfloat16()
    wq = (1 + 0.1 * torch.randn(d, device=DEV, generator=g)).bfloat16()
    wk = (1 + 0.1 * torch.randn(d, device=DEV, generator=g)).bfloat16()
    fr, hp, wp = (3, 30, 52) if n == 4680 else (3, 1, (n + 2) // 3)
    cos, sin = R.rope_tables(R.rope_angles(), 6, fr, hp, wp, DEV)
    cos, sin = cos[:n].contiguous(), sin[:n].contiguous()
    q = torch.empty(n, H, 128, device=DEV, dtype=torch.bfloat16)
    kc = torch.zeros(n + 8, H, 128, device=DEV, dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    ops.qkv_norm_rope(qkv, wq, wk, 1e-6, cos, sin, q, kc[8:], vc[8:])
    qr, kr, vr = qkv.split(d, dim=1)
    q_ref = R.apply_rope(R.rms_norm(qr, wq, 1e-6).view(n, H, 128), cos, sin)
    k_ref = R.apply_rope(R.rms_norm(kr, wk, 1e-6).view(n, H, 128), cos, sin)
    _ulp_close(q, q_ref)
    _ulp_close(kc[8:], k_ref)
    assert torch.equal(vc[8:], vr.reshape(n, H, 128))
    assert not kc[:8].any() and not vc[:8].any()


def test_adaln_modulation_and_affine_match_torch():
    n, d, ft, fr = 4680, 1536, 1560, 3
    g = _gen(1)
    x = (3 * torch.randn(n, d, device=DEV, generator=g) + 0.5).bfloat16()
    em = 0.3 * torch.randn(fr, 6, d, device=DEV, generator=g)
    out = ops.adaln(x, eps=1e-6, shift=em[:, 0], scale=em[:, 1], frame_tokens=ft)
    ref = (R.layer_norm(x, 1e-6).view(fr, -1, d).float() * (1 + em[:, 1:2]) + em[:, 0:1]).bfloat16().view(n, d)
    _ulp_close(out, ref)
    w = (1 + 0.1 * torch.randn(d, device=DEV, generator=g)).bfloat16()
    b = (0.1 * torch.randn(d, device=DEV, generator=g)).bfloat16()
    out = ops.adaln(x, eps=1e-6, weight=w, bias=b)
    _ulp_close(out, R.layer_norm(x, 1e-6, w, b))


def test_rms_norm_and_gate_residual_match_torch():
    n, d, ft, fr = 1000, 1536, 250, 4
    g = _gen(2)
    x = torch.randn(n, 2 * d, device=DEV, generator=g).bfloat16()[:, :d]      # strided rows
    w = (1 + 0.1 * torch.randn(d, device=DEV, generator=g)).bfloat16()
    _ulp_close(ops.rms_norm(x, w, 1e-6), R.rms_norm(x, w, 1e-6))
    base = torch.randn(n, d, device=DEV, generator=g).bfloat16()
    y = torch.randn(n, d, device=DEV, generator=g).bfloat16()
    gate = torch.randn(fr, 6, d, device=DEV, generator=g)[:, 2]
    ref = base + (y.view(fr, -1, d).float() * gate[:, None]).bfloat16().view(n, d)
    got = ops.gate_residual(base.clone(), y, gate=gate, frame_tokens=ft)
    assert torch.equal(got, ref)
    assert torch.equal(ops.gate_residual(base.clone(), y), base + y)


def test_bad_arguments_raise():
    x = torch.zeros(4, 1536, device=DEV, dtype=torch.bfloat16)
    with pytest.raises(ValueError):
        ops.adaln(x, eps=1e-6, shift=torch.zeros(1, 1536, device=DEV), scale=None)
    with pytest.raises(RuntimeError):   # neither modulation nor affine: rejected by the C ABI
        ops.adaln(x, eps=1e-6)


def test_reserve_matches_append():
    cap, H, n = 64 * 6, 2, 100
    g = _gen(3)
    a = KVCache(cap, H, 128, frame_tokens=50, device=DEV)
    b = KVCache(cap, H, 128, frame_tokens=50, device=DEV)
    for start in (0, 100, 100, 200):
        k = torch.randn(n, H, 128, device=DEV, generator=g).bfloat16()
        v = torch.randn(n, H, 128, device=DEV, generator=g).bfloat16()
        a.append(k, v, start)
        rows = b.reserve(n, start)
        rows[0].copy_(k)
        rows[1].copy_(v)
        assert (a.global_end, a.local_end) == (b.global_end, b.local_end)
    assert torch.equal(a.k, b.k) and torch.equal(a.v, b.v)
    # a write that must roll the window is refused
    loc = KVCache(cap, H, 128, frame_tokens=50, local_attn_size=6, device=DEV)
    loc.append(torch.zeros(300, H, 128, device=DEV, dtype=torch.bfloat16),
               torch.zeros(300, H, 128, device=DEV, dtype=torch.bfloat16), 0)
    assert loc.reserve(n, 300) is None and loc.local_end == 300


def test_ffn_gemm_gelu_epilogue_is_the_tanh_form():
    """The fused FFN uses the GEMM's bias+GELU epilogue in place of nn.GELU(approximate='tanh')
    on the GEMM output. (The tanh and erf forms differ by < 5e-4, below bf16 resolution at the
    values where they differ most, so the check is closeness to the tanh form at bf16.)"""
    g = _gen(4)
    x = torch.randn(4680, 1536, device=DEV, generator=g).bfloat16()
    w = (torch.randn(8960, 1536, device=DEV, generator=g) / 40).bfloat16()
    b = (0.1 * torch.randn(8960, device=DEV, generator=g)).bfloat16()
    fused = torch._addmm_activation(b, x, w.t(), use_gelu=True).float()
    lin = torch.addmm(b, x, w.t())
    tanh_ref = torch.nn.functional.gelu(lin, approximate="tanh").float()
    d_tanh = (fused - tanh_ref).abs()
    # one bf16 rounding of the pre-activation apart at most
    assert d_tanh.max() < 0.05 and d_tanh.mean() < 1e-3, (d_tanh.max().item(), d_tanh.mean().item())
