"""Seeded synthetic inputs shared by the GPU parity tests (N(0,1) bf16 Q/K/V, N(0,1/128) router weights)."""
import math

import numpy as np
import torch


def qkv(seed: int, Lq: int, Lk: int, H: int, D: int = 128):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn((Lq, H, D), generator=g).bfloat16()
    k = torch.randn((Lk, H, D), generator=g).bfloat16()
    v = torch.randn((Lk, H, D), generator=g).bfloat16()
    return q, k, v


def router_weights(seed: int, H: int, D: int = 128, R: int = 64):
    g = torch.Generator().manual_seed(seed + 1000)
    wq = torch.randn((H, D, R), generator=g) / math.sqrt(D)
    wk = torch.randn((H, D, R), generator=g) / math.sqrt(D)
    return wq, wk


def np32(t: torch.Tensor) -> np.ndarray:
    return t.float().cpu().numpy()


def assert_attention_close(got: np.ndarray, ref: np.ndarray, max_abs: float = 2e-2, mean_abs: float = 2e-3,
                           nmse: float = 2e-5):
    """The north-star tolerance for bf16 outputs against the fp32-accumulated reference path, plus
    the normalised squared error bound of the reference runtime's own validation of its sparse
    attention (local_experiments/video_runtime_v1/runtime.py:311-323: NMSE < 2e-5)."""
    mask = np.isfinite(ref)
    r = ref[mask].astype(np.float64)
    err = np.abs(got[mask].astype(np.float64) - r)
    assert np.isfinite(got[mask]).all(), "non-finite output"
    assert err.max() <= max_abs, f"max-abs {err.max():.3e} > {max_abs}"
    assert err.mean() <= mean_abs, f"mean-abs {err.mean():.3e} > {mean_abs}"
    e = float((err ** 2).sum() / max(float((r ** 2).sum()), 1e-12))
    assert e < nmse, f"nmse {e:.3e} >= {nmse}"
    return float(err.max()), float(err.mean())
