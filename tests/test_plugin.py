"""The drop-in plugin: patch/restore semantics (CPU) and routed attention through it (GPU)."""
import types

import numpy as np
import pytest
import torch

from helpers import assert_attention_close, np32, qkv, router_weights


def _fake_causal_module():
    mod = types.ModuleType("fake_causal_model")

    def attention(q, k, v):
        return "original"
    mod.attention = attention
    return mod


def test_patch_and_restore_and_nesting():
    from streaming_sparse_b200.plugin import RouterConfig, SparseAttention, SparsePlugin
    mod = _fake_causal_module()
    original = mod.attention
    sparse = SparseAttention(torch.zeros(2, 128, 64), torch.zeros(2, 128, 64), RouterConfig())
    with SparsePlugin(sparse, target=mod):
        assert mod.attention is not original
        with pytest.raises(RuntimeError):
            SparsePlugin(sparse, target=mod).__enter__()
        with pytest.raises(ValueError):
            mod.attention(torch.zeros(1), torch.zeros(1), torch.zeros(1), dropout_p=0.1)
    assert mod.attention is original


def test_router_config_budgets():
    from streaming_sparse_b200.plugin import RouterConfig
    assert RouterConfig(topk=24, density=None).extra(1560, 6240) == 24            # config 1
    assert RouterConfig(density=0.25).extra(4680, 32760) == 54                     # config 2
    c4 = RouterConfig(block=128, density=0.1, rule="rest", sink_tokens=1560)
    from streaming_sparse_b200 import ops
    nf = ops.forced_count(4680, 34320, 128, 1560)
    assert c4.extra(4680, 34320) == int(0.1 * (269 - nf))
    assert RouterConfig(density=0.25).extra(4680, 4680) == 0                        # first chunk: dense


@pytest.mark.gpu
def test_plugin_routes_through_patched_symbol(oracle):
    from streaming_sparse_b200.plugin import RouterConfig, SparseAttention, SparsePlugin
    dev = torch.device("cuda:0")
    Lq, Lk, H = 300, 1500, 2
    q, k, v = qkv(31, Lq, Lk, H)
    wq, wk = router_weights(31, H)
    sparse = SparseAttention(wq.to(dev), wk.to(dev), RouterConfig(density=0.5), validate=True)
    mod = _fake_causal_module()
    with SparsePlugin(sparse, target=mod):
        out = mod.attention(q[None].to(dev), k[None].to(dev), v[None].to(dev))
    assert out.shape == (1, Lq, H, 128) and out.dtype == torch.bfloat16
    extra = RouterConfig(density=0.5).extra(Lq, Lk)
    r = oracle.route(np32(q), np32(k), wq.numpy(), wk.numpy(), 64, extra)
    np.testing.assert_array_equal(sparse.last_ids.cpu().numpy(), r["ids"])
    ref, _ = oracle.attention(np32(q), np32(k), np32(v), r["ids"], 64)
    assert_attention_close(out[0].float().cpu().numpy(), ref)
    # dense mode (the reference's context pass) == every block selected
    sparse.dense = True
    with SparsePlugin(sparse, target=mod):
        dense = mod.attention(q[None].to(dev), k[None].to(dev), v[None].to(dev))
    ref_dense = torch.nn.functional.scaled_dot_product_attention(
        q.float().permute(1, 0, 2), k.float().permute(1, 0, 2), v.float().permute(1, 0, 2)).permute(1, 0, 2)
    assert_attention_close(dense[0].float().cpu().numpy(), ref_dense.numpy())
