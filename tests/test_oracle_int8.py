"""The INT8-QK oracle pinned to the reference's own kernels (tests/golden/int8_qk.npz, produced by
migration/unified_router/opt23/attention.py ``_quant`` and ``_shared`` with INT8=True; see
tests/golden/make_golden_int8.py)."""
import os

import numpy as np

from oracle import oracle

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "int8_qk.npz")


def _g():
    return np.load(GOLD)


def test_k_page_quantisation_bit_exact():
    g = _g()
    ki, ks = oracle.quant_rows(g["k"].transpose(1, 0, 2), oracle.QUANT_PAGE)    # [NK,H,D]
    assert np.array_equal(ki.transpose(1, 0, 2), g["k_i8"])
    assert np.array_equal(ks.view(np.uint32), g["ks"].view(np.uint32))
    assert g["ks"][1, 1] == np.float32(1e-10)      # the all-zero page clamps its scale


def test_shared_loop_matches_reference_kernel():
    g = _g()
    out = oracle.shared_i8_tiles(g["q"], g["k_i8"], g["ks"], g["v"], g["tiles"], int(g["group"]))
    assert np.abs(out - g["out"]).max() <= 2e-6


def test_library_layout_oracle_matches_reference_kernel():
    """attention_i8 (this library's layouts, block = 64, exact float64 softmax) against the
    reference kernel's fp16-P output: the difference is P's fp16 rounding only."""
    g = _g()
    q, k_i8, v = (g[n].transpose(1, 0, 2) for n in ("q", "k_i8", "v"))
    out, lse = oracle.attention_i8(q, k_i8, g["ks"], v, g["page_lists"], 64)
    ref = g["out"].transpose(1, 0, 2)
    err = np.abs(out - ref)
    assert err.max() <= 2e-3 and err.mean() <= 2e-4
    assert np.all(np.isfinite(lse))
    # the all-zero query group scores every key 0: its rows are the plain mean of the selected V
    sel = oracle.selected_tokens(g["page_lists"][0, 0], v.shape[0], 64)
    assert np.allclose(out[32:64, 0], v[sel, 0].astype(np.float64).mean(axis=0), atol=1e-12)


def test_quant_rounds_half_to_even():
    # x / s lands exactly on k + 1/2 (s = 1 when max|x| = 127): ties go to the even integer
    x = np.zeros((32, 1, 128), np.float32)
    x[0, 0, :6] = [127.0, 0.5, 1.5, 2.5, -0.5, -1.5]
    xi, s = oracle.quant_rows(x, 32)
    assert s[0, 0] == 1.0
    assert list(xi[0, 0, :6]) == [127, 0, 2, 2, 0, -2]


def test_128_token_blocks_match_reference_kernel():
    """int8_qk_b128.npz: the same int8 keys, 128-token routing blocks (two pages per block id, the
    window's last block one page): the kernel loop restatement and the library-layout oracle with
    block = 128 against the reference kernel's output."""
    g, g2 = _g(), np.load(GOLD.replace("int8_qk.npz", "int8_qk_b128.npz"))
    out = oracle.shared_i8_tiles(g2["q"], g["k_i8"], g["ks"], g["v"], g2["tiles"], int(g["group"]))
    assert np.abs(out - g2["out"]).max() <= 2e-6
    q, k_i8, v = g2["q"].transpose(1, 0, 2), g["k_i8"].transpose(1, 0, 2), g["v"].transpose(1, 0, 2)
    ref, _ = oracle.attention_i8(q, k_i8, g["ks"], v, g2["block_lists"], 128)
    err = np.abs(ref - g2["out"].transpose(1, 0, 2))
    assert err.max() <= 2e-3 and err.mean() <= 2e-4
