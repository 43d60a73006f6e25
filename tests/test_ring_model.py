"""The ring-buffer cache layout (tests/ring_model.py, the rows ss_cache_append_ring writes) keeps
the window of the reference's shifting cache: over streams with rolls, chunk rewrites, a sink
that is not a multiple of 64 rows and a ring that wraps, every 64-row sub-block read from its
mapped physical start equals the oracle's shifted window (oracle.cache_append, the roll of
wan/modules/causal_model.py:216-246), and a roll writes only the chunk, its mirrored rows and
the sink's copy instead of moving the window."""
import numpy as np
import pytest

from ring_model import RingModel


@pytest.mark.parametrize("cap,sink,chunk,steps", [
    (34320, 1560, 4680, 3),   # config 4: 22 frames of 1560 tokens, a 1-frame sink, 3-frame chunks
    (1000, 100, 150, 2),      # small: the sink ends inside a sub-block, the ring wraps often
    (1000, 0, 130, 1),        # no sink
    (768, 128, 192, 2),       # sink and chunks whole sub-blocks
    (900, 40, 300, 3),        # a sink shorter than one sub-block
])
def test_ring_window_equals_shifted_window(oracle, cap, sink, chunk, steps):
    H = 2
    rng = np.random.default_rng(cap + sink)
    ref_k = np.zeros((cap, H, 128), np.float32)
    ref_v = np.zeros_like(ref_k)
    ring = RingModel(cap, H, sink)
    ge = le = 0
    shift_rows = ring_rows = 0
    for c in range(3 * cap // chunk + 2):
        for step in range(steps):            # the chunk is rewritten at the same position per step
            kn = rng.standard_normal((chunk, H, 128)).astype(np.float32)
            vn = rng.standard_normal((chunk, H, 128)).astype(np.float32)
            start = c * chunk
            rolls = start + chunk > ge and chunk + le > cap
            new_le = oracle.cache_append(ref_k, ref_v, kn, vn, local_attn=True, global_end=ge, local_end=le,
                                         current_start=start, sink_tokens=sink)
            if rolls:
                shift_rows += le - (chunk + le - cap) - sink + chunk   # the rows the shifting cache moves
            assert ring.append(kn, vn, local_attn=True, global_end=ge, local_end=le, current_start=start) == new_le
            if rolls:
                ring_rows += ring.written
                assert ring.written <= chunk + 64 + 2 * (sink % 64) + 64
            ge, le = start + chunk, new_le
            wk, wv = ring.window(le)
            np.testing.assert_array_equal(wk, ref_k[:le])
            np.testing.assert_array_equal(wv, ref_v[:le])
    assert ring.head != 0                       # the stream went round the ring
    assert ring_rows < shift_rows               # and wrote less than the shifting cache moved


def test_sub_rows_are_contiguous_and_in_range():
    ring = RingModel(34320, 1, 1560)
    for head in (0, 1, 23, 24, 25, ring.C - 64, ring.C - 1):
        ring.head = head
        for t0 in range(0, 34320, 64):
            p = ring.sub_row(t0)
            assert 0 <= p and p + 64 <= ring.k.shape[0]
