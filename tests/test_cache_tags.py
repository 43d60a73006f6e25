"""Host-side bookkeeping of the router key tables: the window tag a KVCache gives the router
changes exactly when the history rows change place or content (a roll, a restore, an anchor
rebase, a reset), and not when a denoising call rewrites the current chunk's rows."""
import torch

from streaming_sparse_b200.cache import KVCache
from streaming_sparse_b200.ops import RouterKeys, history_blocks


def test_tag_follows_rolls_and_rewrites():
    c = KVCache(24, num_heads=1, frame_tokens=4, local_attn_size=6, sink_size=1, device="cpu",
                track_positions=False)
    tags = []
    for chunk in range(5):
        for step in range(3):
            start = chunk * 8
            predicted = c.tag_after(8, start)
            c.advance(8, start)
            assert c.history_tag() == predicted
            tags.append(c.history_tag())
    # rewrites of a chunk keep the tag
    for chunk in range(5):
        assert tags[3 * chunk] == tags[3 * chunk + 1] == tags[3 * chunk + 2]
    # chunks 0..2 fill the 24-token cache without a roll (window start 0 each time): the rows
    # already written keep their place; chunks 3 and 4 roll the window
    assert tags[0] == tags[3] == tags[6]
    assert len({tags[6], tags[9], tags[12]}) == 3


def test_tag_bumps_on_restore_and_reset():
    c = KVCache(16, num_heads=1, frame_tokens=4, device="cpu", track_positions=False)
    c.advance(8, 0)
    t0 = c.history_tag()
    snap = c.snapshot()
    c.restore(snap)
    t1 = c.history_tag()
    assert t1 != t0
    c.reset()
    assert c.history_tag() != t1 and c.local_end == 0


def test_router_keys_validity():
    rk = RouterKeys(2, 1000, block=64, device="cpu")
    assert rk.kh.shape == (2, 16, 64)             # 16 blocks, already a multiple of 4
    assert rk.cached(("a", 0, 0)) == 0
    rk.mark(("a", 0, 0), 7)
    assert rk.cached(("a", 0, 0)) == 7 and rk.cached(("a", 1, 0)) == 0
    rk.invalidate()
    assert rk.cached(("a", 0, 0)) == 0
    assert history_blocks(4680, 32760, 64) == 438 and history_blocks(64, 64, 64) == 0
    assert torch.float32 == rk.kh.dtype
