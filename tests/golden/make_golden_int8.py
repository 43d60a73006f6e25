"""Generate tests/golden/int8_qk.npz from the reference's own INT8-QK kernels.

    python tests/golden/make_golden_int8.py --reference <path to jurky123/streaming_sparse>

The reference's INT8-QK attention (migration/unified_router/opt23/attention.py) is two Triton
kernels: ``_quant`` (K quantised per 64-token page and head, :6-14) and ``_shared`` with INT8=True
(Q quantised per G-row tile inside the kernel, int8 dot, base-2 online softmax, :30-58). They run
here unmodified under Triton's CPU interpreter (TRITON_INTERPRET=1), with one substitution: the
interpreter cannot call libdevice, so ``nearbyint`` (round half to even) is replaced by an exact
round-half-even written with floor. V is passed as fp16, the type the reference's Sparge path
gives it (opt24/sparge.py:41 ``self.v=self.pv.half()``): the interpreter's P.V product does not
handle bf16. V is drawn in bf16 (tiny values zeroed), so its values are exact in both types. Pages are made window-global by passing SEG = (number of pages) * 64, so page p covers
tokens [64p, 64p + 64), as in this library.

Two fixtures: int8_qk.npz (64-token routing blocks, one page each) and int8_qk_b128.npz (the same
keys and values, 128-token routing blocks of two pages each, 256 queries).

The reference is read, never modified, and is not needed at test time (the .npz files are committed).
"""
import argparse
import importlib
import os
import sys

os.environ["TRITON_INTERPRET"] = "1"

import numpy as np  # noqa: E402
import torch  # noqa: E402
import triton  # noqa: E402
import triton.language as tl  # noqa: E402

OUT = os.path.dirname(os.path.abspath(__file__))


@triton.jit
def round_half_even(x):
    r = tl.floor(x)
    f = x - r
    odd = (r - 2.0 * tl.floor(r * 0.5)) != 0.0
    return tl.where(f > 0.5, r + 1.0, tl.where(f < 0.5, r, tl.where(odd, r + 1.0, r)))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True)
    a = ap.parse_args()
    sys.path.insert(0, a.reference)
    att = importlib.import_module("migration.unified_router.opt23.attention")
    for kern in (att._quant, att._shared):
        kern.fn.__globals__["nearbyint"] = round_half_even

    g = torch.Generator().manual_seed(8)
    H, N, NK, G, KEEP = 2, 128, 300, 32, 3          # 5 pages, the last one 44 tokens
    pages = -(-NK // 64)
    SEG = pages * 64
    k = torch.randn((H, NK, 128), generator=g).bfloat16()
    k[1, 64:128] = 0                                 # an all-zero page: scale clamps to 1e-10
    k[0, :7, :5] *= 40                               # outliers set a page's scale
    v = torch.randn((H, NK, 128), generator=g).bfloat16()
    v[v.abs() < 1e-3] = 0                           # every value exact in both bf16 and fp16
    v = v.half()
    q = torch.randn((H, N, 128), generator=g).bfloat16()
    q[0, 32:64] = 0                                  # an all-zero query group
    q[1, :32] *= 3
    ki = torch.zeros((H, NK, 128), dtype=torch.int8)
    ks = torch.zeros((H, pages), dtype=torch.float32)
    att._quant[(pages, H)](k, ki, ks, NK, pages, 0, SEG, num_warps=4)

    # page lists: one ascending list per 64-row query block (its two 32-row tiles share it),
    # always holding the last page (the partial one), as a forced current chunk would
    T = N // G
    rng = np.random.default_rng(8)
    lists = np.zeros((H, N // 64, KEEP), np.int32)
    for h in range(H):
        for b in range(N // 64):
            lists[h, b] = np.sort(np.concatenate([rng.choice(pages - 1, KEEP - 1, replace=False), [pages - 1]]))
    tiles = np.repeat(lists, 2, axis=1)              # [H, T, KEEP]
    out = torch.zeros((H, N, 128), dtype=torch.float32)
    att._shared[(T, H, 1)](q, ki, v, ks, torch.from_numpy(tiles), out, out, N, NK, pages, G, T, KEEP, 1, True,
                           SEG, num_warps=4)
    np.savez_compressed(
        os.path.join(OUT, "int8_qk.npz"),
        k=k.float().numpy(), v=v.float().numpy(), q=q.float().numpy(), k_i8=ki.numpy(), ks=ks.numpy(),
        page_lists=lists, tiles=tiles, out=out.numpy(), group=np.int32(G))
    print("wrote int8_qk.npz", out.abs().mean().item())

    # 128-token routing blocks: block id b covers pages 2b and 2b + 1 (the last block's second page
    # lies past the window and is dropped), so a 128-row query block's page list is its blocks'
    # pages; its four 32-row tiles share that list
    g2 = torch.Generator().manual_seed(128)
    N2 = 256
    q2 = torch.randn((H, N2, 128), generator=g2).bfloat16()
    blocks = np.array([[[0, 2], [1, 2]], [[1, 2], [0, 2]]], np.int32)        # [H, 2 query blocks, 2]: 3 pages each
    plists = np.zeros((H, 2, 3), np.int32)
    for h in range(H):
        for b in range(2):
            pg = [2 * x + u for x in blocks[h, b] for u in range(2) if 2 * x + u < pages]
            plists[h, b] = pg
    tiles2 = np.repeat(plists, 4, axis=1)                                       # [H, 8, 3]
    out2 = torch.zeros((H, N2, 128), dtype=torch.float32)
    att._shared[(N2 // G, H, 1)](q2, ki, v, ks, torch.from_numpy(tiles2), out2, out2, N2, NK, pages, G, N2 // G, 3, 1,
                                 True, SEG, num_warps=4)
    np.savez_compressed(os.path.join(OUT, "int8_qk_b128.npz"), q=q2.float().numpy(), block_lists=blocks,
                        tiles=tiles2, out=out2.numpy())
    print("wrote int8_qk_b128.npz", out2.abs().mean().item())


if __name__ == "__main__":
    main()
