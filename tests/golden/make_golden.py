"""Generate the golden vectors in tests/golden/ from the reference's own pure-torch code.

Run from the repository root in a container where the reference checkout is importable:

    python tests/golden/make_golden.py --reference <path to jurky123/streaming_sparse>

The reference is read, never modified; it is not needed at test time (the .npz files are
committed). Each fixture names the reference function that produced it:

* select_v05.npz      streaming_sparse/v05/primitives.py:35-56 ``select`` (stable top-k by score,
                      lower block id on ties, -0 == +0) -- forced blocks enter with +inf score.
* attention_v08.npz   streaming_sparse/v08/attention.py:115-123 ``reference`` (per-query gather of
                      the selected history blocks plus every current token, float64 softmax).
* padded_ids.npz      local_experiments/review_v1/ops.py:113-138 ``RouteOps.select`` (fixed count,
                      own page forced, -1 padding that must not be read).
* merge_vr1.npz       local_experiments/video_runtime_v1/attention.py:40-45 ``merge``.
* positions_adapter.npz  streaming_sparse/integration/self_forcing_adapter.py:50-97 ``_pre``
                      (absolute position of every visible cache slot through roll/evict).
* score_cached.npz    migration/unified_router/fast_route.py:10-34 ``prepare`` + ``score_cached``
                      (block scores: one prototype per key block = the plain mean of its valid
                      tokens, projected by the shared basis; q . k / sqrt(128) + log(count)). The
                      block means are computed here in float64 (the reference builds them with
                      its Triton ``segment`` kernel, opt19/prototype.py:11-49, which reduces to the
                      plain mean with one prototype and does not run without a GPU).
* anchor_rebase.npz   local_experiments/anchor_rebase.py:8-18 ``shift_temporal_`` (temporal RoPE
                      pairs of the anchor frame rotated by a frame offset, float64, back to bf16),
                      with the RoPE table built as wan/modules/model.py:29-37 ``rope_params``
                      concatenated as causal_model.py:500-505 (``wan`` itself is not importable
                      here, so the table is rebuilt from that formula).
"""
import argparse
import inspect
import math
import os
import sys

import numpy as np
import torch

OUT = os.path.dirname(os.path.abspath(__file__))


def select_cases(select):
    torch.manual_seed(701)
    cases = {}
    B = 96
    forced = torch.zeros(B, dtype=torch.bool)
    forced[:5] = True          # sink-like
    forced[70:] = True         # current-chunk-like
    nforced = int(forced.sum())
    for name, scores in [
        ("random", torch.randn(16, B)),
        ("bins1", torch.randint(-1, 1, (16, B)).float()),
        ("bins2", torch.randint(-2, 2, (16, B)).float()),
        ("bins20", torch.randint(-20, 20, (16, B)).float()),
        ("bins4096", torch.randint(-4096, 4096, (16, B)).float()),
    ] + [(f"signed_zero_{s}", torch.full((16, B), -0.0).index_fill_(1, torch.arange(0, B, s), 0.0))
         for s in (2, 3, 9, 47)]:
        for extra in (0, 1, 7, 24, B - nforced):
            ranked = scores.masked_fill(forced[None], float("inf"))
            mask = select(ranked, torch.ones(B), nforced + extra)
            cases[f"{name}_e{extra}_scores"] = scores.numpy()
            cases[f"{name}_e{extra}_mask"] = mask.numpy().astype(np.uint8)
            cases[f"{name}_e{extra}_extra"] = np.array(extra)
    cases["forced"] = forced.numpy().astype(np.uint8)
    np.savez_compressed(os.path.join(OUT, "select_v05.npz"), **cases)


def attention_cases(reference):
    torch.manual_seed(11)
    size, D = 64, 128
    cases = {}
    # inputs are bf16 values (stored as their uint16 bits) so the GPU tests can feed them as-is
    bf = lambda *shape: torch.randn(*shape).bfloat16().double()
    for idx, (nh, nc, nq) in enumerate([(192, 100, 100), (128, 40, 70)]):
        q = bf(nq, D)
        kh, vh = bf(nh, D), bf(nh, D)
        kc, vc = bf(nc, D), bf(nc, D)
        nb = math.ceil(nh / size)
        qblocks = math.ceil(nq / size)
        block_mask = (torch.rand(qblocks, nb) > 0.5).double()
        block_mask[:, 0] = 1
        mask = block_mask.repeat_interleave(size, 0)[:nq]
        out = reference(q, kh, vh, kc, vc, mask, size)
        for key, val in dict(q=q, kh=kh, vh=vh, kc=kc, vc=vc).items():
            cases[f"c{idx}_{key}"] = val.bfloat16().view(torch.int16).numpy().view(np.uint16)
        cases[f"c{idx}_block_mask"] = block_mask.numpy().astype(np.uint8)
        cases[f"c{idx}_out"] = out.float().numpy()
    np.savez_compressed(os.path.join(OUT, "attention_v08.npz"), **cases)


def padded_ids_case(RouteOps, Config):
    torch.manual_seed(192)
    cfg = Config()
    h, t, p = 2, 3, 410
    scores = torch.rand(h, t, p)
    own = torch.tensor([[338, 339, 340]]).expand(h, -1)
    sel = RouteOps.select(scores, own, cfg)
    np.savez_compressed(os.path.join(OUT, "padded_ids.npz"), scores=scores.numpy(), own=own.numpy(),
                        ids=sel["ids"].numpy(), counts=sel["counts"].numpy(), mask=sel["mask"].numpy())


def merge_case(merge):
    torch.manual_seed(5)
    N, H, D = 40, 2, 128
    eo = torch.randn(1, N, H, D)
    el = torch.randn(H, N) * 3
    ap = torch.randn(H, N, D)
    al = torch.randn(H, N) * 3
    al[0, :5] = -float("inf")   # an empty approximate part
    out = merge(eo, el, ap, al)
    np.savez_compressed(os.path.join(OUT, "merge_vr1.npz"), exact=eo.numpy(), exact_lse=el.numpy(),
                        approx=ap.numpy(), approx_lse=al.numpy(), out=out.float().numpy())


class _FakeAttention(torch.nn.Module):
    """Stands in for CausalWanSelfAttention: the adapter only reads these attributes and the
    forward signature; the index update after attention follows causal_model.py:252-253."""

    def __init__(self, local_attn_size, sink_size, frame):
        super().__init__()
        self.local_attn_size, self.sink_size = local_attn_size, sink_size
        self.max_attention_size = 32760 if local_attn_size == -1 else local_attn_size * frame

    def forward(self, x, seq_lens, grid_sizes, freqs, block_mask, kv_cache=None, current_start=0, cache_start=None):
        return x


def positions_case(SelfForcingAdapter):
    cases = {}
    schedules = {
        # the known-answer fixture of streaming_sparse/evaluation/validate.py:57-88
        "validate": dict(frame_hw=(2, 2), local=6, sink=1, cache=24, chunk_frames=3, chunks=3, steps=3, frame=1560),
        # a longer roll: 6-token frames, 4-frame window, sink 1
        "long": dict(frame_hw=(2, 3), local=5, sink=1, cache=30, chunk_frames=2, chunks=9, steps=2, frame=6),
        # no local window (global cache, no eviction)
        "global": dict(frame_hw=(1, 4), local=-1, sink=0, cache=48, chunk_frames=3, chunks=4, steps=2, frame=1560),
    }
    for name, s in schedules.items():
        hh, ww = s["frame_hw"]
        ftok = hh * ww
        n = s["chunk_frames"] * ftok
        module = _FakeAttention(s["local"], s["sink"], s["frame"])
        adapter = SelfForcingAdapter(torch.nn.Module())
        adapter.event = {}
        cache = dict(k=torch.zeros(1, s["cache"], 1, 8), v=torch.zeros(1, s["cache"], 1, 8),
                     global_end_index=torch.tensor([0]), local_end_index=torch.tensor([0]))
        rows = []
        for c in range(s["chunks"]):
            for _ in range(s["steps"]):
                start = c * n
                x = torch.zeros(1, n, 8)
                kwargs = dict(kv_cache=cache, current_start=start)
                args = (x, torch.tensor([n]), torch.tensor([[s["chunk_frames"], hh, ww]]), None, None)
                adapter._pre(0, module, args, kwargs)
                from streaming_sparse.integration.self_forcing_adapter import _active
                ctx = _active.get()
                pos = ctx["positions"]
                flat = (pos[:, 0] * hh * ww + pos[:, 1] * ww + pos[:, 2]).numpy()
                _active.reset(ctx["reset_token"])
                # index update exactly as the model does after attention
                g, l = int(cache["global_end_index"]), int(cache["local_end_index"])
                end = start + n
                if s["local"] != -1 and end > g and n + l > s["cache"]:
                    ev = n + l - s["cache"]
                    l = l + end - g - ev
                else:
                    l = l + end - g
                cache["global_end_index"].fill_(end)
                cache["local_end_index"].fill_(l)
                rows.append((start, n, ctx["history_tokens"], flat))
        cases[f"{name}_meta"] = np.array([ftok, s["local"], s["sink"], s["cache"], n, s["chunks"], s["steps"], s["frame"]])
        cases[f"{name}_calls"] = np.array([(r[0], r[1], r[2], len(r[3])) for r in rows])
        cases[f"{name}_positions"] = np.concatenate([r[3] for r in rows])
    np.savez_compressed(os.path.join(OUT, "positions_adapter.npz"), **cases)


def anchor_rebase_case(shift_temporal_):
    d = 128

    def rope_params(max_seq_len, dim, theta=10000):
        freqs = torch.outer(torch.arange(max_seq_len),
                            1.0 / torch.pow(theta, torch.arange(0, dim, 2).to(torch.float64).div(dim)))
        return torch.polar(torch.ones_like(freqs), freqs)

    freqs = torch.cat([rope_params(1024, d - 4 * (d // 6)), rope_params(1024, 2 * (d // 6)),
                       rope_params(1024, 2 * (d // 6))], dim=1)
    g = torch.Generator().manual_seed(909)
    keys = (3 * torch.randn(2, 64, 2, d, generator=g)).bfloat16()
    bits = lambda t: t.view(torch.int16).numpy()   # bf16 bit patterns
    cases = {"keys": bits(keys)}
    for offset, tokens in ((0, 64), (1, 64), (3, 0), (15, 40), (42, 64), (1023, 64)):
        k = keys.clone()
        shift_temporal_(k, tokens, freqs, offset)
        cases[f"out_{offset}_{tokens}"] = bits(k)
    np.savez_compressed(os.path.join(OUT, "anchor_rebase.npz"), **cases)


def score_cached_case(prepare, score_cached):
    from types import SimpleNamespace
    g = torch.Generator().manual_seed(811)
    Lq, Lk, H, block = 320, 2000, 3, 64           # 32 key blocks, the last one 16 tokens
    q = torch.randn((Lq, H, 128), generator=g).bfloat16().float()
    k = torch.randn((Lk, H, 128), generator=g).bfloat16().float()
    basis = torch.randn((H, 128, 64), generator=g) / math.sqrt(128)

    def means(x):
        L = x.shape[0]
        nb = -(-L // block)
        m = torch.zeros((H, nb, 128), dtype=torch.float64)
        cnt = torch.zeros((H, nb), dtype=torch.float64)
        for j in range(nb):
            rows = x[j * block:min(L, (j + 1) * block)].double()
            m[:, j] = rows.mean(0)
            cnt[:, j] = rows.shape[0]
        return m.float(), cnt.float()

    qm, _ = means(q)
    km, kcount = means(k)
    sketch = SimpleNamespace(key_basis=basis, parts=[SimpleNamespace(key=km[:, :, None], count=kcount[:, :, None],
                                                                      value=None)])
    _, projected = prepare(sketch, "U-Sol")
    score, _ = score_cached(qm, basis, projected)
    # q, k are bf16 values: stored as their bf16 bit patterns (int16)
    np.savez_compressed(os.path.join(OUT, "score_cached.npz"), q_bf16=q.bfloat16().view(torch.int16).numpy(),
                        k_bf16=k.bfloat16().view(torch.int16).numpy(), basis=basis.numpy(),
                        block=block, score=score.numpy(), logcount=kcount.log().numpy())


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True)
    ap.add_argument("--only", default=None, help="write just this fixture (file name without .npz)")
    a = ap.parse_args()
    sys.path.insert(0, a.reference)
    if a.only == "score_cached":
        from migration.unified_router.fast_route import prepare, score_cached
        torch.set_num_threads(4)
        score_cached_case(prepare, score_cached)
        return
    from streaming_sparse.v05.primitives import select
    from streaming_sparse.v08.attention import reference
    from local_experiments.review_v1.ops import RouteOps, Config
    from local_experiments.video_runtime_v1.attention import merge
    from streaming_sparse.integration.self_forcing_adapter import SelfForcingAdapter
    from local_experiments.anchor_rebase import shift_temporal_
    assert "kv_cache" in inspect.signature(_FakeAttention.forward).parameters
    torch.set_num_threads(4)
    select_cases(select)
    attention_cases(reference)
    padded_ids_case(RouteOps, Config)
    merge_case(merge)
    positions_case(SelfForcingAdapter)
    anchor_rebase_case(shift_temporal_)
    from migration.unified_router.fast_route import prepare, score_cached
    score_cached_case(prepare, score_cached)
    for f in sorted(os.listdir(OUT)):
        if f.endswith(".npz"):
            print(f, os.path.getsize(os.path.join(OUT, f)))


if __name__ == "__main__":
    main()
