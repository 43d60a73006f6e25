"""CPU oracle for the routed sparse-attention path -- TEST INFRASTRUCTURE, never the product.

Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline leg of ``bench.py`` import this
module, and only as the checker / timed CPU baseline. The package ``streaming_sparse_b200``
never imports it and has no CPU fallback.

Pieces and the reference code each one restates (paths inside jurky123/streaming_sparse):

* ``route``: exact-fp32 router in C (``ssparse_oracle.c``): block pooling
  (migration/unified_router/opt19/prototype.py:11-49), projection (opt8/projection.py:4-14),
  block-score GEMM (opt16/route.py:34-47), forced sink/current set
  (local_experiments/video_runtime_v1/pipeline_graph.py:140-151), top-k with lower-index ties
  (streaming_sparse/v05/primitives.py:35-56).
* ``attention``: gather-softmax over the selected blocks' valid tokens, float64
  (streaming_sparse/v08/attention.py:115-123 ``reference``; the page gather of
  local_experiments/review_v1/runtime.py:106-121 ``SelectedAttention.fixed``); natural-log LSE as
  returned by ``exact`` (local_experiments/video_runtime_v1/attention.py:15-24).
* ``lse_merge``: local_experiments/video_runtime_v1/attention.py:40-45 ``merge`` generalised to
  P parts (migration/unified_router/opt21/attention.py:7-15).
* ``cache_append``: the roll + write of CausalWanSelfAttention.forward
  (wan/modules/causal_model.py:216-253).
* ``rope_shift``: the anchor rebase ``shift_temporal_`` (local_experiments/anchor_rebase.py:8-18):
  the temporal RoPE pairs of the first tokens rotated by a frame offset in float64.

Parity pins: tests/golden/ holds vectors produced by the reference's own pure-torch functions
(script ``tests/golden/make_golden.py``); ``tests/test_oracle.py`` checks this module against
them before any GPU result is compared with it.
"""
from __future__ import annotations

import ctypes
import math
import os
import subprocess
from functools import lru_cache

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "libssoracle.so")
SRC = os.path.join(HERE, "ssparse_oracle.c")


def build(force: bool = False) -> str:
    """Compile the C restatement (strict IEEE fp32: no contraction, no fast-math)."""
    if force or not os.path.exists(LIB) or os.path.getmtime(LIB) < os.path.getmtime(SRC):
        tmp = LIB + ".tmp"
        subprocess.run(["gcc", "-O2", "-fPIC", "-shared", "-ffp-contract=off", "-fno-fast-math",
                        "-o", tmp, SRC, "-lm"], check=True)
        os.replace(tmp, LIB)
    return LIB


@lru_cache(None)
def _lib():
    lib = ctypes.CDLL(build())
    P = ctypes.c_void_p
    i, i64 = ctypes.c_int, ctypes.c_int64
    lib.oracle_pool_project.argtypes = [P, i64, i, i, i, i, i, P, P, P]
    lib.oracle_pool_project.restype = i
    lib.oracle_scores.argtypes = [P, P, i, i, i, i, P]
    lib.oracle_scores.restype = i64
    lib.oracle_forced.argtypes = [i, i, i, i, P]
    lib.oracle_forced.restype = i
    lib.oracle_select.argtypes = [P, i, i, i, P, i, P, i, P]
    lib.oracle_select.restype = i
    return lib


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(ctypes.c_void_p)


def bf16_round(x: np.ndarray) -> np.ndarray:
    """Round float32 values to bfloat16 (round-to-nearest-even) and return them as float32."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
    return u.astype(np.uint32).view(np.float32)


def nblocks(n: int, block: int) -> int:
    return (n + block - 1) // block


# ----------------------------------------------------------------------------------------------
# router
# ----------------------------------------------------------------------------------------------

def pool_project(x: np.ndarray, w: np.ndarray, block: int):
    """x [L,H,D] fp32 (bf16 values), w [H,D,R] fp32 -> (pooled [H,nb,D], proj [H,nb,R])."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    w = np.ascontiguousarray(w, dtype=np.float32)
    L, H, D = x.shape
    R = w.shape[2]
    nb = nblocks(L, block)
    pooled = np.empty((H, nb, D), np.float32)
    proj = np.empty((H, nb, R), np.float32)
    rc = _lib().oracle_pool_project(_ptr(x), H * D, L, H, D, R, block, _ptr(w), _ptr(pooled), _ptr(proj))
    if rc:
        raise MemoryError("oracle_pool_project failed")
    return pooled, proj


def scores(qh: np.ndarray, kh: np.ndarray):
    """qh [H,qb,R], kh [H,kb,R] -> (S [H,qb,kb] fp32, number of non-finite scores)."""
    qh = np.ascontiguousarray(qh, dtype=np.float32)
    kh = np.ascontiguousarray(kh, dtype=np.float32)
    H, qb, R = qh.shape
    kb = kh.shape[1]
    S = np.empty((H, qb, kb), np.float32)
    bad = _lib().oracle_scores(_ptr(qh), _ptr(kh), H, qb, kb, R, _ptr(S))
    return S, int(bad)


def forced_blocks(Lq: int, Lk: int, block: int, sink_tokens: int = 0) -> np.ndarray:
    kb = nblocks(Lk, block)
    f = np.zeros(kb, np.uint8)
    _lib().oracle_forced(Lq, Lk, block, sink_tokens, _ptr(f))
    return f


def select(S: np.ndarray, forced: np.ndarray, extra: int):
    """Top-`extra` unforced blocks per row plus the forced set -> (ids ascending, mask)."""
    S = np.ascontiguousarray(S, dtype=np.float32)
    forced = np.ascontiguousarray(forced, dtype=np.uint8)
    H, qb, kb = S.shape
    n_ids = int(forced.sum()) + extra
    ids = np.empty((H, qb, n_ids), np.int32)
    mask = np.empty((H, qb, kb), np.uint8)
    rc = _lib().oracle_select(_ptr(S), H, qb, kb, _ptr(forced), extra, _ptr(ids), n_ids, _ptr(mask))
    if rc:
        raise ValueError(f"oracle_select rejected extra={extra} (forced={int(forced.sum())}, kb={kb})")
    return ids, mask.astype(bool)


def route(q, k, wq, wk, block: int, extra: int, sink_tokens: int = 0):
    """Full router: returns dict(ids, mask, scores, qh, kh, nonfinite)."""
    Lq, Lk = q.shape[0], k.shape[0]
    _, qh = pool_project(q, wq, block)
    _, kh = pool_project(k, wk, block)
    S, bad = scores(qh, kh)
    f = forced_blocks(Lq, Lk, block, sink_tokens)
    ids, mask = select(S, f, extra)
    return dict(ids=ids, mask=mask, scores=S, qh=qh, kh=kh, nonfinite=bad, forced=f)


def budget(kb: int, nforced: int, *, topk: int | None = None, density: float | None = None,
           rule: str = "total") -> int:
    """Number of score-chosen blocks per query block.

    * ``topk``: a fixed count outside the forced set (config 1: 24).
    * ``density`` with rule ``"total"``: the row keeps ceil(density*kb) blocks in all, forced
      ones included (config 2).
    * ``density`` with rule ``"rest"``: floor(density*(kb - forced)) extra blocks, the
      ``chunk_history10`` policy of local_experiments/video_runtime_v1/pipeline_graph.py:143-146.
    """
    if topk is not None:
        extra = topk
    elif rule == "total":
        extra = math.ceil(density * kb) - nforced
    elif rule == "rest":
        extra = math.floor(density * (kb - nforced))
    else:
        raise ValueError(rule)
    return max(0, min(extra, kb - nforced))


# ----------------------------------------------------------------------------------------------
# attention
# ----------------------------------------------------------------------------------------------

def selected_tokens(ids_row: np.ndarray, Lk: int, block: int) -> np.ndarray:
    blocks = np.unique(ids_row[ids_row >= 0])
    tok = (blocks[:, None] * block + np.arange(block)[None, :]).reshape(-1)
    return tok[tok < Lk]


def attention_block(q, k, v, ids_row, h: int, r0: int, r1: int, block: int, scale: float, dtype=np.float64):
    """One (head, query block): rows [r0, r1) of head h against the valid tokens of ids_row."""
    tok = selected_tokens(ids_row, k.shape[0], block)
    if len(tok) == 0:
        n = r1 - r0
        return np.zeros((n, q.shape[2]), dtype), np.full(n, -np.inf, dtype)
    kk = np.asarray(k[tok, h, :], dtype)
    vv = np.asarray(v[tok, h, :], dtype)
    z = (np.asarray(q[r0:r1, h, :], dtype) @ kk.T) * dtype(scale)
    m = z.max(axis=1, keepdims=True)
    p = np.exp(z - m)
    s = p.sum(axis=1, keepdims=True)
    return (p @ vv) / s, (m + np.log(s))[:, 0]


def attention(q, k, v, ids, block: int, scale: float | None = None, dtype=np.float64,
              heads=None, qblocks=None):
    """Gather-softmax attention. q [Lq,H,D], k/v [Lk,H,D], ids [H,qb,K] (entries <0 ignored).

    Returns (out [Lq,H,D], lse [H,Lq]) in ``dtype``; rows of skipped heads/qblocks are NaN,
    rows whose list is empty are 0 with LSE -inf.
    """
    Lq, H, D = q.shape
    scale = 1.0 / math.sqrt(D) if scale is None else scale
    qb = nblocks(Lq, block)
    out = np.full((Lq, H, D), np.nan, dtype)
    lse = np.full((H, Lq), np.nan, dtype)
    for h in (range(H) if heads is None else heads):
        for i in (range(qb) if qblocks is None else qblocks):
            r0, r1 = i * block, min(Lq, (i + 1) * block)
            out[r0:r1, h, :], lse[h, r0:r1] = attention_block(q, k, v, ids[h, i], h, r0, r1, block, scale, dtype)
    return out, lse


def lse_merge(o_parts: np.ndarray, lse_parts: np.ndarray):
    """o_parts [P,Lq,H,D], lse_parts [P,H,Lq] natural log -> (out [Lq,H,D], lse [H,Lq])."""
    o = np.asarray(o_parts, np.float64)
    l = np.asarray(lse_parts, np.float64)
    mx = l.max(axis=0)
    safe = np.where(np.isfinite(mx), mx, 0.0)
    w = np.exp(l - safe[None])                      # [P,H,Lq]
    tot = w.sum(axis=0)
    lse = np.where(tot > 0, safe + np.log(np.where(tot > 0, tot, 1.0)), -np.inf)
    wn = np.where(tot[None] > 0, w / np.where(tot > 0, tot, 1.0)[None], 0.0)
    out = np.einsum("phl,plhd->lhd", wn, o)
    return out, lse


# ----------------------------------------------------------------------------------------------
# cache
# ----------------------------------------------------------------------------------------------

def cache_append(k_cache, v_cache, k_new, v_new, *, local_attn: bool, global_end: int,
                 local_end: int, current_start: int, sink_tokens: int):
    """In-place roll + write on numpy caches [cap,H,D]; returns the new local end index.

    Restates wan/modules/causal_model.py:216-246 (the branch taken when a kv_cache is given).
    """
    cap = k_cache.shape[0]
    n = k_new.shape[0]
    current_end = current_start + n
    if local_attn and current_end > global_end and n + local_end > cap:
        evicted = n + local_end - cap
        rolled = local_end - evicted - sink_tokens
        src = slice(sink_tokens + evicted, sink_tokens + evicted + rolled)
        dst = slice(sink_tokens, sink_tokens + rolled)
        k_cache[dst] = k_cache[src].copy()
        v_cache[dst] = v_cache[src].copy()
        new_local_end = local_end + current_end - global_end - evicted
    else:
        new_local_end = local_end + current_end - global_end
    start = new_local_end - n
    k_cache[start:new_local_end] = k_new
    v_cache[start:new_local_end] = v_new
    return new_local_end


# ----------------------------------------------------------------------------------------------

def rope_phase(offset: int, pairs: int = 22, head_dim: int = 128) -> np.ndarray:
    """[pairs, 2] float64 (cos, sin) of offset * theta_p, theta_p = 10000^(-2p / (head_dim - 4*(head_dim//6))):
    the temporal part of the model's RoPE table (wan/modules/model.py:29-37 rope_params with the
    split of causal_model.py:500-505), row `offset`."""
    n = head_dim - 4 * (head_dim // 6)
    theta = 1.0 / np.power(10000.0, np.arange(0, n, 2, dtype=np.float64) / n)
    ang = offset * theta[:pairs]
    return np.stack([np.cos(ang), np.sin(ang)], axis=-1)


def rope_shift(keys: np.ndarray, tokens: int, phase: np.ndarray) -> np.ndarray:
    """keys [..., T, H, D] (bf16 values as float32) -> copy with the first `tokens` rows' first
    `pairs` complex pairs multiplied by phase (float64), rounded to float32 then bf16, as
    ``shift_temporal_`` does (local_experiments/anchor_rebase.py:8-18; the double -> bf16 cast
    goes through float). Spatial pairs and later rows are unchanged."""
    out = np.array(keys, dtype=np.float32, copy=True)
    pairs = phase.shape[0]
    part = out[..., :tokens, :, :2 * pairs].astype(np.float64)
    x, y = part[..., 0::2], part[..., 1::2]
    c, s = phase[:, 0], phase[:, 1]
    re = x * c - y * s
    im = x * s + y * c
    rot = np.empty_like(part)
    rot[..., 0::2], rot[..., 1::2] = re, im
    out[..., :tokens, :, :2 * pairs] = bf16_round(rot.astype(np.float32))
    return out


# ----------------------------------------------------------------------------------------------
# INT8-QK sparse attention (SpargeAttn-style path)
# ----------------------------------------------------------------------------------------------
# Restates migration/unified_router/opt23/attention.py: ``_quant`` (:6-14, K per 64-token page and
# head) and ``_shared`` with INT8=True (:30-58: Q per G-row group and head, quantised in the
# kernel; logits = int32 dot * (qs * ks[page]) * log2(e)/sqrt(128); base-2 online softmax; P cast to
# V's type for the P.V product), used with G = 32 by opt24/pipeline.py:24-25 and opt24/sparge.py.

QUANT_PAGE = 64      # K rows sharing one scale (one page)
QUANT_QGROUP = 32    # Q rows sharing one scale


def quant_rows(x: np.ndarray, rows: int):
    """x [L,H,D] (float32 holding the bf16 values) -> (x_i8 [L,H,D] int8, scale [H,ceil(L/rows)] fp32).

    Per group of ``rows`` consecutive rows and per head: scale = max(max|x| / 127, 1e-10) in fp32,
    x_i8 = round-half-even(x / scale) with an IEEE fp32 divide (opt23/attention.py:10-13,37-39).
    Rows past L count as zeros in their group's maximum.
    """
    x = np.asarray(x, np.float32)
    L, H, D = x.shape
    n = -(-L // rows)
    pad = np.zeros((n * rows, H, D), np.float32)
    pad[:L] = x
    g = pad.reshape(n, rows, H, D)
    amax = np.abs(g).max(axis=(1, 3))                                     # [n,H]
    s = np.maximum(amax / np.float32(127.0), np.float32(1e-10)).astype(np.float32)
    xi = np.rint(g / s[:, None, :, None]).astype(np.int8)
    return xi.reshape(n * rows, H, D)[:L].copy(), np.ascontiguousarray(s.T)


def i8_logit_scale(scale: float) -> np.float32:
    """fp32 multiplier of the scaled int32 logits: scale * log2(e), rounded once to fp32."""
    return np.float32(float(np.float32(scale)) * 1.4426950408889634)


def i8_logits(qi_rows, qs_rows, ki_tok, ks_tok, c):
    """fp32 base-2 logits of ``_shared`` (:47-48): ((int32 dot) * (qs * ks)) * c, each product rounded."""
    # integer dot products, exact in float64 (|dot| <= 127 * 127 * 128 < 2^24) and so in fp32
    dot = qi_rows.astype(np.float64) @ ki_tok.astype(np.float64).T
    t = (qs_rows[:, None].astype(np.float32) * ks_tok[None, :].astype(np.float32)).astype(np.float32)
    return ((dot.astype(np.float32) * t).astype(np.float32) * np.float32(c)).astype(np.float32)


def attention_i8(q, k_i8, ks, v, ids, block: int, scale: float | None = None, heads=None, qblocks=None):
    """INT8-QK block-sparse attention with this library's layouts, exact softmax in float64.

    q [Lq,H,D] (bf16 values), k_i8 [Lk,H,D] int8 and ks [H,ceil(Lk/64)] from ``quant_rows(k, 64)``,
    v [Lk,H,D], ids [H,qb,K] block ids of ``block`` tokens (<0 ignored). Q is quantised per 32-row
    group. Returns (out [Lq,H,D], lse [H,Lq]) in float64 (natural-log LSE); skipped rows are NaN.
    """
    q = np.asarray(q, np.float32)
    Lq, H, D = q.shape
    Lk = k_i8.shape[0]
    scale = 1.0 / math.sqrt(D) if scale is None else scale
    c = i8_logit_scale(scale)
    qi, qs = quant_rows(q, QUANT_QGROUP)
    qb = nblocks(Lq, block)
    out = np.full((Lq, H, D), np.nan)
    lse = np.full((H, Lq), np.nan)
    for h in (range(H) if heads is None else heads):
        for i in (range(qb) if qblocks is None else qblocks):
            r0, r1 = i * block, min(Lq, (i + 1) * block)
            tok = selected_tokens(ids[h, i], Lk, block)
            if len(tok) == 0:
                out[r0:r1, h], lse[h, r0:r1] = 0.0, -np.inf
                continue
            rows = np.arange(r0, r1)
            y = i8_logits(qi[rows, h], qs[h, rows // QUANT_QGROUP], k_i8[tok, h], ks[h, tok // QUANT_PAGE], c)
            z = y.astype(np.float64)
            m = z.max(axis=1, keepdims=True)
            p = np.exp2(z - m)
            s = p.sum(axis=1, keepdims=True)
            out[r0:r1, h] = (p @ np.asarray(v[tok, h], np.float64)) / s
            lse[h, r0:r1] = (m[:, 0] + np.log2(s[:, 0])) * math.log(2.0)
    return out, lse


def shared_i8_tiles(q, k_i8, ks, v, pages, group: int = QUANT_QGROUP, c=None, p_dtype=np.float16):
    """The ``_shared`` kernel's own loop (opt23/attention.py:30-58, INT8=True, SPLITS=1), in its
    layouts: q [H,N,D], k_i8 [H,NK,D], ks [H,B], v [H,NK,D], pages [H,T,KEEP] 64-token page ids per
    ``group``-row tile, visited in list order; P rounded to ``p_dtype`` (V's type) before P.V, fp32
    accumulation. Returns out [H,N,D] float32. Used to pin the restatement to the golden vectors."""
    q = np.asarray(q, np.float32)
    H, N, D = q.shape
    NK = k_i8.shape[1]
    c = np.float32(0.12751743082459617) if c is None else np.float32(c)
    out = np.zeros((H, N, D), np.float32)
    for h in range(H):
        for t in range(pages.shape[1]):
            rows = np.arange(t * group, min(N, (t + 1) * group))
            qt = np.zeros((group, D), np.float32)
            qt[:len(rows)] = q[h, rows]
            qi, qs = quant_rows(qt[:, None, :], group)
            m = np.full(group, -np.inf, np.float32)
            den = np.zeros(group, np.float32)
            acc = np.zeros((group, D), np.float32)
            for page in pages[h, t]:
                ki = page * QUANT_PAGE + np.arange(QUANT_PAGE)
                valid = ki < NK
                kk = np.zeros((QUANT_PAGE, D), np.int8)
                kk[valid] = k_i8[h, ki[valid]]
                y = i8_logits(qi[:, 0], np.full(group, qs[0, 0], np.float32), kk,
                              np.full(QUANT_PAGE, ks[h, page], np.float32), c)
                y = np.where(valid[None, :], y, np.float32(-np.inf))
                nm = np.maximum(m, y.max(axis=1))
                al = np.exp2(m - nm).astype(np.float32)
                pr = np.exp2(y - nm[:, None]).astype(np.float32)
                vv = np.zeros((QUANT_PAGE, D), np.float32)
                vv[valid] = v[h, ki[valid]]
                acc = (acc * al[:, None] + pr.astype(p_dtype).astype(np.float32) @ vv).astype(np.float32)
                den = (den * al + pr.sum(axis=1)).astype(np.float32)
                m = nm
            out[h, rows] = (acc / den[:, None])[:len(rows)]
    return out
