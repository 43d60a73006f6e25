"""Op-level API: the reference's router / sparse-attention / merge / cache ops on libssparse.so.

Every function takes CUDA tensors, enqueues work on the current stream through the C ABI and
raises on a nonzero status; none has a CPU path. Mirrors of the reference's op signatures:

* ``exact(q, k, v, ids, workspace)`` -> (O fp32 [1,N,H,D], natural LSE [H,N]) as
  local_experiments/video_runtime_v1/attention.py:15-24.
* ``merge(exact_output, exact_lse, approx, approx_lse)`` -> bf16 [1,N,H,D] as
  local_experiments/video_runtime_v1/attention.py:40-45.
* ``Workspace`` as local_experiments/video_runtime_v1/attention.py:7-13.
* ``route(q, k, wq, wk, ...)`` replaces the router pipeline (project / pool / score / top-k of
  migration/unified_router/opt16/route.py:90-113 with the forced set of
  local_experiments/video_runtime_v1/pipeline_graph.py:140-151) and returns the page LUT
  ``ids[H, qb, n]`` (ascending, as checked by migration/unified_router/opt28/
  validate_selection.py:30) that ``exact`` consumes.
"""
from __future__ import annotations

import ctypes
import math

import torch

from ._lib import DEV_BADID, DEV_NONFINITE, DEV_TIMEOUT, check, lib

HEAD_DIM = 128


class Workspace:
    """Named, shape-keyed device buffers reused across calls (no per-call allocation)."""

    def __init__(self):
        self.entries = {}

    def tensor(self, name, shape, device, dtype):
        key = (name, tuple(shape), str(device), dtype)
        if key not in self.entries:
            self.entries[key] = torch.empty(shape, device=device, dtype=dtype)
        return self.entries[key]

    def bytes(self):
        return sum(x.numel() * x.element_size() for x in self.entries.values())


_DEFAULT_WS: dict[str, Workspace] = {}


def _ws(workspace, device) -> Workspace:
    if workspace is not None:
        return workspace
    key = str(device)
    if key not in _DEFAULT_WS:
        _DEFAULT_WS[key] = Workspace()
    return _DEFAULT_WS[key]


def _stream(device) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _p(t: torch.Tensor | None):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _require(cond: bool, msg: str):
    if not cond:
        raise ValueError(msg)


def _tokens(x: torch.Tensor, name: str) -> torch.Tensor:
    """Accept [L,H,D] or [1,L,H,D] bf16 CUDA tensors; return the [L,H,D] view."""
    if x.dim() == 4:
        _require(x.shape[0] == 1, f"{name}: batch size must be 1 (got {x.shape[0]})")
        x = x[0]
    _require(x.dim() == 3 and x.shape[-1] == HEAD_DIM, f"{name}: expected [L,H,{HEAD_DIM}], got {tuple(x.shape)}")
    _require(x.is_cuda, f"{name}: must be a CUDA tensor (libssparse has no CPU path)")
    _require(x.dtype == torch.bfloat16, f"{name}: must be bfloat16")
    _require(x.is_contiguous(), f"{name}: must be contiguous")
    return x


def nblocks(n: int, block: int) -> int:
    return (n + block - 1) // block


def forced_count(Lq: int, Lk: int, block: int, sink_tokens: int = 0) -> int:
    """Blocks overlapping the sink [0, sink_tokens) or the current chunk [Lk-Lq, Lk)."""
    return sum(1 for j in range(nblocks(Lk, block))
               if j * block < sink_tokens or min((j + 1) * block, Lk) > Lk - Lq)


def budget(kb: int, nforced: int, *, topk: int | None = None, density: float | None = None,
           rule: str = "total") -> int:
    """Score-chosen blocks per query block (outside the forced set).

    ``topk``: fixed count (config 1: 24). ``density`` + ``rule="total"``: the row keeps
    ceil(density*kb) blocks including the forced ones. ``density`` + ``rule="rest"``:
    floor(density*(kb-forced)) extra blocks (local_experiments/video_runtime_v1/
    pipeline_graph.py:143-146).
    """
    if topk is not None:
        extra = topk
    elif density is None:
        raise ValueError("give topk or density")
    elif rule == "total":
        extra = math.ceil(density * kb) - nforced
    elif rule == "rest":
        extra = math.floor(density * (kb - nforced))
    else:
        raise ValueError(f"unknown budget rule {rule!r}")
    return max(0, min(extra, kb - nforced))


class DeviceStatus:
    """Per-device int32 word the kernels OR their SS_DEV_* bits into."""

    _words: dict[str, torch.Tensor] = {}

    @classmethod
    def word(cls, device) -> torch.Tensor:
        key = str(device)
        if key not in cls._words:
            cls._words[key] = torch.zeros(1, dtype=torch.int32, device=device)
        return cls._words[key]

    @classmethod
    def check(cls, device, reset: bool = True) -> None:
        w = cls.word(device)
        bits = int(w.item())
        if reset:
            w.zero_()
        if bits & DEV_NONFINITE:
            raise FloatingPointError("router produced a non-finite block score")
        if bits & DEV_TIMEOUT:
            raise RuntimeError("attention kernel pipeline wait timed out")
        if bits & DEV_BADID:
            raise IndexError("block id out of range in the attention LUT")


# ----------------------------------------------------------------------------------------------
# router
# ----------------------------------------------------------------------------------------------

def router_workspace_bytes(H: int, Lq: int, Lk: int, R: int = 64, block: int = 64, fast: bool = False) -> int:
    n = ctypes.c_size_t()
    fn = lib().ss_router_fast_workspace_bytes if fast else lib().ss_router_workspace_bytes
    check(fn(H, Lq, Lk, R, block, ctypes.byref(n)), "ss_router_workspace_bytes")
    return n.value


def route(q, k, wq, wk, *, block: int = 64, extra: int, sink_tokens: int = 0, return_mask: bool = False,
          return_scores: bool = False, workspace: Workspace | None = None, out: torch.Tensor | None = None,
          validate: bool = False, keys: RouterKeys | None = None, n_cached: int = 0, k_row0: int = 0,
          fast: bool = False, rescored: torch.Tensor | None = None, ring: Ring | None = None,
          Lk: int | None = None):
    """Block ids per (head, query block): forced blocks plus the ``extra`` best-scoring others.

    q [Lq,H,128] bf16 (current chunk), k [Lk,H,128] bf16 (visible window, current chunk last),
    wq/wk [H,128,R] fp32. Returns ids int32 [H, qb, forced+extra] ascending, and optionally the
    selection mask (bool [H,qb,kb]) and block scores (fp32 [H,qb,kb]).

    ``keys``: a ``RouterKeys`` table whose first ``n_cached`` rows hold this window's key-block
    projections (``ss_router_cached``): only the query blocks and key blocks [n_cached, kb) are
    pooled, their projections written into the table. The ids are those of the uncached call.
    ``k_row0`` (with ``keys``): k holds only the window rows [k_row0, Lk), k_row0 <= n_cached*block
    (a KV-sharded rank: the tail of the window, the history before it represented by ``keys``).

    ``fast`` (R = 32 or 64): the block scores on the tensor cores (``ss_router_fast``), with the
    query blocks whose selection the error bound cannot settle scored again in exact fp32; the ids
    and mask are bit-identical to the exact mode, ``return_scores`` gives the tensor-core scores.
    ``rescored`` (int32 [1] on the device, fast mode): incremented once per query block scored
    again. ``ring`` (with ``Lk``, the window's rows): k is a ring cache [S + C + 64, H, 128]
    (``ss_router_ring``); the result is that of the call on the window's rows in order.
    """
    q = _tokens(q, "q")
    k = _tokens(k, "k")
    Lq, H, _ = q.shape
    _require((ring is None) == (Lk is None), "Lk goes with ring")
    if ring is None:
        Lk = k.shape[0] + k_row0
    else:
        _require(k_row0 == 0 and k.shape[0] == ring.phys_rows(), "a ring cache k holds S + C + 64 rows, k_row0 = 0")
    _require(k_row0 == 0 or (keys is not None and 0 <= k_row0 <= n_cached * block), "k_row0 needs keys covering it")
    _require(k.shape[1] == H and k.device == q.device, "q/k head count or device mismatch")
    _require(wq.shape == wk.shape and wq.dim() == 3 and wq.shape[0] == H and wq.shape[1] == HEAD_DIM,
             "wq/wk must be [H,128,R]")
    wq = wq.to(device=q.device, dtype=torch.float32).contiguous()
    wk = wk.to(device=q.device, dtype=torch.float32).contiguous()
    R = wq.shape[2]
    qb, kb = nblocks(Lq, block), nblocks(Lk, block)
    n_ids = forced_count(Lq, Lk, block, sink_tokens) + extra
    ws = _ws(workspace, q.device)
    nbytes = router_workspace_bytes(H, Lq, Lk, R, block, fast=fast)
    scratch = ws.tensor("router_fast" if fast else "router", (nbytes,), q.device, torch.uint8)
    ids = out if out is not None else torch.empty((H, qb, n_ids), dtype=torch.int32, device=q.device)
    _require(ids.shape == (H, qb, n_ids) and ids.dtype == torch.int32 and ids.is_contiguous(), "bad ids buffer")
    mask = torch.empty((H, qb, kb), dtype=torch.uint8, device=q.device) if return_mask else None
    scores = torch.empty((H, qb, kb), dtype=torch.float32, device=q.device) if return_scores else None
    status = DeviceStatus.word(q.device)
    if keys is not None:
        _require(keys.block == block and keys.R == R and keys.kh.shape[0] == H and keys.kh.device == q.device,
                 "RouterKeys geometry differs from this call")
        _require(0 <= n_cached <= kb and keys.kh.shape[1] >= kb, "n_cached or RouterKeys rows out of range")
    if ring is not None:
        _require(not fast or R in (32, 64), "the fast router needs R = 32 or 64")
        rc = lib().ss_router_ring(_p(q), _p(k), _p(wq), _p(wk), H, Lq, Lk, R, block, sink_tokens, extra,
                                  _p(keys.kh) if keys is not None else None,
                                  keys.kh.shape[1] if keys is not None else 0, int(n_cached), _p(ids), n_ids,
                                  _p(mask), _p(scores), _p(rescored), int(bool(fast)), ring.sink, ring.cap, ring.head,
                                  ring.dev_ptr(), _p(scratch), nbytes, _p(status), _stream(q.device))
        check(rc, "ss_router_ring")
    elif fast:
        _require(R in (32, 64), "the fast router needs R = 32 or 64")
        _require(rescored is None or (rescored.dtype == torch.int32 and rescored.device == q.device),
                 "rescored must be an int32 device tensor")
        rc = lib().ss_router_fast(_p(q), _p(k), int(k_row0), _p(wq), _p(wk), H, Lq, Lk, R, block, sink_tokens, extra,
                                  _p(keys.kh) if keys is not None else None,
                                  keys.kh.shape[1] if keys is not None else 0, int(n_cached), _p(ids), n_ids,
                                  _p(mask), _p(scores), _p(rescored), _p(scratch), nbytes, _p(status),
                                  _stream(q.device))
        check(rc, "ss_router_fast")
    elif keys is None:
        rc = lib().ss_router(_p(q), _p(k), _p(wq), _p(wk), H, Lq, Lk, R, block, sink_tokens, extra, _p(ids), n_ids,
                             _p(mask), _p(scores), _p(scratch), nbytes, _p(status), _stream(q.device))
        check(rc, "ss_router")
    else:
        rc = lib().ss_router_cached(_p(q), _p(k), int(k_row0), _p(wq), _p(wk), H, Lq, Lk, R, block, sink_tokens, extra,
                                    _p(keys.kh), keys.kh.shape[1], int(n_cached), _p(ids), n_ids, _p(mask),
                                    _p(scores), _p(scratch), nbytes, _p(status), _stream(q.device))
        check(rc, "ss_router_cached")
    if validate:
        DeviceStatus.check(q.device)
    res = [ids]
    if return_mask:
        res.append(mask.bool())
    if return_scores:
        res.append(scores)
    return res[0] if len(res) == 1 else tuple(res)


class RouterKeys:
    """One layer's table of key-block projections ``kh [H, rows, R]`` fp32, kept across calls.

    The history's key blocks change only when the window is committed, so their projections are
    pooled once (``pool_keys``, the commit-time ``refresh_history`` of migration/unified_router/
    opt23/pipeline.py:22-29) and reused by every routed call of the chunk, which pools only the
    query blocks and the key blocks from the first one that reaches the current chunk
    (``route(..., keys=...)``, ``Cache.current`` at :30-34). ``tag`` names the window rows the
    first ``n_valid`` rows were pooled from (for a ``KVCache``: its row epoch and window start);
    a different tag means nothing is reusable.
    """

    def __init__(self, H: int, max_tokens: int, *, block: int = 64, R: int = 64, device="cuda"):
        rows = (nblocks(max_tokens, block) + 3) // 4 * 4
        self.block, self.R = block, R
        self.kh = torch.empty((H, rows, R), dtype=torch.float32, device=device)
        self.n_valid = 0
        self.tag = None

    def cached(self, tag) -> int:
        """Leading key blocks whose projections are valid for the window named by ``tag``."""
        return self.n_valid if tag is not None and tag == self.tag else 0

    def mark(self, tag, n_valid: int) -> None:
        self.tag, self.n_valid = tag, int(n_valid)

    def invalidate(self) -> None:
        self.tag, self.n_valid = None, 0


def history_blocks(Lq: int, Lk: int, block: int) -> int:
    """Key blocks that lie wholly in the history [0, Lk - Lq): their projections do not change
    while the chunk is denoised."""
    return (Lk - Lq) // block


def pool_keys(k, wk, keys: RouterKeys, *, j0: int = 0, j1: int | None = None, ring: Ring | None = None,
              Lk: int | None = None) -> None:
    """Pool and project key blocks [j0, j1) of the window k [Lk,H,128] into ``keys.kh``
    (``ss_router_pool_keys``). With ``ring``: k is a ring cache [S + C + 64, H, 128] holding a
    window of ``Lk`` rows (``ss_router_pool_keys_ring``)."""
    k = _tokens(k, "k")
    H = k.shape[1]
    _require((ring is None) == (Lk is None), "Lk goes with ring")
    if ring is None:
        Lk = k.shape[0]
    else:
        _require(k.shape[0] == ring.phys_rows(), "k rows do not match the ring")
    wk = wk.to(device=k.device, dtype=torch.float32).contiguous()
    _require(wk.shape == (H, HEAD_DIM, keys.R), f"wk must be [H,128,{keys.R}]")
    kb = nblocks(Lk, keys.block)
    j1 = kb if j1 is None else j1
    _require(0 <= j0 <= j1 <= kb and keys.kh.shape[0] == H and keys.kh.shape[1] >= kb, "key range or table size")
    st = _p(DeviceStatus.word(k.device))
    if ring is None:
        rc = lib().ss_router_pool_keys(_p(k), _p(wk), H, Lk, keys.R, keys.block, j0, j1, _p(keys.kh), keys.kh.shape[1],
                                       st, _stream(k.device))
    else:
        rc = lib().ss_router_pool_keys_ring(_p(k), _p(wk), H, Lk, keys.R, keys.block, j0, j1, _p(keys.kh),
                                            keys.kh.shape[1], ring.sink, ring.cap, ring.head, ring.dev_ptr(), st,
                                            _stream(k.device))
    check(rc, "ss_router_pool_keys")


# ----------------------------------------------------------------------------------------------
# attention
# ----------------------------------------------------------------------------------------------

def attention_max_ids(Lk: int, block: int = 64) -> int:
    n = ctypes.c_int()
    check(lib().ss_attention_max_ids(Lk, block, ctypes.byref(n)), "ss_attention_max_ids")
    return n.value


_ATTN_WS: dict[tuple, int] = {}


def attention_workspace_bytes(H: int, Lq: int) -> int:
    """Workspace ``ss_attention_ws`` uses to split a small problem's tiles across the SMs (0: none)."""
    key = (H, Lq, torch.cuda.current_device())
    if key not in _ATTN_WS:
        n = ctypes.c_size_t()
        check(lib().ss_attention_workspace_bytes(H, Lq, ctypes.byref(n)), "ss_attention_workspace_bytes")
        _ATTN_WS[key] = n.value
    return _ATTN_WS[key]


def sparse_attention(q, k, v, ids, *, block: int = 64, scale: float | None = None,
                     out_dtype: torch.dtype = torch.bfloat16, return_lse: bool = False,
                     out: torch.Tensor | None = None, lse: torch.Tensor | None = None, validate: bool = False,
                     workspace: Workspace | None = None, split: bool = True, ring: Ring | None = None,
                     Lk: int | None = None):
    """softmax(scale q K_S^T) V_S over the valid tokens of the blocks in ids[h, t // block].

    q [Lq,H,128], k/v [Lk,H,128] bf16; ids int32 [H, ceil(Lq/block), n] (entries < 0 ignored).
    Returns out [Lq,H,128] in ``out_dtype`` (bf16 or fp32), plus the natural-log LSE [H,Lq] fp32
    when ``return_lse``. With ``split`` (default) a problem of fewer 128-row tiles than twice the
    SMs splits its tiles across the SMs (``ss_attention_ws``, workspace from ``workspace``).
    ``ring`` (with ``Lk``, the window's rows): k/v are a ring cache [S + C + 64, H, 128]
    (``ss_attention_ring``).
    """
    q = _tokens(q, "q")
    k = _tokens(k, "k")
    v = _tokens(v, "v")
    Lq, H, D = q.shape
    _require((ring is None) == (Lk is None), "Lk goes with ring")
    if ring is None:
        Lk = k.shape[0]
    else:
        _require(k.shape[0] == ring.phys_rows(), "k/v rows do not match the ring")
    _require(v.shape == k.shape and k.shape[1] == H, "k/v shape mismatch")
    _require(ids.is_cuda and ids.dtype == torch.int32 and ids.dim() == 3, "ids must be int32 CUDA [H,qb,n]")
    _require(ids.shape[0] == H and ids.shape[1] == nblocks(Lq, block), f"ids must be [H,{nblocks(Lq, block)},n]")
    ids = ids.contiguous()
    _require(out_dtype in (torch.bfloat16, torch.float32), "out_dtype must be bf16 or fp32")
    scale = 1.0 / math.sqrt(D) if scale is None else float(scale)
    if out is None:
        out = torch.empty((Lq, H, D), dtype=out_dtype, device=q.device)
    _require(out.shape[-3:] == (Lq, H, D) and out.dtype == out_dtype and out.is_contiguous(), "bad out buffer")
    if return_lse and lse is None:
        lse = torch.empty((H, Lq), dtype=torch.float32, device=q.device)
    status = DeviceStatus.word(q.device)
    nws = attention_workspace_bytes(H, Lq) if split else 0
    if ring is not None:
        ws = _ws(workspace, q.device).tensor("attention_split", (max(nws, 256),), q.device, torch.uint8)
        rc = lib().ss_attention_ring(_p(q), _p(k), _p(v), _p(ids), H, Lq, Lk, block, ids.shape[2], scale, _p(out),
                                     1 if out_dtype == torch.float32 else 0, _p(lse) if return_lse else None,
                                     _p(status), ring.sink, ring.cap, ring.head, ring.dev_ptr(),
                                     _p(ws) if nws else None, nws, _stream(q.device))
        check(rc, "ss_attention_ring")
    elif nws:
        ws = _ws(workspace, q.device).tensor("attention_split", (nws,), q.device, torch.uint8)
        rc = lib().ss_attention_ws(_p(q), _p(k), _p(v), _p(ids), H, Lq, Lk, block, ids.shape[2], scale, _p(out),
                                   1 if out_dtype == torch.float32 else 0, _p(lse) if return_lse else None,
                                   _p(status), _p(ws), nws, _stream(q.device))
        check(rc, "ss_attention_ws")
    else:
        rc = lib().ss_attention(_p(q), _p(k), _p(v), _p(ids), H, Lq, Lk, block, ids.shape[2], scale, _p(out),
                                1 if out_dtype == torch.float32 else 0, _p(lse) if return_lse else None, _p(status),
                                _stream(q.device))
        check(rc, "ss_attention")
    if validate:
        DeviceStatus.check(q.device)
    return (out, lse) if return_lse else out


def sparse_attention_heads(q, k, v, ids, outs, *, out_heads: int, h0: int, block: int = 64,
                           scale: float | None = None, out_dtype: torch.dtype = torch.bfloat16,
                           workspace: Workspace | None = None, validate: bool = False, ring: Ring | None = None,
                           Lk: int | None = None) -> None:
    """``sparse_attention`` over one rank's heads (global heads h0 .. h0 + H - 1 of ``out_heads``)
    whose output rows go into every buffer of ``outs``: device addresses (ints) of the ranks'
    [Lq, out_heads, 128] ``out_dtype`` buffers, this rank's own and the peers' mapped ones
    (``ss_attention_heads``). The kernel's epilogue stores each row to all of them, so a peer
    barrier after the call completes the all-gather of the heads. ``ring`` (with ``Lk``): k/v are
    a ring cache of this rank's heads, as in ``sparse_attention``."""
    q = _tokens(q, "q")
    k = _tokens(k, "k")
    v = _tokens(v, "v")
    Lq, H, D = q.shape
    _require((ring is None) == (Lk is None), "Lk goes with ring")
    if ring is None:
        Lk = k.shape[0]
    else:
        _require(k.shape[0] == ring.phys_rows(), "k/v rows do not match the ring")
    _require(v.shape == k.shape and k.shape[1] == H, "k/v shape mismatch")
    _require(ids.is_cuda and ids.dtype == torch.int32 and ids.dim() == 3, "ids must be int32 CUDA [H,qb,n]")
    _require(ids.shape[0] == H and ids.shape[1] == nblocks(Lq, block), f"ids must be [H,{nblocks(Lq, block)},n]")
    ids = ids.contiguous()
    _require(out_dtype in (torch.bfloat16, torch.float32), "out_dtype must be bf16 or fp32")
    _require(1 <= len(outs) <= 8 and 0 <= h0 and h0 + H <= out_heads, "bad output buffers")
    scale = 1.0 / math.sqrt(D) if scale is None else float(scale)
    arr = (ctypes.c_void_p * len(outs))(*outs)
    nws = attention_workspace_bytes(H, Lq)
    ws = _ws(workspace, q.device).tensor("attention_split", (max(nws, 256),), q.device, torch.uint8)
    status = DeviceStatus.word(q.device)
    rs = (ring.sink, ring.cap, ring.head, ring.dev_ptr()) if ring is not None else (0, 0, 0, None)
    rc = lib().ss_attention_heads(_p(q), _p(k), _p(v), _p(ids), H, Lq, Lk, block, ids.shape[2], scale, arr,
                                  len(outs), out_heads, h0, 1 if out_dtype == torch.float32 else 0, None, _p(status),
                                  *rs, _p(ws) if nws else None, nws, _stream(q.device))
    check(rc, "ss_attention_heads")
    if validate:
        DeviceStatus.check(q.device)


PAGE_TOKENS = 64


def quant_pages(Lk: int) -> int:
    """Key pages (64 tokens, the last one possibly partial) of a window of Lk tokens."""
    return (Lk + PAGE_TOKENS - 1) // PAGE_TOKENS


def quant_k_pages(k, *, p0: int = 0, p1: int | None = None, k_i8: torch.Tensor | None = None,
                  ks: torch.Tensor | None = None, ring: "Ring | None" = None, Lk: int | None = None):
    """Quantise key pages [p0, p1) of k [Lk,H,128] bf16 to int8 (``ss_quant_k_pages``).

    Returns (k_i8 [Lk,H,128] int8, ks [H,ceil(Lk/64)] fp32); pass the previous buffers to update
    only some pages (history pages once per commit, the current chunk's pages per call, as
    ``Quantized.history`` / ``.current`` of migration/unified_router/opt23/attention.py:16-28).
    ``ring`` (with ``Lk``, the window's rows): k is a ring cache's physical rows and k_i8 gets the
    same rows (``ss_quant_k_pages_ring``).
    """
    k = _tokens(k, "k")
    _require((ring is None) == (Lk is None), "Lk goes with ring")
    H = k.shape[1]
    if ring is None:
        Lk = k.shape[0]
    else:
        _require(k.shape[0] == ring.phys_rows(), "k rows do not match the ring")
    npg = quant_pages(Lk)
    p1 = npg if p1 is None else p1
    if k_i8 is None:
        k_i8 = torch.empty((Lk, H, HEAD_DIM), dtype=torch.int8, device=k.device)
    if ks is None:
        ks = torch.empty((H, npg), dtype=torch.float32, device=k.device)
    _require(k_i8.shape == k.shape and k_i8.dtype == torch.int8 and k_i8.is_contiguous(), "bad k_i8 buffer")
    _require(ks.shape == (H, npg) and ks.dtype == torch.float32 and ks.is_contiguous(), "bad ks buffer")
    if ring is None:
        rc = lib().ss_quant_k_pages(_p(k), H, Lk, p0, p1, _p(k_i8), _p(ks), _stream(k.device))
    else:
        rc = lib().ss_quant_k_pages_ring(_p(k), H, Lk, p0, p1, _p(k_i8), _p(ks), ring.sink, ring.cap, ring.head,
                                         ring.dev_ptr(), _stream(k.device))
    check(rc, "ss_quant_k_pages")
    return k_i8, ks


def attention_i8_workspace_bytes(H: int, Lq: int) -> int:
    """Workspace bytes ss_attention_i8 uses to split tiles on the current device (0: never splits)."""
    n = ctypes.c_size_t(0)
    check(lib().ss_attention_i8_workspace_bytes(H, Lq, ctypes.byref(n)), "ss_attention_i8_workspace_bytes")
    return int(n.value)


def sparse_attention_i8(q, k_i8, ks, v, ids, *, block: int = 64, scale: float | None = None,
                        out_dtype: torch.dtype = torch.bfloat16, return_lse: bool = False,
                        out: torch.Tensor | None = None, lse: torch.Tensor | None = None, validate: bool = False,
                        workspace: Workspace | None = None, split: bool = True, ring: "Ring | None" = None,
                        Lk: int | None = None):
    """INT8-QK block-sparse attention (``ss_attention_i8``): ``sparse_attention`` with the scores
    taken from int8 Q (32-row groups, quantised in the kernel) and int8 K pages (``quant_k_pages``),
    as the reference's INT8 path (migration/unified_router/opt23/attention.py:30-58). With ``split``
    (default) a problem that would leave a partial wave cuts its tiles into equal pieces merged by
    LSE (workspace from ``workspace``). ``ring`` (with ``Lk``): k_i8 and v are a ring cache's
    physical rows (``ss_attention_i8_ring``)."""
    q = _tokens(q, "q")
    v = _tokens(v, "v")
    Lq, H, D = q.shape
    _require((ring is None) == (Lk is None), "Lk goes with ring")
    if ring is None:
        Lk = v.shape[0]
    else:
        _require(v.shape[0] == ring.phys_rows(), "v rows do not match the ring")
    _require(k_i8.is_cuda and k_i8.dtype == torch.int8 and k_i8.shape == v.shape and k_i8.is_contiguous(),
             "k_i8 must be int8 CUDA [Lk,H,128] like v")
    _require(ks.is_cuda and ks.dtype == torch.float32 and ks.shape == (H, quant_pages(Lk)) and ks.is_contiguous(),
             f"ks must be fp32 CUDA [H,{quant_pages(Lk)}]")
    _require(ids.is_cuda and ids.dtype == torch.int32 and ids.dim() == 3, "ids must be int32 CUDA [H,qb,n]")
    _require(ids.shape[0] == H and ids.shape[1] == nblocks(Lq, block), f"ids must be [H,{nblocks(Lq, block)},n]")
    ids = ids.contiguous()
    _require(out_dtype in (torch.bfloat16, torch.float32), "out_dtype must be bf16 or fp32")
    scale = 1.0 / math.sqrt(D) if scale is None else float(scale)
    if out is None:
        out = torch.empty((Lq, H, D), dtype=out_dtype, device=q.device)
    _require(out.shape == (Lq, H, D) and out.dtype == out_dtype and out.is_contiguous(), "bad out buffer")
    if return_lse and lse is None:
        lse = torch.empty((H, Lq), dtype=torch.float32, device=q.device)
    status = DeviceStatus.word(q.device)
    nws = attention_i8_workspace_bytes(H, Lq) if split else 0
    ws = _ws(workspace, q.device).tensor("attention_i8_split", (nws,), q.device, torch.uint8) if nws else None
    if ring is None:
        rc = lib().ss_attention_i8(_p(q), _p(k_i8), _p(ks), _p(v), _p(ids), H, Lq, Lk, block, ids.shape[2], scale,
                                   _p(out), 1 if out_dtype == torch.float32 else 0, _p(lse) if return_lse else None,
                                   _p(status), _p(ws), nws, _stream(q.device))
    else:
        rc = lib().ss_attention_i8_ring(_p(q), _p(k_i8), _p(ks), _p(v), _p(ids), H, Lq, Lk, block, ids.shape[2],
                                        scale, _p(out), 1 if out_dtype == torch.float32 else 0,
                                        _p(lse) if return_lse else None, _p(status), ring.sink, ring.cap, ring.head,
                                        ring.dev_ptr(), _p(ws), nws, _stream(q.device))
    check(rc, "ss_attention_i8")
    if validate:
        DeviceStatus.check(q.device)
    return (out, lse) if return_lse else out


def exact(q, k, v, ids, workspace: Workspace | None = None):
    """Reference mirror: q/k/v [1,N,H,D] bf16, ids [H, N//64, count] -> (O fp32 [1,N,H,D], lse [H,N])."""
    ws = _ws(workspace, q.device)
    _, n, h, d = q.shape
    out = ws.tensor("exact", (1, n, h, d), q.device, torch.float32)
    lse = ws.tensor("exact_lse", (h, n), q.device, torch.float32)
    ids = ids.to(torch.int32)
    sparse_attention(q, k, v, ids, block=64, out_dtype=torch.float32, return_lse=True, out=out[0], lse=lse)
    return out, lse


# ----------------------------------------------------------------------------------------------
# merge
# ----------------------------------------------------------------------------------------------

def lse_merge(o_parts: torch.Tensor, lse_parts: torch.Tensor, *, out_dtype: torch.dtype = torch.bfloat16,
              return_lse: bool = False):
    """o_parts fp32 [P,Lq,H,128], lse_parts fp32 [P,H,Lq] natural log -> merged [Lq,H,128] (+ LSE)."""
    _require(o_parts.is_cuda and o_parts.dtype == torch.float32 and o_parts.dim() == 4, "o_parts: fp32 CUDA [P,Lq,H,D]")
    P, Lq, H, D = o_parts.shape
    _require(D == HEAD_DIM and lse_parts.shape == (P, H, Lq) and lse_parts.dtype == torch.float32, "lse_parts: [P,H,Lq]")
    o_parts = o_parts.contiguous()
    lse_parts = lse_parts.contiguous()
    out = torch.empty((Lq, H, D), dtype=out_dtype, device=o_parts.device)
    lse = torch.empty((H, Lq), dtype=torch.float32, device=o_parts.device) if return_lse else None
    rc = lib().ss_lse_merge(_p(o_parts), _p(lse_parts), P, H, Lq, _p(out), 1 if out_dtype == torch.float32 else 0,
                            _p(lse), _stream(o_parts.device))
    check(rc, "ss_lse_merge")
    return (out, lse) if return_lse else out


def merge(exact_output, exact_lse, approx, approx_lse):
    """Reference mirror: exact [1,N,H,D] + LSE [H,N] with approx [H,N,D] + LSE [H,N] -> bf16 [1,N,H,D]."""
    parts = torch.stack((exact_output[0].float(), approx.float().transpose(0, 1)))
    lses = torch.stack((exact_lse.float(), approx_lse.float()))
    return lse_merge(parts, lses, out_dtype=torch.bfloat16)[None]


# ----------------------------------------------------------------------------------------------
# cache
# ----------------------------------------------------------------------------------------------

def cache_append(k_cache, v_cache, k_new, v_new, *, local_attn: bool, global_end: int, local_end: int,
                 current_start: int, sink_tokens: int) -> int:
    """Roll (evict) + write one chunk into [cap,H,128] (or [1,cap,H,128]) bf16 caches in place.

    Returns the new local end index; the visible window is cache[max(0, end - W) : end].
    """
    kc = k_cache[0] if k_cache.dim() == 4 else k_cache
    vc = v_cache[0] if v_cache.dim() == 4 else v_cache
    kn = k_new[0] if k_new.dim() == 4 else k_new
    vn = v_new[0] if v_new.dim() == 4 else v_new
    for name, t in (("k_cache", kc), ("v_cache", vc), ("k_new", kn), ("v_new", vn)):
        _require(t.is_cuda and t.dtype == torch.bfloat16 and t.shape[-1] == HEAD_DIM, f"{name}: bf16 CUDA [...,128]")
    _require(kc.is_contiguous() and vc.is_contiguous() and kc.shape == vc.shape, "caches must be contiguous and equal")
    cap, H, _ = kc.shape
    _require(kn.shape == vn.shape and kn.shape[1] == H and kn.stride() == vn.stride(), "k_new/v_new mismatch")
    _require(kn.stride(2) == 1 and kn.stride(1) == HEAD_DIM, "k_new rows must be [H,128] contiguous")
    new_end = ctypes.c_int64()
    rc = lib().ss_cache_append(_p(kc), _p(vc), cap, H, _p(kn), _p(vn), kn.stride(0), kn.shape[0], int(bool(local_attn)),
                               int(global_end), int(local_end), int(current_start), int(sink_tokens),
                               ctypes.byref(new_end), _stream(kc.device))
    check(rc, "ss_cache_append")
    return new_end.value


class Ring(tuple):
    """Geometry of a ring-buffer KV cache: (sink rows S, ring rows C, head). Window row t >= S lives
    at physical row S + ((t - S + head) mod C); see ``ss_router_ring`` in include/ssparse.h.
    ``head_dev`` (optional int32 [1] device tensor) holds the same head in device memory: the
    kernels then read it at run time, so calls captured in a CUDA graph follow later rolls."""

    def __new__(cls, sink: int, cap: int, head: int, head_dev: torch.Tensor | None = None):
        r = super().__new__(cls, (int(sink), int(cap), int(head)))
        r.head_dev = head_dev
        return r

    def with_head(self, head: int) -> "Ring":
        return Ring(self[0], self[1], head, self.head_dev)

    def dev_ptr(self):
        return None if self.head_dev is None else self.head_dev.data_ptr()

    @property
    def sink(self) -> int:
        return self[0]

    @property
    def cap(self) -> int:
        return self[1]

    @property
    def head(self) -> int:
        return self[2]

    def phys_rows(self) -> int:
        return self[0] + self[1] + 64


def cache_append_ring(k_cache, v_cache, k_new, v_new, *, cap: int, local_attn: bool, global_end: int,
                      local_end: int, current_start: int, sink_tokens: int, ring: Ring) -> tuple[int, int]:
    """``cache_append`` on a ring cache [S + C + 64, H, 128] (``ss_cache_append_ring``): the same
    window, but a roll only moves the ring's head. Returns (new local end, new head)."""
    kc = k_cache[0] if k_cache.dim() == 4 else k_cache
    vc = v_cache[0] if v_cache.dim() == 4 else v_cache
    kn = k_new[0] if k_new.dim() == 4 else k_new
    vn = v_new[0] if v_new.dim() == 4 else v_new
    for name, t in (("k_cache", kc), ("v_cache", vc), ("k_new", kn), ("v_new", vn)):
        _require(t.is_cuda and t.dtype == torch.bfloat16 and t.shape[-1] == HEAD_DIM, f"{name}: bf16 CUDA [...,128]")
    _require(kc.is_contiguous() and vc.is_contiguous() and kc.shape == vc.shape, "caches must be contiguous and equal")
    _require(ring.sink == sink_tokens and kc.shape[0] == ring.phys_rows(), "cache rows do not match the ring")
    H = kc.shape[1]
    _require(kn.shape == vn.shape and kn.shape[1] == H and kn.stride() == vn.stride(), "k_new/v_new mismatch")
    _require(kn.stride(2) == 1 and kn.stride(1) == HEAD_DIM, "k_new rows must be [H,128] contiguous")
    new_end, new_head = ctypes.c_int64(), ctypes.c_int()
    rc = lib().ss_cache_append_ring(_p(kc), _p(vc), int(cap), H, _p(kn), _p(vn), kn.stride(0), kn.shape[0],
                                    int(bool(local_attn)), int(global_end), int(local_end), int(current_start),
                                    int(sink_tokens), ring.cap, ring.head, ring.dev_ptr(), ctypes.byref(new_end),
                                    ctypes.byref(new_head), _stream(kc.device))
    check(rc, "ss_cache_append_ring")
    return new_end.value, new_head.value


def ring_refresh(k_cache, v_cache, ring: Ring) -> None:
    """Rewrite a ring cache's copy of the sink's last S mod 64 rows (``ss_cache_ring_refresh``)."""
    kc = k_cache[0] if k_cache.dim() == 4 else k_cache
    vc = v_cache[0] if v_cache.dim() == 4 else v_cache
    rc = lib().ss_cache_ring_refresh(_p(kc), _p(vc), kc.shape[1], ring.sink, ring.cap, ring.head, ring.dev_ptr(),
                                     _stream(kc.device))
    check(rc, "ss_cache_ring_refresh")


def rope_shift(src: torch.Tensor, dst: torch.Tensor, phase: torch.Tensor) -> torch.Tensor:
    """dst = src with the first P complex pairs of every head rotated by phase [P, 2] float64
    (cos, sin) on the device (`ss_cache_rope_shift`). src/dst [n, H, 128] bf16 (rows may be
    strided; dst may be src). The anchor rebase of local_experiments/anchor_rebase.py:8-18."""
    for name, t in (("src", src), ("dst", dst)):
        _require(t.is_cuda and t.dtype == torch.bfloat16 and t.dim() == 3 and t.shape[-1] == HEAD_DIM and
                 t.stride(2) == 1 and t.stride(1) == HEAD_DIM, f"{name}: bf16 CUDA [n, H, 128] rows")
    _require(src.shape == dst.shape, "src and dst must have the same shape")
    _require(phase.is_cuda and phase.dtype == torch.float64 and phase.is_contiguous() and phase.dim() == 2 and
             phase.shape[1] == 2, "phase: float64 CUDA [P, 2]")
    n, H, _ = src.shape
    rc = lib().ss_cache_rope_shift(_p(src), src.stride(0), _p(dst), dst.stride(0), n, H, phase.shape[0], _p(phase),
                                   _stream(src.device))
    check(rc, "ss_cache_rope_shift")
    return dst


# ----------------------------------------------------------------------------------------------
# per-token kernels of the DiT layer around the attention (csrc/dit.cu), used by the rollout
# ----------------------------------------------------------------------------------------------
def _rows(t: torch.Tensor, name: str, width: int) -> int:
    """Row stride of a CUDA tensor whose last dim holds `width` contiguous values per row."""
    _require(t.is_cuda, f"{name}: must be a CUDA tensor")
    _require(t.stride(-1) == 1 and t.shape[-1] >= width, f"{name}: rows of {width} contiguous values expected")
    return t.stride(-2) if t.dim() >= 2 else width


def qkv_norm_rope(qkv: torch.Tensor, norm_q: torch.Tensor, norm_k: torch.Tensor, eps: float, cos: torch.Tensor,
                  sin: torch.Tensor, q_out: torch.Tensor, k_out: torch.Tensor, v_out: torch.Tensor, *,
                  model_heads: int | None = None, h0: int = 0) -> torch.Tensor:
    """q/k RMSNorm + weight + 3-D RoPE, v copied, from one fused projection (`ss_qkv_norm_rope`).

    qkv [n, >=3d] bf16 (q | k | v columns, d = H*128); norm_q/norm_k [d] bf16; cos/sin [n, 64]
    fp32; q_out [n, H, 128] bf16; k_out/v_out [n, H, 128] bf16 with equal row strides (for
    example the cache rows of the chunk). Returns q_out. ``model_heads`` (head sharding): qkv holds
    all ``model_heads`` heads (the norm runs over the whole width) and only heads h0 .. h0 + h - 1
    are written, h = q_out.shape[1] (``ss_qkv_norm_rope_heads``).
    """
    n, H = q_out.shape[0], q_out.shape[1]
    if model_heads is not None:
        return _qkv_heads(qkv, norm_q, norm_k, eps, cos, sin, q_out, k_out, v_out, model_heads, h0)
    d = H * HEAD_DIM
    _require(qkv.dtype == torch.bfloat16 and qkv.dim() == 2 and qkv.shape[0] == n, "qkv: bf16 [n, 3d]")
    ld = _rows(qkv, "qkv", 3 * d)
    for name, t in (("q_out", q_out), ("k_out", k_out), ("v_out", v_out)):
        _require(t.dtype == torch.bfloat16 and t.shape == (n, H, HEAD_DIM) and t.stride(2) == 1 and
                 t.stride(1) == HEAD_DIM, f"{name}: bf16 [n, H, 128] rows")
    _require(k_out.stride(0) == v_out.stride(0), "k_out and v_out must share a row stride")
    for name, t in (("norm_q", norm_q), ("norm_k", norm_k)):
        _require(t.dtype == torch.bfloat16 and t.is_contiguous() and t.numel() == d, f"{name}: bf16 [{d}]")
    for name, t in (("cos", cos), ("sin", sin)):
        _require(t.dtype == torch.float32 and t.is_contiguous() and t.shape == (n, HEAD_DIM // 2),
                 f"{name}: fp32 [n, 64]")
    rc = lib().ss_qkv_norm_rope(_p(qkv), ld, n, H, _p(norm_q), _p(norm_k), float(eps), _p(cos), _p(sin), _p(q_out),
                                q_out.stride(0), _p(k_out), _p(v_out), k_out.stride(0), _stream(qkv.device))
    check(rc, "ss_qkv_norm_rope")
    return q_out


def _qkv_heads(qkv, norm_q, norm_k, eps, cos, sin, q_out, k_out, v_out, model_heads: int, h0: int,
               ring: Ring | None = None, t0: int = 0, evicted: int = 0) -> torch.Tensor:
    """``ss_qkv_norm_rope_heads``: the norm over all ``model_heads`` heads of qkv, heads
    h0 .. h0 + h - 1 written to q_out [n, h, 128] and k_out / v_out (rows of h heads, plain or a
    ring cache)."""
    n, h = q_out.shape[0], q_out.shape[1]
    d = model_heads * HEAD_DIM
    _require(qkv.dtype == torch.bfloat16 and qkv.dim() == 2 and qkv.shape[0] == n, "qkv: bf16 [n, 3d]")
    _require(0 <= h0 and h0 + h <= model_heads, "head range outside the model's heads")
    ld = _rows(qkv, "qkv", 3 * d)
    _require(q_out.dtype == torch.bfloat16 and q_out.stride(2) == 1 and q_out.stride(1) == HEAD_DIM,
             "q_out: bf16 [n, h, 128] rows")
    for name, t in (("k_out", k_out), ("v_out", v_out)):
        _require(t.dtype == torch.bfloat16 and t.shape[1:] == (h, HEAD_DIM) and t.stride(2) == 1 and
                 t.stride(1) == HEAD_DIM, f"{name}: bf16 [rows, h, 128]")
    _require(k_out.stride(0) == v_out.stride(0), "k_out and v_out must share a row stride")
    for name, t in (("norm_q", norm_q), ("norm_k", norm_k)):
        _require(t.dtype == torch.bfloat16 and t.is_contiguous() and t.numel() == d, f"{name}: bf16 [{d}]")
    for name, t in (("cos", cos), ("sin", sin)):
        _require(t.dtype == torch.float32 and t.is_contiguous() and t.shape == (n, HEAD_DIM // 2),
                 f"{name}: fp32 [n, 64]")
    if ring is not None:
        _require(ring.head_dev is not None, "the ring's head must live in device memory")
        _require(k_out.is_contiguous() and v_out.is_contiguous() and k_out.shape[0] == ring.phys_rows(),
                 "caches must be contiguous ring caches of the ring's geometry")
        rs = (ring.sink, ring.cap, int(t0), ring.dev_ptr(), int(evicted))
    else:
        _require(k_out.shape[0] == n and v_out.shape[0] == n, "k_out / v_out: the chunk's n rows")
        rs = (0, 0, 0, None, 0)
    rc = lib().ss_qkv_norm_rope_heads(_p(qkv), ld, n, model_heads, _p(norm_q), _p(norm_k), float(eps), _p(cos),
                                      _p(sin), h0, h, _p(q_out), q_out.stride(0), _p(k_out), _p(v_out),
                                      k_out.stride(0), *rs, _stream(qkv.device))
    check(rc, "ss_qkv_norm_rope_heads")
    return q_out


def qkv_norm_rope_ring(qkv: torch.Tensor, norm_q: torch.Tensor, norm_k: torch.Tensor, eps: float, cos: torch.Tensor,
                       sin: torch.Tensor, q_out: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, *,
                       ring: Ring, t0: int, evicted: int, model_heads: int | None = None, h0: int = 0) -> torch.Tensor:
    """``qkv_norm_rope`` with k and v written into a ring-buffer cache [S + C + 64, H, 128] at the
    rows of window rows t0 .. t0 + n - 1, placed by the device head moved on by ``evicted``
    (``ss_qkv_norm_rope_ring``; ``ring.head_dev`` required). Follow it with ``ring_commit``.
    ``model_heads`` / ``h0``: as in ``qkv_norm_rope`` (a cache of h0 .. h0 + h - 1)."""
    n, H = q_out.shape[0], q_out.shape[1]
    d = H * HEAD_DIM
    kc = k_cache[0] if k_cache.dim() == 4 else k_cache
    vc = v_cache[0] if v_cache.dim() == 4 else v_cache
    if model_heads is not None:
        return _qkv_heads(qkv, norm_q, norm_k, eps, cos, sin, q_out, kc, vc, model_heads, h0, ring=ring, t0=t0,
                          evicted=evicted)
    _require(ring.head_dev is not None, "the ring's head must live in device memory")
    _require(qkv.dtype == torch.bfloat16 and qkv.dim() == 2 and qkv.shape[0] == n, "qkv: bf16 [n, 3d]")
    ld = _rows(qkv, "qkv", 3 * d)
    _require(q_out.dtype == torch.bfloat16 and q_out.shape == (n, H, HEAD_DIM) and q_out.stride(2) == 1 and
             q_out.stride(1) == HEAD_DIM, "q_out: bf16 [n, H, 128] rows")
    _require(kc.is_contiguous() and vc.is_contiguous() and kc.shape == vc.shape and kc.shape[0] == ring.phys_rows()
             and kc.shape[1] == H, "caches must be contiguous ring caches of the ring's geometry")
    rc = lib().ss_qkv_norm_rope_ring(_p(qkv), ld, n, H, _p(norm_q), _p(norm_k), float(eps), _p(cos), _p(sin),
                                     _p(q_out), q_out.stride(0), _p(kc), _p(vc), kc.stride(0), ring.sink, ring.cap,
                                     int(t0), ring.dev_ptr(), int(evicted), _stream(qkv.device))
    check(rc, "ss_qkv_norm_rope_ring")
    return q_out


def ring_commit(k_cache, v_cache, ring: Ring, *, evicted: int, refresh: bool) -> None:
    """After ``qkv_norm_rope_ring``: the sink's copy before the new head (when the write rolled or
    wrote sink rows), then the device head moved on by ``evicted`` (``ss_cache_ring_commit``)."""
    kc = k_cache[0] if k_cache.dim() == 4 else k_cache
    vc = v_cache[0] if v_cache.dim() == 4 else v_cache
    _require(ring.head_dev is not None, "the ring's head must live in device memory")
    rc = lib().ss_cache_ring_commit(_p(kc), _p(vc), kc.shape[1], ring.sink, ring.cap, ring.dev_ptr(), int(evicted),
                                    int(bool(refresh)), _stream(kc.device))
    check(rc, "ss_cache_ring_commit")


def adaln(x: torch.Tensor, *, eps: float, shift: torch.Tensor | None = None, scale: torch.Tensor | None = None,
          frame_tokens: int = 0, weight: torch.Tensor | None = None, bias: torch.Tensor | None = None,
          out: torch.Tensor | None = None) -> torch.Tensor:
    """LayerNorm of x [n, d] bf16 with per-frame modulation (shift/scale fp32 rows [frames, d],
    any row stride) or with an affine bf16 weight/bias (`ss_adaln`)."""
    _require(x.dtype == torch.bfloat16 and x.dim() == 2 and x.is_contiguous() and x.is_cuda,
             "x: contiguous bf16 [n, d]")
    n, d = x.shape
    out = torch.empty_like(x) if out is None else out
    _require(out.shape == x.shape and out.dtype == x.dtype and out.is_contiguous(), "bad out buffer")
    mod_ld = 0
    if shift is not None or scale is not None:
        _require(shift is not None and scale is not None, "shift and scale go together")
        _require(shift.dtype == scale.dtype == torch.float32, "shift/scale: fp32")
        mod_ld = _rows(shift, "shift", d)
        _require(_rows(scale, "scale", d) == mod_ld, "shift and scale must share a row stride")
        _require(frame_tokens > 0 and shift.shape[-2] * frame_tokens >= n, "frame_tokens must cover the rows")
    rc = lib().ss_adaln(_p(x), n, d, int(frame_tokens), _p(shift), _p(scale), mod_ld, _p(weight), _p(bias), float(eps),
                        _p(out), _stream(x.device))
    check(rc, "ss_adaln")
    return out


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float, out: torch.Tensor | None = None) -> torch.Tensor:
    """WanRMSNorm of the rows of x [n, d] bf16 (any row stride) with a bf16 weight (`ss_rms_norm`)."""
    _require(x.dtype == torch.bfloat16 and x.dim() == 2, "x: bf16 [n, d]")
    n, d = x.shape
    x_ld = _rows(x, "x", d)
    _require(weight.dtype == torch.bfloat16 and weight.is_contiguous() and weight.numel() == d, f"weight: bf16 [{d}]")
    out = torch.empty((n, d), dtype=x.dtype, device=x.device) if out is None else out
    _require(out.shape == (n, d) and out.dtype == x.dtype and out.is_contiguous(), "bad out buffer")
    rc = lib().ss_rms_norm(_p(x), x_ld, n, d, _p(weight), float(eps), _p(out), _stream(x.device))
    check(rc, "ss_rms_norm")
    return out


def gate_residual(x: torch.Tensor, y: torch.Tensor, *, gate: torch.Tensor | None = None,
                  frame_tokens: int = 0) -> torch.Tensor:
    """In place: x = x + y * gate[frame] (or x + y), bf16 [n, d] (`ss_gate_residual`)."""
    _require(x.dtype == y.dtype == torch.bfloat16 and x.dim() == 2 and x.is_contiguous(), "x: contiguous bf16 [n, d]")
    n, d = x.shape
    _require(y.shape == x.shape, "y must match x")
    y_ld = _rows(y, "y", d)
    g_ld = 0
    if gate is not None:
        _require(gate.dtype == torch.float32, "gate: fp32")
        g_ld = _rows(gate, "gate", d)
        _require(frame_tokens > 0 and gate.shape[-2] * frame_tokens >= n, "frame_tokens must cover the rows")
    rc = lib().ss_gate_residual(_p(x), _p(y), y_ld, n, d, int(frame_tokens), _p(gate), g_ld, _stream(x.device))
    check(rc, "ss_gate_residual")
    return x


__all__ = ["Workspace", "DeviceStatus", "route", "router_workspace_bytes", "RouterKeys", "pool_keys",
           "history_blocks", "sparse_attention", "sparse_attention_heads", "exact",
           "attention_max_ids", "attention_workspace_bytes", "lse_merge", "merge", "cache_append", "budget", "forced_count", "nblocks",
           "Ring", "cache_append_ring", "ring_refresh", "qkv_norm_rope_ring", "ring_commit",
           "rope_shift", "qkv_norm_rope", "adaln", "rms_norm", "gate_residual"]

# keep the status-bit names importable from here
DEV_BITS = dict(nonfinite=DEV_NONFINITE, timeout=DEV_TIMEOUT, badid=DEV_BADID)
