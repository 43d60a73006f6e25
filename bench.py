"""Benchmark: routed sparse attention (router + block-sparse attention) for one chunk-layer.

Workload (config 2): a 4680-query chunk against a 32760-token KV window, 12 heads, D=128,
64-token router blocks, 25% block density (74 forced current-chunk blocks + 54 routed),
seeded N(0,1) bf16 Q/K/V, N(0,1/128) router weights. One step = router + attention on inputs
already resident in HBM. Two input sets alternate (215 MB each, larger than the 126 MB L2).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

N>1 runs under torchrun: every rank processes its own stream (weak scaling, no collective on
the data path); ``value`` is the sum over ranks of effective FLOPs / the slowest rank's time.
``--impl reference`` times the CPU restatement of the reference's path (oracle/) on the host
cores, rank 0 only.

The line also carries ``rollout`` (config 3, unless ``--no-rollout``): latent frames/s of one
Self-Forcing rollout stream per GPU through a random-init Wan-1.3B DiT with the plugin in every
self-attention layer, next to the same model with dense attention; and ``other_configs`` (unless
``--no-configs``): router + attention at the shapes of configs 1, 4 and a grid of config 5;
``hbm_kernels``: the rolling cache append, the 8-part LSE merge and the anchor rebase, each alone;
``e2e`` (the plugin call with the whole KV window uploaded from the host every step) and
``e2e_streaming`` (the window resident in a KVCache, only the chunk's q/k/v uploaded per step);
``int8_qk`` (unless ``--no-int8``): the INT8-QK attention path on config 2's inputs and ids.
"""
from __future__ import annotations

import argparse
import datetime
import json
import math
import os
import statistics
import threading
import time

import numpy as np
import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
LQ, LK, H, D, BLOCK, DENSITY = 4680, 32760, 12, 128, 64, 0.25
WORKLOAD = "config2 chunk-layer: 4680 q x 32760 KV tokens, 12 heads, D=128, block 64, 25% density, router+attention"
METRIC = "routed sparse-attn effective TFLOP/s per chunk-layer (router + block-sparse attention)"


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["bf16_tflops"]), float(p["hbm_gbs"]), "measured"
    except Exception:
        return 1590.0, 6650.0, "fallback"


# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) of one attention launch at config 2,
# from the ncu capture summarised in profiles/attention_sm100_config2.md (same command given there).
ATTN_TRAFFIC_BYTES = 297295104
ATTN_TRAFFIC_SOURCE = "ncu --set full capture of one config-2 attention launch (profiles/attention_sm100_config2.md)"


def make_inputs(seed: int, device):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn((LQ, H, D), generator=g).bfloat16()
    k = torch.randn((LK, H, D), generator=g).bfloat16()
    v = torch.randn((LK, H, D), generator=g).bfloat16()
    wq = torch.randn((H, D, 64), generator=g) / math.sqrt(D)
    wk = torch.randn((H, D, 64), generator=g) / math.sqrt(D)
    if device is None:
        return q, k, v, wq, wk
    return tuple(t.to(device) for t in (q, k, v, wq, wk))


def effective_flops(ids: np.ndarray, Lq: int = LQ, Lk: int = LK, block: int = BLOCK) -> float:
    """4*D*sum over heads and query rows of the valid tokens in the row's selected blocks."""
    valid = np.minimum(block, Lk - np.arange(math.ceil(Lk / block)) * block)
    tok = np.where(ids >= 0, valid[np.clip(ids, 0, None)], 0).sum(-1)          # [H, qb]
    rows = np.minimum(block, Lq - np.arange(ids.shape[1]) * block)             # [qb]
    return float(4 * D * (tok * rows[None]).sum())


class ClockSampler:
    """NVML SM clock / throttle-reason samples taken while the timed region runs (read only)."""

    REASONS = {0x8: "hw_slowdown", 0x40: "hw_thermal_slowdown", 0x20: "sw_thermal_slowdown", 0x4: "sw_power_cap",
               0x80: "hw_power_brake_slowdown", 0x2: "applications_clocks_setting"}

    def __init__(self, index: int):
        self.samples, self.reasons, self.max_mhz = [], set(), None
        self._stop = threading.Event()
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nvml = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
        except Exception:
            self.nvml = None

    def _run(self):
        while not self._stop.is_set():
            self.sample()
            time.sleep(0.002)

    def sample(self):
        if self.nvml is None:
            return
        try:
            self.samples.append(self.nvml.nvmlDeviceGetClockInfo(self.h, self.nvml.NVML_CLOCK_SM))
            bits = self.nvml.nvmlDeviceGetCurrentClocksEventReasons(self.h)
            for b, name in self.REASONS.items():
                if bits & b:
                    self.reasons.add(name)
        except Exception:
            pass

    def __enter__(self):
        self.t = threading.Thread(target=self._run, daemon=True)
        self.t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        self.t.join()
        self.sample()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["nvml unavailable"], "samples": 0}
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples)}


# ----------------------------------------------------------------------------------------------
# CPU baseline (the oracle restatement of the reference's path, timed on the host cores)
# ----------------------------------------------------------------------------------------------

class CpuPort:
    """The CPU restatement of the reference's path (oracle/: exact-fp32 C router + fp32 numpy
    gather-softmax attention) on the config-2 workload, run on the host cores."""

    def __init__(self):
        import sys
        sys.path.insert(0, ROOT)
        from oracle import oracle as o
        self.o = o
        self.threads = len(os.sched_getaffinity(0))
        q, k, v, wq, wk = make_inputs(0, None)
        self.q, self.k, self.v = (t.float().numpy() for t in (q, k, v))
        self.wq, self.wk = wq.numpy(), wk.numpy()
        self.extra = o.budget(512, 74, density=DENSITY)
        self.ids = None
        self.order = None
        self.pos = 0

    def route(self) -> float:
        t0 = time.perf_counter()
        r = self.o.route(self.q, self.k, self.wq, self.wk, BLOCK, self.extra)
        dt = time.perf_counter() - t0
        self.ids = r["ids"]
        if self.order is None:
            self.order = [(h, i) for i in range(self.ids.shape[1]) for h in range(H)]
            np.random.default_rng(0).shuffle(self.order)
        return dt

    def attend(self, seconds: float = 1e9, max_pairs: int | None = None):
        """Attention over (head, query block) pairs until the budget is spent -> (flops, s, pairs)."""
        flops, t_att, done = 0.0, 0.0, 0
        while t_att < seconds and (max_pairs is None or done < max_pairs):
            h, i = self.order[self.pos % len(self.order)]
            self.pos += 1
            t1 = time.perf_counter()
            r0, r1 = i * BLOCK, min(LQ, (i + 1) * BLOCK)
            self.o.attention_block(self.q, self.k, self.v, self.ids[h, i], h, r0, r1, BLOCK, 1.0 / math.sqrt(D),
                                   dtype=np.float32)
            t_att += time.perf_counter() - t1
            sub = np.full_like(self.ids, -1)
            sub[h, i] = self.ids[h, i]
            flops += effective_flops(sub)
            done += 1
        return flops, t_att, done

    def charged(self, flops, t_att, pairs, t_router):
        """Time charged to a sample: its attention plus the router pro rata to its rows."""
        t = t_att + t_router * pairs / len(self.order)
        return flops / t / 1e12, t


def cpu_baseline(seconds: float):
    port = CpuPort()
    t_router = port.route()
    flops, t_att, pairs = port.attend(seconds=seconds)
    val, _ = port.charged(flops, t_att, pairs, t_router)
    return {"value": val, "unit": "TFLOP/s", "cores": port.threads, "kind": "port",
            "sample": f"{pairs} (head, query-block) pairs of config 2 ({t_att:.1f} s of fp32 numpy attention) plus "
                      f"the exact-fp32 C router charged pro rata ({t_router:.2f} s per full chunk-layer)"}


def run_reference(args, rank: int):
    if rank != 0:
        return
    port = CpuPort()
    times, vals = [], []
    for s in range(args.warmup + args.steps):
        t_router = port.route()
        flops, t_att, pairs = port.attend(max_pairs=args.ref_pairs)
        val, t = port.charged(flops, t_att, pairs, t_router)
        if s >= args.warmup:
            times.append(t)
            vals.append(val)
    value = statistics.median(vals)
    sample = (f"per step: the full C router + {args.ref_pairs} (head, query-block) pairs of config-2 attention "
              f"(fp32 numpy), router time charged pro rata")
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * statistics.median(times),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": WORKLOAD, "parallelism": "rank 0 host cores"},
        "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": port.threads, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


# ----------------------------------------------------------------------------------------------
# GPU arm
# ----------------------------------------------------------------------------------------------

def cache_append_bench(dev, inputs, args):
    """Time ss_cache_append writing the current chunk (4680 tokens of K and V) into a 32760-token
    global cache; algorithmic bytes = chunk read + chunk written, for K and V. Four (chunk, cache)
    pairs rotate, so each append's 57.5 MB come from and go to HBM rather than L2 (4 x 229 MB)."""
    from streaming_sparse_b200 import ops
    start = LK - LQ
    if inputs is not None:
        _, k, v, _, _ = inputs
        k, v = k[start:], v[start:]
    else:
        k = torch.randn((LQ, H, D), device=dev).to(torch.bfloat16)
        v = torch.randn((LQ, H, D), device=dev).to(torch.bfloat16)
    pairs = []
    for r in range(4):
        kc = torch.zeros((LK, H, D), dtype=torch.bfloat16, device=dev)
        vc = torch.zeros_like(kc)
        kn = torch.roll(k, r, 0).contiguous()
        vn = torch.roll(v, r, 0).contiguous()
        pairs.append((kc, vc, kn, vn))

    def once(i):
        kc, vc, kn, vn = pairs[i % len(pairs)]
        ops.cache_append(kc, vc, kn, vn, local_attn=False, global_end=start, local_end=start,
                         current_start=start, sink_tokens=0)

    for i in range(4):
        once(i)
    torch.cuda.synchronize()
    reps = 8
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for i in range(reps):
            once(i)
    g.replay()
    n = max(5, args.steps // reps)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    a.record()
    for _ in range(n):
        g.replay()
    b.record()
    torch.cuda.synchronize()
    us = 1e3 * a.elapsed_time(b) / (n * reps)
    kc, vc, kn, vn = pairs[0]
    nbytes = 2 * 2 * kn.numel() * kn.element_size()
    assert torch.equal(kc[start:], kn) and torch.equal(vc[start:], vn)
    del pairs
    return {"us": us, "bytes": nbytes, "gbs": nbytes / (us * 1e-6) / 1e9,
            "note": "chunk of 4680 tokens x 12 heads x 128 (K and V, bf16) read + written; 4 rotating "
                    "(chunk, cache) pairs larger than L2; CUDA-graph replay"}


def _graph_us(fn, reps: int, steps: int) -> float:
    """Mean us per call of fn(i), i = 0..reps-1 captured in one CUDA graph, replayed back to back
    (eager warm-up first)."""
    for i in range(reps):
        fn(i)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for i in range(reps):
            fn(i)
    g.replay()
    n = max(5, steps // reps)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    a.record()
    for _ in range(n):
        g.replay()
    b.record()
    torch.cuda.synchronize()
    del g
    return 1e3 * a.elapsed_time(b) / (n * reps)


def _replay_ms(graphs, n: int) -> float:
    """Mean ms per replay of the given graphs replayed round-robin n times (after one warm-up round)."""
    for g in graphs:
        g.replay()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for i in range(n):
        graphs[i % len(graphs)].replay()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) / n


def hbm_kernels_bench(dev, args, hbm_gbs: float) -> dict:
    """The HBM-bound kernels beside the attention, each timed alone with CUDA events over graph
    replays, inputs rotating over buffers larger than L2 where the kernel's traffic allows:

    * ``cache_append_roll``: a chunk write into a full rolling window (config 4: 22 frames of
      1560 tokens with a 1-frame sink, 4680-token chunk): 28080 rows shifted left by 4680 in six
      copies, then the chunk written; (28080 + 4680) rows x 3 KB x (K, V) read + written.
    * ``cache_append_ring_roll``: the same roll on a ring-buffer cache: the ring's head moves by
      4680 rows and only the chunk (with at most 64 mirrored rows and the sink's last 24 rows
      repeated before the head) is written.
    * ``lse_merge_8``: the KV-sharded merge of 8 partial outputs (fp32 [8, 4680, 12, 128] + LSE)
      into bf16, the combine step of 8-GPU KV-block sharding.
    * ``anchor_rebase``: one layer's anchor rebase (1560 canonical key rows copied into the
      cache, their 22 temporal RoPE pairs rotated); L2-resident, so latency-bound.
    Each is checked once against a torch expression before it is timed."""
    from streaming_sparse_b200 import ops
    from streaming_sparse_b200.cache import temporal_phase
    out = {}
    gen = torch.Generator(device=dev)
    gen.manual_seed(7)
    row_bytes = H * D * 2

    # ---- rolling append, config-4 window
    ft, sink, n = 1560, 1560, LQ
    cap = 22 * ft
    evicted, rolled = n, cap - n - sink
    caches = [(torch.randn((cap, H, D), generator=gen, device=dev).to(torch.bfloat16),
               torch.randn((cap, H, D), generator=gen, device=dev).to(torch.bfloat16)) for _ in range(2)]
    chunks = [(torch.randn((n, H, D), generator=gen, device=dev).to(torch.bfloat16),
               torch.randn((n, H, D), generator=gen, device=dev).to(torch.bfloat16)) for _ in range(2)]
    g_end = 10 * n

    def roll(i):
        (kc, vc), (kn, vn) = caches[i % 2], chunks[i % 2]
        ops.cache_append(kc, vc, kn, vn, local_attn=True, global_end=g_end, local_end=cap, current_start=g_end,
                         sink_tokens=sink)

    kc, vc = caches[0]
    want_k = torch.cat((kc[:sink], kc[sink + evicted:], chunks[0][0]))
    want_v = torch.cat((vc[:sink], vc[sink + evicted:], chunks[0][1]))
    roll(0)
    torch.cuda.synchronize()
    assert torch.equal(kc, want_k) and torch.equal(vc, want_v), "rolling append differs from the window roll"
    del want_k, want_v
    us = _graph_us(roll, 2, args.steps)
    nbytes = (rolled + n) * row_bytes * 2 * 2
    out["cache_append_roll"] = {"us": us, "bytes": nbytes, "gbs": nbytes / (us * 1e-6) / 1e9,
                                "frac": nbytes / (us * 1e-6) / 1e9 / hbm_gbs, "launches": rolled // evicted + 1}

    # ---- the same roll on a ring-buffer cache: the head moves, only the chunk (plus the mirrored
    # rows and the sink's copy before the head) is written
    ring0 = ops.Ring(sink, cap - sink + 64, 10 * n % (cap - sink + 64))
    rcaches = [(torch.randn((ring0.phys_rows(), H, D), generator=gen, device=dev).to(torch.bfloat16),
                torch.randn((ring0.phys_rows(), H, D), generator=gen, device=dev).to(torch.bfloat16)) for _ in range(2)]

    def ring_roll(i):
        (kc, vc), (kn, vn) = rcaches[i % 2], chunks[i % 2]
        return ops.cache_append_ring(kc, vc, kn, vn, cap=cap, local_attn=True, global_end=g_end, local_end=cap,
                                     current_start=g_end, sink_tokens=sink, ring=ring0)

    def window_of(kc, r):
        t = torch.arange(cap, device=dev)
        rows = torch.where(t < r.sink, t, r.sink + torch.remainder(t - r.sink + r.head, r.cap))
        return kc.index_select(0, rows)

    kc, vc = rcaches[0]
    before = window_of(kc, ring0)
    want_k = torch.cat((before[:sink], before[sink + evicted:], chunks[0][0]))
    _, head = ring_roll(0)
    torch.cuda.synchronize()
    assert torch.equal(window_of(kc, ops.Ring(sink, ring0.cap, head)), want_k), "ring roll differs from the window roll"
    del before, want_k
    us = _graph_us(ring_roll, 2, args.steps)
    a = sink % 64
    rows_written = n + min(n, 64) + a + 64   # chunk, mirrored rows (at most 64), sink copy (+ its mirror, at most)
    nbytes = (n + a) * row_bytes * 2 * 2     # read + written, K and V: the chunk and the sink's copy
    out["cache_append_ring_roll"] = {"us": us, "bytes": nbytes, "gbs": nbytes / (us * 1e-6) / 1e9,
                                     "frac": nbytes / (us * 1e-6) / 1e9 / hbm_gbs,
                                     "rows_written_max": rows_written,
                                     "vs_shift_bytes": out["cache_append_roll"]["bytes"]}
    del caches, chunks, rcaches

    # ---- 8-part LSE merge
    P = 8
    parts = [(torch.randn((P, LQ, H, D), generator=gen, device=dev),
              4.0 * torch.randn((P, H, LQ), generator=gen, device=dev)) for _ in range(2)]
    o, l = parts[0]
    ref = (torch.softmax(l, 0).permute(0, 2, 1)[..., None] * o).sum(0)
    got = ops.lse_merge(o, l, out_dtype=torch.bfloat16)
    torch.cuda.synchronize()
    assert torch.allclose(got.float(), ref, atol=2e-2, rtol=1e-2), "lse_merge differs from the softmax-weighted sum"
    del ref, got

    def merge(i):
        ops.lse_merge(*parts[i % 2], out_dtype=torch.bfloat16)

    us = _graph_us(merge, 2, args.steps)
    nbytes = P * LQ * H * D * 4 + P * H * LQ * 4 + LQ * H * D * 2
    out["lse_merge_8"] = {"us": us, "bytes": nbytes, "gbs": nbytes / (us * 1e-6) / 1e9,
                          "frac": nbytes / (us * 1e-6) / 1e9 / hbm_gbs}
    del parts

    # ---- anchor rebase of one layer (canonical rows -> cache rows, temporal pairs rotated)
    anchor = torch.randn((ft, H, D), generator=gen, device=dev).to(torch.bfloat16)
    kc = torch.zeros((cap, H, D), dtype=torch.bfloat16, device=dev)
    phase = temporal_phase(5 * 3, dev, D)
    ops.rope_shift(anchor, kc[:ft], temporal_phase(0, dev, D))
    torch.cuda.synchronize()
    assert torch.equal(kc[:ft], anchor), "a zero-offset rebase must restore the saved rows"

    def rebase(i):
        ops.rope_shift(anchor, kc[:ft], phase)

    us = _graph_us(rebase, 4, args.steps)
    pairs = phase.shape[0]
    nbytes = 2 * ft * row_bytes + 2 * ft * H * pairs * 4
    out["anchor_rebase"] = {"us": us, "bytes": nbytes, "gbs": nbytes / (us * 1e-6) / 1e9,
                            "note": "rows copied + temporal pairs rotated in place; L2-resident"}
    out["hbm_peak_gbs"] = hbm_gbs
    return out


def config_points():
    """(short name, long name, Lq, Lk, block, sink tokens, budget rule) of every shape the bench
    times besides the headline: config 1, config 4 and a grid of config 5's sweep."""
    pts = [("c1", "config1", 1560, 6240, 64, 0, dict(topk=24)),
           ("c4", "config4", 4680, 34320, 128, 1560, dict(density=0.10, rule="rest"))]
    # c = 1 (the window is the chunk: every block forced, dense), then c = 2, 14, 21
    pts.append(("c5/4680", "config5 Lk=4680 (all forced) b=64", 4680, 4680, 64, 0, dict(density=0.25)))
    for lk in (9360, 65520, 98280):
        for dens in (0.05, 0.10, 0.25, 0.5):
            pts.append((f"c5/{lk}/{round(dens * 100)}", f"config5 Lk={lk} d={dens:g} b=64", 4680, lk, 64, 0,
                        dict(density=dens)))
    for dens in (0.05, 0.5):
        pts.append((f"c5/98280/{round(dens * 100)}/b128", f"config5 Lk=98280 d={dens:g} b=128", 4680, 98280, 128, 0,
                    dict(density=dens)))
    return pts


def configs_bench(dev, args):
    """Router + attention at the other shapes of the reference's configs: config 1, config 4
    (128-token blocks, a one-frame sink, 10 % of the unforced blocks) and a grid of config 5's
    sweep (windows of c = 1, 2, 14 and 21 chunks of 4680 tokens, densities 5/10/25/50 %, blocks 64
    and 128). Seeded N(0,1) inputs. As in the headline step, the history's key blocks are pooled at
    commit and a routed call pools the rest: per point, the median of graph replays of (cached
    route + attention) with a 256 MB L2 flush before each, plus a quarter of the commit's median
    (one commit per four denoising calls). The cached route's ids are checked against the full
    route's, bit for bit, at every point."""
    from streaming_sparse_b200 import ops

    peak, _, _ = peaks()
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    g = torch.Generator(device=dev).manual_seed(55)
    out = []
    reps = max(5, min(20, args.steps // 10))

    def median_us(graph):
        ms = []
        for _ in range(reps):
            flush.fill_(1)
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            graph.replay()
            b.record()
            torch.cuda.synchronize()
            ms.append(a.elapsed_time(b))
        return 1e3 * statistics.median(ms)

    for short, name, lq, lk, block, sink, rule in config_points():
        q = torch.randn((lq, H, D), device=dev, generator=g).bfloat16()
        k = torch.randn((lk, H, D), device=dev, generator=g).bfloat16()
        v = torch.randn((lk, H, D), device=dev, generator=g).bfloat16()
        wq = torch.randn((H, D, 64), device=dev, generator=g) / math.sqrt(D)
        wk = torch.randn((H, D, 64), device=dev, generator=g) / math.sqrt(D)
        kb = ops.nblocks(lk, block)
        nf = ops.forced_count(lq, lk, block, sink)
        extra = ops.budget(kb, nf, **rule)
        ws = ops.Workspace()
        ids = torch.empty((H, ops.nblocks(lq, block), nf + extra), dtype=torch.int32, device=dev)
        o = torch.empty_like(q)
        keys = ops.RouterKeys(H, lk, block=block, device=dev)
        n_hist = ops.history_blocks(lq, lk, block)

        def commit():
            ops.pool_keys(k, wk, keys, j0=0, j1=n_hist)

        def step():
            ops.route(q, k, wq, wk, block=block, extra=extra, sink_tokens=sink, workspace=ws, out=ids, keys=keys,
                      n_cached=n_hist)
            ops.sparse_attention(q, k, v, ids, block=block, out=o)

        commit()
        for _ in range(3):
            step()
        torch.cuda.synchronize()
        ops.DeviceStatus.check(dev)
        full = ops.route(q, k, wq, wk, block=block, extra=extra, sink_tokens=sink, workspace=ws)
        assert torch.equal(full, ids), f"{name}: cached route differs from the full route"
        gs = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gs):
            step()
        gc = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gc):
            commit()
        step_us, commit_us = median_us(gs), median_us(gc)
        us = step_us + commit_us / 4
        fl = effective_flops(ids.cpu().numpy(), lq, lk, block)
        out.append({"short": short, "name": name, "Lq": lq, "Lk": lk, "block": block, "sink_tokens": sink,
                    "blocks_per_query_block": nf + extra, "us": us, "step_us": step_us, "commit_us": commit_us,
                    "effective_gflop": fl / 1e9, "tflops": fl / (us * 1e-6) / 1e12,
                    "frac_of_peak": fl / (us * 1e-6) / 1e12 / peak})
        del gs, gc, q, k, v, ids, o, ws, keys, full
    del flush
    torch.cuda.empty_cache()
    return out


def rollout_bench(dev, args, world: int):
    """Config 3: one Self-Forcing rollout stream per GPU (21 latent frames = 7 chunks x (4 denoising
    + 1 clean pass) x 30 layers of a random-init Wan-1.3B DiT), the sparse plugin (25% density) in
    every self-attention layer, CUDA-graph replay per (chunk, phase). Timed region per rollout:
    pinned-host noise and text -> device, the rollout, latents -> pinned host. Streams are
    independent (weak scaling); the time is the max over ranks. The same model with dense
    attention (scaled-dot-product, no plugin) is timed beside it."""
    import torch.distributed as dist
    from streaming_sparse_b200 import rollout as R
    from streaming_sparse_b200.plugin import RouterConfig, SparseAttention, init_router_weights

    cfg = R.WanConfig()
    rank = dist.get_rank() if world > 1 else 0
    model = R.build_model(cfg, device=dev, seed=0)
    g = torch.Generator(device="cpu").manual_seed(100 + rank)
    noise_h = torch.randn((cfg.frames, cfg.in_dim, cfg.latent_h, cfg.latent_w), generator=g).pin_memory()
    text_h = torch.randn((cfg.text_len, cfg.text_dim), generator=g).pin_memory()
    out_h = torch.empty_like(noise_h).pin_memory()
    noise_d, text_d = torch.empty_like(noise_h, device=dev), torch.empty_like(text_h, device=dev)
    wq, wk = init_router_weights(cfg.num_heads, device=dev)
    dg = torch.Generator(device=dev)
    res = {}
    for name, sparse in (("sparse", SparseAttention(wq, wk, RouterConfig(density=DENSITY))), ("dense", None)):
        ro = R.Rollout(model, sparse=sparse, graphs=True)

        def once():
            noise_d.copy_(noise_h, non_blocking=True)
            text_d.copy_(text_h, non_blocking=True)
            out = ro.run(noise_d, text_d, generator=dg.manual_seed(7))
            out_h.copy_(out, non_blocking=True)

        for _ in range(2):      # eager warm-up, then capture of every (chunk, phase) graph
            once()
        torch.cuda.synchronize()
        reps = max(1, min(3, args.steps // 50))
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(reps):
            once()
        b.record()
        torch.cuda.synchronize()
        ms = torch.tensor([a.elapsed_time(b) / reps], dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(ms, op=dist.ReduceOp.MAX)
        ok = bool(torch.isfinite(out_h).all())
        res[name] = (float(ms), ok)
        ro.release_graphs()
        del ro
    del model
    torch.cuda.empty_cache()
    ms_s, ok_s = res["sparse"]
    ms_d, ok_d = res["dense"]
    frames = cfg.frames * world
    c4 = rollout4_bench(dev, args) if world == 1 else None
    if c4 is not None:
        c4r = rollout4_bench(dev, args, ring=True)
        c4["ring_cache"] = {"value": c4r["value"], "ms_per_rollout": c4r["ms_per_rollout"],
                            "latents_equal": bool(torch.equal(c4r.pop("latents"), c4["latents"]))}
        c4.pop("latents")
    return {"metric": "latent frames/s (config 3 rollout, all streams)", "value": frames / (ms_s * 1e-3),
            "unit": "frames/s", "streams": world, "frames_per_stream": cfg.frames, "ms_per_rollout": ms_s,
            "dense_value": frames / (ms_d * 1e-3), "dense_ms_per_rollout": ms_d, "speedup_vs_dense": ms_d / ms_s,
            "finite": ok_s and ok_d, "reps": reps,
            "h2d_bytes_per_rollout": noise_h.numel() * 4 + text_h.numel() * 4,
            "d2h_bytes_per_rollout": out_h.numel() * 4,
            "model": "random-init Wan-1.3B causal DiT (30 blocks, dim 1536, 12 heads, FFN 8960), bf16",
            "note": "7 chunks x 3 latent frames (60x104), 4 denoising steps + 1 clean pass per chunk, global "
                    "KV cache 32760 tokens, text 512 x 4096 N(0,1); routed at 25% density in the denoising "
                    "passes, dense (every block) in the clean pass; dense_value: same model with "
                    "scaled-dot-product attention; timed region includes host<->device copies",
            "config4_long_horizon": c4}


def rollout4_bench(dev, args, ring: bool = False, head_parallel: bool = False):
    """Config 4's stream on one GPU: 120 latent frames in 40 chunks through a rolling window of 21
    frames + 1 sink frame (34320 tokens), 128-token router blocks at 10 % of the unforced blocks;
    the window rolls on every chunk's first call from chunk 7 on. One timed rollout after an eager
    warm-up and a capture run (routed only; the dense model is timed by
    `python -m streaming_sparse_b200.rollout --config4 --dense`). ``ring``: the layers' KV caches
    as ring buffers (a roll moves the head; heads in device memory under graph replay).
    ``head_parallel`` (under torchrun): the same stream with every layer's attention split by
    heads over the ranks (each rank's caches hold its heads; the fused head gather returns all
    heads to every rank; the rest of the model runs on every rank), timed between barriers, max
    over ranks."""
    import torch.distributed as dist
    from streaming_sparse_b200 import rollout as R
    from streaming_sparse_b200.plugin import RouterConfig, SparseAttention, init_router_weights

    cfg = R.WanConfig(frames=120, cache_frames=22, local_attn_frames=22, sink_frames=1, ring_cache=ring)
    model = R.build_model(cfg, device=dev, seed=0)
    g = torch.Generator(device=dev)
    noise = torch.randn((cfg.frames, cfg.in_dim, cfg.latent_h, cfg.latent_w), device=dev, generator=g.manual_seed(3))
    text = torch.randn((cfg.text_len, cfg.text_dim), device=dev, generator=g.manual_seed(4))
    wq, wk = init_router_weights(cfg.num_heads, device=dev)
    sp = SparseAttention(wq, wk, RouterConfig(block=128, density=0.10, rule="rest", sink_tokens=cfg.frame_tokens))
    ro = R.Rollout(model, sparse=sp, graphs=True, head_parallel=head_parallel)
    for _ in range(2):
        ro.run(noise, text, generator=g.manual_seed(5))
    torch.cuda.synchronize()
    if head_parallel:
        dist.barrier()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    out = ro.run(noise, text, generator=g.manual_seed(5))
    b.record()
    torch.cuda.synchronize()
    ms = a.elapsed_time(b)
    if head_parallel:
        t = torch.tensor([ms], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t)
    res = {"value": cfg.frames / (ms * 1e-3), "unit": "frames/s", "ms_per_rollout": ms, "frames": cfg.frames,
           "graphs": len(ro._graph), "finite": bool(torch.isfinite(out).all()), "ring_cache": ring,
           "latents": out}
    ro.close()
    if head_parallel:
        dist.barrier()
    del ro, model
    torch.cuda.empty_cache()
    return res


def sharded_bench(dev, args, rank: int, world: int) -> dict:
    """Config 4's chunk-layer (4680 queries against a 34320-token window with a sink frame,
    128-token blocks, 10 % of the unforced blocks) split over the N GPUs, next to the same call on
    one GPU (every rank builds the same seeded window):

    * ``kv``: KV-block sharding. Each rank stores its own blocks, the history keys are pooled by
      their owners and all-gathered at commit (outside the timed region, once per chunk), and a
      call routes, attends over the rank's blocks with the epilogue pushing each partial row to
      the rank that owns it, then every rank's merge kernel (after a flag barrier it makes
      itself) merges its own rows and stores them into all ranks' outputs, and a second barrier
      ends the call. ``kv_pull``: the same call with the partials pulled over peer memory by one
      merge kernel per rank (every row). Both are timed as ``attend`` (route, attention,
      exchange), as the single-GPU call finds the chunk already in its window; writing the
      chunk's rows into the shards (``write_chunk``) is reported beside it.
    * ``heads``: head sharding, each rank routing and attending over its heads, then one NCCL
      all_gather of the outputs.
    * ``heads_fused``: the same heads, the gather fused into the attention: the kernel's epilogue
      stores every output row into all ranks' buffers over NVLink, then a flag barrier.
    * ``stream4_heads`` (unless ``--no-rollout``): config 4's whole stream (120 frames) with every
      layer's attention split by heads this way, frames/s max over ranks; rank 0 also runs the
      stream on one GPU for the ratio and the latents' difference (split-mode tiles at 6 heads
      per rank merge in fp32, so the latents agree to rounding, not bit for bit).
    * ``c5_98280``: config 5's longest window (98280 tokens, 64-token blocks, 10 %), KV push and
      fused heads.
    Each is checked once against the single-GPU output (router ids bit for bit for ``kv``; max-abs,
    mean-abs and NMSE of the output), then timed as CUDA-graph replays (two calls per graph),
    max over ranks. The KV-sharded speed-ups are against the one-GPU call that also routes with
    the history keys pooled at commit (``single_gpu_cached_us``); the head-sharded ones against
    the plain one-GPU call (both route the whole window per call). ``merge_share``: the part of a
    KV-sharded call that a graph without the barrier and merge does not take."""
    import torch.distributed as dist
    from streaming_sparse_b200 import ops
    from streaming_sparse_b200.distributed import HeadShardedAttention, KVShardedAttention, head_shard, local_ids
    from streaming_sparse_b200.plugin import RouterConfig, SparseAttention

    lq, lk, block, sink = 4680, 34320, 128, 1560
    cfg = RouterConfig(block=block, density=0.10, rule="rest", sink_tokens=sink)
    g = torch.Generator().manual_seed(404)
    q = torch.randn((lq, H, D), generator=g).bfloat16().to(dev)
    k = torch.randn((lk, H, D), generator=g).bfloat16().to(dev)
    v = torch.randn((lk, H, D), generator=g).bfloat16().to(dev)
    wq = (torch.randn((H, D, 64), generator=g) / math.sqrt(D)).to(dev)
    wk = (torch.randn((H, D, 64), generator=g) / math.sqrt(D)).to(dev)
    sp = SparseAttention(wq, wk, cfg)
    whole = sp.forward_one(q, k, v)
    whole_ids = sp.last_ids.clone()
    reps = max(10, min(50, args.steps))

    def graph_us(calls):
        """us per call: a graph of two calls, replayed `reps` times after warm-up, max over ranks."""
        for _ in range(2):
            calls()
        torch.cuda.synchronize()
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr):
            calls()
        for _ in range(3):
            gr.replay()
        torch.cuda.synchronize()
        dist.barrier()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(reps):
            gr.replay()
        b.record()
        torch.cuda.synchronize()
        t = torch.tensor([a.elapsed_time(b) * 1e3 / (2 * reps)], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dist.barrier()
        del gr
        return float(t)

    def err(x):
        d = (x.float() - whole.float()).abs()
        return {"max_abs": float(d.max()), "mean_abs": float(d.mean()),
                "nmse": float((d.double() ** 2).sum() / (whole.double() ** 2).sum())}

    o1 = torch.empty_like(q)
    single = graph_us(lambda: (sp.forward_one(q, k, v, out=o1), sp.forward_one(q, k, v, out=o1)))

    def cached_single(q_, k_, v_, cfg_, sink_):
        """us of the one-GPU call with the history keys pooled at commit (as the KV-sharded ranks
        route): cached route + attention."""
        lq_, lk_ = q_.shape[0], k_.shape[0]
        keys = ops.RouterKeys(H, lk_, block=cfg_.block, device=dev)
        nh = ops.history_blocks(lq_, lk_, cfg_.block)
        ops.pool_keys(k_, wk, keys, j0=0, j1=nh)
        ws1, o_ = ops.Workspace(), torch.empty_like(q_)

        def call():
            ids = ops.route(q_, k_, wq, wk, block=cfg_.block, extra=cfg_.extra(lq_, lk_), sink_tokens=sink_,
                            workspace=ws1, keys=keys, n_cached=nh)
            ops.sparse_attention(q_, k_, v_, ids, block=cfg_.block, out=o_, workspace=ws1)
        return graph_us(lambda: (call(), call()))

    single_cached = cached_single(q, k, v, cfg, sink)
    res = {"config": "config4 chunk-layer: 4680 q x 34320 KV (21 frames + 1 sink frame), b128, 10% of unforced",
           "single_gpu_us": single, "single_gpu_cached_us": single_cached}

    # ---- KV blocks
    c0 = lk - lq
    kc, vc = k[c0:].clone(), v[c0:].clone()
    ob = torch.empty_like(q)
    lo, ll = torch.empty_like(q), torch.empty((H, lq), dtype=torch.float32, device=dev)
    for exchange in ("push", "pull"):
        shard = KVShardedAttention(SparseAttention(wq, wk, cfg), lq, lk, dev, exchange=exchange)
        shard.commit(k, v)
        out = shard(q, kc, vc).clone()
        torch.cuda.synchronize()
        ops.DeviceStatus.check(dev)
        kv = dict(err(out), ids_equal=bool(torch.equal(shard.last_ids, whole_ids)))
        # timed: route + attention + exchange over the window as written (the single-GPU call
        # likewise finds the chunk in its window); the chunk's write into the shards apart
        if exchange == "push":
            kv["us"] = graph_us(lambda: (shard.attend(q), shard.attend(q)))
            kv["write_chunk_us"] = graph_us(lambda: (shard.write_chunk(kc, vc), shard.write_chunk(kc, vc)))
            push_out = out
        else:
            kv["us"] = graph_us(lambda: (shard.attend(q, out=ob), shard.attend(q, out=ob)))
            kv["equals_push"] = bool(torch.equal(out, push_out))

            def local_part():
                ids = shard.route(q)
                ops.sparse_attention(q, shard.k_local[:shard.Lk_local], shard.v_local[:shard.Lk_local],
                                     local_ids(ids, rank, world), block=block, return_lse=True, out=lo, lse=ll)
            kv["local_us"] = graph_us(lambda: (local_part(), local_part()))
            kv["merge_share"] = max(0.0, 1.0 - kv["local_us"] / kv["us"])
        # against the one-GPU call that also routes with the keys pooled at commit
        kv["speedup_vs_1gpu"] = single_cached / kv["us"]
        torch.cuda.synchronize()
        ops.DeviceStatus.check(dev)
        dist.barrier()
        shard.close()
        res["kv" if exchange == "push" else "kv_pull"] = kv

    # ---- heads
    sph = SparseAttention(head_shard(wq, rank, world, 0), head_shard(wk, rank, world, 0), cfg)
    hq, hk, hv = head_shard(q, rank, world), head_shard(k, rank, world), head_shard(v, rank, world)
    hs = HeadShardedAttention(sph, H)
    hout = hs(hq, hk, hv)
    torch.cuda.synchronize()
    heads = dict(err(hout), bit_exact=bool(torch.equal(hout, whole)))
    heads["us"] = graph_us(lambda: (hs(hq, hk, hv), hs(hq, hk, hv)))
    heads["speedup_vs_1gpu"] = single / heads["us"]
    res["heads"] = heads

    # ---- heads, the gather fused into the attention (epilogue stores to every rank's buffer)
    hf = HeadShardedAttention(SparseAttention(head_shard(wq, rank, world, 0), head_shard(wk, rank, world, 0), cfg),
                              H, Lq=lq, device=dev)
    fout = hf(hq, hk, hv).clone()
    torch.cuda.synchronize()
    ops.DeviceStatus.check(dev)
    fused = dict(err(fout), equals_all_gather=bool(torch.equal(fout, hout)))
    fused["us"] = graph_us(lambda: (hf(hq, hk, hv), hf(hq, hk, hv)))
    fused["speedup_vs_1gpu"] = single / fused["us"]
    torch.cuda.synchronize()
    ops.DeviceStatus.check(dev)
    dist.barrier()
    hf.close()
    res["heads_fused"] = fused
    del shard, hs
    torch.cuda.empty_cache()

    # ---- config 5's longest window (98280 tokens, 64-token blocks, 10 %): KV push, fused heads
    lq5, lk5 = 4680, 98280
    cfg5 = RouterConfig(block=64, density=0.10)
    g5 = torch.Generator().manual_seed(505)
    q5, k5, v5 = (torch.randn((n, H, D), generator=g5).bfloat16().to(dev) for n in (lq5, lk5, lk5))
    sp5 = SparseAttention(wq, wk, cfg5)
    whole5 = sp5.forward_one(q5, k5, v5)
    ids5 = sp5.last_ids.clone()
    o5 = torch.empty_like(q5)
    c5 = {"config": "config5 chunk-layer: 4680 q x 98280 KV, b64, 10%",
          "single_gpu_us": graph_us(lambda: (sp5.forward_one(q5, k5, v5, out=o5), sp5.forward_one(q5, k5, v5, out=o5))),
          "single_gpu_cached_us": cached_single(q5, k5, v5, cfg5, 0)}
    sh5 = KVShardedAttention(SparseAttention(wq, wk, cfg5), lq5, lk5, dev)
    sh5.commit(k5, v5)                     # the whole window, the chunk's rows included
    out5 = sh5.attend(q5).clone()
    torch.cuda.synchronize()
    ops.DeviceStatus.check(dev)
    c5["kv"] = {"us": graph_us(lambda: (sh5.attend(q5), sh5.attend(q5))),
                "ids_equal": bool(torch.equal(sh5.last_ids, ids5)),
                "max_abs": float((out5.float() - whole5.float()).abs().max())}
    c5["kv"]["speedup_vs_1gpu"] = c5["single_gpu_cached_us"] / c5["kv"]["us"]
    torch.cuda.synchronize()
    dist.barrier()
    sh5.close()
    hf5 = HeadShardedAttention(SparseAttention(head_shard(wq, rank, world, 0), head_shard(wk, rank, world, 0), cfg5),
                               H, Lq=lq5, device=dev)
    a5 = (head_shard(q5, rank, world), head_shard(k5, rank, world), head_shard(v5, rank, world))
    hout5 = hf5(*a5).clone()
    torch.cuda.synchronize()
    ops.DeviceStatus.check(dev)
    c5["heads_fused"] = {"us": graph_us(lambda: (hf5(*a5), hf5(*a5))),
                         "max_abs": float((hout5.float() - whole5.float()).abs().max())}
    c5["heads_fused"]["speedup_vs_1gpu"] = c5["single_gpu_us"] / c5["heads_fused"]["us"]
    torch.cuda.synchronize()
    dist.barrier()
    hf5.close()
    res["c5_98280"] = c5
    del sp5, sh5, hf5, q5, k5, v5, a5, whole5
    torch.cuda.empty_cache()

    # ---- config 4's stream, every layer's attention split by heads (fused gather)
    if not args.no_rollout:
        hp = rollout4_bench(dev, args, ring=True, head_parallel=True)
        stream = {"frames_s": hp["value"], "ms_per_rollout": hp["ms_per_rollout"], "finite": hp["finite"]}
        if rank == 0:   # the same stream on one GPU, same box, for the ratio and the latents
            one = rollout4_bench(dev, args, ring=True)
            d = (hp["latents"].float() - one["latents"].float()).abs()
            stream.update(single_frames_s=one["value"], speedup_vs_1gpu=hp["value"] / one["value"],
                          latents_max_abs=float(d.max()), latents_mean_abs=float(d.mean()))
            del one
        del hp
        dist.barrier()
        res["stream4_heads"] = stream
    torch.cuda.empty_cache()
    return res


def e2e_streaming_bench(dev, sets, sparse, flops, args, world: int, stream) -> dict:
    """The config-2 chunk-layer as a streaming caller makes it (the reference's per-layer
    ``self_attn.forward(..., kv_cache, current_start)``, wan/modules/causal_model.py:216-253):
    the 32760-token window is resident in a ``KVCache`` kept across calls, and every step uploads
    only the chunk's q, k, v from pinned host memory, writes k/v into the window
    (``KVCache.append``; a denoising call rewrites its chunk's rows, no roll), routes and attends
    over the window, and reads the output back. The chunk's q, k, v are staged in one pinned
    buffer, so a step is one upload; pipelined like ``e2e``: step i+1's upload overlaps step i. One window per input set; the output of a warm-up step is checked bit for bit against
    the plugin call on the same q/k/v."""
    import torch.distributed as dist
    from streaming_sparse_b200.cache import KVCache
    start = LK - LQ
    caches = []
    for q, k, v, _, _ in sets:
        c = KVCache(LK, H, D, local_attn_size=-1, device=dev, track_positions=False)
        c.append(k, v, 0)                       # the history (and this chunk) written once, outside timing
        caches.append(c)
        sparse.attach(c)                        # history key projections pooled once, reused per call
    # the chunk's q, k, v staged in one pinned buffer [3, Lq, H, D]: one upload per step
    host = [torch.stack((q, k[start:], v[start:])).cpu().pin_memory() for q, k, v, _, _ in sets]
    dev_in = [torch.empty(h.shape, dtype=h.dtype, device=dev) for h in host]
    outs = [torch.empty((LQ, H, D), dtype=torch.bfloat16).pin_memory() for _ in range(2)]
    h2d = host[0].numel() * host[0].element_size()
    d2h = outs[0].numel() * outs[0].element_size()
    up, down = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    copied = [torch.cuda.Event() for _ in range(2)]
    done = [torch.cuda.Event() for _ in range(2)]

    def upload(i):
        s_ = i % 2
        with torch.cuda.stream(up):
            if i >= 2:
                up.wait_event(done[s_])
            dev_in[s_].copy_(host[s_], non_blocking=True)
            copied[s_].record(up)

    def compute(i):
        s_ = i % 2
        stream.wait_event(copied[s_])
        q, k_new, v_new = dev_in[s_].unbind(0)
        cache = caches[s_]
        cache.append(k_new, v_new, start)
        kw, vw = cache.window()
        res = sparse.forward_one(q, kw, vw)
        done[s_].record(stream)
        with torch.cuda.stream(down):
            down.wait_event(done[s_])
            outs[s_].copy_(res, non_blocking=True)
        res.record_stream(down)

    def run(n):
        upload(0)
        for i in range(n):
            if i + 1 < n:
                upload(i + 1)
            compute(i)

    run(2)
    torch.cuda.synchronize()
    ref = sparse(sets[0][0][None], sets[0][1][None], sets[0][2][None])[0].cpu()
    assert torch.equal(outs[0], ref), "streaming call differs from the plugin call on the same inputs"
    n = max(3, min(args.steps, 20))
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(up)
    run(n)
    down.wait_stream(stream)
    b.record(down)
    torch.cuda.synchronize()
    ms = a.elapsed_time(b)
    fl = sum(flops[i % 2] for i in range(n))
    t = torch.tensor([ms, fl], dtype=torch.float64, device=dev)
    if world > 1:
        mx = t.clone()
        dist.all_reduce(mx[:1], op=dist.ReduceOp.MAX)
        sm = t.clone()
        dist.all_reduce(sm[1:], op=dist.ReduceOp.SUM)
        ms, fl = float(mx[0]), float(sm[1])
    else:
        ms, fl = float(t[0]), float(t[1])
    return {"value": fl / (ms * 1e-3) / 1e12, "unit": "TFLOP/s", "h2d_bytes_per_step": h2d,
            "d2h_bytes_per_step": d2h, "steps": n, "ms_per_step": ms / n,
            "api": "KVCache.append(k_new, v_new, current_start) + SparseAttention.forward_one(q, *cache.window()) "
                   "with the chunk's q, k, v in one pinned host buffer and a pinned output; the window stays "
                   "resident across calls"}


def int8_bench(dev, sets, ids_buf, flops, args, peak) -> dict:
    """The INT8-QK path (migration/unified_router/opt23/attention.py, INT8=True) at
    config 2 on the bench's own inputs and router ids: the history's key pages quantised once per
    commit, the pages the current chunk touches quantised per call, then ss_attention_i8. Each stage
    is one CUDA graph per input set, replayed alternately (two 215 MB sets, > L2); its output is
    compared with the bf16 kernel's on the same ids (the difference is the int8 rounding of Q and K)."""
    from streaming_sparse_b200 import ops
    npg = ops.quant_pages(LK)
    p_cur = (LK - LQ) // 64                       # first page holding a current-chunk token
    qk = [ops.quant_k_pages(s_[1]) for s_ in sets]
    out8 = [torch.empty((LQ, H, D), dtype=torch.bfloat16, device=dev) for _ in sets]
    ws = ops.Workspace()

    def commit(s):
        ops.quant_k_pages(sets[s][1], p0=0, p1=p_cur, k_i8=qk[s][0], ks=qk[s][1])

    def quant_chunk(s):
        ops.quant_k_pages(sets[s][1], p0=p_cur, p1=npg, k_i8=qk[s][0], ks=qk[s][1])

    def attend(s):
        q, k, v, _, _ = sets[s]
        ops.sparse_attention_i8(q, qk[s][0], qk[s][1], v, ids_buf[s], block=BLOCK, out=out8[s], workspace=ws)

    for s in range(2):
        commit(s), quant_chunk(s), attend(s)
    torch.cuda.synchronize()
    ops.DeviceStatus.check(dev)
    graphs = {}
    for name, fn in (("commit", commit), ("quant_chunk", quant_chunk), ("attend", attend)):
        graphs[name] = []
        for s in range(2):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                fn(s)
            graphs[name].append(g)
    n = max(10, min(args.steps, 100))
    res = {}
    for name, gs in graphs.items():
        for i in range(max(3, args.warmup)):
            gs[i % 2].replay()
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(n)]
        torch.cuda.synchronize()
        for i in range(n):
            evs[i][0].record()
            gs[i % 2].replay()
            evs[i][1].record()
        torch.cuda.synchronize()
        res[name] = statistics.mean(a.elapsed_time(b) for a, b in evs) * 1e3
    ref = torch.empty((LQ, H, D), dtype=torch.float32, device=dev)
    dif = []
    for s in range(2):
        q, k, v, _, _ = sets[s]
        ops.sparse_attention(q, k, v, ids_buf[s], block=BLOCK, out=ref, out_dtype=torch.float32)
        d = out8[s].float() - ref
        dif.append((float(d.abs().max()), float((d * d).sum() / (ref * ref).sum())))
    eff = statistics.mean(flops)
    tf = eff / (res["attend"] * 1e-6) / 1e12
    return {"attention_us": res["attend"], "quant_chunk_us": res["quant_chunk"], "commit_quant_us": res["commit"],
            "pieces_workspace_bytes": ops.attention_i8_workspace_bytes(H, LQ),
            "tflops": tf, "frac_of_peak": tf / peak, "step_tflops": eff / ((res["attend"] + res["quant_chunk"]) * 1e-6) / 1e12,
            "vs_bf16_max_abs": max(x[0] for x in dif), "vs_bf16_nmse": max(x[1] for x in dif),
            "kernel": "ss::i8::attention_i8_kernel (tcgen05.mma kind::i8 scores, kind::f16 P.V)"}


def run_ours(args, rank: int, world: int, local_rank: int):
    import torch.distributed as dist
    from streaming_sparse_b200 import ops
    from streaming_sparse_b200.plugin import RouterConfig, SparseAttention

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    lib_ok = ops.attention_max_ids(LK, BLOCK) >= 128
    assert lib_ok
    if args.only_hbm_kernels:   # the cache / merge kernels alone (e.g. under a profiler), rank 0
        if rank == 0:
            _, hbm, _ = peaks()
            hbm_k = hbm_kernels_bench(dev, args, hbm)   # first: its first 7 copy launches are one rolling append
            cache = cache_append_bench(dev, None, args)
            line = {"cache_append": dict(cache, hbm_peak_gbs=hbm, frac=cache["gbs"] / hbm), "hbm_kernels": hbm_k}
            print(json.dumps(line), flush=True)
        return
    sets = [make_inputs(1000 * rank + s, dev) for s in range(2)]
    extra = RouterConfig(density=DENSITY).extra(LQ, LK)
    ws = ops.Workspace()
    n_ids = ops.forced_count(LQ, LK, BLOCK) + extra
    ids_buf = [torch.empty((H, math.ceil(LQ / BLOCK), n_ids), dtype=torch.int32, device=dev) for _ in sets]
    out = torch.empty((LQ, H, D), dtype=torch.bfloat16, device=dev)
    # Each input set is one layer's window: its history key blocks are pooled at commit
    # (ss_router_pool_keys) and every routed call pools only the query blocks and the key blocks
    # from the chunk boundary on (ss_router_cached), as the reference's streaming pipeline does
    # (refresh_history once per chunk, current per call: migration/unified_router/opt23/pipeline.py).
    n_hist = ops.history_blocks(LQ, LK, BLOCK)
    keys = [ops.RouterKeys(H, LK, block=BLOCK, device=dev) for _ in sets]

    def commit(s):
        _, k, _, _, wk = sets[s]
        ops.pool_keys(k, wk, keys[s], j0=0, j1=n_hist)

    def route(s):
        q, k, v, wq, wk = sets[s]
        ops.route(q, k, wq, wk, block=BLOCK, extra=extra, workspace=ws, out=ids_buf[s], keys=keys[s], n_cached=n_hist)

    def route_uncached(s):
        q, k, v, wq, wk = sets[s]
        ops.route(q, k, wq, wk, block=BLOCK, extra=extra, workspace=ws, out=ids_buf[s])

    fast_ids = [torch.empty_like(b) for b in ids_buf]

    def route_fast(s):   # the tensor-core router mode (same ids), timed beside the exact one
        q, k, v, wq, wk = sets[s]
        ops.route(q, k, wq, wk, block=BLOCK, extra=extra, workspace=ws, out=fast_ids[s], keys=keys[s],
                  n_cached=n_hist, fast=True)

    def attend(s):
        q, k, v, wq, wk = sets[s]
        ops.sparse_attention(q, k, v, ids_buf[s], block=BLOCK, out=out)

    for s in range(2):
        commit(s)
    for s in range(max(3, args.warmup)):
        route(s % 2)
        attend(s % 2)
    torch.cuda.synchronize()
    ops.DeviceStatus.check(dev)
    cached_ids = [b.clone() for b in ids_buf]
    for s in range(2):
        route_uncached(s)
        route_fast(s)
    torch.cuda.synchronize()
    assert all(torch.equal(a, b) for a, b in zip(cached_ids, ids_buf)), "cached route differs from the full route"
    fast_equal = all(torch.equal(a, b) for a, b in zip(cached_ids, fast_ids))
    assert fast_equal, "the fast router's ids differ from the exact router's"
    flops = [effective_flops(b.cpu().numpy()) for b in ids_buf]
    # router FLOPs (reported separately): pooled projections + block-score GEMM
    qb, kb = math.ceil(LQ / BLOCK), math.ceil(LK / BLOCK)
    router_flops = 2 * H * qb * kb * 64 + 2 * H * (qb + kb) * D * 64

    # one CUDA graph per (stage, input set): a step replays the router graph (after the commit
    # graph on the set's every fourth call: a chunk's four denoising calls share one commit), then
    # the attention graph
    g_commit, g_route, g_attn, g_full, g_fast = [], [], [], [], []
    for s in range(2):
        for fn, lst in ((commit, g_commit), (route, g_route), (attend, g_attn), (route_uncached, g_full),
                        (route_fast, g_fast)):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                fn(s)
            lst.append(g)
    for s in range(2):
        g_commit[s].replay()
        g_route[s].replay()
        g_attn[s].replay()
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream(dev)

    def is_commit(i):
        return (i // 2) % 4 == 0

    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(args.steps)]
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(dev.index if "CUDA_VISIBLE_DEVICES" not in os.environ else 0) as clk:
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        t0.record(stream)
        for i in range(args.steps):
            e = evs[i]
            e[0].record(stream)
            if is_commit(i):
                g_commit[i % 2].replay()
            g_route[i % 2].replay()
            e[1].record(stream)
            g_attn[i % 2].replay()
            e[2].record(stream)
        t1.record(stream)
        torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    elapsed_ms = t0.elapsed_time(t1)
    att_ms = [e[1].elapsed_time(e[2]) for e in evs]
    rt_ms = [e[0].elapsed_time(e[1]) for e in evs]
    my_flops = sum(flops[i % 2] for i in range(args.steps))
    t = torch.tensor([elapsed_ms, my_flops], dtype=torch.float64, device=dev)
    if world > 1:
        mx = t.clone()
        dist.all_reduce(mx[:1], op=dist.ReduceOp.MAX)
        sm = t.clone()
        dist.all_reduce(sm[1:], op=dist.ReduceOp.SUM)
        elapsed_ms, total_flops = float(mx[0]), float(sm[1])
    else:
        total_flops = my_flops
    value = total_flops / (elapsed_ms * 1e-3) / 1e12
    launches = sum(3 + (1 if is_commit(i) else 0) for i in range(args.steps))
    # untimed beside it: the commit-time pooling alone and the router that pools every key block
    commit_us = 1e3 * _replay_ms(g_commit, 20)
    route_full_us = 1e3 * _replay_ms(g_full, 20)
    route_cached_us = 1e3 * _replay_ms(g_route, 20)
    route_fast_us = 1e3 * _replay_ms(g_fast, 20)
    del g_commit, g_full, g_fast

    # ---- e2e: the public plugin call with host buffers (pinned), copies inside the timed region
    sparse = SparseAttention(sets[0][3], sets[0][4], RouterConfig(density=DENSITY), workspace=ws)
    host = [tuple(t.cpu().pin_memory() for t in s_[:3]) for s_ in sets]
    dev_in = [tuple(torch.empty_like(t) for t in s_[:3]) for s_ in sets]
    host_out = torch.empty((1, LQ, H, D), dtype=torch.bfloat16).pin_memory()
    h2d = sum(t.numel() * t.element_size() for t in host[0])
    d2h = host_out.numel() * host_out.element_size()

    # Pipelined as a streaming caller would run it: step i+1's host->device copy (its own stream)
    # overlaps step i's router + attention, and step i's result goes back on a third stream.
    # Two device input slots and two pinned output buffers alternate.
    up, down = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    copied = [torch.cuda.Event() for _ in range(2)]
    done = [torch.cuda.Event() for _ in range(2)]
    outs = [torch.empty_like(host_out).pin_memory() for _ in range(2)]

    def upload(i):
        s_ = i % 2
        with torch.cuda.stream(up):
            if i >= 2:
                up.wait_event(done[s_])            # step i-2 has finished reading this slot
            for dst, src in zip(dev_in[s_], host[s_]):
                dst.copy_(src, non_blocking=True)
            copied[s_].record(up)

    def compute(i):
        s_ = i % 2
        stream.wait_event(copied[s_])
        q, k, v = dev_in[s_]
        res = sparse(q[None], k[None], v[None])
        done[s_].record(stream)
        with torch.cuda.stream(down):
            down.wait_event(done[s_])
            outs[s_].copy_(res, non_blocking=True)
        res.record_stream(down)

    def run_e2e(n):
        upload(0)
        for i in range(n):
            if i + 1 < n:
                upload(i + 1)
            compute(i)

    run_e2e(2)
    torch.cuda.synchronize()
    e_steps = max(3, min(args.steps, 20))
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(up)
    run_e2e(e_steps)
    down.wait_stream(stream)
    b.record(down)
    torch.cuda.synchronize()
    e2e_ms = a.elapsed_time(b)
    e2e_flops = sum(flops[i % 2] for i in range(e_steps))
    te = torch.tensor([e2e_ms, e2e_flops], dtype=torch.float64, device=dev)
    if world > 1:
        mx = te.clone()
        dist.all_reduce(mx[:1], op=dist.ReduceOp.MAX)
        sm = te.clone()
        dist.all_reduce(sm[1:], op=dist.ReduceOp.SUM)
        e2e_ms, e2e_flops = float(mx[0]), float(sm[1])
    e2e_value = e2e_flops / (e2e_ms * 1e-3) / 1e12
    streaming = e2e_streaming_bench(dev, sets, sparse, flops, args, world, stream)

    # ---- cache append (the chunk write of config 2 into a 32760-token window), HBM-bound
    cache = cache_append_bench(dev, sets[0], args)
    _, hbm_gbs, _ = peaks()
    hbm_k = hbm_kernels_bench(dev, args, hbm_gbs)

    # ---- the INT8-QK path on the same inputs and ids
    int8 = None if args.no_int8 else int8_bench(dev, sets, ids_buf, flops, args, peaks()[0])

    # ---- config 4's chunk-layer split over the GPUs (KV blocks / heads), N > 1
    sharded = sharded_bench(dev, args, rank, world) if world > 1 and not args.no_sharded else None

    # ---- config 3: streaming rollout of the DiT with the plugin in every layer (latent frames/s)
    rollout = None
    if not args.no_rollout:
        rollout = rollout_bench(dev, args, world)
    # ---- the other configs' shapes (router + attention, per shape)
    other = None if args.no_configs else configs_bench(dev, args)

    if rank != 0:
        return
    peak, hbm, peak_kind = peaks()
    att_avg = statistics.mean(att_ms)
    achieved = (sum(flops) / 2) / (att_avg * 1e-3) / 1e12
    cpu = None if args.no_cpu_baseline else cpu_baseline(args.cpu_seconds)
    # Detail records first, one JSON object per line; the last line is the bench line proper,
    # short enough that a reader keeping only the tail of stdout still sees every headline figure.
    details = {"e2e_streaming": streaming, "cache_append": dict(cache, hbm_peak_gbs=hbm, frac=cache["gbs"] / hbm),
               "hbm_kernels": hbm_k, "rollout": rollout, "other_configs": other, "sharded": sharded, "int8_qk": int8}
    for name, rec in details.items():
        if rec is not None:
            print(json.dumps({"detail": name, "record": rec}), flush=True)

    def r(x, nd=1):
        return None if x is None else round(float(x), nd)

    line = {
        "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": elapsed_ms / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": WORKLOAD, "parallelism": f"streams x{world} (one replica per GPU)",
                   "timing": "CUDA-graph replays, events between them; history keys pooled at commit (every 4th "
                             "call of a window), current chunk pooled per call",
                   "l2": "2 alternating input sets of 215 MB each (> 126 MB L2)", "density": DENSITY,
                   "blocks_per_query_block": n_ids},
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                     "frac": achieved / peak, "traffic": ATTN_TRAFFIC_BYTES, "peak_kind": peak_kind,
                     "kernel": "ss::attn::sparse_attention_kernel", "traffic_source": ATTN_TRAFFIC_SOURCE},
        "cpu_baseline": cpu,
        "e2e": {"value": e2e_value, "unit": "TFLOP/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "steps": e_steps, "api": "plugin.SparseAttention(q,k,v), pinned host q/k/v (whole window) and output"},
        # per timed step: pool_project + score_select + attention, plus pool_project at each commit
        "gpu_launches": launches,
        "clocks": clk.summary(),
        "us_per_chunk_layer": r(1e3 * elapsed_ms / args.steps),
        "attention_us": r(1e3 * att_avg), "router_us": r(1e3 * statistics.mean(rt_ms)),
        "router": {"cached_us": r(route_cached_us), "commit_pool_us": r(commit_us), "full_us": r(route_full_us),
                   "fast_cached_us": r(route_fast_us), "fast_ids_equal": fast_equal},
        "roll": {"shift_us": r(hbm_k["cache_append_roll"]["us"]), "shift_mb": r(hbm_k["cache_append_roll"]["bytes"] / 1e6),
                 "ring_us": r(hbm_k["cache_append_ring_roll"]["us"]),
                 "ring_mb": r(hbm_k["cache_append_ring_roll"]["bytes"] / 1e6)},
        "effective_gflop": r(statistics.mean(flops) / 1e9), "router_gflop": r(router_flops / 1e9, 3),
        "e2e_streaming": {"value": r(streaming["value"]), "ms_per_step": r(streaming["ms_per_step"], 3),
                          "h2d_bytes_per_step": streaming["h2d_bytes_per_step"]},
        "rollout": None if rollout is None else {
            "frames_s": r(rollout["value"], 2), "dense_frames_s": r(rollout["dense_value"], 2),
            "streams": rollout["streams"],
            "config4_frames_s": None if rollout["config4_long_horizon"] is None else
            r(rollout["config4_long_horizon"]["value"], 2),
            "config4_ring_frames_s": None if rollout["config4_long_horizon"] is None else
            r(rollout["config4_long_horizon"]["ring_cache"]["value"], 2)},
        "int8_qk": None if int8 is None else {
            "attention_us": r(int8["attention_us"]), "quant_chunk_us": r(int8["quant_chunk_us"]),
            "tflops": r(int8["tflops"]), "frac": r(int8["frac_of_peak"], 3),
            "vs_bf16_nmse": int8["vs_bf16_nmse"]},
        "configs_frac": None if other is None else {o["short"]: [r(o["us"]), r(o["frac_of_peak"], 3)] for o in other},
        "sharded": None if sharded is None else {
            "c4_1gpu_us": r(sharded["single_gpu_us"]), "c4_1gpu_cached_us": r(sharded["single_gpu_cached_us"]),
            "kv": {"us": r(sharded["kv"]["us"]), "x": r(sharded["kv"]["speedup_vs_1gpu"], 2),
                   "write_chunk_us": r(sharded["kv"]["write_chunk_us"]), "ids_equal": sharded["kv"]["ids_equal"],
                   "max_abs": r(sharded["kv"]["max_abs"], 5), "nmse": sharded["kv"]["nmse"]},
            "kv_pull": {"us": r(sharded["kv_pull"]["us"]), "x": r(sharded["kv_pull"]["speedup_vs_1gpu"], 2),
                        "merge_share": r(sharded["kv_pull"]["merge_share"], 3),
                        "equals_push": sharded["kv_pull"]["equals_push"]},
            "heads": {"us": r(sharded["heads"]["us"]), "x": r(sharded["heads"]["speedup_vs_1gpu"], 2),
                      "bit_exact": sharded["heads"]["bit_exact"], "max_abs": r(sharded["heads"]["max_abs"], 5),
                      "nmse": sharded["heads"]["nmse"]},
            "heads_fused": {"us": r(sharded["heads_fused"]["us"]), "x": r(sharded["heads_fused"]["speedup_vs_1gpu"], 2),
                            "equals_all_gather": sharded["heads_fused"]["equals_all_gather"],
                            "max_abs": r(sharded["heads_fused"]["max_abs"], 5)},
            "c5_98280": {"1gpu_us": r(sharded["c5_98280"]["single_gpu_us"]),
                         "1gpu_cached_us": r(sharded["c5_98280"]["single_gpu_cached_us"]),
                         "kv_us": r(sharded["c5_98280"]["kv"]["us"]),
                         "kv_x": r(sharded["c5_98280"]["kv"]["speedup_vs_1gpu"], 2),
                         "kv_ids_equal": sharded["c5_98280"]["kv"]["ids_equal"],
                         "heads_fused_us": r(sharded["c5_98280"]["heads_fused"]["us"]),
                         "heads_fused_x": r(sharded["c5_98280"]["heads_fused"]["speedup_vs_1gpu"], 2)},
            "stream4_heads": sharded.get("stream4_heads") and {
                k_: (r(v_, 3) if isinstance(v_, float) else v_) for k_, v_ in sharded["stream4_heads"].items()}},
    }
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--ref-pairs", type=int, default=48)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-rollout", action="store_true", help="skip the config-3 rollout measurement")
    ap.add_argument("--no-int8", action="store_true", help="skip the INT8-QK path measurement")
    ap.add_argument("--no-configs", action="store_true", help="skip the per-shape measurements of configs 1, 4, 5")
    ap.add_argument("--no-sharded", action="store_true", help="skip the KV-block / head sharded config-4 chunk-layer")
    ap.add_argument("--only-hbm-kernels", action="store_true",
                    help="measure only the cache append / roll, LSE merge and anchor rebase kernels")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank)
        return
    import torch.distributed as dist
    if world > 1:
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    try:
        run_ours(args, rank, world, local_rank)
    finally:
        if world > 1:
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
