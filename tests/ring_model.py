"""A numpy model of the ring-buffer KV cache (test infrastructure): what ss_cache_append_ring
writes, row for row, and where a window row is read from. Checked against the oracle's
shift-left cache (tests/test_ring_model.py) and used as the expected physical rows of the GPU
cache (tests/test_gpu_ring.py)."""
import numpy as np


class RingModel:
    def __init__(self, cap: int, H: int, sink: int, D: int = 128):
        self.cap, self.S = cap, sink
        self.C = cap - sink + 64
        self.k = np.zeros((sink + self.C + 64, H, D), np.float32)
        self.v = np.zeros_like(self.k)
        self.head = 0
        self.written = 0          # physical rows written by the last append

    def sub_row(self, t0: int) -> int:
        """Physical row of the 64-row sub-block starting at window row t0."""
        if t0 + 64 <= self.S:
            return t0
        return self.S + (t0 - self.S + self.head) % self.C

    def row(self, t: int) -> int:
        return t if t < self.S else self.S + (t - self.S + self.head) % self.C

    def _ring_write(self, k, v, pos0: int):
        for i in range(k.shape[0]):
            p = (pos0 + i) % self.C
            self.k[self.S + p], self.v[self.S + p] = k[i], v[i]
            self.written += 1
            if p < 64:
                self.k[self.S + self.C + p], self.v[self.S + self.C + p] = k[i], v[i]
                self.written += 1

    def append(self, k_new, v_new, *, local_attn: bool, global_end: int, local_end: int, current_start: int):
        """The index arithmetic of the oracle's cache_append; returns the new local end."""
        n = k_new.shape[0]
        end = current_start + n
        self.written = 0
        if local_attn and end > global_end and n + local_end > self.cap:
            evicted = n + local_end - self.cap
            assert local_end - evicted - self.S >= 0
            self.head = (self.head + evicted) % self.C
            new_end = local_end + end - global_end - evicted
        else:
            new_end = local_end + end - global_end
        start = new_end - n
        ns = max(0, min(self.S, new_end) - start)
        self.k[start:start + ns], self.v[start:start + ns] = k_new[:ns], v_new[:ns]
        self.written += ns
        if n > ns:
            t0 = start + ns
            self._ring_write(k_new[ns:], v_new[ns:], (t0 - self.S + self.head) % self.C)
        a = self.S % 64
        if a:
            self._ring_write(self.k[self.S - a:self.S].copy(), self.v[self.S - a:self.S].copy(),
                             (self.head - a) % self.C)
        return new_end

    def window(self, Lk: int):
        """The window's rows in order, read 64-row sub-block by sub-block from their physical start
        (as the kernels read them)."""
        rows = []
        for t0 in range(0, Lk, 64):
            p = self.sub_row(t0)
            rows.append(np.arange(p, p + min(64, Lk - t0)))
        idx = np.concatenate(rows) if rows else np.zeros(0, np.int64)
        return self.k[idx], self.v[idx]
