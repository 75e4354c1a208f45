"""Device timing helpers (CUDA events on the launching stream)."""
from __future__ import annotations

from typing import List

import torch


class StepTimer:
    """Records a (start, end) CUDA-event pair around every engine step's device work
    (first H2D copy to the D2H read of the sampled ids); ``total_ms`` sums them, which
    excludes the host-side scheduling gaps between steps."""

    def __init__(self):
        self.pairs: List[tuple] = []
        self._cur = None

    def begin(self) -> None:
        ev = torch.cuda.Event(enable_timing=True)
        ev.record()
        self._cur = ev

    def end(self) -> None:
        ev = torch.cuda.Event(enable_timing=True)
        ev.record()
        self.pairs.append((self._cur, ev))
        self._cur = None

    def reset(self) -> None:
        self.pairs = []

    def total_ms(self) -> float:
        torch.cuda.synchronize()
        return sum(a.elapsed_time(b) for a, b in self.pairs)


def time_cuda(fn, iters: int = 10, warmup: int = 3, flush_bytes: int = 0) -> float:
    """Median ms of ``fn()`` over ``iters`` runs, CUDA events, optional L2 flush between runs."""
    flush = torch.empty(flush_bytes // 4, dtype=torch.float32, device="cuda") if flush_bytes else None
    for _ in range(warmup):
        fn()
    times = []
    for _ in range(iters):
        if flush is not None:
            flush.zero_()
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        b.synchronize()
        times.append(a.elapsed_time(b))
    times.sort()
    return times[len(times) // 2]
