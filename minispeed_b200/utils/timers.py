"""Named timers.

:class:`Timers` keeps the reference's wall-clock API (``engine.timers``,
reference ``minispeed/utils.py:14-60``): ``timers("name")``,
``with timers.timer("name")``, ``names()``, ``reset()`` and a rank-0
``log()`` string ``"name: 0.123s | ..."``.  Like the reference it does not
synchronize the GPU, so on CUDA it measures host time.

:class:`DeviceTimers` measures the same kind of named sections on the GPU
with CUDA events recorded on the current stream; ``elapsed_ms()`` syncs
once and sums every completed interval.  ``max_over_ranks`` reduces a value
with MAX across the process group, which is how multi-GPU times are
reported.

With ``MINISPEED_NVTX=1`` every named section is also an NVTX range
(``torch.cuda.nvtx``), so the engine's gather / backward / step / reduce
phases show up in a timeline profiler.
"""

from __future__ import annotations

import os
import time
from contextlib import contextmanager
from typing import Dict, Iterator, List

import torch

_NVTX = os.environ.get("MINISPEED_NVTX", "0") == "1"


class Timer:
    def __init__(self, name: str):
        self.name = name
        self.elapsed = 0.0
        self.started_at = None

    @contextmanager
    def section(self) -> Iterator[None]:
        t0 = time.perf_counter()
        try:
            yield
        finally:
            self.elapsed += time.perf_counter() - t0

    def start(self) -> None:
        self.started_at = time.perf_counter()

    def stop(self) -> None:
        if self.started_at is not None:
            self.elapsed += time.perf_counter() - self.started_at
            self.started_at = None

    def reset(self) -> None:
        self.elapsed = 0.0


class Timers:
    def __init__(self) -> None:
        self._timers: Dict[str, Timer] = {}

    def __call__(self, name: str) -> Timer:
        t = self._timers.get(name)
        if t is None:
            t = self._timers[name] = Timer(name)
        return t

    @contextmanager
    def timer(self, name: str) -> Iterator[None]:
        nvtx = _NVTX and torch.cuda.is_available()
        if nvtx:
            torch.cuda.nvtx.range_push(name)
        try:
            with self(name).section():
                yield
        finally:
            if nvtx:
                torch.cuda.nvtx.range_pop()

    def names(self) -> List[str]:
        return list(self._timers)

    def reset(self) -> None:
        for t in self._timers.values():
            t.reset()

    def log(self, rank0_only: bool = True) -> str:
        from .. import comm

        if rank0_only and comm.get_rank() != 0:
            return ""
        return " | ".join(f"{n}: {t.elapsed:.3f}s" for n, t in self._timers.items())


class DeviceTimers:
    """CUDA-event section timers (no-ops on CPU).

    Once more than ``fold_after`` intervals of a section are pending, the
    oldest ones whose end event has completed are folded into the totals
    (events recorded on one stream complete in order, so the scan stops at
    the first that has not).  If the GPU is so far behind that more than
    ``2 * fold_after`` stay pending, the oldest half is waited for: a long
    run that never reads the timers holds a bounded number of events."""

    def __init__(self, fold_after: int = 256) -> None:
        self._pending: Dict[str, list] = {}
        self._done: Dict[str, float] = {}
        self._fold_after = fold_after

    def _fold_completed(self, name: str) -> None:
        pend = self._pending.get(name, [])
        if len(pend) > 2 * self._fold_after:
            pend[len(pend) // 2][1].synchronize()
        n = 0
        total = self._done.get(name, 0.0)
        for a, b in pend:
            if not b.query():
                break
            total += a.elapsed_time(b)
            n += 1
        self._done[name] = total
        del pend[:n]

    @contextmanager
    def timer(self, name: str) -> Iterator[None]:
        if not torch.cuda.is_available() or torch.cuda.is_current_stream_capturing():
            # inside a CUDA-graph capture the replay is timed as a whole
            yield
            return
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record()
        try:
            yield
        finally:
            b.record()
            pend = self._pending.setdefault(name, [])
            pend.append((a, b))
            if len(pend) > self._fold_after:
                self._fold_completed(name)

    def elapsed_ms(self) -> Dict[str, float]:
        if self._pending:
            torch.cuda.synchronize()
        for name, pairs in self._pending.items():
            self._done[name] = self._done.get(name, 0.0) + sum(a.elapsed_time(b) for a, b in pairs)
        self._pending.clear()
        return dict(self._done)

    def reset(self) -> None:
        self._pending.clear()
        self._done.clear()


def max_over_ranks(value: float) -> float:
    """The largest ``value`` over the process group (device times are reported
    as the slowest rank's)."""
    from .. import comm

    if not comm.is_distributed():
        return float(value)
    dev = torch.device("cuda", torch.cuda.current_device()) if (
        torch.cuda.is_available() and torch.distributed.get_backend() == "nccl") else "cpu"
    t = torch.tensor([float(value)], dtype=torch.float64, device=dev)
    comm.all_reduce(t, op="max")
    return float(t.item())


def set_seed(seed: int) -> None:
    torch.manual_seed(seed)
    if torch.cuda.is_available():
        torch.cuda.manual_seed_all(seed)
