"""Progress timer with named scopes, windowed averages and ETA
(reference: mvp_engine/utils/log/timer.py:8-168).

Host clock only; device-side step timing lives in :class:`CudaStepTimer`,
which brackets a step with CUDA events and reports the max over ranks.
"""

from __future__ import annotations

import time
from collections import defaultdict, deque
from contextlib import contextmanager
from typing import Iterator, Optional

import torch
import torch.distributed as dist


def format_time(seconds: float) -> str:
    seconds = max(0, int(seconds))
    d, rem = divmod(seconds, 86400)
    h, rem = divmod(rem, 3600)
    m, s = divmod(rem, 60)
    return f"{d}d {h:02d}:{m:02d}:{s:02d}" if d else f"{h:02d}:{m:02d}:{s:02d}"


class Timer:
    def __init__(self, total_progress: Optional[float] = None, window_size: int = 100) -> None:
        self.total_progress = total_progress
        self.window_size = int(window_size)
        self.reset()

    def reset(self) -> "Timer":
        self._start = None
        self._last_tick = None
        self.progress = 0.0
        self._start_progress = 0.0
        self._tick_times: deque = deque(maxlen=self.window_size)
        self._scopes: dict = defaultdict(lambda: deque(maxlen=self.window_size))
        self._open: dict = {}
        return self

    def start(self) -> "Timer":
        now = time.perf_counter()
        self._start = now
        self._last_tick = now
        self._start_progress = self.progress
        return self

    def set_progress(self, current_progress: float, total_progress: Optional[float] = None) -> None:
        self.progress = float(current_progress)
        self._start_progress = self.progress
        if total_progress is not None:
            self.total_progress = total_progress

    def tick(self, progress_increment: float = 1.0) -> float:
        now = time.perf_counter()
        if self._start is None:
            self.start()
            return 0.0
        elapsed = now - self._last_tick
        self._last_tick = now
        self.progress += progress_increment
        self._tick_times.append(elapsed / max(progress_increment, 1e-12))
        return elapsed

    def start_scope(self, scope: str) -> None:
        self._open[scope] = time.perf_counter()

    def end_scope(self, scope: str) -> float:
        t0 = self._open.pop(scope, None)
        if t0 is None:
            return 0.0
        elapsed = time.perf_counter() - t0
        self._scopes[scope].append(elapsed)
        return elapsed

    @contextmanager
    def scope(self, scope: str) -> Iterator[None]:
        self.start_scope(scope)
        try:
            yield
        finally:
            self.end_scope(scope)

    def record_scope(self, scope: str, elapsed: float) -> None:
        self._scopes[scope].append(float(elapsed))

    @property
    def total_elapsed(self) -> float:
        return 0.0 if self._start is None else time.perf_counter() - self._start

    @property
    def remaining_progress(self) -> float:
        if self.total_progress is None:
            return 0.0
        return max(0.0, float(self.total_progress) - self.progress)

    @property
    def progress_time(self) -> float:
        return sum(self._tick_times) / len(self._tick_times) if self._tick_times else 0.0

    @property
    def progress_time_latest(self) -> float:
        return self._tick_times[-1] if self._tick_times else 0.0

    @property
    def eta(self) -> float:
        return self.progress_time * self.remaining_progress

    @property
    def eta_string(self) -> str:
        return format_time(self.eta)

    @property
    def elapsed_string(self) -> str:
        return format_time(self.total_elapsed)

    def get_scope_time(self, scope: str) -> float:
        vals = self._scopes.get(scope)
        return sum(vals) / len(vals) if vals else 0.0

    def get_scope_time_latest(self, scope: str) -> float:
        vals = self._scopes.get(scope)
        return vals[-1] if vals else 0.0

    def get_stats(self) -> dict:
        return {
            "elapsed": self.total_elapsed,
            "progress": self.progress,
            "progress_time": self.progress_time,
            "eta": self.eta,
            "scopes": {k: self.get_scope_time(k) for k in self._scopes},
        }


class CudaStepTimer:
    """Device-side step time: CUDA events on the current stream around a step.

    ``stop()`` synchronises and returns milliseconds; ``max_over_ranks`` reduces
    a duration with MAX over the default group, which is how every multi-GPU
    step time in this engine is reported.
    """

    def __init__(self) -> None:
        self._s = None
        self._e = None

    def start(self) -> None:
        if torch.cuda.is_available():
            self._s = torch.cuda.Event(enable_timing=True)
            self._e = torch.cuda.Event(enable_timing=True)
            self._s.record()
        else:
            self._t0 = time.perf_counter()

    def stop(self) -> float:
        if self._s is not None:
            self._e.record()
            self._e.synchronize()
            return float(self._s.elapsed_time(self._e))
        return (time.perf_counter() - self._t0) * 1e3

    @staticmethod
    def max_over_ranks(ms: float, device: Optional[torch.device] = None) -> float:
        if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
            return ms
        dev = device or (torch.device("cuda", torch.cuda.current_device()) if torch.cuda.is_available()
                         else torch.device("cpu"))
        t = torch.tensor([ms], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())
