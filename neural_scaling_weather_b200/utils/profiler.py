"""NVTX ranges and CUDA-profiler windows, plus device-side phase timers.

Reference behaviour (``utils/profiler_utils.py:9-96``): a global profiler, enabled by
``profiler.enabled`` for the ranks in ``profiler.profile_ranks``, pushes NVTX ranges
through ``@profile(name)`` / ``profile_range(name)`` and brackets ``profile_epoch`` with
``cudaProfilerStart/Stop`` (for ``nsys -c cudaProfilerApi``).  Range names are kept
identical so timelines of the two frameworks line up.

Added here: :class:`DeviceTimer`, CUDA-event timing of named phases without host syncs
inside the step (events are read once, at the end).
"""

from __future__ import annotations

import functools
from contextlib import contextmanager
from typing import Dict, List, Optional

import torch


def _world_rank() -> int:
    import torch.distributed as dist

    return dist.get_rank() if dist.is_initialized() else 0


class Profiler:
    def __init__(self, cfg):
        prof = cfg.profiler
        self.enabled = bool(prof.enabled)
        self.profile_ranks = list(prof.profile_ranks)
        self.profile_epoch = int(prof.profile_epoch)
        self.current_rank = _world_rank()
        self.current_epoch = 0
        self.is_profiling = False

    def should_profile(self) -> bool:
        return self.enabled and self.current_rank in self.profile_ranks

    def should_start_cuda_profiler(self) -> bool:
        return self.should_profile() and self.current_epoch == self.profile_epoch

    def set_epoch(self, epoch: int) -> None:
        if self.is_profiling:
            torch.cuda.profiler.stop()
            self.is_profiling = False
        self.current_epoch = epoch
        if self.should_start_cuda_profiler() and torch.cuda.is_available():
            torch.cuda.profiler.start()
            self.is_profiling = True

    @contextmanager
    def profile_range(self, name: str):
        if not self.should_profile() or not torch.cuda.is_available():
            yield
            return
        torch.cuda.nvtx.range_push(name)
        try:
            yield
        finally:
            torch.cuda.nvtx.range_pop()


class NoOpProfiler:
    enabled = False

    def should_profile(self) -> bool:
        return False

    def set_epoch(self, _epoch) -> None:
        pass

    @contextmanager
    def profile_range(self, _name):
        yield


_profiler: Optional[Profiler] = None


def init_profiler(cfg) -> Profiler:
    global _profiler
    _profiler = Profiler(cfg)
    return _profiler


def get_profiler():
    return _profiler if _profiler is not None else NoOpProfiler()


def profile(name: Optional[str] = None):
    def deco(fn):
        @functools.wraps(fn)
        def wrapper(*args, **kwargs):
            with get_profiler().profile_range(name or fn.__name__):
                return fn(*args, **kwargs)

        return wrapper

    return deco


@contextmanager
def profile_range(name: str):
    with get_profiler().profile_range(name):
        yield


class DeviceTimer:
    """Accumulates CUDA-event durations of named phases; read with :meth:`summary`."""

    def __init__(self, enabled: bool = True):
        self.enabled = enabled and torch.cuda.is_available()
        self._events: Dict[str, List] = {}

    @contextmanager
    def phase(self, name: str):
        if not self.enabled:
            yield
            return
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        start.record()
        try:
            yield
        finally:
            end.record()
            self._events.setdefault(name, []).append((start, end))

    def summary(self) -> Dict[str, float]:
        """Total milliseconds per phase (synchronises once)."""
        if not self.enabled:
            return {}
        torch.cuda.synchronize()
        out = {k: sum(s.elapsed_time(e) for s, e in v) for k, v in self._events.items()}
        self._events.clear()
        return out
