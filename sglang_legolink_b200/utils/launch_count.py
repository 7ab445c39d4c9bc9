"""Counts this package's own kernel launches (eager calls + CUDA-graph
replays), for the benchmark's ``gpu_launches`` field."""

from __future__ import annotations

import threading

_lock = threading.Lock()
_count = [0]
_active = [False]


def add(n: int) -> None:
    if _active[0]:
        with _lock:
            _count[0] += n


def raw() -> int:
    return _count[0]


class LaunchCounter:
    def start(self) -> None:
        with _lock:
            _count[0] = 0
            _active[0] = True

    def stop(self) -> int:
        with _lock:
            _active[0] = False
            return _count[0]


class Recorder:
    """Counts launches while capturing a CUDA graph, regardless of whether a
    LaunchCounter is active, so replays can be credited later."""

    def __init__(self):
        self.n = 0

    def __enter__(self):
        self._prev = _active[0]
        with _lock:
            self._base = _count[0]
            _active[0] = True
        return self

    def __exit__(self, *a):
        with _lock:
            self.n = _count[0] - self._base
            _count[0] = self._base
            _active[0] = self._prev
