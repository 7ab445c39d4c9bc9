"""Runtime observability: JSONL trace, host timing spans, CUDA-event timers.

* ``emit_trace(event, **details)`` appends one JSON record to
  ``$SGLANG_PIC_TRACE_PATH`` (one held O_APPEND descriptor per path; nothing
  is formatted -- and no device value is read -- when tracing is off).  Each
  record carries ``schema_version``, ``timestamp_unix_s``,
  ``timestamp_monotonic_s``, ``event``, ``pid`` and ``rank``; prompts and
  token contents are never written (reference ``pic_runtime.py:31-125,
  1652-1745``).  Long lists are truncated head/tail to
  ``$SGLANG_PIC_TRACE_MAX_ITEMS`` (default 32).
* :class:`HostTimer` -- nested perf-counter spans (``SGLANG_PIC_HOST_TIMING_ENABLED``).
* :class:`CudaTimer` -- pooled CUDA event pairs per named span, resolved with
  one synchronize at :meth:`CudaTimer.finalize` (``SGLANG_PIC_CUDA_EVENTS``).
"""

from __future__ import annotations

import json
import os
import threading
import time
from contextlib import contextmanager
from typing import Any, Optional

TRACE_SCHEMA_VERSION = 1
_fds: dict[str, int] = {}
_fd_lock = threading.Lock()


def trace_enabled() -> bool:
    return bool(os.getenv("SGLANG_PIC_TRACE_PATH"))


def _max_items() -> int:
    try:
        return max(2, int(os.getenv("SGLANG_PIC_TRACE_MAX_ITEMS", "32")))
    except ValueError:
        return 32


def _jsonable(v: Any, limit: int) -> Any:
    try:
        import torch

        if isinstance(v, torch.Tensor):
            v = v.detach().cpu().tolist()
    except Exception:  # pragma: no cover
        pass
    if callable(v):
        v = v()
    if isinstance(v, (list, tuple)):
        if len(v) > limit:
            h = limit // 2
            return {"count": len(v), "head": [_jsonable(x, limit) for x in v[:h]],
                    "tail": [_jsonable(x, limit) for x in v[-h:]]}
        return [_jsonable(x, limit) for x in v]
    if isinstance(v, dict):
        return {str(k): _jsonable(x, limit) for k, x in v.items()}
    if isinstance(v, (str, int, float, bool)) or v is None:
        return v
    return str(v)


def _fd(path: str) -> int:
    with _fd_lock:
        fd = _fds.get(path)
        if fd is None:
            os.makedirs(os.path.dirname(os.path.abspath(path)) or ".", exist_ok=True)
            fd = os.open(path, os.O_WRONLY | os.O_CREAT | os.O_APPEND, 0o644)
            _fds[path] = fd
        return fd


def emit_trace(event: str, **details: Any) -> bool:
    """Append one trace record; returns False (doing no work) when disabled.
    Values may be zero-argument callables, evaluated only when written."""
    path = os.getenv("SGLANG_PIC_TRACE_PATH")
    if not path:
        return False
    lim = _max_items()
    rec = {
        "schema_version": TRACE_SCHEMA_VERSION,
        "timestamp_unix_s": time.time(),
        "timestamp_monotonic_s": time.monotonic(),
        "event": event,
        "pid": os.getpid(),
        "rank": int(os.getenv("RANK", "0")),
    }
    for k, v in details.items():
        rec[k] = _jsonable(v, lim)
    os.write(_fd(path), (json.dumps(rec, separators=(",", ":")) + "\n").encode())
    return True


def close_traces() -> None:
    with _fd_lock:
        for fd in _fds.values():
            try:
                os.close(fd)
            except OSError:
                pass
        _fds.clear()


class HostTimer:
    def __init__(self, stage: str = "runtime", enabled: Optional[bool] = None):
        self.stage = stage
        self.enabled = (os.getenv("SGLANG_PIC_HOST_TIMING_ENABLED", "0") == "1") if enabled is None else enabled
        self.spans: dict[str, float] = {}

    @contextmanager
    def span(self, name: str):
        if not self.enabled:
            yield
            return
        t0 = time.perf_counter_ns()
        try:
            yield
        finally:
            self.add_ns(name, time.perf_counter_ns() - t0)

    def add_ns(self, name: str, ns: int) -> None:
        self.spans[name] = self.spans.get(name, 0.0) + ns / 1e6

    def record(self) -> dict:
        return {"stage": self.stage, "spans_ms": dict(self.spans)}


class CudaTimer:
    """Named spans timed with CUDA events on the current stream."""

    _pool: list = []

    def __init__(self, enabled: Optional[bool] = None):
        import torch

        if enabled is None:
            enabled = os.getenv("SGLANG_PIC_CUDA_EVENTS", "0") == "1"
        self.enabled = bool(enabled) and torch.cuda.is_available()
        self._open: list[tuple[str, Any, Any]] = []
        self.ms: dict[str, float] = {}

    def _pair(self):
        import torch

        if CudaTimer._pool:
            return CudaTimer._pool.pop()
        return torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)

    @contextmanager
    def span(self, name: str):
        if not self.enabled:
            yield
            return
        a, b = self._pair()
        a.record()
        try:
            yield
        finally:
            b.record()
            self._open.append((name, a, b))

    def finalize(self) -> dict[str, float]:
        if not self._open:
            return self.ms
        self._open[-1][2].synchronize()
        for name, a, b in self._open:
            self.ms[name] = self.ms.get(name, 0.0) + a.elapsed_time(b)
            CudaTimer._pool.append((a, b))
        self._open.clear()
        return self.ms
