"""Host-side profiling of the control plane.

* :class:`HostTimingRecorder` -- nested ``perf_counter_ns`` spans of one
  pipeline stage, emitted as one JSONL row (``NOC_HOST_TIMING_ENABLED=1``,
  ``NOC_HOST_TIMING_PATH``).  Rows carry a wall-clock anchor so they can be
  placed on the same time axis as the runtime's trace rows.
* :func:`profile_range` -- a ``torch.profiler.record_function`` region
  (``NOC_PROFILE_RANGES_ENABLED=1``) and/or an NVTX range with bounded
  request metadata in its name (``NOC_NVTX_ENABLED=1``).
* :class:`ProfilerWindowConfig` -- a validated wait / warmup / active
  schedule for ``torch.profiler`` windows.
* :class:`NcuRunConfig` -- the Nsight Compute command for one kernel of a
  small case, with the flags this deployment requires (clock control off,
  one kernel, few launches).

Reference: ``noc_context_manager/profiling.py:25-250`` (the environment flag
names and the row's ``measurement_kind`` are kept so that rows from either
implementation are read the same way).
"""

from __future__ import annotations

import contextlib
import json
import os
import threading
import time
from dataclasses import asdict, dataclass
from pathlib import Path
from typing import Any, Iterator, Optional

SCHEMA_VERSION = 1
_BOUNDED_KEYS = ("request_id", "task_id", "variant", "phase", "concurrency", "k", "decode_iteration")
_lock = threading.Lock()


def _flag(name: str) -> bool:
    return os.getenv(name, "0").lower() in {"1", "true", "yes", "on"}


def bounded_metadata(meta: Optional[dict]) -> dict:
    """Only a fixed set of small identity fields travels with a range or row."""
    if not meta:
        return {}
    return {k: meta[k] for k in _BOUNDED_KEYS if meta.get(k) is not None}


def nvtx_range_name(name: str, meta: Optional[dict] = None) -> str:
    m = bounded_metadata(meta)
    return name if not m else name + "[" + ",".join(f"{k}={v}" for k, v in m.items()) + "]"


@contextlib.contextmanager
def profile_range(name: str, *, metadata: Optional[dict] = None) -> Iterator[None]:
    rec, nvtx = _flag("NOC_PROFILE_RANGES_ENABLED"), _flag("NOC_NVTX_ENABLED")
    if not (rec or nvtx):
        yield
        return
    try:
        import torch
    except (ImportError, OSError):
        torch = None
    ctx = torch.profiler.record_function(name) if (rec and torch is not None) else contextlib.nullcontext()
    use_nvtx = bool(nvtx and torch is not None and torch.cuda.is_available())
    with ctx:
        if use_nvtx:
            torch.cuda.nvtx.range_push(nvtx_range_name(name, metadata))
        try:
            yield
        finally:
            if use_nvtx:
                torch.cuda.nvtx.range_pop()


def append_jsonl(path, row: dict) -> None:
    p = Path(path)
    with _lock:
        p.parent.mkdir(parents=True, exist_ok=True)
        with p.open("a", encoding="utf-8") as f:
            f.write(json.dumps(row, ensure_ascii=False, separators=(",", ":"), default=str) + "\n")


class HostTimingRecorder:
    def __init__(self, stage: str, *, metadata: Optional[dict] = None, output_path=None, enabled=None):
        self.enabled = _flag("NOC_HOST_TIMING_ENABLED") if enabled is None else bool(enabled)
        self.stage = stage
        self.metadata = bounded_metadata(metadata)
        path = output_path or os.getenv("NOC_HOST_TIMING_PATH")
        self.output_path = Path(path) if path else None
        self.t0 = time.perf_counter_ns() if self.enabled else 0
        self.t0_unix = time.time_ns() if self.enabled else 0
        self.spans: list[dict] = []
        self._depth = 0
        self._done = False

    @contextlib.contextmanager
    def span(self, name: str) -> Iterator[None]:
        if not self.enabled:
            yield
            return
        start, depth = time.perf_counter_ns(), self._depth
        self._depth += 1
        try:
            yield
        finally:
            self._depth -= 1
            end = time.perf_counter_ns()
            self.spans.append({"name": name, "depth": depth, "started_ns": start, "ended_ns": end,
                               "elapsed_ns": max(0, end - start)})

    def emit(self, *, status: str = "ok", error: Optional[str] = None) -> dict:
        if not self.enabled or self._done:
            return {}
        self._done = True
        end = time.perf_counter_ns()
        row = {"schema_version": SCHEMA_VERSION, "metric_level": "request",
               "measurement_kind": "diagnostic_host_timing", "profiling_type": "host_timing",
               "formal_latency": False, "diagnostic": True, "event": "noc_host_timing", "stage": self.stage,
               "status": status, "started_ns": self.t0, "started_unix_ns": self.t0_unix, "ended_ns": end,
               "wall_elapsed_ns": max(0, end - self.t0), "spans": list(self.spans), **self.metadata}
        if error:
            row["error"] = error
        if self.output_path is not None:
            append_jsonl(self.output_path, row)
        return row

    def span_totals_ms(self) -> dict:
        out: dict = {}
        for s in self.spans:
            out[s["name"]] = out.get(s["name"], 0.0) + s["elapsed_ns"] / 1e6
        return out


@dataclass(frozen=True)
class ProfilerWindowConfig:
    wait: int = 1
    warmup: int = 2
    active: int = 5
    repeat: int = 1
    record_shapes: bool = False
    profile_memory: bool = False
    with_stack: bool = False

    def __post_init__(self):
        if min(self.wait, self.warmup, self.active, self.repeat) < 0:
            raise ValueError("profiler schedule values cannot be negative")
        if self.active < 1 or self.repeat < 1:
            raise ValueError("profiler active and repeat must be at least one")

    @property
    def total_steps(self) -> int:
        return (self.wait + self.warmup + self.active) * self.repeat

    def schedule(self):
        import torch

        return torch.profiler.schedule(wait=self.wait, warmup=self.warmup, active=self.active, repeat=self.repeat)

    def to_dict(self) -> dict:
        return asdict(self)


@dataclass(frozen=True)
class NcuRunConfig:
    """One kernel of a small case under Nsight Compute.  Clock control is
    always off (the GPU's clocks are left as found) and the capture is bounded
    to ``launch_count`` launches of kernels matching ``kernel_regex``."""

    output: str
    command: tuple
    kernel_regex: str
    launch_skip: int = 0
    launch_count: int = 1
    section_set: str = "full"

    def __post_init__(self):
        if not (1 <= self.launch_count <= 3):
            raise ValueError("capture 1 to 3 launches of one kernel")

    def ncu_command(self) -> list[str]:
        return ["ncu", "--set", self.section_set, "--clock-control", "none", "-k", f"regex:{self.kernel_regex}",
                "-s", str(self.launch_skip), "-c", str(self.launch_count), "-o", self.output, *self.command]

    def manifest(self, *, role: str) -> dict[str, Any]:
        return {"schema_version": SCHEMA_VERSION, "metric_level": "ncu_run",
                "measurement_kind": "diagnostic_nsight_compute", "profiling_type": "nsight_compute",
                "formal_latency": False, "diagnostic": True, "role": role, "output": self.output,
                "command": self.ncu_command()}
