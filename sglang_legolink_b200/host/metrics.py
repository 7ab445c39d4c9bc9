"""Metric rows of agent turns and their aggregation.

One row per agent turn / request, appended to a JSONL file
(:class:`MetricsRecorder`), then aggregated to per-variant statistics
(:func:`aggregate_experiment`) with p50 / p95 by linear interpolation between
order statistics.  The row field names are the reference's metric schema
(``noc_context_manager/metrics.py:13-115``; aggregation
``experiment_metrics.py:44-211``; stream metrics ``inference_metrics.py:24-112``)
so that rows from either implementation aggregate together.

Rows of an original-server (non-LegoLink) variant carry no LegoLink fields:
normalisation blanks them so that a comparison never averages a cache ratio
that the baseline arm did not have.
"""

from __future__ import annotations

import json
import statistics
import threading
from collections import defaultdict
from dataclasses import asdict, dataclass, field
from pathlib import Path
from typing import Any, Iterable, Optional, Sequence

FORMAL_KINDS = frozenset({"formal_latency", "paired_replay", "official_agent", "wildclaw_long_running"})
BASELINE_VARIANTS = frozenset({"full_context_original_sglang", "selected_context_original_sglang",
                               "original_sglang"})
LEGOLINK_FIELDS = ("compiled_blocks", "compiled_tokens", "cache_hits", "cache_misses", "linked_tokens",
                   "reused_tokens", "recomputed_tokens", "cache_reuse_ratio", "recompute_ratio",
                   "average_reuse_count_per_block", "superseded_blocks", "invalidated_blocks", "evicted_blocks",
                   "evicted_tokens", "fallback_count", "recovery_success_count")


def percentile(values: Sequence[float], q: float) -> Optional[float]:
    """Linear interpolation between the two nearest order statistics
    (position ``q * (n - 1)``); None for no samples."""
    if not values:
        return None
    xs = sorted(float(v) for v in values)
    pos = q * (len(xs) - 1)
    lo = int(pos)
    hi = min(lo + 1, len(xs) - 1)
    return xs[lo] + (xs[hi] - xs[lo]) * (pos - lo)


def summary_stats(values: Iterable[Optional[float]]) -> dict:
    xs = [float(v) for v in values if v is not None]
    if not xs:
        return {"sample_count": 0, "mean": None, "std": None, "p50": None, "p95": None, "min": None, "max": None}
    return {"sample_count": len(xs), "mean": statistics.fmean(xs),
            "std": statistics.stdev(xs) if len(xs) > 1 else 0.0,
            "p50": percentile(xs, 0.5), "p95": percentile(xs, 0.95), "min": min(xs), "max": max(xs)}


@dataclass
class AgentMetric:
    """One agent turn.  Identity, context sizes, segmentation / selection,
    compile and reuse accounting, latencies, agent-loop counters, outcome."""

    task_id: str
    agent_id: str
    request_id: str
    session_revision: int
    loop_stage: str
    objective: str
    variant: str
    operation_mode: str
    measurement_kind: str = "formal_latency"
    # context sizes
    full_session_tokens: Optional[int] = None
    candidate_context_tokens: Optional[int] = None
    selected_context_tokens: Optional[int] = None
    mutable_tokens: Optional[int] = None
    context_reduction_tokens: Optional[int] = None
    context_reduction_ratio: Optional[float] = None
    selected_sub_context_count: Optional[int] = None
    excluded_sub_context_count: Optional[int] = None
    # segmentation / selection
    segmentation_model: Optional[str] = None
    segmentation_latency_ms: Optional[float] = None
    segment_count: Optional[int] = None
    validation_status: Optional[str] = None
    repair_count: Optional[int] = None
    segmentation_fallback_used: Optional[bool] = None
    selection_model: Optional[str] = None
    selection_latency_ms: Optional[float] = None
    token_budget: Optional[int] = None
    selected_ids: list = field(default_factory=list)
    excluded_ids: list = field(default_factory=list)
    # compile / reuse
    compile_decisions: list = field(default_factory=list)
    compile_requests: Optional[int] = None
    compiled_blocks: Optional[int] = None
    compiled_tokens: Optional[int] = None
    compile_latency_ms: Optional[float] = None
    duplicate_compile_avoided: Optional[int] = None
    requested_cache_keys: list = field(default_factory=list)
    cache_hits: Optional[int] = None
    cache_misses: Optional[int] = None
    stale_blocks: Optional[int] = None
    incompatible_blocks: Optional[int] = None
    reused_tokens: Optional[int] = None
    recomputed_tokens: Optional[int] = None
    cache_reuse_ratio: Optional[float] = None
    recompute_ratio: Optional[float] = None
    eviction_count: Optional[int] = None
    fallback_reason: Optional[str] = None
    # latencies
    lookup_latency_ms: Optional[float] = None
    link_plan_latency_ms: Optional[float] = None
    link_latency_ms: Optional[float] = None
    native_prefill_latency_ms: Optional[float] = None
    ttft_ms: Optional[float] = None
    decode_latency_ms: Optional[float] = None
    itl_ms: Optional[float] = None
    itl_p50_ms: Optional[float] = None
    itl_p95_ms: Optional[float] = None
    queue_wait_ms: Optional[float] = None
    request_latency_ms: Optional[float] = None
    prompt_tokens: Optional[int] = None
    output_tokens: Optional[int] = None
    output_tokens_per_second: Optional[float] = None
    # agent loop
    agent_steps: Optional[int] = None
    planner_calls: Optional[int] = None
    replanner_calls: Optional[int] = None
    llm_calls: Optional[int] = None
    tool_calls: Optional[int] = None
    successful_tool_calls: Optional[int] = None
    failed_tool_calls: Optional[int] = None
    repeated_action_count: Optional[int] = None
    invalid_tool_call_count: Optional[int] = None
    tool_execution_time_ms: Optional[float] = None
    total_llm_latency_ms: Optional[float] = None
    context_management_latency_ms: Optional[float] = None
    e2e_latency_ms: Optional[float] = None
    # outcome and residency
    task_success: Optional[bool] = None
    verifier_pass: Optional[bool] = None
    timeout: Optional[bool] = None
    error: Optional[str] = None
    unique_semantic_blocks: Optional[int] = None
    average_reuse_count_per_block: Optional[float] = None
    superseded_blocks: Optional[int] = None
    invalidated_blocks: Optional[int] = None
    evicted_blocks: Optional[int] = None
    evicted_tokens: Optional[int] = None
    fallback_count: Optional[int] = None
    recovery_success_count: Optional[int] = None
    concurrent_tasks: Optional[int] = None
    warmup: bool = False

    def finalize(self) -> "AgentMetric":
        if self.full_session_tokens is not None and self.selected_context_tokens is not None:
            self.context_reduction_tokens = self.full_session_tokens - self.selected_context_tokens
            self.context_reduction_ratio = (self.context_reduction_tokens / self.full_session_tokens
                                            if self.full_session_tokens else 0.0)
        if self.reused_tokens is not None and self.recomputed_tokens is not None:
            tot = self.reused_tokens + self.recomputed_tokens
            self.cache_reuse_ratio = self.reused_tokens / tot if tot else 0.0
            self.recompute_ratio = self.recomputed_tokens / tot if tot else 0.0
        return self

    def to_dict(self) -> dict:
        return asdict(self.finalize())


class MetricsRecorder:
    """Appends metric rows to a JSONL file (thread-safe, one row per line)."""

    def __init__(self, path):
        self.path = Path(path)
        self._lock = threading.Lock()

    def record(self, row) -> dict:
        d = row.to_dict() if isinstance(row, AgentMetric) else dict(row)
        line = json.dumps(d, ensure_ascii=False, separators=(",", ":"), default=str)
        with self._lock:
            self.path.parent.mkdir(parents=True, exist_ok=True)
            with self.path.open("a", encoding="utf-8") as f:
                f.write(line + "\n")
        return d

    def rows(self) -> list[dict]:
        return read_jsonl(self.path)


def read_jsonl(path) -> list[dict]:
    p = Path(path)
    if not p.exists():
        return []
    out = []
    for line in p.read_text(encoding="utf-8").splitlines():
        line = line.strip()
        if line:
            try:
                out.append(json.loads(line))
            except json.JSONDecodeError:
                continue  # a torn last line of a concurrent writer
    return out


def normalize_row(row: dict) -> dict:
    r = dict(row)
    r.setdefault("warmup", False)
    r.setdefault("formal_latency", r.get("measurement_kind") in FORMAL_KINDS)
    r.setdefault("diagnostic", not r["formal_latency"])
    if r.get("variant") in BASELINE_VARIANTS:
        for f in LEGOLINK_FIELDS:
            r[f] = None
    return r


def formal_rows(rows: Iterable[dict]) -> list[dict]:
    return [normalize_row(r) for r in rows
            if not r.get("warmup") and r.get("measurement_kind") in FORMAL_KINDS and not r.get("diagnostic")]


def _total(rows, name) -> int:
    return sum(int(r.get(name) or 0) for r in rows)


def aggregate_agent_steps(rows: Iterable[dict]) -> list[dict]:
    """Step rows -> one task row per (variant, task, trial, concurrency)."""
    groups = defaultdict(list)
    for r in map(normalize_row, rows):
        groups[(r.get("variant"), r.get("task_id"), r.get("trial_id"), r.get("concurrency") or 1)].append(r)
    out = []
    counters = ("planner_calls", "replanner_calls", "llm_calls", "tool_calls", "successful_tool_calls",
                "failed_tool_calls", "repeated_action_count", "invalid_tool_call_count")
    for key in sorted(groups, key=lambda k: tuple(map(str, k))):
        items = groups[key]
        row = {"metric_level": "task", "measurement_kind": "official_agent", "variant": key[0], "task_id": key[1],
               "trial_id": key[2], "concurrency": key[3], "agent_steps": len(items),
               "step_latency_ms": summary_stats(r.get("step_latency_ms") for r in items)}
        row.update({c: _total(items, c) for c in counters})
        out.append(normalize_row(row))
    return out


def aggregate_experiment(rows: Iterable[dict]) -> list[dict]:
    """Rows -> one row per (variant, kind, concurrency, phase, k) with latency
    statistics, throughput and reuse totals (warm-up rows dropped)."""
    groups = defaultdict(list)
    for r in map(normalize_row, rows):
        if r.get("warmup"):
            continue
        groups[(r.get("variant"), r.get("measurement_kind"), r.get("concurrency") or 1, r.get("phase"),
                r.get("k"))].append(r)
    out = []
    for key in sorted(groups, key=lambda k: tuple(map(str, k))):
        variant, kind, conc, phase, k = key
        items = groups[key]
        wall = sum(float(r.get("e2e_latency_ms") or 0.0) for r in items)
        done = sum(bool(r.get("task_success") or r.get("verifier_pass")) for r in items)
        base = variant in BASELINE_VARIANTS
        reused = None if base else _total(items, "reused_tokens")
        recomputed = None if base else _total(items, "recomputed_tokens")
        linked = None if base else reused + recomputed
        out.append(normalize_row({
            "metric_level": "experiment", "measurement_kind": kind, "variant": variant, "concurrency": conc,
            "phase": phase, "k": k, "sample_count": len(items),
            "request_latency_ms_stats": summary_stats(r.get("request_latency_ms") for r in items),
            "ttft_ms_stats": summary_stats(r.get("ttft_ms") for r in items),
            "e2e_latency_ms_stats": summary_stats(r.get("e2e_latency_ms") for r in items),
            "completed_tasks": done, "failed_tasks": len(items) - done,
            "verifier_pass_rate": done / len(items) if items else None,
            "steps_per_minute": 60_000.0 * _total(items, "agent_steps") / wall if wall else None,
            "tasks_per_hour": 3_600_000.0 * len(items) / wall if wall else None,
            "reused_tokens": reused, "recomputed_tokens": recomputed,
            "cache_reuse_ratio": reused / linked if linked else None,
            "recompute_ratio": recomputed / linked if linked else None,
        }))
    return out


def compute_stream_metrics(*, request_started_ns: int, token_ready_ns: Sequence[int], request_completed_ns: int,
                           prompt_tokens: Optional[int] = None, output_tokens: Optional[int] = None,
                           reused_tokens: Optional[int] = None, recomputed_tokens: Optional[int] = None,
                           **stage_ns: Optional[int]) -> dict:
    """TTFT, inter-token latency (mean, p50, p95), decode time and output
    tokens/s from monotonic per-token arrival timestamps; extra ``*_ns``
    keyword stage durations are passed through with their ``*_ms`` forms."""
    ts = list(token_ready_ns)
    if request_completed_ns < request_started_ns:
        raise ValueError("request completion precedes request start")
    if any(t < request_started_ns for t in ts):
        raise ValueError("token timestamp precedes request start")
    if ts != sorted(ts):
        raise ValueError("token timestamps must be monotonic")

    def ms(v):
        return None if v is None else float(v) / 1e6

    first = ts[0] if ts else None
    gaps = [b - a for a, b in zip(ts, ts[1:])]
    dur_s = (request_completed_ns - request_started_ns) / 1e9
    linked = (int(reused_tokens) + int(recomputed_tokens)
              if reused_tokens is not None and recomputed_tokens is not None else None)
    out = {
        "request_latency_ns": request_completed_ns - request_started_ns,
        "request_latency_ms": ms(request_completed_ns - request_started_ns),
        "ttft_ns": None if first is None else first - request_started_ns,
        "ttft_ms": None if first is None else ms(first - request_started_ns),
        "decode_ns": None if first is None else request_completed_ns - first,
        "decode_ms": None if first is None else ms(request_completed_ns - first),
        "itl_ms": ms(sum(gaps) / len(gaps)) if gaps else None,
        "itl_p50_ms": ms(percentile(gaps, 0.5)) if gaps else None,
        "itl_p95_ms": ms(percentile(gaps, 0.95)) if gaps else None,
        "output_tokens_per_second": (float(output_tokens) / dur_s
                                     if output_tokens is not None and dur_s > 0 else None),
        "prompt_tokens": prompt_tokens, "output_tokens": output_tokens, "linked_tokens": linked,
        "reused_tokens": reused_tokens, "recomputed_tokens": recomputed_tokens,
        "cache_reuse_ratio": (float(reused_tokens) / linked if linked else None),
    }
    for k, v in stage_ns.items():
        out[k] = v
        if k.endswith("_ns"):
            out[k[:-3] + "_ms"] = ms(v)
    return out
