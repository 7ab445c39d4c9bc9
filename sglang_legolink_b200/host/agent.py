"""Agent-side wrappers of the host pipeline.

* :class:`AgentLLM` -- one agent turn: OpenAI messages (+ tools) -> session
  events -> :meth:`RequestPipeline.execute` -> the completion text, and one
  :class:`~.metrics.AgentMetric` row (reuse accounting, compile requests,
  residency recovery, latencies) appended to the metrics JSONL.  The
  reference's agent LLM does the same per turn
  (``terminal_bench_integration/noc_sglang_agent.py:540-1033``).
* :class:`ReplayDriver` -- scripted turns (recorded messages or raw event
  tuples) through an :class:`AgentLLM`, for examples and regression runs
  (reference ``terminal_bench_integration/replay.py:71``).

Only the newest messages of each turn are new events: the session's event
collector deduplicates by source id and content digest, so a client that
resends the whole conversation every turn still produces one revision per
changed source.
"""

from __future__ import annotations

import time
import uuid
from dataclasses import dataclass, field
from typing import Callable, Iterable, Optional, Sequence

from .adapter import PipelineExecution, PipelineRoute, RequestPipeline
from .ingress import SourceLedger, openai_request_events
from .metrics import AgentMetric, MetricsRecorder


@dataclass
class TurnResult:
    text: str
    execution: PipelineExecution
    metric: dict


class AgentLLM:
    def __init__(self, pipeline: RequestPipeline, *, task_id: str, agent_id: str = "agent",
                 variant: str = "selected_context_radixcache_legolink", recorder: Optional[MetricsRecorder] = None,
                 route: PipelineRoute = PipelineRoute.SELECTED_CONTEXT_LEGOLINK,
                 measurement_kind: str = "formal_latency"):
        self.pipeline = pipeline
        self.task_id = task_id
        self.agent_id = agent_id
        self.variant = variant
        self.recorder = recorder
        self.route = route
        self.measurement_kind = measurement_kind
        self.turns = 0

    def call(self, messages: Sequence[dict], tools: Optional[list] = None, *, objective: str = "",
             loop_stage: str = "act", events: Optional[list] = None, warmup: bool = False) -> TurnResult:
        self.turns += 1
        if events is None:
            # what this call adds to the session: sources it already holds with
            # the same text are skipped, an earlier request becomes history
            held = self.pipeline.manager.collector.events()
            events = openai_request_events(list(messages), tools=tools, ledger=SourceLedger.from_events(held),
                                           first_turn=not held)
        evs = list(events)
        query = objective or next((m.get("content") or "" for m in reversed(list(messages))
                                   if m.get("role") == "user" and isinstance(m.get("content"), str)), "")
        t0 = time.perf_counter()
        error = None
        try:
            ex = self.pipeline.execute(evs, route=self.route, query=query, tools=tools)
        except Exception as e:  # a failed turn still leaves a row
            error = f"{type(e).__name__}: {e}"
            ex = None
        e2e_ms = (time.perf_counter() - t0) * 1e3
        row = self._metric(ex, e2e_ms, objective or query, loop_stage, error, warmup)
        d = self.recorder.record(row) if self.recorder is not None else row.to_dict()
        if ex is None:
            raise RuntimeError(error)
        return TurnResult(ex.result.text, ex, d)

    def _metric(self, ex: Optional[PipelineExecution], e2e_ms: float, objective: str, loop_stage: str,
                error: Optional[str], warmup: bool) -> AgentMetric:
        m = AgentMetric(task_id=self.task_id, agent_id=self.agent_id, request_id=uuid.uuid4().hex[:16],
                        session_revision=int(self.pipeline.manager.collector.revision),
                        loop_stage=loop_stage, objective=objective[:200], variant=self.variant,
                        operation_mode=self.route.value, measurement_kind=self.measurement_kind, warmup=warmup,
                        e2e_latency_ms=e2e_ms, agent_steps=1, llm_calls=1, error=error)
        if ex is None:
            return m
        m.request_latency_ms = ex.result.latency_s * 1e3
        m.compile_requests = ex.compile_requests
        m.compile_latency_ms = ex.compile_latency_s * 1e3
        m.context_management_latency_ms = sum(v for k, v in ex.timings_ms.items() if k in ("ingest", "plan", "frame"))
        m.link_latency_ms = ex.timings_ms.get("link")
        rec = ex.result.recovery or {}
        recovered = list(rec.get("recovered_cache_keys") or [])
        m.fallback_count = 1 if rec.get("outcome", "not_needed") != "not_needed" else 0
        m.recovery_success_count = len(recovered)
        if ex.plan is not None:
            d = ex.plan.to_dict()
            acc = d.get("reuse_accounting") or {}
            m.reused_tokens = acc.get("reused_tokens")
            m.recomputed_tokens = (acc.get("recompute_tokens") or 0) + (acc.get("repair_tokens") or 0)
            m.selected_context_tokens = acc.get("total_tokens")
            m.selected_ids = list(d.get("manifest", {}).get("selected_sub_context_ids", []))
            m.selected_sub_context_count = len(m.selected_ids)
            m.compiled_blocks = len(ex.plan.compile_on_miss_contexts)
            m.requested_cache_keys = [r.cache_key for r in ex.plan.records] if ex.plan.records else []
        usage = (ex.result.response or {}).get("usage") or {}
        m.prompt_tokens = usage.get("prompt_tokens")
        m.output_tokens = usage.get("completion_tokens")
        return m


@dataclass
class ReplayDriver:
    """Runs scripted turns.  A turn is either a list of OpenAI messages
    (``{"messages": [...], "tools": [...]}``) or a list of raw event tuples
    (``{"events": [...]}``)."""

    agent: AgentLLM
    objective: str = ""
    results: list = field(default_factory=list)

    def run(self, turns: Iterable[dict], on_turn: Optional[Callable[[int, TurnResult], None]] = None) -> list:
        for i, turn in enumerate(turns):
            res = self.agent.call(turn.get("messages") or [], turn.get("tools"), objective=self.objective,
                                  events=turn.get("events"), loop_stage=turn.get("loop_stage", "act"),
                                  warmup=bool(turn.get("warmup")))
            self.results.append(res)
            if on_turn is not None:
                on_turn(i, res)
        return self.results
