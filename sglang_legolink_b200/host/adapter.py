"""Runtime adapter, transports, single-flight residency recovery and the
request pipeline (host stages 9-10).

* Transports: :class:`JSONHTTPTransport` (non-streamed chat, latency) and
  :func:`post_chat_stream` (SSE; TTFT taken at the first non-empty content
  delta; an SSE ``error`` frame raises :class:`ChatStreamError`).  Any
  callable ``payload -> response dict`` (e.g. an in-process runtime) works.
* :class:`ResidencyRecoveryCoordinator` -- per (runtime, cache key) flights:
  the first request to see a key gone becomes the *owner* and recompiles it;
  concurrent requests become *waiters*; a request that observed the abort
  before a later successful recovery is *settled*; waits are bounded
  (default 300 s) and an owner always completes its flight in ``finally``.
* :class:`RuntimeAdapter` -- Compile (``max_tokens=1``, ``extra_key``,
  ``sub_context``), Link (``pic_link``), the native baselines, failure
  classification and the Link retry loop with recovery.
* :class:`RequestPipeline` -- one agent turn: ingest -> select -> plan ->
  stitch -> frame -> Compile-on-miss -> Link (route C), or the native routes
  A (full context) / B (selected context).
"""

from __future__ import annotations

import json
import threading
import time
import urllib.error
import urllib.request
from dataclasses import dataclass, field
from enum import Enum
from typing import Any, Callable, Hashable, Optional

from ..contract import PIC_LINK_RUNTIME_OWNED_FIELDS, parse_residency_recovery
from .framing import (ChatTokenLayout, RepairDecision, RepairWindowPlanner, Stitcher, StitchedContext,
                      UniformRepairWindow, build_layout, compile_payload, frame_link, framing_spec_for)
from .manager import ContextManager
from .token_reuse import RequestTokenSource, SharedTokenCache, host_token_reuse_enabled
from .planner import CacheCatalog, ExecutionPlan, Planner


class TransportError(RuntimeError):
    def __init__(self, message: str, status: Optional[int] = None):
        super().__init__(message)
        self.status = status


class ChatStreamError(TransportError):
    pass


class JSONHTTPTransport:
    def __init__(self, api_base: str, timeout: float = 1200.0):
        self.api_base = api_base.rstrip("/")
        self.timeout = timeout

    def __call__(self, payload: dict) -> dict:
        req = urllib.request.Request(self.api_base + "/chat/completions", data=json.dumps(payload).encode(),
                                     headers={"Content-Type": "application/json"})
        t0 = time.perf_counter()
        try:
            with urllib.request.urlopen(req, timeout=self.timeout) as r:
                body = json.loads(r.read())
        except urllib.error.HTTPError as e:
            raise TransportError(e.read().decode("utf-8", "replace"), e.code) from None
        except urllib.error.URLError as e:
            raise TransportError(f"transport failure: {e.reason}") from None
        body.setdefault("_latency_s", time.perf_counter() - t0)
        return body


def post_chat_stream(api_base: str, payload: dict, timeout: float = 1200.0) -> dict:
    """Streams a chat completion; returns text, ttft_s, latency_s."""
    p = dict(payload, stream=True)
    req = urllib.request.Request(api_base.rstrip("/") + "/chat/completions", data=json.dumps(p).encode(),
                                 headers={"Content-Type": "application/json", "Accept": "text/event-stream"})
    t0 = time.perf_counter()
    ttft, parts = None, []
    try:
        with urllib.request.urlopen(req, timeout=timeout) as r:
            for raw in r:
                line = raw.decode().strip()
                if not line.startswith("data:"):
                    continue
                data = line[5:].strip()
                if data == "[DONE]":
                    break
                ev = json.loads(data)
                if "error" in ev:
                    raise ChatStreamError(json.dumps(ev["error"]))
                for ch in ev.get("choices") or []:
                    piece = (ch.get("delta") or {}).get("content") or ""
                    if piece and ttft is None:
                        ttft = time.perf_counter() - t0
                    parts.append(piece)
    except urllib.error.HTTPError as e:
        raise TransportError(e.read().decode("utf-8", "replace"), e.code) from None
    return {"text": "".join(parts), "ttft_s": ttft, "latency_s": time.perf_counter() - t0}


# ------------------------------------------------------------ recovery
class Role(str, Enum):
    OWNER = "owner"
    WAITER = "waiter"
    SETTLED = "settled"
    FAILED = "failed"


@dataclass
class Flight:
    key: tuple
    done: threading.Event = field(default_factory=threading.Event)
    ok: bool = False
    error: Optional[str] = None
    waiters: int = 0


@dataclass
class Ticket:
    role: Role
    key: tuple
    flight: Optional[Flight] = None
    error: Optional[str] = None


class ResidencyRecoveryCoordinator:
    def __init__(self, wait_timeout_s: float = 300.0):
        self.wait_timeout_s = wait_timeout_s
        self._lock = threading.Lock()
        self._flights: dict[tuple, Flight] = {}
        self._last_ok: dict[tuple, int] = {}
        self._last_fail: dict[tuple, tuple[int, str]] = {}
        self.completions = 0
        self.counters = {"owners": 0, "waiters": 0, "settled": 0, "compiles": 0, "failures": 0}

    def claim(self, runtime_id: Hashable, cache_key: str, *, observed: int) -> Ticket:
        k = (runtime_id, cache_key)
        with self._lock:
            f = self._flights.get(k)
            if f is not None and not f.done.is_set():
                f.waiters += 1
                self.counters["waiters"] += 1
                return Ticket(Role.WAITER, k, f)
            if self._last_ok.get(k, 0) > observed:
                self.counters["settled"] += 1
                return Ticket(Role.SETTLED, k)
            f = self._flights[k] = Flight(k)
            self.counters["owners"] += 1
            return Ticket(Role.OWNER, k, f)

    def complete(self, t: Ticket, *, ok: bool, error: Optional[str] = None) -> None:
        if t.role != Role.OWNER or t.flight is None:
            return
        with self._lock:
            self.completions += 1
            t.flight.ok, t.flight.error = ok, error
            if ok:
                self._last_ok[t.key] = self.completions
            else:
                self._last_fail[t.key] = (self.completions, error or "recovery failed")
                self.counters["failures"] += 1
            self._flights.pop(t.key, None)
            t.flight.done.set()

    def wait(self, t: Ticket) -> bool:
        if t.role != Role.WAITER or t.flight is None:
            return t.role == Role.SETTLED
        if not t.flight.done.wait(self.wait_timeout_s):
            raise TimeoutError(f"residency recovery of {t.key[1]} did not finish in {self.wait_timeout_s}s")
        return t.flight.ok


# ------------------------------------------------------------- the adapter
def classify_failure(message: str) -> str:
    d = parse_residency_recovery(message)
    if any(d.values()):
        return "residency"
    low = message.lower()
    if "allocatable" in low or "capacity" in low or "out of pages" in low:
        return "capacity"
    if "pic_link" in low or "contract" in low or "hash mismatch" in low or "unknown fields" in low:
        return "contract"
    if "transport failure" in low:
        return "transport"
    return "other"


@dataclass
class AdapterResult:
    route: str
    text: str = ""
    response: dict = field(default_factory=dict)
    latency_s: float = 0.0
    compile_requests: int = 0
    compile_latency_s: float = 0.0
    link_attempts: int = 0
    recovery: dict = field(default_factory=dict)
    audit: Optional[dict] = None
    error: Optional[str] = None


class RuntimeAdapter:
    def __init__(self, transport: Callable[[dict], dict], *, model: str, tokenizer, catalog: Optional[CacheCatalog] = None,
                 coordinator: Optional[ResidencyRecoveryCoordinator] = None, runtime_id: Hashable = "runtime-0",
                 repair_planner: Optional[RepairWindowPlanner] = None, recovery_attempts: int = 2,
                 generation: Optional[dict] = None, formal: bool = False, execution_profile: Optional[dict] = None,
                 model_id: Optional[str] = None):
        self.transport = transport
        self.model = model
        self.tokenizer = tokenizer
        self.catalog = catalog or CacheCatalog()
        self.coordinator = coordinator or ResidencyRecoveryCoordinator()
        self.runtime_id = runtime_id
        self.repair_planner = repair_planner or RepairWindowPlanner()
        self.recovery_attempts = recovery_attempts
        self.generation = dict(generation or {"max_tokens": 16, "temperature": 0.0})
        self.formal = formal
        self.execution_profile = execution_profile
        self.model_id = model_id or model
        self._rid = 0

    def _next_rid(self) -> str:
        self._rid += 1
        return f"host-{id(self) & 0xffff:x}-{self._rid}"

    def _send(self, payload: dict) -> dict:
        return self.transport(payload)

    # ---- Compile
    def compile_segment(self, seg) -> tuple[int, float]:
        with self.catalog.lock(seg.cache_key):
            if self.catalog.is_compiled(seg.cache_key):
                return 0, 0.0
            t0 = time.perf_counter()
            self._send(compile_payload(seg, model=self.model, fingerprints={
                "tokenizer_fingerprint": self.tokenizer.fingerprint}))
            dt = time.perf_counter() - t0
            self.catalog.mark_compiled(seg.cache_key, token_count=len(seg.token_ids))
            return 1, dt

    def compile_plan(self, layout: ChatTokenLayout) -> tuple[int, float]:
        n, dt = 0, 0.0
        for seg in layout.link_segments:
            a, b = self.compile_segment(seg)
            n += a
            dt += b
        return n, dt

    # ---- Link with recovery
    def link(self, stitched: StitchedContext, layout: ChatTokenLayout, *, task_id: str = "task") -> AdapterResult:
        decision = self.repair_planner.plan(layout)
        rid = self._next_rid()
        payload, audit = frame_link(stitched, layout, decision, request_id=rid, task_id=task_id, model=self.model,
                                    generation=self.generation, formal=self.formal,
                                    framing_spec=framing_spec_for(self.tokenizer, self.model_id),
                                    execution_profile=self.execution_profile)
        assert not (set(payload["pic_link"]) & PIC_LINK_RUNTIME_OWNED_FIELDS)
        res = AdapterResult("selected_context_radixcache_legolink", audit=audit.to_dict())
        rec = {"attempts": 0, "owners": 0, "waiters": 0, "outcome": "not_needed", "recovered_cache_keys": []}
        t0 = time.perf_counter()
        for attempt in range(self.recovery_attempts + 1):
            observed = self.coordinator.completions
            res.link_attempts += 1
            try:
                resp = self._send(payload)
                res.response = resp
                res.text = _text_of(resp)
                if rec["attempts"]:
                    rec["outcome"] = "recovered_after_source_missing"
                break
            except TransportError as e:
                msg = str(e)
                kind = classify_failure(msg)
                if kind != "residency" or attempt == self.recovery_attempts:
                    res.error = msg
                    rec["outcome"] = "failed" if rec["attempts"] else rec["outcome"]
                    raise
                gone = parse_residency_recovery(msg)
                keys = list(dict.fromkeys(gone["missing"] + gone["stale"] + gone["incompatible"]))
                rec["attempts"] += 1
                n, dt = self._recover(keys, layout, observed, rec)
                res.compile_requests += n
                res.compile_latency_s += dt
        res.latency_s = time.perf_counter() - t0
        res.recovery = rec
        return res

    def _recover(self, keys, layout: ChatTokenLayout, observed: int, rec: dict) -> tuple[int, float]:
        segs = {s.cache_key: s for s in layout.link_segments}
        n, dt = 0, 0.0
        for k in keys:
            self.catalog.invalidate(k)
            t = self.coordinator.claim(self.runtime_id, k, observed=observed)
            if t.role == Role.OWNER:
                rec["owners"] += 1
                try:
                    if k not in segs:
                        raise KeyError(f"runtime reported {k} gone but this Link does not use it")
                    a, b = self.compile_segment(segs[k])
                    n, dt = n + a, dt + b
                    self.coordinator.counters["compiles"] += a
                    self.coordinator.complete(t, ok=True)
                    rec["recovered_cache_keys"].append(k)
                except Exception as e:
                    self.coordinator.complete(t, ok=False, error=str(e))
                    raise
            elif t.role == Role.WAITER:
                rec["waiters"] += 1
                if not self.coordinator.wait(t):
                    raise TransportError(f"recovery of {k} failed in another request")
                self.catalog.mark_compiled(k)
                rec["recovered_cache_keys"].append(k)
            else:
                self.catalog.mark_compiled(k)
        return n, dt

    # ---- native baselines
    def native(self, messages: list[dict], route: str) -> AdapterResult:
        t0 = time.perf_counter()
        resp = self._send({"model": self.model, "messages": messages, **self.generation})
        return AdapterResult(route, _text_of(resp), resp, time.perf_counter() - t0)


def _text_of(resp: dict) -> str:
    try:
        return resp["choices"][0]["message"]["content"] or ""
    except (KeyError, IndexError, TypeError):
        return ""


# ------------------------------------------------------------ the pipeline
class PipelineRoute(str, Enum):
    FULL_CONTEXT_ORIGINAL = "full_context_original_sglang"
    SELECTED_CONTEXT_ORIGINAL = "selected_context_original_sglang"
    SELECTED_CONTEXT_LEGOLINK = "selected_context_radixcache_legolink"


@dataclass
class PipelineExecution:
    route: PipelineRoute
    result: AdapterResult
    plan: Optional[ExecutionPlan] = None
    stitched: Optional[StitchedContext] = None
    layout: Optional[ChatTokenLayout] = None
    compile_requests: int = 0
    compile_latency_s: float = 0.0
    timings_ms: dict = field(default_factory=dict)

    def metrics_row(self) -> dict:
        row = {"route": self.route.value, "compile_requests": self.compile_requests,
               "compile_latency_s": round(self.compile_latency_s, 6), "latency_s": round(self.result.latency_s, 6),
               "link_attempts": self.result.link_attempts, "residency_recovery": self.result.recovery,
               "host_timings_ms": self.timings_ms}
        if self.plan is not None:
            d = self.plan.to_dict()
            row["block_planning"] = d["block_planning"]
            row["reuse_accounting"] = d["reuse_accounting"]
            row.update(self.plan.namespace_config)
            rec = (self.result.recovery or {}).get("recovered_cache_keys", [])
            row["namespace"] = self.plan.namespace_summary(recovered_cache_keys=rec)
        if self.layout is not None:
            row["framing"] = self.layout.diagnostics()
        return row


class RequestPipeline:
    def __init__(self, manager: ContextManager, adapter: RuntimeAdapter, planner: Optional[Planner] = None,
                 stitcher: Optional[Stitcher] = None, namespace: str = "default"):
        self.manager = manager
        self.adapter = adapter
        self.planner = planner or Planner(catalog=adapter.catalog)
        self.stitcher = stitcher or Stitcher(tokenizer=None)
        self.namespace = namespace
        self.shared_tokens = SharedTokenCache()  # immutable texts' ids across requests (host token reuse)

    def execute(self, events, route: PipelineRoute = PipelineRoute.SELECTED_CONTEXT_LEGOLINK, query: str = "",
                tools=None) -> PipelineExecution:
        tm = {}
        t = time.perf_counter()
        self.manager.ingest(events)
        tm["ingest"] = (time.perf_counter() - t) * 1e3
        t = time.perf_counter()
        manifest = self.manager.select(query)
        contexts = self.manager.contexts()
        plan = self.planner.plan(manifest, contexts)
        tm["plan"] = (time.perf_counter() - t) * 1e3
        if route == PipelineRoute.FULL_CONTEXT_ORIGINAL or route == PipelineRoute.SELECTED_CONTEXT_ORIGINAL:
            text = self.stitcher.baseline_text(plan)
            res = self.adapter.native([{"role": "user", "content": text}], route.value)
            return PipelineExecution(route, res, plan, timings_ms=tm)
        if not plan.linked_contexts:
            text = self.stitcher.baseline_text(plan)
            res = self.adapter.native([{"role": "user", "content": text}], "legolink_no_reusable_block")
            return PipelineExecution(route, res, plan, timings_ms=tm)
        t = time.perf_counter()
        stitched = self.stitcher.stitch(plan)
        tok = self.adapter.tokenizer
        source = None
        if host_token_reuse_enabled():
            # framing reads the ids the stored sub-contexts already hold
            source = RequestTokenSource(tok, shared=self.shared_tokens)
            for v in plan.linked_contexts:
                source.adopt(v)
            for v in stitched.linked_views:  # block + separator: immutable, shared across turns
                source.mark_immutable(v.raw_text)
            tok = source
        layout = build_layout(stitched, tok, tools=tools)
        tm["frame"] = (time.perf_counter() - t) * 1e3
        if source is not None:
            tm["token_reuse"] = source.counts()
        t = time.perf_counter()
        nc, cdt = self.adapter.compile_plan(layout)
        self.planner.after_compile(plan)
        tm["compile"] = (time.perf_counter() - t) * 1e3
        t = time.perf_counter()
        res = self.adapter.link(stitched, layout, task_id=self.manager.task_id)
        self.planner.after_link(plan)
        tm["link"] = (time.perf_counter() - t) * 1e3
        return PipelineExecution(route, res, plan, stitched, layout, nc + res.compile_requests,
                                 cdt + res.compile_latency_s, tm)


def make_pipeline(transport: Callable[[dict], dict], *, task_id: str, model: str = "legolink", tokenizer=None,
                  catalog: Optional[CacheCatalog] = None, coordinator: Optional[ResidencyRecoveryCoordinator] = None,
                  namespace_mode="global", cross_namespace_pairs=(), resolver=None, repair_tokens: int = 16,
                  generation: Optional[dict] = None) -> RequestPipeline:
    """One agent session's pipeline.  Sessions that talk to one runtime
    should share ``catalog`` (one host view of the runtime's blocks, which
    the namespace resolver reads across tasks) and ``coordinator``.
    ``namespace_mode`` / ``cross_namespace_pairs`` are validated here, at
    construction (reference ``cache_namespace.py:502``); a ``resolver``
    built once may be passed instead."""
    from .namespaces import NamespacePolicy, NamespaceResolver

    if resolver is None:
        resolver = NamespaceResolver(namespace_mode, NamespacePolicy(cross_namespace_pairs=list(cross_namespace_pairs)))
    cm = ContextManager(task_id, tokenizer=tokenizer) if tokenizer is not None else ContextManager(task_id)
    catalog = catalog if catalog is not None else CacheCatalog()
    ad = RuntimeAdapter(transport, model=model, tokenizer=cm.tokenizer, catalog=catalog, coordinator=coordinator,
                        repair_planner=RepairWindowPlanner(UniformRepairWindow(repair_tokens)), generation=generation)
    return RequestPipeline(cm, ad, planner=Planner(catalog=catalog, resolver=resolver))

