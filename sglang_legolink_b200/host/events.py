"""Session events, field-first extraction and OpenAI-request ingress.

Stages 1-2 of the host pipeline (reference ``noc_context_manager/
real_ingress.py`` and ``session.py``): agent inputs become revisioned,
de-duplicated :class:`SessionEvent` records; each event's source is assigned
one of seven context fields by a fixed table; hidden sources (oracle /
grader / solution files) are dropped before anything is segmented.
"""

from __future__ import annotations

import hashlib
import json
from dataclasses import asdict, dataclass, field
from datetime import datetime, timezone
from enum import Enum
from pathlib import PurePath
from typing import Any, Iterable, Optional

CONTEXT_FIELDS = (
    "user_prompt",
    "task_instruction",
    "tool_definitions",
    "tool_history_output",
    "conversation_history",
    "workspace_evidence",
    "task_metadata",
)


class EventType(str, Enum):
    USER_REQUEST = "user_request"
    TASK_INSTRUCTION = "task_instruction"
    PLANNER_OUTPUT = "planner_output"
    TOOL_DEFINITION = "tool_definition"
    TOOL_CALL = "tool_call"
    TOOL_OUTPUT = "tool_output"
    CONVERSATION_MESSAGE = "conversation_message"
    WORKSPACE_FILE = "workspace_file"
    TASK_METADATA = "task_metadata"
    UNCLASSIFIED = "unclassified"


FIELD_OF_EVENT = {
    EventType.USER_REQUEST: "user_prompt",
    EventType.TASK_INSTRUCTION: "task_instruction",
    EventType.PLANNER_OUTPUT: "conversation_history",
    EventType.TOOL_DEFINITION: "tool_definitions",
    EventType.TOOL_CALL: "tool_history_output",
    EventType.TOOL_OUTPUT: "tool_history_output",
    EventType.CONVERSATION_MESSAGE: "conversation_history",
    EventType.WORKSPACE_FILE: "workspace_evidence",
    EventType.TASK_METADATA: "task_metadata",
}

HIDDEN_PATH_PARTS = frozenset(
    {"oracle", "grader", "graders", "solution", "solutions", "hidden_answer", "answer_key", "verifier"})
HIDDEN_NAME_MARKERS = ("oracle", "grader", "solution", "answer_key", "test_answer", "expected_answer", "verifier")


class FieldClassificationError(ValueError):
    pass


def utc_now() -> str:
    return datetime.now(timezone.utc).isoformat(timespec="milliseconds")


@dataclass(frozen=True)
class SourceSpan:
    source_id: str
    start: int
    end: int
    source_path: str = ""

    def to_dict(self) -> dict:
        return asdict(self)


@dataclass(frozen=True)
class SessionEvent:
    event_id: str
    task_id: str
    session_revision: int
    event_type: EventType
    source_id: str
    raw_text: str
    timestamp: str
    sequence_number: int
    metadata: dict = field(default_factory=dict)

    def to_dict(self) -> dict:
        d = asdict(self)
        d["event_type"] = self.event_type.value
        return d

    @classmethod
    def from_dict(cls, d: dict) -> "SessionEvent":
        return cls(str(d["event_id"]), str(d["task_id"]), int(d["session_revision"]), EventType(d["event_type"]),
                   str(d["source_id"]), str(d.get("raw_text") or ""), str(d["timestamp"]),
                   int(d["sequence_number"]), dict(d.get("metadata") or {}))


EventTuple = tuple  # (event_type, source_id, raw_text, metadata)


class EventCollector:
    """Accepts events in batches; each accepted batch is one new revision.
    An event identical (type, source, text) to one already accepted is
    dropped.  :meth:`checkpoint` / :meth:`rollback` make an ingest
    transactional."""

    def __init__(self, task_id: str):
        self.task_id = task_id
        self._events: list[SessionEvent] = []
        self._digests: list[str] = []
        self._seen: set[str] = set()
        self._revision = 0

    @property
    def revision(self) -> int:
        return self._revision

    def events(self, revision: Optional[int] = None) -> list[SessionEvent]:
        if revision is None:
            return list(self._events)
        return [e for e in self._events if e.session_revision <= revision]

    def checkpoint(self) -> tuple[int, int]:
        return len(self._events), self._revision

    def rollback(self, cp: tuple[int, int]) -> list[SessionEvent]:
        n, rev = cp
        if n > len(self._events) or rev > self._revision:
            raise ValueError("cannot roll back to a checkpoint from the future")
        removed = self._events[n:]
        del self._events[n:]
        self._seen.difference_update(self._digests[n:])
        del self._digests[n:]
        self._revision = rev
        return removed

    def add_events(self, values: Iterable[EventTuple], *, timestamp: Optional[str] = None) -> list[SessionEvent]:
        fresh, pending = [], set()
        for et, sid, text, meta in values:
            kind = EventType(et)
            dg = hashlib.sha256(f"{kind.value}\0{sid}\0{text}".encode()).hexdigest()
            if dg in self._seen or dg in pending:
                continue
            pending.add(dg)
            fresh.append((kind, str(sid), str(text), dict(meta or {}), dg))
        if not fresh:
            return []
        self._revision += 1
        out = []
        for kind, sid, text, meta, dg in fresh:
            ev = SessionEvent(f"evt-{dg[:20]}", self.task_id, self._revision, kind, sid, text, timestamp or utc_now(),
                              len(self._events) + 1, meta)
            self._events.append(ev)
            self._digests.append(dg)
            self._seen.add(dg)
            out.append(ev)
        return out


@dataclass(frozen=True)
class ExtractedSource:
    context_field: str
    event_id: str
    source_id: str
    raw_text: str
    sequence_number: int
    source_path: str = ""
    metadata: dict = field(default_factory=dict)
    revision: int = 0


@dataclass(frozen=True)
class FieldExtraction:
    task_id: str
    session_revision: int
    fields: dict
    filtered_event_ids: tuple = ()

    def sources(self) -> list[ExtractedSource]:
        return sorted((s for v in self.fields.values() for s in v), key=lambda s: s.sequence_number)


def is_hidden_source(ev: SessionEvent) -> bool:
    m = ev.metadata
    if any(bool(m.get(k)) for k in ("hidden", "oracle", "grader", "answer")):
        return True
    path = str(m.get("path") or m.get("file_path") or "").replace("\\", "/")
    pp = PurePath(path)
    parts = {p.lower() for p in pp.parts}
    name = pp.name.lower()
    return bool(parts & HIDDEN_PATH_PARTS) or any(x in name for x in HIDDEN_NAME_MARKERS)


class FieldExtractor:
    """Table-driven field assignment; an optional ``classifier(event) -> field``
    decides only event types the table does not cover (else fail closed)."""

    def __init__(self, classifier=None):
        self.classifier = classifier

    def field_for(self, ev: SessionEvent) -> tuple[str, Optional[dict]]:
        f = FIELD_OF_EVENT.get(ev.event_type)
        if f is not None:
            return f, None
        if self.classifier is None:
            raise FieldClassificationError(
                f"event {ev.event_id} has type {ev.event_type.value!r}, which no field table covers, and no field "
                "classifier is configured")
        f = self.classifier(ev)
        if f not in CONTEXT_FIELDS:
            raise FieldClassificationError(f"classifier returned unknown field {f!r}")
        return f, {"classifier": getattr(self.classifier, "__name__", "custom"), "field": f}

    def extract(self, events: Iterable[SessionEvent]) -> FieldExtraction:
        ordered = sorted(events, key=lambda e: e.sequence_number)
        tasks = {e.task_id for e in ordered}
        if len(tasks) > 1:
            raise ValueError("field extraction cannot mix task ids")
        latest = {e.source_id: e for e in ordered}  # only the newest revision of a source is active
        fields: dict[str, list] = {f: [] for f in CONTEXT_FIELDS}
        filtered = []
        for ev in sorted(latest.values(), key=lambda e: e.sequence_number):
            if is_hidden_source(ev):
                filtered.append(ev.event_id)
                continue
            f, cls = self.field_for(ev)
            meta = dict(ev.metadata)
            if cls is not None:
                meta["field_classification"] = cls
            fields[f].append(ExtractedSource(f, ev.event_id, ev.source_id, ev.raw_text, ev.sequence_number,
                                             str(meta.get("path") or meta.get("file_path") or ""), meta,
                                             ev.session_revision))
        return FieldExtraction(next(iter(tasks), ""), max((e.session_revision for e in ordered), default=0),
                               {k: tuple(v) for k, v in fields.items()}, tuple(filtered))


# ------------------------------------------------------------------ ingress
def canonical_tool_schema(tool: dict) -> str:
    """Byte-stable text of one tool definition (sorted keys, compact)."""
    return json.dumps(tool, sort_keys=True, separators=(",", ":"), ensure_ascii=False)


def _content_text(content: Any) -> str:
    if content is None:
        return ""
    if isinstance(content, str):
        return content
    if isinstance(content, list):
        return "".join(p.get("text", "") for p in content if isinstance(p, dict) and p.get("type") == "text")
    return str(content)


def openai_request_events(messages: list[dict], tools: Optional[list[dict]] = None) -> list[EventTuple]:
    """Stateless, position-keyed variant: OpenAI chat messages (+tools) ->
    event tuples (system -> task instruction, the last user message -> user
    request, other user / assistant -> conversation, tool -> tool output,
    each tool definition -> tool definition).  Agents that resend their whole
    conversation use the session-aware ``host.ingress.openai_request_events``
    (content-derived ids and a source ledger)."""
    out: list[EventTuple] = []
    for i, tool in enumerate(tools or []):
        name = ((tool.get("function") or {}).get("name")) or tool.get("name") or f"tool-{i}"
        out.append((EventType.TOOL_DEFINITION, f"tool-def:{name}", canonical_tool_schema(tool), {"tool_name": name}))
    last_user = max((i for i, m in enumerate(messages) if m.get("role") == "user"), default=-1)
    for i, m in enumerate(messages):
        role = m.get("role")
        text = _content_text(m.get("content"))
        if role == "system":
            out.append((EventType.TASK_INSTRUCTION, f"system:{i}", text, {"message_role": "system"}))
        elif role == "user":
            kind = EventType.USER_REQUEST if i == last_user else EventType.CONVERSATION_MESSAGE
            out.append((kind, f"user:{i}", text, {"message_role": "user"}))
        elif role == "assistant":
            if text:
                out.append((EventType.CONVERSATION_MESSAGE, f"assistant:{i}", text, {"message_role": "assistant"}))
            for j, call in enumerate(m.get("tool_calls") or []):
                out.append((EventType.TOOL_CALL, f"tool-call:{call.get('id', f'{i}.{j}')}",
                            canonical_tool_schema(call), {"message_role": "assistant"}))
        elif role == "tool":
            out.append((EventType.TOOL_OUTPUT, f"tool-output:{m.get('tool_call_id', i)}", text,
                         {"message_role": "tool", "tool_call_id": m.get("tool_call_id")}))
    return out


def tool_output_event(call_id: str, text: str, **meta) -> EventTuple:
    return (EventType.TOOL_OUTPUT, f"tool-output:{call_id}", text, dict(meta))
