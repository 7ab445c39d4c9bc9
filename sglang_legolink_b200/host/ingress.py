"""Session-aware structured ingress: what one agent request adds to a session.

An agent resends its whole conversation on every call.  The events of a
call are therefore derived so that what the session already holds is not
ingested again, and ids never depend on a message's position:

* source ids come from content: a chat message is ``message-<digest(role,
  text)>``, a tool call ``tool-call:<digest(canonical call)>``, a tool result
  ``tool-output:<digest(tool name, text)>``, a tool schema
  ``tool-schema:<name>`` (a changed schema under the same name is a new
  revision of that source; two tools of one name get a digest suffix);
* :class:`SourceLedger` -- ``source_id -> (latest type, text digest)`` of the
  session: a source held with the same text is skipped whatever type it
  comes back as; a user message that was the current request of an earlier
  call and is history now is re-emitted as a conversation message under the
  same id (the extractor keeps a source's latest revision);
* the last message of a call is the current request -- except on the first
  call of a session, whose prompt is the task instruction;
* :class:`PromptRegistry` and :func:`terminus_turn_events` -- for agents
  that call ``call(prompt, message_history)`` and declare how they assembled
  ``prompt`` (:class:`PromptPart`: tool output vs their own directive).  A
  declaration is used only if its parts join to the prompt byte for byte;
  when that prompt returns as one history message, its parts are settled
  instead of ingesting the text twice.

The id formulas and event kinds are kept as the reference's so sessions
persisted by either host dedupe the same way.  Reference:
``noc_context_manager/real_ingress.py:40-472``.
"""

from __future__ import annotations

import hashlib
import json
from dataclasses import dataclass, field
from typing import Any, Callable, Iterable, Mapping, Optional, Sequence

from .events import EventType

INGRESS_VERSION = "real-ingress-v1"
KIND_TOOL_OUTPUT = "tool_output"
KIND_AGENT_DIRECTIVE = "agent_directive"

EventTuple = tuple  # (EventType, source_id, raw_text, metadata)


def canonical_json(value: Any) -> str:
    return json.dumps(value, sort_keys=True, separators=(",", ":"), ensure_ascii=False)


def content_digest(*parts: str, size: int = 20) -> str:
    return hashlib.sha256("\0".join(parts).encode("utf-8")).hexdigest()[:size]


def message_source_id(role: str, content: str) -> str:
    return "message-" + content_digest(role, content)


def message_text(content: Any) -> str:
    """OpenAI text or multi-part content as plain text."""
    if content is None:
        return ""
    if isinstance(content, str):
        return content
    if isinstance(content, list):
        out = []
        for item in content:
            if isinstance(item, dict):
                if item.get("type") == "text":
                    out.append(str(item.get("text") or ""))
                elif "content" in item:
                    out.append(str(item.get("content") or ""))
            else:
                out.append(str(item))
        return "\n".join(p for p in out if p)
    return str(content)


def _meta(ingress: str, **kw) -> dict:
    return {"ingress": ingress, "ingress_version": INGRESS_VERSION, **kw}


# --------------------------------------------------------------- tools
def _tool_name(tool: Mapping) -> str:
    fn = tool.get("function") if isinstance(tool.get("function"), Mapping) else None
    return str((fn or tool).get("name") or "")


def tool_definition_events(tools: Optional[Sequence[Mapping]], *,
                           functions: Optional[Sequence[Mapping]] = None) -> list:
    """One TOOL_DEFINITION per tool (``tools`` and the legacy ``functions``);
    adding, removing or reordering one tool never invalidates another."""
    declared = [dict(t) for t in (tools or [])] + [{"type": "function", "function": dict(f)} for f in (functions or [])]
    names = [_tool_name(t) for t in declared]
    out = []
    for i, tool in enumerate(declared):
        text = canonical_json(tool)
        name = names[i] or f"tool-{i}"
        sid = f"tool-schema:{name}"
        if names.count(names[i]) > 1:
            sid += "#" + content_digest(text, size=8)
        out.append((EventType.TOOL_DEFINITION, sid, text, _meta("openai.tools", tool_name=name)))
    return out


def _decoded(arguments: Any) -> Any:
    if isinstance(arguments, str):
        try:
            return json.loads(arguments)
        except ValueError:
            return arguments
    return arguments


def tool_call_event(call_id: str, tool_name: str, arguments: Any, *, ingress: str) -> EventTuple:
    """The call as canonical ``{"arguments", "tool_name"}`` text; the call id is
    execution bookkeeping and stays in metadata."""
    text = canonical_json({"tool_name": tool_name, "arguments": _decoded(arguments)})
    return (EventType.TOOL_CALL, "tool-call:" + content_digest(text), text,
            _meta(ingress, tool_call_id=call_id, tool_name=tool_name))


def tool_output_event(call_id: str, tool_name: str, content: str, *, ingress: str,
                      extra: Optional[Mapping] = None) -> EventTuple:
    """A tool result; the text is exactly what the tool returned."""
    return (EventType.TOOL_OUTPUT, "tool-output:" + content_digest(tool_name, content), content,
            _meta(ingress, tool_call_id=call_id, tool_name=tool_name, **dict(extra or {})))


# --------------------------------------------------------------- ledger
@dataclass
class SourceLedger:
    latest: dict = field(default_factory=dict)  # source_id -> (EventType, text digest)

    @classmethod
    def from_events(cls, events: Iterable[Any]) -> "SourceLedger":
        led = cls()
        for e in sorted(events, key=lambda x: x.sequence_number):
            led.latest[e.source_id] = (EventType(e.event_type), content_digest(e.raw_text, size=32))
        return led

    def type_of(self, source_id: str) -> Optional[EventType]:
        held = self.latest.get(source_id)
        return None if held is None else held[0]

    def admit(self, batch: list, event: EventTuple) -> bool:
        """Appends ``event`` unless the session or this batch holds that
        source with that text.  Returns whether it was appended."""
        _kind, sid, text, _md = event
        d = content_digest(text, size=32)
        held = self.latest.get(sid)
        if held is not None and held[1] == d:
            return False
        if any(e[1] == sid and content_digest(e[2], size=32) == d for e in batch):
            return False
        batch.append(event)
        return True

    def record(self, events: Iterable[EventTuple]) -> None:
        """Marks a batch as ingested (when the caller does not rebuild the
        ledger from the collector)."""
        for kind, sid, text, _md in events:
            self.latest[sid] = (EventType(kind), content_digest(text, size=32))


def _chat_kind(role: str) -> EventType:
    return EventType.TASK_INSTRUCTION if role in ("system", "developer") else EventType.CONVERSATION_MESSAGE


def _message(batch: list, ledger: SourceLedger, role: str, text: str, kind: EventType, ingress: str,
             **extra) -> None:
    sid = message_source_id(role, text)
    if kind is EventType.CONVERSATION_MESSAGE and ledger.type_of(sid) is EventType.USER_REQUEST:
        # the request of an earlier call is history now: settle it
        batch.append((kind, sid, text, _meta(ingress, message_role=role, settled_from="user_request", **extra)))
        return
    ledger.admit(batch, (kind, sid, text, _meta(ingress, message_role=role, **extra)))


def openai_request_events(messages: Sequence[Mapping], *, tools: Optional[Sequence[Mapping]] = None,
                          functions: Optional[Sequence[Mapping]] = None, ledger: SourceLedger,
                          first_turn: bool) -> list:
    """The events one OpenAI chat request adds to a session (role, position
    of the last message, tool calls / results and the ``tools`` field are the
    only evidence used)."""
    batch: list = []
    for ev in tool_definition_events(tools, functions=functions):
        ledger.admit(batch, ev)
    call_names: dict = {}
    last = len(messages) - 1
    for i, m in enumerate(messages):
        role = str(m.get("role") or "user")
        text = message_text(m.get("content"))
        calls = m.get("tool_calls") or []
        if role == "assistant" or calls:
            if text.strip():
                _message(batch, ledger, role, text, EventType.CONVERSATION_MESSAGE, "openai.messages")
            for call in calls:
                fn = call.get("function") if isinstance(call.get("function"), Mapping) else call
                name, cid = str(fn.get("name") or ""), str(call.get("id") or "")
                call_names[cid] = name
                ledger.admit(batch, tool_call_event(cid, name, fn.get("arguments"), ingress="openai.messages"))
            continue
        if role in ("tool", "function"):
            cid = str(m.get("tool_call_id") or "")
            name = str(m.get("name") or call_names.get(cid) or "")
            ledger.admit(batch, tool_output_event(cid, name, text, ingress="openai.messages",
                                                  extra={"message_role": role}))
            continue
        if role == "user" and i == last:
            kind = EventType.TASK_INSTRUCTION if first_turn else EventType.USER_REQUEST
        else:
            kind = _chat_kind(role)
        _message(batch, ledger, role, text, kind, "openai.messages")
    return batch


# ------------------------------------------------------- declared prompts
@dataclass(frozen=True)
class PromptPart:
    """A piece of one prompt, as the agent that assembled it declares it."""
    kind: str  # KIND_TOOL_OUTPUT | KIND_AGENT_DIRECTIVE
    text: str
    metadata: Mapping = field(default_factory=dict)


def verified_parts(prompt: str, parts: Optional[Sequence[PromptPart]]) -> Optional[tuple]:
    """The declared parts if they join to ``prompt`` byte for byte (the
    agent says *what* it assembled; it is never trusted to say it right)."""
    if not parts or any(p.kind not in (KIND_TOOL_OUTPUT, KIND_AGENT_DIRECTIVE) for p in parts):
        return None
    if "".join(p.text for p in parts) != prompt:
        return None
    return tuple(p for p in parts if p.text)


def split_around(prompt: str, needle: str, *, needle_kind: str = KIND_TOOL_OUTPUT,
                 needle_metadata: Optional[Mapping] = None) -> Optional[tuple]:
    """directive / ``needle`` / directive, when ``prompt`` holds ``needle`` once."""
    if not needle or prompt.count(needle) != 1:
        return None
    before, after = prompt.split(needle, 1)
    parts = (PromptPart(KIND_AGENT_DIRECTIVE, before), PromptPart(needle_kind, needle, dict(needle_metadata or {})),
             PromptPart(KIND_AGENT_DIRECTIVE, after))
    return tuple(p for p in parts if p.text)


def part_event(part: PromptPart, *, ingress: str, current: bool) -> EventTuple:
    """A tool-output part keeps its exact bytes; an agent directive is the
    agent's own text to the model (the request when it ends the prompt) and
    its seam whitespace is trimmed (a block that starts or ends with newlines
    tokenizes differently next to the stitch separator)."""
    if part.kind == KIND_TOOL_OUTPUT:
        md = dict(part.metadata)
        return tool_output_event(str(md.pop("tool_call_id", "")), str(md.pop("tool_name", "terminal")), part.text,
                                 ingress=ingress, extra=md)
    text = part.text.strip()
    return (EventType.USER_REQUEST if current else EventType.CONVERSATION_MESSAGE, message_source_id("user", text),
            text, _meta(ingress, message_role="user", prompt_part=part.kind, **dict(part.metadata)))


class PromptRegistry:
    """How each declared prompt was split, so that when the prompt comes back
    as one history message its parts are settled rather than the whole text
    ingested again."""

    def __init__(self):
        self._parts: dict = {}

    @staticmethod
    def key(prompt: str) -> str:
        return content_digest(prompt, size=32)

    def remember(self, prompt: str, parts: tuple) -> None:
        self._parts[self.key(prompt)] = parts

    def lookup(self, prompt: str) -> Optional[tuple]:
        return self._parts.get(self.key(prompt))


def _value(message: Any, name: str, default: Any = "") -> Any:
    if isinstance(message, Mapping):
        return message.get(name, default)
    return getattr(message, name, default)


def terminus_turn_events(prompt: str, history: Sequence[Any], *, ledger: SourceLedger, registry: PromptRegistry,
                         declared: Optional[Sequence[PromptPart]], first_turn: bool,
                         message_value: Callable[[Any, str, Any], Any] = _value,
                         ingress: str = "terminus.call") -> tuple:
    """(events, structure) of one ``call(prompt, message_history)``: the
    history (user / assistant messages only -- no system message, tool
    schema or structured tool result exists at this boundary), then the
    prompt, split by the agent's verified declaration when there is one."""
    batch: list = []
    for m in history:
        role = str(message_value(m, "role", "user"))
        text = str(message_value(m, "content", ""))
        earlier = registry.lookup(text) if role == "user" else None
        if earlier is not None:
            for part in earlier:
                if part.kind == KIND_AGENT_DIRECTIVE:
                    ev = part_event(part, ingress=ingress, current=False)
                    if ev[2].strip() and ledger.type_of(ev[1]) is EventType.USER_REQUEST:
                        batch.append(ev)
            continue
        _message(batch, ledger, role, text, _chat_kind(role), ingress)
    parts = verified_parts(prompt, declared)
    structure = {"declared": declared is not None, "verified": parts is not None,
                 "parts": [p.kind for p in parts] if parts else []}
    if parts is not None and not first_turn:
        registry.remember(prompt, parts)
        present = [p for p in parts if p.text.strip()]
        for i, part in enumerate(present):
            # only the end of the turn can be the current request: agent text
            # that introduces more of the same prompt is framing, ingested as
            # conversation now so it keeps its place before what it introduces
            ledger.admit(batch, part_event(part, ingress=ingress, current=i == len(present) - 1))
        return batch, structure
    kind = EventType.TASK_INSTRUCTION if first_turn else EventType.USER_REQUEST
    ledger.admit(batch, (kind, message_source_id("user", prompt), prompt, _meta(ingress, message_role="user")))
    return batch, structure
