"""Agent integrations: LLM clients an agent framework calls as
``call(prompt, message_history)``, and a terminal agent loop over them.

* :class:`PICLLM` -- direct Compile/Link client (no host context manager):
  every history message is cut into tagged text blocks of at most
  ``block_chars``; blocks never compiled before are compiled (one Compile
  request each, ``max_tokens=1``), then the turn is one Link naming every
  block, with the last chunk of the current prompt as the mutable suffix.
  Reference: ``terminal_bench_integration/sglang_pic_agent.py:129-590``.
* :class:`NOCLLM` -- the same call through the host pipeline: the turn's
  events come from :func:`~.ingress.terminus_turn_events` (session ledger,
  prompt registry, the agent's verified prompt declaration), then
  :meth:`RequestPipeline.execute` plans, compiles and links; one metrics row
  per call.  Reference: ``noc_sglang_agent.py:147-1033``.
* :class:`TerminalAgent` -- a Terminus-style loop: the model answers with
  JSON ``{"commands": [{"keystrokes", "is_blocking", "timeout_sec"}],
  "is_task_complete"}``; commands go to a :class:`TerminalSession`; the
  terminal output is the next prompt.  Invalid answers get a bounded
  re-ask; an identical command batch repeated ``max_repeats`` times ends
  the loop.  :class:`NOCTerminalAgent` runs it on :class:`NOCLLM`;
  :class:`NOCTerminus2Agent` also declares each prompt's structure (agent
  directive around the tool output) so the output is ingested as a tool
  result, not as the user's request.  Reference: ``sglang_pic_agent.py:594-1320``,
  ``noc_sglang_agent.py:1090-1240``.

terminal-bench is not a dependency: a terminal is anything with
``send_keys`` / ``capture`` (:class:`TerminalSession`);
:class:`TmuxSessionAdapter` wraps an object exposing terminal-bench's
``send_keys(keys, block=..., max_timeout_sec=...)`` / ``capture_pane()``, and
:class:`SubprocessTerminal` runs commands in a local shell.
"""

from __future__ import annotations

import hashlib
import json
import re
import subprocess
import time
import uuid
from dataclasses import dataclass, field
from typing import Any, Callable, Optional, Protocol, Sequence

from ..contract import validate_pic_link_request
from .ingress import (KIND_AGENT_DIRECTIVE, KIND_TOOL_OUTPUT, PromptPart, PromptRegistry, SourceLedger,
                      split_around, terminus_turn_events)
from .metrics import AgentMetric, MetricsRecorder


def _text_of(resp: dict) -> str:
    try:
        return resp["choices"][0]["message"]["content"] or ""
    except (KeyError, IndexError, TypeError):
        return ""


def split_text(text: str, max_chars: int) -> list:
    """Chunks of at most ``max_chars``, cut at a blank line, else a line end,
    else hard (a cut in the first half of the window is not taken)."""
    rest, out = text.strip(), []
    while rest:
        if len(rest) <= max_chars:
            out.append(rest)
            break
        cut = rest.rfind("\n\n", 0, max_chars + 1)
        if cut < max_chars // 2:
            cut = rest.rfind("\n", 0, max_chars + 1)
        if cut < max_chars // 2:
            cut = max_chars
        out.append(rest[:cut].rstrip())
        rest = rest[cut:].lstrip()
    return out or [""]


def _value(message: Any, name: str, default: str = "") -> str:
    v = message.get(name, default) if isinstance(message, dict) else getattr(message, name, default)
    return str(v if v is not None else default)


# ------------------------------------------------------------- PIC client
class PICLLM:
    """Direct Compile/Link client over a runtime transport (a callable that
    posts one OpenAI chat body and returns the response dict)."""

    def __init__(self, transport: Callable[[dict], dict], *, model: str, recompute_mode: str = "batched",
                 legolink_k: int = 256, first_block_k: Optional[int] = None, max_tokens: int = 1024,
                 temperature: float = 0.0, block_chars: int = 6000, recorder: Optional[MetricsRecorder] = None):
        if recompute_mode not in ("batched", "full_causal"):
            raise ValueError("recompute_mode must be batched or full_causal")
        if legolink_k < 0 or (first_block_k is not None and first_block_k < 0) or max_tokens <= 0 \
                or block_chars <= 0:
            raise ValueError("invalid LegoLink K, max_tokens or block_chars")
        self.transport, self.model = transport, model
        self.recompute_mode = recompute_mode
        self.k = int(legolink_k)
        self.first_k = int(first_block_k) if first_block_k is not None else int(legolink_k)
        self.max_tokens, self.temperature, self.block_chars = int(max_tokens), float(temperature), int(block_chars)
        self.recorder = recorder
        self.session_id = uuid.uuid4().hex
        self.task_id = "unknown"
        self.turn = 0
        self.compiled: dict = {}  # cache_key -> prompt tokens

    def set_task_context(self, task_id: str) -> None:
        self.task_id = str(task_id)

    def _blocks(self, role: str, content: str, *, force_two: bool = False) -> list:
        chunks = split_text(content, self.block_chars)
        if force_two and len(chunks) == 1 and len(chunks[0]) > 1:
            mid = len(chunks[0]) // 2
            chunks = [chunks[0][:mid], chunks[0][mid:]]
        out = []
        for i, c in enumerate(chunks):
            text = f"<agent_message role={role} chunk={i + 1}/{len(chunks)}>\n{c}\n</agent_message>"
            out.append((hashlib.sha256(f"{self.model}\0{text}".encode()).hexdigest(), text))
        return out

    def prepare_turn(self, prompt: str, history: Sequence[Any]) -> tuple:
        """(blocks to link, mutable text): every history message, then all but
        the last chunk of the prompt.  The first user message and a prompt
        without history are cut in two, so a Link always has a block and a
        mutable suffix."""
        blocks = []
        for i, m in enumerate(history):
            role = _value(m, "role", "user")
            blocks += self._blocks(role, _value(m, "content"), force_two=(i == 0 and role == "user"))
        cur = self._blocks("user", prompt, force_two=not history)
        return blocks + cur[:-1], cur[-1][1]

    def block_id(self, cache_key: str) -> str:
        """The id a block is compiled and linked under (stable across turns)."""
        return f"agent::{self.task_id}::{cache_key[:16]}"

    def _compile(self, key: str, text: str) -> tuple:
        body = {"model": self.model, "messages": [{"role": "user", "content": text}], "max_tokens": 1,
                "temperature": 0.0, "extra_key": key,
                "sub_context": {"cache_key": key, "semantic_block_id": self.block_id(key), "task_id": self.task_id,
                                "pic_storage_mode": "reference"}}
        t0 = time.perf_counter()
        resp = self.transport(body)
        return int((resp.get("usage") or {}).get("prompt_tokens") or 0), time.perf_counter() - t0

    def call(self, prompt: str, message_history: Optional[Sequence[Any]] = None, **kw) -> str:
        self.turn += 1
        blocks, mutable = self.prepare_turn(prompt, message_history or [])
        compiles, compile_s = 0, 0.0
        for key, text in blocks:
            if key in self.compiled:
                continue
            n, dt = self._compile(key, text)
            self.compiled[key] = n
            compiles, compile_s = compiles + 1, compile_s + dt
        keys = [k for k, _ in blocks]
        link = {"request_id": f"agent::{self.session_id}::turn-{self.turn}", "task_id": self.task_id,
                "variant": "full_causal" if self.recompute_mode == "full_causal" else f"adaptive_l{self.k}",
                "cache_keys": keys, "block_ids": [self.block_id(k) for k in keys], "recompute_mode": self.recompute_mode,
                "recompute_initial_tokens": self.k, "recompute_first_block": self.first_k > 0,
                "recompute_first_block_tokens": self.first_k}
        validate_pic_link_request(dict(link))
        body = {"model": self.model, "messages": [{"role": "user", "content": mutable}], "pic_link": link,
                "max_tokens": int(kw.get("max_tokens", self.max_tokens)), "temperature": self.temperature}
        t0 = time.perf_counter()
        resp = self.transport(body)
        link_s = time.perf_counter() - t0
        if self.recorder is not None:
            m = AgentMetric(task_id=self.task_id, agent_id="pic-llm", request_id=link["request_id"],
                            session_revision=self.turn, loop_stage="act", objective="", variant="picruntime_owner",
                            operation_mode="pic_link", compile_requests=compiles,
                            compile_latency_ms=compile_s * 1e3, link_latency_ms=link_s * 1e3,
                            requested_cache_keys=keys, compiled_blocks=compiles, llm_calls=1,
                            prompt_tokens=(resp.get("usage") or {}).get("prompt_tokens"),
                            output_tokens=(resp.get("usage") or {}).get("completion_tokens"))
            self.recorder.record(m)
        return _text_of(resp)

    def count_tokens(self, messages: Sequence[dict]) -> int:
        """Estimate (characters / 4) for the agent's context accounting."""
        return sum(len(str(m.get("content") or "")) for m in messages) // 4 + 1


# --------------------------------------------------------------- NOC client
class NOCLLM:
    """``call(prompt, message_history)`` through the host pipeline."""

    def __init__(self, pipeline, *, recorder: Optional[MetricsRecorder] = None, agent_id: str = "noc-llm",
                 variant: str = "selected_context_radixcache_legolink"):
        from .adapter import PipelineRoute

        self.pipeline = pipeline
        self.recorder = recorder
        self.agent_id, self.variant = agent_id, variant
        self.route = PipelineRoute.SELECTED_CONTEXT_LEGOLINK
        self.registry = PromptRegistry()
        self._declared: Optional[tuple] = None
        self.turn = 0
        self.last_structure: dict = {}

    def declare_prompt_structure(self, parts: Optional[Sequence[PromptPart]]) -> None:
        """The agent says how it assembled the NEXT prompt (checked against it)."""
        self._declared = tuple(parts) if parts else None

    def turn_events(self, prompt: str, history: Sequence[Any]) -> list:
        held = self.pipeline.manager.collector.events()
        events, self.last_structure = terminus_turn_events(
            prompt, history, ledger=SourceLedger.from_events(held), registry=self.registry, declared=self._declared,
            first_turn=not held)
        self._declared = None
        return events

    def call(self, prompt: str, message_history: Optional[Sequence[Any]] = None, **kw) -> str:
        self.turn += 1
        events = self.turn_events(prompt, message_history or [])
        t0 = time.perf_counter()
        error, ex = None, None
        try:
            ex = self.pipeline.execute(events, route=self.route, query=prompt[-2000:])
        except Exception as e:  # noqa: BLE001 - a failed turn still leaves a row
            error = f"{type(e).__name__}: {e}"
        if self.recorder is not None:
            m = AgentMetric(task_id=self.pipeline.manager.task_id, agent_id=self.agent_id,
                            request_id=uuid.uuid4().hex[:16],
                            session_revision=int(self.pipeline.manager.collector.revision), loop_stage="act",
                            objective=prompt[:200], variant=self.variant, operation_mode=self.route.value,
                            e2e_latency_ms=(time.perf_counter() - t0) * 1e3, llm_calls=1, error=error,
                            compile_requests=ex.compile_requests if ex else None)
            row = m.to_dict()
            row["ingress_structure"] = dict(self.last_structure)
            self.recorder.record(row)
        if ex is None:
            raise RuntimeError(error)
        return ex.result.text


# ------------------------------------------------------------- terminals
class TerminalSession(Protocol):
    def send_keys(self, keys: str, *, block: bool = False, timeout_sec: float = 180.0) -> None: ...

    def capture(self) -> str: ...


class SubprocessTerminal:
    """Runs each command line in a local shell (bounded by its timeout) and
    keeps the transcript."""

    def __init__(self, cwd: Optional[str] = None, shell: str = "/bin/bash"):
        self.cwd, self.shell = cwd, shell
        self.transcript = ""

    def send_keys(self, keys: str, *, block: bool = False, timeout_sec: float = 180.0) -> None:
        cmd = keys.rstrip("\n")
        if not cmd.strip():
            return
        try:
            r = subprocess.run([self.shell, "-lc", cmd], cwd=self.cwd, capture_output=True, text=True,
                               timeout=max(1.0, float(timeout_sec)))
            out = r.stdout + r.stderr
        except subprocess.TimeoutExpired as e:
            out = f"{e.stdout or ''}{e.stderr or ''}\n[command timed out after {timeout_sec}s]\n"
        self.transcript += f"$ {cmd}\n{out}"

    def capture(self) -> str:
        return self.transcript


class TmuxSessionAdapter:
    """Any object with terminal-bench's ``send_keys(keys, block=...,
    max_timeout_sec=...)`` and ``capture_pane()`` as a :class:`TerminalSession`."""

    def __init__(self, session: Any):
        self.session = session

    def send_keys(self, keys: str, *, block: bool = False, timeout_sec: float = 180.0) -> None:
        self.session.send_keys(keys, block=block, max_timeout_sec=timeout_sec)

    def capture(self) -> str:
        return self.session.capture_pane()


# ------------------------------------------------------------ the agent
@dataclass
class AgentCommand:
    keystrokes: str
    is_blocking: bool = False
    timeout_sec: float = 180.0


@dataclass
class AgentResponse:
    commands: list
    is_task_complete: bool
    raw: str


@dataclass
class AgentResult:
    steps: int
    is_task_complete: bool
    failure_mode: str  # "none" | "max_steps" | "repeated_actions" | "invalid_responses" | "llm_error"
    commands_run: int
    invalid_responses: int
    repeated_action_count: int
    transcript: list = field(default_factory=list)


_FENCE = re.compile(r"```(?:json)?\s*(\{.*\})\s*```", re.S)


def parse_agent_response(text: str) -> AgentResponse:
    """The model's JSON answer (bare, or in a code fence); ValueError if it
    is not an object with a ``commands`` list of keystroke objects."""
    m = _FENCE.search(text)
    body = m.group(1) if m else text[text.find("{"): text.rfind("}") + 1]
    data = json.loads(body)
    if not isinstance(data, dict) or not isinstance(data.get("commands", []), list):
        raise ValueError("the answer must be a JSON object with a commands list")
    cmds = []
    for c in data.get("commands", []):
        if not isinstance(c, dict) or not isinstance(c.get("keystrokes"), str):
            raise ValueError("each command needs a keystrokes string")
        cmds.append(AgentCommand(c["keystrokes"], bool(c.get("is_blocking", False)),
                                 float(c.get("timeout_sec", 180.0))))
    return AgentResponse(cmds, bool(data.get("is_task_complete", False)), text)


INSTRUCTION_TEMPLATE = (
    "You operate a Linux terminal to complete the task below. Answer ONLY with a JSON object: "
    '{{"commands": [{{"keystrokes": "<command>\\n", "is_blocking": true, "timeout_sec": 60}}], '
    '"is_task_complete": false}}. Set is_task_complete to true when the task is done.\n\nTask:\n{instruction}\n\n'
    "Current terminal state:\n{terminal}")
OBSERVATION_DIRECTIVE = "Output of your last commands:\n"
OBSERVATION_TAIL = "\n\nWhat next? Answer with the JSON object only."
INVALID_DIRECTIVE = "Your last answer was not valid ({error}). Answer with the JSON object only."


class TerminalAgent:
    """Terminus-style loop over an LLM with ``call(prompt, message_history)``."""

    declare_structure = False

    def __init__(self, llm, *, max_steps: int = 50, max_output_chars: int = 6000, max_invalid: int = 3,
                 max_repeats: int = 3):
        self.llm = llm
        self.max_steps, self.max_output_chars = max_steps, max_output_chars
        self.max_invalid, self.max_repeats = max_invalid, max_repeats

    @staticmethod
    def name() -> str:
        return "legolink-terminal-agent"

    def _compact(self, out: str) -> str:
        out = out.strip()
        if len(out) <= self.max_output_chars:
            return out
        half = self.max_output_chars // 2
        return out[:half] + "\n[... output truncated ...]\n" + out[-half:]

    def _declare(self, prompt: str, observation: str) -> None:
        if self.declare_structure and hasattr(self.llm, "declare_prompt_structure"):
            self.llm.declare_prompt_structure(split_around(prompt, observation,
                                                           needle_metadata={"tool_name": "terminal"}))

    def perform_task(self, instruction: str, session: TerminalSession) -> AgentResult:
        history: list = []
        prompt = INSTRUCTION_TEMPLATE.format(instruction=instruction, terminal=self._compact(session.capture()))
        invalid = repeats = ran = 0
        last_batch = None
        transcript = []
        for step in range(1, self.max_steps + 1):
            try:
                answer = self.llm.call(prompt, list(history))
            except Exception as e:  # noqa: BLE001
                return AgentResult(step, False, "llm_error", ran, invalid, repeats, transcript + [repr(e)[:500]])
            history += [{"role": "user", "content": prompt}, {"role": "assistant", "content": answer}]
            try:
                resp = parse_agent_response(answer)
            except (ValueError, json.JSONDecodeError) as e:
                invalid += 1
                if invalid > self.max_invalid:
                    return AgentResult(step, False, "invalid_responses", ran, invalid, repeats, transcript)
                prompt = INVALID_DIRECTIVE.format(error=str(e)[:200])
                continue
            batch = tuple((c.keystrokes, c.is_blocking) for c in resp.commands)
            repeats = repeats + 1 if (batch and batch == last_batch) else 0
            last_batch = batch
            if repeats >= self.max_repeats:
                return AgentResult(step, False, "repeated_actions", ran, invalid, repeats, transcript)
            for c in resp.commands:
                session.send_keys(c.keystrokes, block=c.is_blocking, timeout_sec=c.timeout_sec)
                ran += 1
                transcript.append(c.keystrokes)
            if resp.is_task_complete:
                return AgentResult(step, True, "none", ran, invalid, repeats, transcript)
            observation = self._compact(session.capture())
            prompt = OBSERVATION_DIRECTIVE + observation + OBSERVATION_TAIL
            self._declare(prompt, observation)
        return AgentResult(self.max_steps, False, "max_steps", ran, invalid, repeats, transcript)


class NOCTerminalAgent(TerminalAgent):
    """The loop on the host context manager (:class:`NOCLLM`)."""

    @staticmethod
    def name() -> str:
        return "legolink-noc-agent"


class NOCTerminus2Agent(NOCTerminalAgent):
    """As :class:`NOCTerminalAgent`, declaring every observation prompt as
    directive + tool output + directive, so terminal output is ingested as a
    tool result (its own namespace and cache key) and the directive alone is
    the user's request."""

    declare_structure = True

    @staticmethod
    def name() -> str:
        return "legolink-noc-terminus2-agent"


__all__ = ["PICLLM", "NOCLLM", "TerminalAgent", "NOCTerminalAgent", "NOCTerminus2Agent", "TerminalSession",
           "SubprocessTerminal", "TmuxSessionAdapter", "AgentCommand", "AgentResponse", "AgentResult",
           "parse_agent_response", "split_text", "KIND_AGENT_DIRECTIVE", "KIND_TOOL_OUTPUT"]
