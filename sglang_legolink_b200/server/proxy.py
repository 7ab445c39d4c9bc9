"""OpenAI-compatible proxy in front of the host pipeline.

An agent framework talks plain OpenAI ``/v1/chat/completions`` to this proxy;
the proxy keeps one host session per conversation and turns every request
into a LegoLink turn (events -> plan -> Compile-on-miss -> Link) through
:class:`~sglang_legolink_b200.host.agent.AgentLLM`, writing one metric row
per turn.  Reference: ``terminal_bench_integration/noc_openai_proxy.py:470-779``
and ``proxy_sessions.py:117``.

* Session key: ``session_id`` in the body, else the ``X-Session-Id`` header,
  else a digest of the conversation's opening (its system messages and first
  user message), so a client that resends the growing conversation lands in
  the same session.
* JSON guardrail: when the request asks for a JSON response
  (``response_format`` json_object / json_schema), an output that does not
  parse is re-requested with a corrective user message, up to
  ``json_retries`` times (each retry is one more LegoLink turn in the same
  session); the response reports the attempts.
* Passthrough control arm (``--passthrough``): the request is forwarded
  unchanged to the runtime's native chat route; no host pipeline runs.
* Sessions idle longer than ``session_ttl_s`` are dropped (their runtime
  blocks stay resident until the runtime evicts them).
"""

from __future__ import annotations

import argparse
import hashlib
import json
import secrets
import threading
import time
import uuid
from http.server import BaseHTTPRequestHandler, ThreadingHTTPServer
from typing import Callable, Optional

from ..host.adapter import ResidencyRecoveryCoordinator, make_pipeline
from ..host.agent import AgentLLM
from ..host.metrics import MetricsRecorder
from ..host.namespaces import NamespacePolicy, NamespaceResolver
from ..host.planner import CacheCatalog


DERIVED_PREFIX = "derived-"


def normalize_model_name(model: str) -> str:
    """Strips a LiteLLM provider prefix ("openai/Qwen/..." -> "Qwen/...")."""
    m = str(model or "")
    return m[len("openai/"):] if m.startswith("openai/") else m


def message_content_to_text(content) -> str:
    """OpenAI message content as text: a string as is; a list of content
    parts as the newline-joined text of its text parts (image and other
    parts carry no text and are skipped)."""
    if content is None:
        return ""
    if isinstance(content, str):
        return content
    if isinstance(content, list):
        out = []
        for part in content:
            if isinstance(part, str):
                out.append(part)
            elif isinstance(part, dict):
                t = part.get("text", part.get("content"))
                if isinstance(t, str):
                    out.append(t)
        return "\n".join(out)
    return str(content)


def transcript_digest(messages: list) -> str:
    """sha256 of a transcript's (role, text) turns."""
    turns = [[str(m.get("role") or "user"), message_content_to_text(m.get("content"))] for m in messages]
    return hashlib.sha256(json.dumps(turns, separators=(",", ":"), ensure_ascii=False).encode()).hexdigest()


class TranscriptIndex:
    """Continuation of sessions that name no identity.  After each turn the
    proxy records the digest of the transcript it has seen, ending with its
    own reply; a later request continues that session only if its messages
    start with that whole transcript.  Knowing a conversation's opening
    prompt is therefore not enough to join it (the opening prompt is task
    text, not a capability): the caller must present every earlier turn,
    including the replies this proxy gave.  Bounded LRU."""

    def __init__(self, max_entries: int = 4096):
        self.max_entries = max_entries
        self._by_digest: dict = {}
        self._lock = threading.Lock()

    def remember(self, key: str, transcript: list) -> None:
        with self._lock:
            self._by_digest.pop(transcript_digest(transcript), None)
            self._by_digest[transcript_digest(transcript)] = key
            while len(self._by_digest) > self.max_entries:
                self._by_digest.pop(next(iter(self._by_digest)))

    def continuation(self, messages: list) -> Optional[str]:
        """The session whose recorded transcript is the longest prefix of
        ``messages`` ending with an assistant turn, if any."""
        with self._lock:
            for i in range(len(messages) - 1, -1, -1):
                if messages[i].get("role") == "assistant":
                    key = self._by_digest.get(transcript_digest(messages[: i + 1]))
                    if key is not None:
                        return key
        return None


class SessionRegistry:
    """session key -> (AgentLLM, last use); built lazily by ``factory``."""

    def __init__(self, factory: Callable[[str], AgentLLM], ttl_s: float = 3600.0, max_sessions: int = 1024):
        self.factory = factory
        self.ttl_s = ttl_s
        self.max_sessions = max_sessions
        self._sessions: dict = {}
        self._locks: dict = {}
        self._lock = threading.Lock()

    def get(self, key: str) -> tuple[AgentLLM, threading.Lock]:
        now = time.monotonic()
        with self._lock:
            self._expire(now)
            ent = self._sessions.get(key)
            if ent is None:
                if len(self._sessions) >= self.max_sessions:
                    oldest = min(self._sessions, key=lambda k: self._sessions[k][1])
                    self._sessions.pop(oldest)
                    self._locks.pop(oldest, None)
                ent = [self.factory(key), now]
                self._sessions[key] = ent
                self._locks[key] = threading.Lock()
            ent[1] = now
            return ent[0], self._locks[key]

    def _expire(self, now: float) -> None:
        for k in [k for k, v in self._sessions.items() if now - v[1] > self.ttl_s]:
            self._sessions.pop(k)
            self._locks.pop(k, None)

    def __len__(self) -> int:
        return len(self._sessions)


def wants_json(payload: dict) -> bool:
    rf = payload.get("response_format") or {}
    return isinstance(rf, dict) and rf.get("type") in ("json_object", "json_schema")


def parses_as_json(text: str) -> bool:
    t = text.strip()
    if t.startswith("```"):
        t = t.strip("`")
        t = t[t.find("\n") + 1:] if "\n" in t else t
    try:
        json.loads(t)
        return True
    except (ValueError, TypeError):
        return False


JSON_REPAIR_INSTRUCTION = ("Your previous reply was not valid JSON. Reply again with only one JSON value, "
                           "no prose and no code fences.")


class LegoLinkProxy:
    def __init__(self, transport, *, model: str = "legolink", tokenizer=None, repair_tokens: int = 16,
                 metrics_path: Optional[str] = None, passthrough: bool = False, json_retries: int = 2,
                 session_ttl_s: float = 3600.0, namespace_mode: str = "global", cross_namespace_pairs=(),
                 command_guardrail: bool = False):
        # command_guardrail: terminal-agent replies whose keystrokes break a
        # rule of host/command_guardrail.py are re-asked (json_retries times),
        # then replaced by a parser-safe diagnostic reply
        self.command_guardrail = command_guardrail
        self.transport = transport
        self.model = model
        self.tokenizer = tokenizer
        self.repair_tokens = repair_tokens
        # one view of the runtime's blocks for every session (the namespace
        # resolver reads it across tasks); the mode is checked here
        self.resolver = NamespaceResolver(namespace_mode,
                                          NamespacePolicy(cross_namespace_pairs=list(cross_namespace_pairs)))
        self.catalog = CacheCatalog()
        self.coordinator = ResidencyRecoveryCoordinator()
        self.recorder = MetricsRecorder(metrics_path) if metrics_path else None
        self.passthrough = passthrough
        self.json_retries = json_retries
        self.sessions = SessionRegistry(self._new_session, ttl_s=session_ttl_s)
        self.transcripts = TranscriptIndex()
        self.stats = {"requests": 0, "json_retries": 0, "passthrough": 0}

    def _new_session(self, key: str) -> AgentLLM:
        pipe = make_pipeline(self.transport, task_id=key, model=self.model, tokenizer=self.tokenizer,
                             catalog=self.catalog, coordinator=self.coordinator, resolver=self.resolver,
                             repair_tokens=self.repair_tokens)
        return AgentLLM(pipe, task_id=key, recorder=self.recorder)

    def session_key(self, payload: dict, headers: Optional[dict] = None) -> str:
        """An explicit identity (``session_id`` field, ``X-Session-Id``
        header, or the OpenAI ``user`` field) gives a stable key; otherwise
        the request continues the session whose whole transcript it repeats,
        or gets a fresh opaque key.  Never derived from message content."""
        hdr = {str(k).lower(): v for k, v in (headers or {}).items()}
        explicit = payload.get("session_id") or hdr.get("x-session-id")
        if explicit:
            return str(explicit)
        if payload.get("user"):
            return "user:" + str(payload["user"])
        cont = self.transcripts.continuation(list(payload.get("messages") or []))
        return cont if cont is not None else DERIVED_PREFIX + secrets.token_hex(12)

    def chat_completion(self, payload: dict, headers: Optional[dict] = None) -> dict:
        self.stats["requests"] += 1
        if self.passthrough:
            self.stats["passthrough"] += 1
            return self.transport(dict(payload))
        key = self.session_key(payload, headers)
        agent, lock = self.sessions.get(key)
        messages = list(payload.get("messages") or [])
        tools = payload.get("tools")
        attempts = 0
        with lock:  # one turn at a time per session: the host session is not reentrant
            res = agent.call(messages, tools)
            text = res.text
            attempts = 1
            while wants_json(payload) and not parses_as_json(text) and attempts <= self.json_retries:
                self.stats["json_retries"] += 1
                messages = messages + [{"role": "assistant", "content": text},
                                       {"role": "user", "content": JSON_REPAIR_INSTRUCTION}]
                res = agent.call(messages, tools, loop_stage="replan")
                text = res.text
                attempts += 1
            if self.command_guardrail:
                from ..host.command_guardrail import command_violation, replan_prompt, safe_diagnostic_response

                retries = 0
                violation = command_violation(text)
                while violation is not None and retries < self.json_retries:
                    self.stats["guardrail_replans"] = self.stats.get("guardrail_replans", 0) + 1
                    messages = messages + [{"role": "assistant", "content": text},
                                           {"role": "user", "content": replan_prompt(violation)}]
                    res = agent.call(messages, tools, loop_stage="replan")
                    text = res.text
                    attempts += 1
                    retries += 1
                    violation = command_violation(text)
                if violation is not None:
                    self.stats["guardrail_blocked"] = self.stats.get("guardrail_blocked", 0) + 1
                    text = safe_diagnostic_response(violation)
                else:
                    from ..host.command_guardrail import inject_verification

                    # commands that change files silently print what they changed
                    text, probed = inject_verification(text)
                    if probed is not None:
                        self.stats["verification_probes"] = self.stats.get("verification_probes", 0) + 1
        self.transcripts.remember(key, list(payload.get("messages") or []) + [{"role": "assistant", "content": text}])
        usage = (res.execution.result.response or {}).get("usage") or {}
        return {"id": "chatcmpl-" + uuid.uuid4().hex[:24], "object": "chat.completion", "created": int(time.time()),
                "model": normalize_model_name(payload.get("model") or self.model),
                "choices": [{"index": 0, "message": {"role": "assistant", "content": text},
                             "finish_reason": "stop"}],
                "usage": usage,
                "legolink": {"session": key, "attempts": attempts,
                             "compile_requests": res.execution.compile_requests,
                             "reused_tokens": res.metric.get("reused_tokens"),
                             "route": res.execution.route.value}}


def make_handler(proxy: LegoLinkProxy):
    class Handler(BaseHTTPRequestHandler):
        protocol_version = "HTTP/1.1"

        def log_message(self, *a):
            pass

        def _send(self, code: int, body: dict):
            data = json.dumps(body).encode()
            self.send_response(code)
            self.send_header("Content-Type", "application/json")
            self.send_header("Content-Length", str(len(data)))
            self.end_headers()
            self.wfile.write(data)

        def do_GET(self):
            if self.path in ("/health", "/v1/models"):
                self._send(200, {"status": "ok", "sessions": len(proxy.sessions), "stats": proxy.stats,
                                 "data": [{"id": proxy.model, "object": "model"}]})
            else:
                self._send(404, {"error": "not found"})

        def do_POST(self):
            n = int(self.headers.get("Content-Length") or 0)
            try:
                payload = json.loads(self.rfile.read(n) or b"{}")
            except json.JSONDecodeError:
                self._send(400, {"error": {"message": "invalid JSON body"}})
                return
            if self.path != "/v1/chat/completions":
                self._send(404, {"error": {"message": f"unknown route {self.path}"}})
                return
            if payload.get("stream"):
                self._send(400, {"error": {"message": "the proxy answers non-streamed completions only"}})
                return
            try:
                self._send(200, proxy.chat_completion(payload, dict(self.headers)))
            except Exception as e:  # the proxy stays up; the request fails closed
                self._send(502, {"error": {"message": f"{type(e).__name__}: {e}"}})

    return Handler


def serve(proxy: LegoLinkProxy, host: str = "127.0.0.1", port: int = 8100) -> ThreadingHTTPServer:
    srv = ThreadingHTTPServer((host, port), make_handler(proxy))
    threading.Thread(target=srv.serve_forever, daemon=True).start()
    return srv


def main():
    from ..host.adapter import JSONHTTPTransport

    ap = argparse.ArgumentParser(description="OpenAI-compatible LegoLink proxy")
    ap.add_argument("--runtime", default="http://127.0.0.1:30000/v1", help="LegoLink runtime API base (.../v1)")
    ap.add_argument("--host", default="127.0.0.1")
    ap.add_argument("--port", type=int, default=8100)
    ap.add_argument("--repair-tokens", type=int, default=16)
    ap.add_argument("--metrics", default=None, help="metrics JSONL path")
    ap.add_argument("--passthrough", action="store_true", help="control arm: forward requests unchanged")
    ap.add_argument("--json-retries", type=int, default=2)
    ap.add_argument("--command-guardrail", action="store_true",
                    help="re-ask, then block, terminal-agent replies whose keystrokes break a guardrail rule")
    ap.add_argument("--semantic-cache-namespace-mode", default="global",
                    choices=["global", "hard_namespace", "logical_namespace"])
    ap.add_argument("--cross-namespace-pairs", default="",
                    help="logical mode: comma-separated requester->serving root pairs, e.g. workspace<->tool_output")
    a = ap.parse_args()
    from ..host.tokenizer import RuntimeTokenizer

    transport = JSONHTTPTransport(a.runtime)
    proxy = LegoLinkProxy(transport, tokenizer=RuntimeTokenizer(a.runtime), repair_tokens=a.repair_tokens,
                          metrics_path=a.metrics, passthrough=a.passthrough, json_retries=a.json_retries,
                          namespace_mode=a.semantic_cache_namespace_mode,
                          cross_namespace_pairs=[x for x in a.cross_namespace_pairs.split(",") if x.strip()],
                          command_guardrail=a.command_guardrail)
    srv = ThreadingHTTPServer((a.host, a.port), make_handler(proxy))
    print(f"LegoLink proxy on http://{a.host}:{a.port} -> {a.runtime}", flush=True)
    srv.serve_forever()


if __name__ == "__main__":
    main()
