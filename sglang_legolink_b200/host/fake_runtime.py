"""Runtimes for host tests without a GPU.

* :class:`StrictFakeRuntime` -- enforces the contract with no model: a
  Compile registers its tokens, a Link must name resident keys (else it
  aborts with the residency-recovery JSON), the runtime-owned fields are
  refused, and plain generation is refused.  ``evict_everything()`` is the
  fault injector (reference ``examples/strict_fake_runtime.py:25-93``).
* :class:`ServiceTransport` -- calls a real in-process
  :class:`~sglang_legolink_b200.server.http_server.RuntimeService` (the
  engine on CPU or GPU) and turns request-scoped rejections into
  :class:`~sglang_legolink_b200.host.adapter.TransportError`, exactly as the
  HTTP transport would.
* :func:`serve_callable` -- puts any ``payload -> response`` callable behind
  a local HTTP server, so the JSON transport is exercised too.
"""

from __future__ import annotations

import json
import threading
from http.server import BaseHTTPRequestHandler, ThreadingHTTPServer

from ..contract import (ContractError, residency_recovery_message, validate_physical_token_input,
                        validate_pic_link_request)
from .adapter import TransportError


class StrictFakeRuntime:
    def __init__(self):
        self.blocks: dict[str, list[int]] = {}
        self.requests: list[dict] = []
        self._lock = threading.Lock()

    def __call__(self, payload: dict) -> dict:
        with self._lock:
            self.requests.append(json.loads(json.dumps(payload)))
            sc, link = payload.get("sub_context"), payload.get("pic_link")
            if sc is not None and link is not None:
                raise TransportError("a request is either a Compile or a Link", 400)
            try:
                if sc is not None:
                    ids = validate_physical_token_input(sc, label="sub_context") or []
                    self.blocks[str(sc["cache_key"])] = ids
                    return _resp("", kind="compile")
                if link is not None:
                    validate_pic_link_request(dict(link), require_formal=False, allow_legacy_fields=False)
                    gone = [k for k in link["cache_keys"] if k not in self.blocks]
                    if gone:
                        raise TransportError(residency_recovery_message(missing=gone), 400)
                    n = sum(len(self.blocks[k]) for k in link["cache_keys"])
                    return _resp(f"linked {len(link['cache_keys'])} blocks ({n} tokens)", kind="link")
            except ContractError as e:
                raise TransportError(str(e), 400) from None
            raise TransportError("LegoLink-only runtime: plain generation is refused", 400)

    def evict_everything(self) -> list[str]:
        with self._lock:
            gone = list(self.blocks)
            self.blocks.clear()
            return gone

    def compile_requests(self, since: int = 0) -> list[dict]:
        return [r for r in self.requests[since:] if r.get("sub_context") is not None]

    def link_requests(self, since: int = 0) -> list[dict]:
        return [r for r in self.requests[since:] if r.get("pic_link") is not None]

    def plain_generation_requests(self) -> list[dict]:
        return [r for r in self.requests if r.get("sub_context") is None and r.get("pic_link") is None]


def _resp(text: str, **meta) -> dict:
    return {"object": "chat.completion", "choices": [{"index": 0, "message": {"role": "assistant", "content": text},
                                                      "finish_reason": "stop"}], "meta_info": meta}


class ServiceTransport:
    def __init__(self, service):
        self.service = service
        self.requests: list[dict] = []

    def __call__(self, payload: dict) -> dict:
        from ..runtime.scheduler import RequestRejected

        self.requests.append(payload)
        try:
            return self.service.complete(payload)
        except (RequestRejected, ContractError, ValueError) as e:
            raise TransportError(str(e), 400) from None

    def compile_requests(self, since: int = 0) -> list[dict]:
        return [r for r in self.requests[since:] if r.get("sub_context") is not None]


def serve_callable(fn, host: str = "127.0.0.1", port: int = 0) -> ThreadingHTTPServer:
    class H(BaseHTTPRequestHandler):
        protocol_version = "HTTP/1.1"

        def log_message(self, *a):
            pass

        def do_POST(self):
            n = int(self.headers.get("Content-Length") or 0)
            body = json.loads(self.rfile.read(n) or b"{}")
            try:
                out, code = fn(body), 200
            except TransportError as e:
                out, code = {"object": "error", "message": str(e)}, e.status or 400
            data = json.dumps(out).encode()
            self.send_response(code)
            self.send_header("Content-Type", "application/json")
            self.send_header("Content-Length", str(len(data)))
            self.end_headers()
            self.wfile.write(data)

    srv = ThreadingHTTPServer((host, port), H)
    threading.Thread(target=srv.serve_forever, daemon=True).start()
    return srv
