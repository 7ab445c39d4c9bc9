"""OpenAI-compatible HTTP runtime with the Compile / Link contract.

Endpoints (reference ``patched_sglang_files/python/sglang/srt/entrypoints/
http_server.py``, ``openai/protocol.py:696-709``, ``serving_chat.py:397-423``):

* ``POST /v1/chat/completions`` -- body fields ``sub_context`` (a Compile),
  ``pic_link`` (a Link) and ``extra_key``; ``stream: true`` answers with SSE
  (``data: {...}`` chunks, ``data: [DONE]``; an error mid-stream is an
  ``error`` frame).  A plain chat request is refused in LegoLink-only mode.
* ``POST /v1/completions`` -- the same over a text/ids prompt.
* ``POST /v1/tokenize`` -- ``prompt`` (text) or ``messages`` (+ ``tools``,
  ``add_generation_prompt``, ``continue_final_message``) with the model's
  chat template -> ``{"tokens": [...], "count": n}``; the host's
  authoritative tokenizer.
* ``GET /v1/models``, ``GET /model_info``, ``GET /health``,
  ``POST /start_profile`` / ``/stop_profile`` (torch profiler window).

``--tp-size`` / ``--dp-size`` start one process per GPU (``server/launch.py``).

Startup warmup sends one Compile and one Link (a plain-generation warmup
would be refused by a LegoLink-only server), reference
``pic_runtime.py:1381-1508``.
"""

from __future__ import annotations

import argparse
import itertools
import json
import os
import threading
import time
import uuid
from http.server import BaseHTTPRequestHandler, ThreadingHTTPServer
from typing import Any, Optional

from ..contract import (ContractError, physical_token_ids_sha256, validate_physical_token_input,
                        validate_pic_link_request)
from ..runtime.scheduler import Request, RequestRejected, Scheduler
from ..runtime.sampling import SamplingParams


def asks_input_logprobs(payload: dict) -> bool:
    """Whether a request asks for log-probabilities of its INPUT tokens: the
    OpenAI completions form (``echo`` with ``logprobs``), an explicit
    ``input_logprobs``, or the native form (``return_logprob`` with a
    ``logprob_start_len`` >= 0; -1, the default, asks for output tokens
    only).  A Link's input rows are linked, not computed, so it has none
    (reference ``tests/test_security_l1_link_input_logprobs.py``)."""
    if payload.get("input_logprobs"):
        return True
    if payload.get("echo") and payload.get("logprobs"):
        return True
    start = payload.get("logprob_start_len")
    if payload.get("return_logprob") and start is not None:
        try:
            return int(start) >= 0
        except (TypeError, ValueError):
            return True  # unreadable: treated as asking
    return False


def _prompt_ids(tokenizer, payload: dict) -> list[int]:
    msgs = payload.get("messages") or []
    return list(tokenizer.tokenize_messages(msgs, tools=payload.get("tools"),
                                            chat_template_kwargs=payload.get("chat_template_kwargs")))


class RuntimeService:
    """Turns API payloads into scheduler requests (no HTTP here, so tests and
    in-process hosts call it directly)."""

    def __init__(self, scheduler: Scheduler, tokenizer, model_name: str = "default"):
        self.scheduler = scheduler
        self.tokenizer = tokenizer
        self.model_name = model_name
        self.eos = getattr(tokenizer, "eos_token_id", None)
        self._profiler = None

    def build_request(self, payload: dict) -> Request:
        import copy

        # The runtime publishes its resolved plan into the pic_link dict; work
        # on a copy so an in-process caller's payload is never modified.
        sc, link = copy.deepcopy(payload.get("sub_context")), copy.deepcopy(payload.get("pic_link"))
        if sc is not None and link is not None:
            raise RequestRejected("a request is either a Compile (sub_context) or a Link (pic_link), not both")
        if link is not None and asks_input_logprobs(payload):
            raise RequestRejected("a Link may not request input logprobs: its input rows are linked, not computed")
        max_new = int(payload.get("max_tokens") or payload.get("max_completion_tokens") or 16)
        stop = (self.eos,) if (self.eos is not None and not payload.get("ignore_eos")) else ()
        stop = stop + tuple(int(t) for t in (payload.get("stop_token_ids") or ()))
        sampling = SamplingParams.from_request(payload)
        rid = str(payload.get("rid") or (link or {}).get("request_id") or uuid.uuid4().hex[:16])
        if sc is not None:
            if not isinstance(sc, dict):
                raise RequestRejected("sub_context must be an object")
            ids = validate_physical_token_input(sc, label="sub_context")
            if ids is None:
                ids = _prompt_ids(self.tokenizer, payload)
            return Request("compile", rid, ids, 1, stop, sub_context=sc)
        if link is not None:
            # the request contract is checked on arrival (a copy: the engine
            # checks it again against its own state)
            validate_pic_link_request(copy.deepcopy(link))
            if isinstance(link, dict) and link.get("physical_token_layout_version") is not None:
                ids = validate_physical_token_input(link, label="pic_link")
            else:
                ids = _prompt_ids(self.tokenizer, payload)
            return Request("link", rid, list(ids or []), max_new, stop, pic_link=link, sampling=sampling)
        if "prompt" in payload:
            p = payload["prompt"]
            ids = list(p) if isinstance(p, list) else list(self.tokenizer.tokenize(str(p)))
        else:
            ids = _prompt_ids(self.tokenizer, payload)
        return Request("plain", rid, ids, max_new, stop, sampling=sampling)

    def complete(self, payload: dict) -> dict:
        req = self.build_request(payload)
        t0 = time.perf_counter()
        out = self.scheduler.run_sync(req)
        toks = out["tokens"]
        text = self.tokenizer.decode(toks) if hasattr(self.tokenizer, "decode") else ""
        choice = {"index": 0, "message": {"role": "assistant", "content": text}, "finish_reason": out.get(
            "finish_reason", "length")}
        return {"id": f"chatcmpl-{req.rid}", "object": "chat.completion", "created": int(time.time()),
                "model": self.model_name, "choices": [choice],
                "usage": {"prompt_tokens": len(req.input_ids), "completion_tokens": len(toks),
                          "total_tokens": len(req.input_ids) + len(toks)},
                "meta_info": {"output_ids": toks, "ttft_s": out.get("ttft_s"), "e2e_s": time.perf_counter() - t0,
                              "kind": req.kind, **({"compile": out["compile"]} if "compile" in out else {}),
                              **({"link": out["link"]} if "link" in out else {})}}

    def stream(self, payload: dict):
        """Yields SSE chunk dicts.  Arrival refusals (the request contract,
        the scheduler's arrival checks) raise RequestRejected / ContractError
        when the generator first runs, before any chunk."""
        req = self.build_request(payload)
        self.scheduler.check(req)
        self.scheduler.submit(req)
        cid = f"chatcmpl-{req.rid}"
        while True:
            kind, val = req.events.get(timeout=600)
            if kind == "token":
                text = self.tokenizer.decode([val]) if hasattr(self.tokenizer, "decode") else ""
                yield {"id": cid, "object": "chat.completion.chunk", "model": self.model_name,
                       "choices": [{"index": 0, "delta": {"content": text}, "finish_reason": None}],
                       "meta_info": {"token_id": val}}
            elif kind == "done":
                yield {"id": cid, "object": "chat.completion.chunk", "model": self.model_name,
                       "choices": [{"index": 0, "delta": {}, "finish_reason": val.get("finish_reason")}]}
                return
            else:
                yield {"error": {"message": str(val), "type": "legolink_request_failed"}}
                return

    def tokenize(self, payload: dict) -> dict:
        if "messages" in payload:
            ids = self.tokenizer.tokenize_messages(
                payload["messages"], tools=payload.get("tools"),
                continue_final_message=bool(payload.get("continue_final_message")),
                chat_template_kwargs=payload.get("chat_template_kwargs"),
                **({"add_generation_prompt": payload["add_generation_prompt"]}
                   if "add_generation_prompt" in payload else {}))
        else:
            ids = self.tokenizer.tokenize(str(payload.get("prompt", "")))
        ids = [int(i) for i in ids]
        return {"tokens": ids, "count": len(ids), "max_model_len": self.scheduler.max_context}

    def model_info(self) -> dict:
        eng = self.scheduler.engine
        return {"model_path": self.model_name, "model_config": eng.cfg.to_hf_dict(),
                "tokenizer_fingerprint": self.tokenizer.fingerprint,
                "chat_template_sha256": getattr(self.tokenizer, "chat_template_sha256", None),
                "eos_token_id": self.eos, "legolink_only": self.scheduler.legolink_only,
                "page_size": eng.page_size, "kv_pages": eng.kv.num_pages,
                "legolink_stats": eng.registry.stats(), "engine_stats": eng.stats}

    def warmup(self, block_tokens: int = 256, k: int = 16) -> dict:
        """One Compile + one Link of synthetic tokens (LegoLink-only safe)."""
        vocab = self.scheduler.engine.cfg.vocab_size
        ids = [(7 * i + 3) % max(2, vocab - 8) + 1 for i in range(block_tokens)]
        key = "legolink-warmup-" + physical_token_ids_sha256(ids)[:16]
        sc = {"cache_key": key, "physical_token_layout_version": "noc-single-chat-template-split-v1",
              "physical_input_ids": ids, "physical_token_count": len(ids),
              "physical_token_ids_sha256": physical_token_ids_sha256(ids)}
        t0 = time.perf_counter()
        self.complete({"messages": [], "sub_context": sc, "max_tokens": 1})
        t1 = time.perf_counter()
        self.complete({"messages": [{"role": "user", "content": "warmup"}], "max_tokens": 8, "ignore_eos": True,
                       "pic_link": {"cache_keys": [key], "recompute_initial_tokens": k, "request_id": "warmup"}})
        return {"compile_s": t1 - t0, "link_s": time.perf_counter() - t1}


def make_handler(svc: RuntimeService):
    class Handler(BaseHTTPRequestHandler):
        protocol_version = "HTTP/1.1"

        def log_message(self, *a):
            pass

        def _json(self, code: int, body: dict) -> None:
            data = json.dumps(body).encode()
            self.send_response(code)
            self.send_header("Content-Type", "application/json")
            self.send_header("Content-Length", str(len(data)))
            self.end_headers()
            self.wfile.write(data)

        def _body(self) -> dict:
            n = int(self.headers.get("Content-Length") or 0)
            return json.loads(self.rfile.read(n) or b"{}")

        def do_GET(self):
            if self.path.rstrip("/") in ("/health", "/health_generate"):
                return self._json(200, {"status": "ok"})
            if self.path.rstrip("/") == "/v1/models":
                return self._json(200, {"object": "list", "data": [{"id": svc.model_name, "object": "model",
                                                                     "owned_by": "legolink-b200"}]})
            if self.path.rstrip("/") in ("/model_info", "/get_model_info"):
                return self._json(200, svc.model_info())
            return self._json(404, {"object": "error", "message": f"no route {self.path}"})

        def do_POST(self):
            try:
                body = self._body()
            except ValueError as e:
                return self._json(400, {"object": "error", "message": f"bad JSON: {e}"})
            path = self.path.rstrip("/")
            try:
                if path == "/v1/tokenize":
                    return self._json(200, svc.tokenize(body))
                if path == "/start_profile":
                    import torch

                    svc._profiler = torch.profiler.profile(profile_memory=bool(body.get("profile_memory")))
                    svc._profiler.__enter__()
                    return self._json(200, {"status": "profiling"})
                if path == "/stop_profile":
                    if svc._profiler is not None:
                        svc._profiler.__exit__(None, None, None)
                        out = body.get("output_path") or "legolink_profile.json"
                        svc._profiler.export_chrome_trace(out)
                        svc._profiler = None
                        return self._json(200, {"status": "saved", "path": out})
                    return self._json(400, {"object": "error", "message": "no profile running"})
                if path in ("/v1/chat/completions", "/v1/completions"):
                    if body.get("stream"):
                        return self._stream(body)
                    return self._json(200, svc.complete(body))
            except (RequestRejected, ContractError, ValueError) as e:
                return self._json(400, {"object": "error", "message": str(e), "type": "BadRequestError",
                                        "code": 400})
            return self._json(404, {"object": "error", "message": f"no route {self.path}"})

        def _stream(self, body: dict):
            gen = svc.stream(body)
            # the request is validated when the generator first runs: take the
            # first chunk before any header, so a refused request is a 400
            first = next(gen)
            self.send_response(200)
            self.send_header("Content-Type", "text/event-stream")
            self.send_header("Cache-Control", "no-cache")
            self.send_header("Connection", "close")
            self.end_headers()
            for chunk in itertools.chain((first,), gen):
                self.wfile.write(b"data: " + json.dumps(chunk).encode() + b"\n\n")
                self.wfile.flush()
            self.wfile.write(b"data: [DONE]\n\n")
            self.wfile.flush()
            self.close_connection = True

    return Handler


def serve(svc: RuntimeService, host: str = "127.0.0.1", port: int = 30000) -> ThreadingHTTPServer:
    srv = ThreadingHTTPServer((host, port), make_handler(svc))
    threading.Thread(target=srv.serve_forever, daemon=True).start()
    return srv


def build_service(model: str = "tiny-qwen2", *, device: str = "cpu", tokenizer: Optional[str] = None,
                  legolink_only: Optional[bool] = True, page_size: int = 16, num_pages: Optional[int] = None,
                  max_context: int = 32768, seed: int = 0, layerwise_markers: bool = False) -> RuntimeService:
    import torch

    from ..host.tokenizer import HashTokenizer, HFTokenizer
    from ..models.config import get_config
    from ..models.qwen import QwenModel
    from ..runtime.engine import Engine

    dtype = torch.bfloat16 if device.startswith("cuda") else torch.float32
    if os.path.isdir(model) and any(f.endswith(".safetensors") for f in os.listdir(model)):
        m = QwenModel.from_pretrained(model, device=device, dtype=dtype)
    else:
        m = QwenModel.random_init(get_config(model), seed=seed, device=device, dtype=dtype)
    if layerwise_markers:
        from ..utils.layer_markers import LayerMarkers

        m.markers = LayerMarkers(True)
    tok = HFTokenizer(tokenizer) if tokenizer else HashTokenizer(m.cfg.vocab_size, name=m.cfg.name)
    eng = Engine(m, page_size=page_size, num_pages=num_pages, max_context=max_context)
    sch = Scheduler(eng, legolink_only=legolink_only)
    sch.start()
    return RuntimeService(sch, tok, model_name=m.cfg.name)


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(description="LegoLink B200 runtime server")
    ap.add_argument("--model", default="tiny-qwen2", help="preset name or HF checkpoint directory")
    ap.add_argument("--tokenizer", default=None, help="HF tokenizer path (default: hash tokenizer)")
    ap.add_argument("--device", default="cuda:0")
    ap.add_argument("--host", default="127.0.0.1")
    ap.add_argument("--port", type=int, default=30000)
    ap.add_argument("--page-size", type=int, default=16)
    ap.add_argument("--context-length", type=int, default=32768)
    ap.add_argument("--allow-plain-generation", action="store_true",
                    help="serve plain generation too (default: SGLANG_PIC_LEGOLINK_ONLY, on unless set to 0)")
    ap.add_argument("--skip-warmup", action="store_true")
    ap.add_argument("--enable-layerwise-nvtx-marker", action="store_true",
                    help="LegoLink::Attention / FFN / LMHead / Sampling profiler regions and NVTX ranges")
    ap.add_argument("--tp-size", type=int, default=1, help="shard the model over this many GPUs (one process each)")
    ap.add_argument("--dp-size", type=int, default=1, help="replicas sharing one block directory (one GPU each)")
    ap.add_argument("--pp-size", type=int, default=1, help="pipeline parallelism: refused unless 1")
    ap.add_argument("--tp-comm", choices=("fused", "nccl"), default="fused",
                    help="TP boundary: fused NVLink kernels, or the collective library")
    ap.add_argument("--dp-base-port", type=int, default=0, help="replica r > 0 listens on this + r (default --port)")
    ap.add_argument("--dist-timeout", type=int, default=600, help="process-group timeout, seconds")
    ap.add_argument("--seed", type=int, default=0)
    a = ap.parse_args(argv)
    if a.tp_size > 1 or a.dp_size > 1 or a.pp_size != 1:
        from .launch import launch

        launch(a)
        return
    svc = build_service(a.model, device=a.device, tokenizer=a.tokenizer,
                        legolink_only=False if a.allow_plain_generation else None, page_size=a.page_size,
                        max_context=a.context_length, layerwise_markers=a.enable_layerwise_nvtx_marker)
    if not a.skip_warmup and os.getenv("SGLANG_PIC_WARMUP", "1") != "0":
        print("warmup", svc.warmup(int(os.getenv("SGLANG_PIC_WARMUP_BLOCK_TOKENS", "256")),
                                   int(os.getenv("SGLANG_PIC_WARMUP_LEGOLINK_K", "16"))), flush=True)
    srv = serve(svc, a.host, a.port)
    print(f"serving on http://{a.host}:{a.port}", flush=True)
    try:
        threading.Event().wait()
    except KeyboardInterrupt:
        srv.shutdown()


if __name__ == "__main__":
    main()
