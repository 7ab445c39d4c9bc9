#!/usr/bin/env python3
"""Compile -> Link -> decode walk-through of the host pipeline.

Five scripted agent turns drive the real host pipeline (events -> fields ->
segmentation -> sub-context store -> selection -> compile policy -> layout
feasibility -> Compile-on-miss + Link with residency recovery).  Then every
block is evicted from the runtime and the last turn shows the host
recovering them.

Runtimes:
  (default)      a strict fake runtime in this process (CPU, no model)
  --engine       the real engine in this process (tiny random Qwen2 on CPU,
                 or --device cuda:0 --model qwen2.5-7b on a GPU)
  --fake-http    the fake behind a local HTTP server (exercises the JSON transport)
"""

import argparse
import json
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from sglang_legolink_b200.contract import PIC_LINK_RUNTIME_OWNED_FIELDS  # noqa: E402
from sglang_legolink_b200.host.adapter import JSONHTTPTransport, RequestPipeline, RuntimeAdapter  # noqa: E402
from sglang_legolink_b200.host.fake_runtime import ServiceTransport, StrictFakeRuntime, serve_callable  # noqa: E402
from sglang_legolink_b200.host.framing import RepairWindowPlanner, UniformRepairWindow  # noqa: E402
from sglang_legolink_b200.host.manager import ContextManager  # noqa: E402
from sglang_legolink_b200.host.tokenizer import HashTokenizer  # noqa: E402

OBJECTIVE = "fix the failing parser test: run pytest, read the tool output, continue the conversation"
SCRIPT = [
    [("task_instruction", "task", "Fix the failing parser test. " * 40, {})],
    [("conversation_message", "assistant-1", "I will run the pytest tests first. " * 40, {"message_role": "assistant"})],
    [("tool_output", "pytest-1", "FAILED tests/test_parser.py::test_empty parser error " * 40, {})],
    [("conversation_message", "assistant-2", "The parser test fails on empty input, patching it now. " * 40,
      {"message_role": "assistant"}),
     ("tool_output", "pytest-2", "PASSED tests/test_parser.py::test_empty parser fixed " * 40, {})],
    [],
]


def run(transport, tokenizer, counter, k=16, max_tokens=8):
    cm = ContextManager("example-task", tokenizer=tokenizer)
    ad = RuntimeAdapter(transport, model="legolink", tokenizer=tokenizer,
                        repair_planner=RepairWindowPlanner(UniformRepairWindow(k)),
                        generation={"max_tokens": max_tokens, "temperature": 0.0})
    pipe = RequestPipeline(cm, ad)
    report = []
    for i, events in enumerate(SCRIPT):
        seen = counter()
        ex = pipe.execute(events, query=OBJECTIVE)
        link = ex.result.audit or {}
        row = ex.metrics_row()
        report.append({"turn": i + 1, "compile_requests": ex.compile_requests,
                       "reused_tokens": row["reuse_accounting"]["reused_tokens"],
                       "linked_blocks": len(ex.layout.link_segments) if ex.layout else 0,
                       "output": ex.result.text[:60]})
    return pipe, report


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--engine", action="store_true")
    ap.add_argument("--fake-http", action="store_true")
    ap.add_argument("--device", default="cpu")
    ap.add_argument("--model", default="tiny-qwen2")
    a = ap.parse_args()
    fake = None
    server = None
    if a.engine:
        from sglang_legolink_b200.server.http_server import build_service

        svc = build_service(a.model, device=a.device, num_pages=4096 if a.device == "cpu" else None)
        tok = svc.tokenizer
        transport = ServiceTransport(svc)
        counter = lambda: len(transport.requests)  # noqa: E731
    else:
        fake = StrictFakeRuntime()
        tok = HashTokenizer(1024)
        transport = fake
        if a.fake_http:
            server = serve_callable(fake)
            transport = JSONHTTPTransport(f"http://127.0.0.1:{server.server_address[1]}/v1")
        counter = lambda: len(fake.requests)  # noqa: E731
    pipe, report = run(transport, tok, counter)
    log = fake.requests if fake else transport.requests
    owned = sorted({f for r in log if r.get("pic_link") for f in r["pic_link"]} & PIC_LINK_RUNTIME_OWNED_FIELDS)
    # evict everything in the runtime, then replay the last turn: the host recovers
    if fake is not None:
        gone = fake.evict_everything()
    else:
        eng = svc.scheduler.engine
        gone = eng.registry.keys()
        eng.registry.clear()
    before = counter()
    ex = pipe.execute([], query=OBJECTIVE + " (after the runtime evicted everything)")
    rec = ex.result.recovery
    out = {"turns": report, "runtime_owned_fields_on_the_wire": owned,
           "after_eviction": {"blocks_evicted": len(gone), "outcome": rec.get("outcome"),
                              "recovered_cache_keys": len(rec.get("recovered_cache_keys", [])),
                              "compile_requests_sent": sum(1 for r in log[before:] if r.get("sub_context")),
                              "plain_generation_requests_ever_sent": sum(
                                  1 for r in log if r.get("sub_context") is None and r.get("pic_link") is None)}}
    print(json.dumps(out, indent=1))
    ok = (not owned and out["after_eviction"]["outcome"] == "recovered_after_source_missing"
          and out["after_eviction"]["plain_generation_requests_ever_sent"] == 0)
    if server is not None:
        server.shutdown()
    return 0 if ok else 1


if __name__ == "__main__":
    sys.exit(main())
