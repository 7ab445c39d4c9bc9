"""Metric rows and aggregation, host timing, the agent-turn wrapper, replay,
and the OpenAI-compatible proxy (sessions, JSON guardrail, passthrough arm)
against the strict fake runtime (CPU, no model)."""

import json
import urllib.request

import pytest

from sglang_legolink_b200.host.adapter import RequestPipeline, RuntimeAdapter
from sglang_legolink_b200.host.agent import AgentLLM, ReplayDriver
from sglang_legolink_b200.host.fake_runtime import StrictFakeRuntime
from sglang_legolink_b200.host.framing import RepairWindowPlanner, UniformRepairWindow
from sglang_legolink_b200.host.manager import ContextManager
from sglang_legolink_b200.host.metrics import (AgentMetric, MetricsRecorder, aggregate_agent_steps,
                                               aggregate_experiment, compute_stream_metrics, formal_rows,
                                               percentile, read_jsonl, summary_stats)
from sglang_legolink_b200.host.profiling import HostTimingRecorder, NcuRunConfig, ProfilerWindowConfig
from sglang_legolink_b200.host.tokenizer import HashTokenizer
from sglang_legolink_b200.server.proxy import LegoLinkProxy, parses_as_json, serve


def test_percentile_and_summary():
    assert percentile([], 0.5) is None
    assert percentile([3.0], 0.95) == 3.0
    assert percentile([1, 2, 3, 4], 0.5) == 2.5
    assert percentile(list(range(101)), 0.95) == pytest.approx(95.0)
    s = summary_stats([1, None, 3])
    assert s["sample_count"] == 2 and s["p50"] == 2.0 and s["min"] == 1.0


def test_metric_row_ratios_and_aggregation(tmp_path):
    rec = MetricsRecorder(tmp_path / "m.jsonl")
    for i in range(4):
        m = AgentMetric(task_id="t", agent_id="a", request_id=str(i), session_revision=i, loop_stage="act",
                        objective="o", variant="selected_context_radixcache_legolink", operation_mode="link",
                        reused_tokens=300, recomputed_tokens=100, full_session_tokens=1000,
                        selected_context_tokens=400, request_latency_ms=10.0 * (i + 1), e2e_latency_ms=20.0,
                        agent_steps=1, task_success=True, warmup=(i == 0))
        rec.record(m)
    rec.record({"variant": "original_sglang", "measurement_kind": "formal_latency", "reused_tokens": 5,
                "request_latency_ms": 50.0, "e2e_latency_ms": 60.0})
    rows = read_jsonl(tmp_path / "m.jsonl")
    assert rows[1]["cache_reuse_ratio"] == 0.75 and rows[1]["context_reduction_ratio"] == 0.6
    agg = {r["variant"]: r for r in aggregate_experiment(rows)}
    ll = agg["selected_context_radixcache_legolink"]
    assert ll["sample_count"] == 3  # the warm-up row is dropped
    assert ll["request_latency_ms_stats"]["p50"] == 30.0
    assert ll["reused_tokens"] == 900 and ll["cache_reuse_ratio"] == 0.75
    assert agg["original_sglang"]["reused_tokens"] is None  # baseline arm carries no LegoLink fields
    assert len(formal_rows(rows)) == 4
    steps = aggregate_agent_steps([{"variant": "v", "task_id": "t", "step_latency_ms": 5, "tool_calls": 2}] * 3)
    assert steps[0]["agent_steps"] == 3 and steps[0]["tool_calls"] == 6


def test_stream_metrics():
    ms = 1_000_000
    out = compute_stream_metrics(request_started_ns=0, token_ready_ns=[10 * ms, 12 * ms, 15 * ms],
                                 request_completed_ns=16 * ms, output_tokens=3, reused_tokens=90,
                                 recomputed_tokens=10, link_ns=4 * ms)
    assert out["ttft_ms"] == 10.0 and out["itl_ms"] == 2.5 and out["decode_ms"] == 6.0
    assert out["cache_reuse_ratio"] == 0.9 and out["link_ms"] == 4.0
    with pytest.raises(ValueError):
        compute_stream_metrics(request_started_ns=0, token_ready_ns=[5, 3], request_completed_ns=9)


def test_host_timing_spans_and_configs(tmp_path):
    h = HostTimingRecorder("plan", metadata={"request_id": "r1", "secret": "x"}, output_path=tmp_path / "h.jsonl",
                           enabled=True)
    with h.span("outer"):
        with h.span("inner"):
            pass
    row = h.emit()
    assert [s["name"] for s in row["spans"]] == ["inner", "outer"]
    assert row["spans"][0]["depth"] == 1 and "secret" not in row and row["request_id"] == "r1"
    assert h.emit() == {}  # one row per recorder
    assert len(read_jsonl(tmp_path / "h.jsonl")) == 1
    assert ProfilerWindowConfig(wait=1, warmup=1, active=2, repeat=2).total_steps == 8
    with pytest.raises(ValueError):
        ProfilerWindowConfig(active=0)
    cmd = NcuRunConfig("out", ("python", "x.py"), "gemm").ncu_command()
    assert "--clock-control" in cmd and cmd[cmd.index("--clock-control") + 1] == "none"
    with pytest.raises(ValueError):
        NcuRunConfig("out", ("python",), "gemm", launch_count=10)


def _agent(tmp_path, fake):
    tok = HashTokenizer(vocab_size=4096)
    cm = ContextManager("agent-task", tokenizer=tok)
    ad = RuntimeAdapter(fake, model="legolink", tokenizer=tok, repair_planner=RepairWindowPlanner(
        UniformRepairWindow(8)), generation={"max_tokens": 4, "temperature": 0.0})
    return AgentLLM(RequestPipeline(cm, ad), task_id="agent-task", recorder=MetricsRecorder(tmp_path / "a.jsonl"))


def test_agent_turns_record_reuse(tmp_path):
    fake = StrictFakeRuntime()
    agent = _agent(tmp_path, fake)
    sys_msg = {"role": "system", "content": "You fix failing tests in this repository. " * 30}
    turns = [
        {"messages": [sys_msg, {"role": "user", "content": "run the tests"}]},
        {"messages": [sys_msg, {"role": "user", "content": "run the tests"},
                      {"role": "assistant", "content": "running pytest now " * 30},
                      {"role": "user", "content": "what failed?"}]},
    ]
    res = ReplayDriver(agent, objective="fix tests").run(turns)
    assert len(res) == 2
    rows = read_jsonl(tmp_path / "a.jsonl")
    assert len(rows) == 2 and rows[0]["task_id"] == "agent-task"
    assert rows[1]["reused_tokens"] and rows[1]["reused_tokens"] > 0
    assert not fake.plain_generation_requests()


def test_proxy_sessions_json_guardrail_and_passthrough(tmp_path):
    fake = StrictFakeRuntime()
    px = LegoLinkProxy(fake, tokenizer=HashTokenizer(vocab_size=4096), repair_tokens=8,
                       metrics_path=str(tmp_path / "p.jsonl"), json_retries=1)
    sys_msg = {"role": "system", "content": "You are a careful agent. " * 40}
    msgs = [sys_msg, {"role": "user", "content": "list the files"}]
    a = px.chat_completion({"messages": msgs})
    b = px.chat_completion({"messages": msgs + [{"role": "assistant", "content": a["choices"][0]["message"][
        "content"]}, {"role": "user", "content": "now read setup.py"}]})
    # no identity named: an opaque key, continued because b repeats the whole
    # transcript including the proxy's reply
    assert a["legolink"]["session"] == b["legolink"]["session"]
    assert a["legolink"]["session"].startswith("derived-")
    assert len(px.sessions) == 1
    # the same opening prompt without the earlier reply is a new session
    d = px.chat_completion({"messages": msgs})
    assert d["legolink"]["session"] != a["legolink"]["session"] and len(px.sessions) == 2
    # the fake's replies are not JSON: the guardrail re-asks json_retries times
    c = px.chat_completion({"messages": msgs, "response_format": {"type": "json_object"}, "session_id": "s2"})
    assert c["legolink"]["attempts"] == 2 and px.stats["json_retries"] == 1
    assert parses_as_json('```json\n{"a": 1}\n```') and not parses_as_json("not json")
    # over HTTP
    srv = serve(px, port=0)
    try:
        port = srv.server_address[1]
        req = urllib.request.Request(f"http://127.0.0.1:{port}/v1/chat/completions",
                                     data=json.dumps({"messages": msgs}).encode(),
                                     headers={"Content-Type": "application/json"})
        with urllib.request.urlopen(req, timeout=30) as r:
            body = json.loads(r.read())
        assert body["object"] == "chat.completion"
    finally:
        srv.shutdown()
    assert len(read_jsonl(tmp_path / "p.jsonl")) >= 4
    # passthrough arm forwards the request unchanged (the LegoLink-only fake refuses plain generation)
    pt = LegoLinkProxy(fake, passthrough=True)
    with pytest.raises(Exception):
        pt.chat_completion({"messages": msgs})
    assert fake.plain_generation_requests()


def test_proxy_session_identity_helpers():
    """Explicit identities give stable keys (field, header in any case, the
    OpenAI ``user``); content parts flatten to text; the LiteLLM provider
    prefix is stripped; a continuation must repeat the proxy's own reply."""
    from sglang_legolink_b200.server.proxy import (TranscriptIndex, message_content_to_text, normalize_model_name,
                                                   transcript_digest)

    assert normalize_model_name("openai/Qwen/Qwen2.5-7B") == "Qwen/Qwen2.5-7B"
    assert normalize_model_name("Qwen/Qwen2.5-7B") == "Qwen/Qwen2.5-7B"
    parts = [{"type": "text", "text": "first"}, {"type": "image_url", "image_url": {"url": "x"}}, {"content": "second"}]
    assert message_content_to_text(parts) == "first\nsecond" and message_content_to_text(None) == ""
    assert transcript_digest([{"role": "user", "content": parts}]) == transcript_digest(
        [{"role": "user", "content": "first\nsecond"}])
    px = LegoLinkProxy(StrictFakeRuntime(), tokenizer=HashTokenizer(vocab_size=4096))
    m = [{"role": "user", "content": "hi"}]
    assert px.session_key({"messages": m, "session_id": "s"}) == "s"
    assert px.session_key({"messages": m}, {"x-session-id": "h"}) == "h"
    assert px.session_key({"messages": m, "user": "u1"}) == "user:u1"
    k1, k2 = px.session_key({"messages": m}), px.session_key({"messages": m})
    assert k1 != k2 and k1.startswith("derived-")
    idx = TranscriptIndex(max_entries=2)
    t = m + [{"role": "assistant", "content": "reply"}]
    idx.remember("k", t)
    assert idx.continuation(t + [{"role": "user", "content": "more"}]) == "k"
    assert idx.continuation(m + [{"role": "assistant", "content": "forged"}, {"role": "user", "content": "x"}]) is None
    idx.remember("k2", [{"role": "assistant", "content": "a"}])
    idx.remember("k3", [{"role": "assistant", "content": "b"}])
    assert idx.continuation(t) is None  # bounded: the oldest entry was dropped
