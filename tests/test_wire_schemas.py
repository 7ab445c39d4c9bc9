"""The reference's JSON wire shapes (``noc_*`` schemas built from the tables
in ``host/wire.py``): the committed schema files match the tables; objects a
reference host writes validate; and the objects this host emits -- session
events, sub-contexts, manifests, execution plans, LegoLink requests, metric
rows -- validate after export."""

import json
import os

import pytest

from sglang_legolink_b200 import schemas as S
from sglang_legolink_b200.host import wire as W
from sglang_legolink_b200.host.adapter import RequestPipeline, RuntimeAdapter
from sglang_legolink_b200.host.agent import AgentLLM
from sglang_legolink_b200.host.fake_runtime import StrictFakeRuntime
from sglang_legolink_b200.host.framing import RepairWindowPlanner, UniformRepairWindow
from sglang_legolink_b200.host.manager import ContextManager
from sglang_legolink_b200.host.metrics import MetricsRecorder, read_jsonl
from sglang_legolink_b200.host.tokenizer import HashTokenizer

H64 = "ab" * 32


@pytest.mark.parametrize("name", S.NOC_SCHEMA_NAMES)
def test_committed_noc_schemas_match_the_tables(name):
    with open(os.path.join(S.HERE, f"{name}.schema.json"), encoding="utf-8") as f:
        assert json.load(f) == S.build_noc_schema(name)


def test_table_sizes():
    assert len(W.EXPERIMENT_METRICS) == 127 and len(W.SEMANTIC_SUBCONTEXT) == 28
    assert len(W.AGENT_CONTEXT_MANIFEST) == 18 and len(W.REQUEST_EXECUTION_PLAN) == 15


# ------------------------------------------------- objects a reference host writes
REF_OBJECTS = {
    "noc_legolink_request": {"request_id": "r-1", "semantic_block_ids": ["sc-1"], "cache_keys": [H64],
                             "mutable_text": "what next?", "generation_parameters": {"max_tokens": 16}},
    "noc_session_event": {"event_id": "e1", "task_id": "t", "session_revision": 1, "event_type": "tool_output",
                          "source_id": "tool-output:x", "raw_text": "ok", "timestamp": "2026-01-01T00:00:00Z",
                          "sequence_number": 3, "metadata": {"ingress": "openai.messages"}},
    "noc_agent_context_manifest": {
        "task_id": "t", "agent_id": "a", "request_id": "r", "session_revision": 2, "objective": "fix",
        "selected_sub_context_ids": ["s1", "s2"], "selected_cache_keys": [H64, H64], "mutable_text": "q",
        "full_session_tokens": 900, "candidate_context_tokens": 800, "selected_context_tokens": 500,
        "context_reduction_tokens": 400, "context_reduction_ratio": 0.44, "selection_reason": {"s1": "rule"},
        "excluded_reason": {}, "selection_order": ["s1", "s2"], "excluded_sub_context_ids": [],
        "context_token_budget": 4096},
    "noc_semantic_subcontext": {
        "sub_context_id": "s1", "task_id": "t", "session_revision": 1, "context_field": "tool_history_output",
        "title": "t", "question_or_objective": "", "raw_text": "x", "canonical_text": "x",
        "source_spans": [{"source_id": "src", "start": 0, "end": 1}], "content_hash": H64, "cache_key": H64,
        "version": 1, "token_count": 1, "token_ids": [5], "tokenizer_fingerprint": "tok", "model_fingerprint": "m",
        "recompute_policy_version": "v", "is_mutable": False, "reuse_candidate": True,
        "semantic_independence_reason": "r", "segmentation_confidence": 0.9, "policy_version": "p",
        "created_at": "2026-01-01T00:00:00Z", "updated_at": "2026-01-01T00:00:00Z", "supersedes": None,
        "invalidated": False},
    "noc_request_execution_plan": {
        "manifest": {}, "selected_order": ["s1"], "reuse_cached": ["s1"], "compile_on_miss": [], "keep_mutable": [],
        "excluded": [], "expected_cache_keys": [H64], "baseline_selected_text": "x", "text_separator": "\n\n",
        "decisions": [{"action": "compile"}],
        "block_planning": [{"semantic_candidate": True, "cache_availability": "host_catalog_entry",
                            "reuse_eligibility": "exact_safe", "effective_decision": "REUSE_CACHED",
                            "feasibility_reason": "none"}],
        "profitability": {"enforced": False, "profitability_mode": "observe_only"}},
    "noc_experiment_metrics": {"metric_level": "request", "variant": "selected_context_radixcache_legolink",
                               "measurement_kind": "formal_latency", "ttft_ms": 80.3, "link_ms": 80.3,
                               "reused_tokens": 11000, "cache_reuse_ratio": 0.7, "concurrency": 8,
                               "selected_blocks": ["s1"], "profiling_type": None, "any_extra_field": 1},
}


@pytest.mark.parametrize("name", sorted(REF_OBJECTS))
def test_reference_shaped_objects_validate(name):
    S.validate(name, REF_OBJECTS[name])


@pytest.mark.parametrize("name,mutate", [
    ("noc_legolink_request", lambda d: d.update(mutable_text="")),
    ("noc_legolink_request", lambda d: d.update(imp_indices=[1])),
    ("noc_session_event", lambda d: d.update(event_type="oracle")),
    ("noc_semantic_subcontext", lambda d: d.update(cache_key="XYZ")),
    ("noc_semantic_subcontext", lambda d: d.update(source_spans=[])),
    ("noc_agent_context_manifest", lambda d: d.update(context_reduction_ratio=1.5)),
    ("noc_request_execution_plan", lambda d: d["block_planning"][0].update(imp_indices=[3])),
    ("noc_request_execution_plan", lambda d: d.update(profitability={"enforced": True})),
    ("noc_experiment_metrics", lambda d: d.update(variant="mine")),
    ("noc_experiment_metrics", lambda d: d.update(concurrency=0)),
])
def test_wire_violations_are_caught(name, mutate):
    obj = json.loads(json.dumps(REF_OBJECTS[name]))
    mutate(obj)
    with pytest.raises(S.SchemaValidationError):
        S.validate(name, obj)


# --------------------------------------------------- this host's objects, exported
def test_this_hosts_objects_export_to_the_wire(tmp_path):
    tok = HashTokenizer(vocab_size=4096)
    cm = ContextManager("wire-task", tokenizer=tok, capture_token_ids=True)
    ad = RuntimeAdapter(StrictFakeRuntime(), model="legolink", tokenizer=tok,
                        repair_planner=RepairWindowPlanner(UniformRepairWindow(8)),
                        generation={"max_tokens": 4, "temperature": 0.0})
    agent = AgentLLM(RequestPipeline(cm, ad), task_id="wire-task", recorder=MetricsRecorder(tmp_path / "m.jsonl"))
    sysm = {"role": "system", "content": "You fix failing tests in this repository. " * 20}
    r1 = agent.call([sysm, {"role": "user", "content": "run the tests"}])
    agent.call([sysm, {"role": "user", "content": "run the tests"}, {"role": "assistant", "content": "ran " * 40},
                {"role": "user", "content": "what failed?"}])
    for ev in cm.collector.events():
        S.validate("noc_session_event", W.session_event_wire(ev))
    for v in cm.contexts():
        S.validate("noc_semantic_subcontext", W.subcontext_wire(v))
    plan = r1.execution.plan
    wire_plan = W.execution_plan_wire(plan, request_id="r1")
    S.validate("noc_request_execution_plan", wire_plan)
    S.validate("noc_agent_context_manifest", wire_plan["manifest"])
    S.validate("noc_legolink_request", W.legolink_request_wire(plan, request_id="r1", generation={"max_tokens": 4}))
    rows = W.export_rows(read_jsonl(tmp_path / "m.jsonl"))
    assert len(rows) == 2
    for row in rows:
        S.validate("noc_experiment_metrics", row)
    assert rows[1]["reused_tokens"] and rows[1]["formal_latency"] is True
