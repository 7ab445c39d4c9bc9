"""Host pipeline: events, segmentation, identities, policy gates, framing,
contract and residency recovery (CPU, no model)."""

import json
import os
import subprocess
import sys
import threading

import pytest

from sglang_legolink_b200.contract import (PIC_LINK_RUNTIME_OWNED_FIELDS, ContractError, parse_residency_recovery,
                                           physical_token_ids_sha256, residency_recovery_message,
                                           validate_pic_link_request)
from sglang_legolink_b200.host.adapter import ResidencyRecoveryCoordinator, Role, classify_failure
from sglang_legolink_b200.host.events import EventCollector, EventType, FieldExtractor, openai_request_events
from sglang_legolink_b200.host.framing import (RepairWindowPlanner, Stitcher, UniformRepairWindow, build_layout,
                                               frame_link)
from sglang_legolink_b200.host.manager import (ContextManager, DeterministicSegmenter, Segment, SegmentationError,
                                               validate_segments)
from sglang_legolink_b200.host.planner import (CompileAction, CompilePolicy, PersistentCacheCatalog, Planner,
                                               PolicyContext)
from sglang_legolink_b200.host.store import semantic_cache_key, semantic_identity
from sglang_legolink_b200.host.tokenizer import HashTokenizer, RegexTokenizer

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_collector_dedup_revisions_and_rollback():
    c = EventCollector("t")
    a = c.add_events([("tool_output", "s1", "x", {}), ("tool_output", "s1", "x", {})])
    assert len(a) == 1 and c.revision == 1
    assert c.add_events([("tool_output", "s1", "x", {})]) == []
    cp = c.checkpoint()
    c.add_events([("tool_output", "s2", "y", {})])
    c.rollback(cp)
    assert c.revision == 1 and len(c.events()) == 1
    assert len(c.add_events([("tool_output", "s2", "y", {})])) == 1  # re-offered after rollback


def test_hidden_sources_are_filtered_and_unknown_types_fail_closed():
    c = EventCollector("t")
    c.add_events([("workspace_file", "f1", "secret", {"path": "tests/oracle/answer.txt"}),
                  ("workspace_file", "f2", "ok", {"path": "src/main.py"})])
    ext = FieldExtractor().extract(c.events())
    assert [s.source_id for s in ext.sources()] == ["f2"] and len(ext.filtered_event_ids) == 1
    c.add_events([("unclassified", "u", "?", {})])
    with pytest.raises(ValueError):
        FieldExtractor().extract(c.events())


def test_openai_ingress_roles():
    ev = openai_request_events([{"role": "system", "content": "sys"}, {"role": "user", "content": "q1"},
                                {"role": "assistant", "content": "a1"}, {"role": "tool", "tool_call_id": "c1",
                                                                         "content": "out"},
                                {"role": "user", "content": "q2"}],
                               tools=[{"type": "function", "function": {"name": "run"}}])
    kinds = [e[0] for e in ev]
    assert kinds[0] == EventType.TOOL_DEFINITION and EventType.USER_REQUEST in kinds
    assert kinds.count(EventType.USER_REQUEST) == 1


def test_segmentation_budget_split_tiles_the_source():
    tok = RegexTokenizer()
    seg = DeterministicSegmenter(tok, max_segment_tokens=50)
    text = "".join(f"line {i} with some words here\n" for i in range(60))
    from sglang_legolink_b200.host.events import ExtractedSource

    segs = seg.segment(ExtractedSource("tool_history_output", "e", "s", text, 1))
    validate_segments(text, segs)
    assert len(segs) > 1 and all(tok.count(text[s.start:s.end]) <= 50 for s in segs)
    with pytest.raises(SegmentationError):
        validate_segments("abc", [Segment(0, 1), Segment(2, 3)])


def test_identity_is_content_not_provenance():
    a = semantic_identity(context_field="tool_definitions", raw_text="same")
    b = semantic_identity(context_field="tool_definitions", raw_text="same")
    assert a == b and a != semantic_identity(context_field="task_instruction", raw_text="same")
    k1 = semantic_cache_key(semantic_identity=a, context_field="tool_definitions", model_fingerprint="m",
                            tokenizer_fingerprint="t", segmentation_policy_version="s", recompute_policy_version="r")
    k2 = semantic_cache_key(semantic_identity=a, context_field="tool_definitions", model_fingerprint="m2",
                            tokenizer_fingerprint="t", segmentation_policy_version="s", recompute_policy_version="r")
    assert k1 != k2


@pytest.mark.parametrize("n,action", [(63, CompileAction.KEEP_MUTABLE), (64, CompileAction.COMPILE),
                                      (65, CompileAction.COMPILE)])
def test_legacy_fixed_64_floor(n, action):
    from dataclasses import replace

    cm = ContextManager("t", tokenizer=HashTokenizer())
    cm.ingest([("task_instruction", "task", " ".join(["w"] * n), {})])
    v = cm.contexts()[0]
    v = replace(v, token_count=n)
    assert CompilePolicy().decide(v, PolicyContext()).action == action


def _session(tok):
    cm = ContextManager("task", tokenizer=tok)
    cm.ingest([("task_instruction", "task", "Fix the bug. " * 30, {})])
    cm.ingest([("conversation_message", "a1", "I will run the tests. " * 30, {})])
    cm.ingest([("tool_output", "t1", "FAILED test_x " * 30, {})])
    return cm


def test_planner_layout_prefix_and_mutable_suffix():
    tok = HashTokenizer()
    cm = _session(tok)
    plan = Planner().plan(cm.select("continue"), cm.contexts())
    cats = [r.planner_category for r in plan.records]
    assert cats[:2] == ["compile_on_miss", "compile_on_miss"] and cats[-1] == "mutable"
    # linked blocks form a prefix of the included order
    inc = [v.sub_context_id for v in plan.included_contexts]
    assert inc[: len(plan.linked_contexts)] == [v.sub_context_id for v in plan.linked_contexts]


def test_stitch_framing_and_link_payload_contract():
    tok = HashTokenizer()
    cm = _session(tok)
    plan = Planner().plan(cm.select("continue please"), cm.contexts())
    st = Stitcher(tokenizer=tok).stitch(plan)
    assert "".join(v.raw_text for v in st.linked_views) + st.mutable_text == st.selected_text
    lay = build_layout(st, tok)
    assert lay.assembled_token_ids == lay.baseline_token_ids
    md = lay.link_metadata()
    assert md["expected_complete_token_ids_sha256"] == physical_token_ids_sha256(lay.baseline_token_ids)
    dec = RepairWindowPlanner(UniformRepairWindow(16)).plan(lay)
    payload, audit = frame_link(st, lay, dec, request_id="r", task_id="t", model="m")
    wire = payload["pic_link"]
    assert not set(wire) & PIC_LINK_RUNTIME_OWNED_FIELDS
    assert wire["recompute_tokens_per_block"][0] > 0  # block 0 sits behind the chat prefix
    validate_pic_link_request(dict(wire))


def test_runtime_owned_and_unknown_fields_refused():
    with pytest.raises(ContractError):
        validate_pic_link_request({"cache_keys": ["a"], "imp_indices": [1]})
    with pytest.raises(ContractError):
        validate_pic_link_request({"cache_keys": ["a"], "expected_cache_keys": ["a"]})
    with pytest.raises(ContractError):
        validate_pic_link_request({"cache_keys": ["a"], "recompute_initial_tokens": True})
    with pytest.raises(ContractError):
        validate_pic_link_request({"cache_keys": ["a"], "recompute_mode": "fast"})
    with pytest.raises(ContractError):
        validate_pic_link_request({"cache_keys": ["a"], "execution_mode": "formal"})
    validate_pic_link_request({"cache_keys": ["a"], "imp_indices": [1]}, allow_legacy_fields=True)


def test_recovery_message_roundtrip_and_classification():
    m = residency_recovery_message(missing=["k1"], stale=["k2"])
    d = parse_residency_recovery(m)
    assert d == {"missing": ("k1",), "stale": ("k2",), "incompatible": ()}
    body = json.dumps({"object": "error", "message": m})
    assert parse_residency_recovery(body)["missing"] == ("k1",)
    assert classify_failure(m) == "residency"


def test_single_flight_recovery_one_owner_per_key():
    co = ResidencyRecoveryCoordinator(wait_timeout_s=5)
    roles, barrier = [], threading.Barrier(8)

    def worker():
        barrier.wait()
        t = co.claim("rt", "key", observed=0)
        roles.append(t.role)
        if t.role == Role.OWNER:
            import time

            time.sleep(0.05)
            co.complete(t, ok=True)
        else:
            co.wait(t)

    ths = [threading.Thread(target=worker) for _ in range(8)]
    [t.start() for t in ths]
    [t.join() for t in ths]
    assert roles.count(Role.OWNER) == 1
    assert co.claim("rt", "key", observed=0).role == Role.SETTLED


def test_persistent_catalog_shared_between_instances(tmp_path):
    p = str(tmp_path / "catalog.jsonl")
    a, b = PersistentCacheCatalog(p), PersistentCacheCatalog(p)
    a.mark_compiled("k", token_count=3)
    assert b.is_compiled("k")
    with open(p, "a") as f:
        f.write('{"op": "compiled", "key": "torn"')  # torn last line is ignored
    assert not b.is_compiled("torn")
    a.invalidate("k")
    assert not b.is_compiled("k")


@pytest.mark.parametrize("mode", [[], ["--fake-http"], ["--engine"]])
def test_example_compile_link_decode(mode):
    r = subprocess.run([sys.executable, os.path.join(ROOT, "examples", "compile_link_decode.py"), *mode],
                       capture_output=True, text=True, timeout=600, env={**os.environ, "CUDA_VISIBLE_DEVICES": ""})
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
    out = json.loads(r.stdout)
    assert [t["compile_requests"] for t in out["turns"]] == [1, 0, 1, 1, 0]
    assert out["after_eviction"]["outcome"] == "recovered_after_source_missing"
    assert out["after_eviction"]["plain_generation_requests_ever_sent"] == 0
    assert out["runtime_owned_fields_on_the_wire"] == []
