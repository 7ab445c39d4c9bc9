"""Wire schemas: every schema is a valid draft 2020-12 schema, the objects the
host pipeline and the runtime contract really produce match them, what the
contract refuses the schemas refuse too, and each schema's field set stays in
step with the code that writes the object (CPU only)."""

import dataclasses
import json
import pathlib

import pytest

from sglang_legolink_b200 import contract as C
from sglang_legolink_b200 import schemas as S
from sglang_legolink_b200.host.agent import ReplayDriver
from sglang_legolink_b200.host.events import EventCollector, SessionEvent
from sglang_legolink_b200.host.fake_runtime import StrictFakeRuntime
from sglang_legolink_b200.host.manager import ContextManager
from sglang_legolink_b200.host.metrics import AgentMetric, read_jsonl
from sglang_legolink_b200.host.planner import Planner
from sglang_legolink_b200.host.store import SubContext
from sglang_legolink_b200.host.tokenizer import HashTokenizer


def test_schema_files_are_valid_and_complete():
    S.check_schemas()
    here = pathlib.Path(S.HERE)
    assert sorted(p.name for p in here.glob("*.schema.json")) == sorted(f"{n}.schema.json" for n in S.SCHEMA_NAMES)
    with pytest.raises(KeyError):
        S.load("no_such_schema")


@pytest.fixture(scope="module")
def session(tmp_path_factory):
    """Two replayed agent turns against the strict fake runtime: the bodies it
    received are what a host sends over the wire."""
    from test_host_agent_proxy import _agent

    tmp = tmp_path_factory.mktemp("schemas")
    fake = StrictFakeRuntime()
    agent = _agent(tmp, fake)
    sys_msg = {"role": "system", "content": "You fix failing tests in this repository. " * 30}
    turns = [{"messages": [sys_msg, {"role": "user", "content": "run the tests"}]},
             {"messages": [sys_msg, {"role": "user", "content": "run the tests"},
                           {"role": "assistant", "content": "running pytest now " * 30},
                           {"role": "user", "content": "what failed?"}]}]
    ReplayDriver(agent, objective="fix tests").run(turns)
    return fake.requests, read_jsonl(tmp / "a.jsonl")


def test_wire_requests_and_metric_rows_match(session):
    requests, rows = session
    compiles = [r for r in requests if r.get("sub_context") is not None]
    links = [r for r in requests if r.get("pic_link") is not None]
    assert compiles and links and rows
    for body in requests:
        S.validate("legolink_request", body)
    for body in links:
        S.validate("pic_link", body["pic_link"])
        C.validate_pic_link_field_types(body["pic_link"])  # the runtime's own check agrees
    for row in rows:
        S.validate("metric_row", row)


def _wire(obj):
    """The JSON form of an object, which is what the schemas describe."""
    return json.loads(json.dumps(obj))


def test_host_objects_match():
    tok = HashTokenizer()
    cm = ContextManager("task", tokenizer=tok)
    events = cm.ingest([("task_instruction", "task", "Fix the bug. " * 30, {})])
    events += cm.ingest([("tool_output", "t1", "FAILED test_x " * 30, {"path": "log.txt"})])
    assert events
    for e in events:
        S.validate("session_event", _wire(e.to_dict()))
    assert cm.contexts()
    for v in cm.contexts():
        d = _wire(v.to_dict())
        S.validate("sub_context", d)
        assert SubContext.from_dict(d) == v
    manifest = cm.select("continue")
    S.validate("agent_context_manifest", _wire(manifest.to_dict()))
    S.validate("execution_plan", _wire(Planner().plan(manifest, cm.contexts()).to_dict()))
    c = EventCollector("t")
    for e in c.add_events([("tool_output", "s1", "x", {})]):
        S.validate("session_event", _wire(e.to_dict()))


def _good_link():
    return {"cache_keys": ["k0", "k1"], "request_id": "r1", "recompute_initial_tokens": 16,
            "recompute_tokens_per_block": [16, 16], "recompute_mode": "batched"}


@pytest.mark.parametrize("field", sorted(C.PIC_LINK_RUNTIME_OWNED_FIELDS))
def test_runtime_owned_fields_refused_by_schema_and_contract(field):
    bad = dict(_good_link(), **{field: [0]})
    assert S.errors("pic_link", bad)
    with pytest.raises(C.ContractError):
        C.validate_pic_link_request(bad, profile={}, require_formal=False)


@pytest.mark.parametrize("patch", [
    {"unknown_field": 1},
    {"recompute_initial_tokens": True},  # booleans are not integers on this wire
    {"recompute_initial_tokens": C.PIC_LINK_MAX_INTEGER + 1},
    {"recompute_initial_tokens": -1},
    {"recompute_mode": "sideways"},
    {"recompute_tokens_per_block": [16, "16"]},
    {"cache_keys": []},
])
def test_malformed_pic_link_refused_by_schema_and_contract(patch):
    bad = dict(_good_link(), **patch)
    assert S.errors("pic_link", bad), patch
    with pytest.raises(C.ContractError):
        C.validate_pic_link_request(bad, profile={}, require_formal=False)


def test_good_pic_link_and_request_shapes():
    S.validate("pic_link", _good_link())
    C.validate_pic_link_request(_good_link(), profile={}, require_formal=False)
    S.validate("pic_link", dict(_good_link(), recompute_mode="BATCHED"))  # the contract lower-cases the mode
    body = {"model": "m", "messages": [{"role": "user", "content": "hi"}], "pic_link": _good_link()}
    S.validate("legolink_request", body)
    with pytest.raises(S.SchemaValidationError):  # one request is a Compile or a Link, not both
        S.validate("legolink_request", dict(body, sub_context={"cache_key": "k0"}))
    with pytest.raises(S.SchemaValidationError) as ei:  # a nested violation names its path
        S.validate("legolink_request", dict(body, pic_link=dict(_good_link(), imp_indices=[1])))
    assert ei.value.path == ["pic_link"]


def test_schema_field_sets_follow_the_code():
    props = lambda n: set(S.load(n)["properties"])
    assert props("pic_link") == set(C.PIC_LINK_REQUEST_FIELDS)
    assert not props("pic_link") & C.PIC_LINK_RUNTIME_OWNED_FIELDS
    assert set(S.load("pic_link")["properties"]["framing_spec"]["required"]) == C.FRAMING_SPEC_FIELDS
    assert set(S.load("pic_link")["properties"]["repair_decision"]["required"]) == C.REPAIR_DECISION_FIELDS
    assert props("session_event") == {f.name for f in dataclasses.fields(SessionEvent)}
    assert props("sub_context") == {f.name for f in dataclasses.fields(SubContext)}
    assert props("metric_row") == {f.name for f in dataclasses.fields(AgentMetric)}
    tok = HashTokenizer()
    cm = ContextManager("task", tokenizer=tok)
    cm.ingest([("task_instruction", "task", "Fix the bug. " * 30, {})])
    m = cm.select("go")
    assert props("agent_context_manifest") == set(m.to_dict())
    assert props("execution_plan") == set(Planner().plan(m, cm.contexts()).to_dict())


def test_command_line_validator(tmp_path, capsys, session):
    from sglang_legolink_b200.schemas.__main__ import main

    _, rows = session
    good = tmp_path / "m.jsonl"
    good.write_text("".join(json.dumps(r) + "\n" for r in rows) + "\n")
    assert main(["metric_row", str(good)]) == 0 and capsys.readouterr().out.strip() == f"ok {len(rows)}"
    bad = tmp_path / "link.json"
    bad.write_text(json.dumps(dict(_good_link(), imp_indices=[3])))
    assert main(["pic_link", str(bad)]) == 1 and "imp_indices" in capsys.readouterr().out
    assert main(["no_such_schema", str(bad)]) == 2
