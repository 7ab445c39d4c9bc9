"""Session-aware ingress (content-derived ids, source ledger, prompt
registry, Terminus turns; reference ``noc_context_manager/real_ingress.py``)
and the agent integrations (direct Compile/Link client, NOC client, terminal
agent loops; reference ``terminal_bench_integration/``) on CPU."""

import json

import pytest

from sglang_legolink_b200.host.adapter import RequestPipeline, RuntimeAdapter
from sglang_legolink_b200.host.agents import (NOCLLM, PICLLM, NOCTerminus2Agent, SubprocessTerminal, TerminalAgent,
                                              TmuxSessionAdapter, parse_agent_response, split_text)
from sglang_legolink_b200.host.events import EventType
from sglang_legolink_b200.host.fake_runtime import StrictFakeRuntime
from sglang_legolink_b200.host.framing import RepairWindowPlanner, UniformRepairWindow
from sglang_legolink_b200.host.ingress import (KIND_AGENT_DIRECTIVE, KIND_TOOL_OUTPUT, PromptPart, PromptRegistry,
                                               SourceLedger, message_source_id, openai_request_events, split_around,
                                               terminus_turn_events, tool_call_event, tool_definition_events,
                                               verified_parts)
from sglang_legolink_b200.host.manager import ContextManager
from sglang_legolink_b200.host.metrics import MetricsRecorder, read_jsonl
from sglang_legolink_b200.host.tokenizer import HashTokenizer

SYS = {"role": "system", "content": "You are a coding agent."}
TOOLS = [{"type": "function", "function": {"name": "run", "parameters": {"type": "object"}}}]


def _ingest(ledger, events):
    ledger.record(events)
    return events


# ------------------------------------------------------------------ ingress
def test_first_call_prompt_is_the_task_instruction_then_requests():
    led = SourceLedger()
    ev = _ingest(led, openai_request_events([SYS, {"role": "user", "content": "fix the build"}], tools=TOOLS,
                                            ledger=led, first_turn=True))
    kinds = [e[0] for e in ev]
    assert kinds == [EventType.TOOL_DEFINITION, EventType.TASK_INSTRUCTION, EventType.TASK_INSTRUCTION]
    again = openai_request_events([SYS, {"role": "user", "content": "fix the build"},
                                   {"role": "assistant", "content": "running make"},
                                   {"role": "user", "content": "it failed"}], tools=TOOLS, ledger=led,
                                  first_turn=False)
    assert [(e[0], e[2]) for e in again] == [(EventType.CONVERSATION_MESSAGE, "running make"),
                                             (EventType.USER_REQUEST, "it failed")]


def test_a_past_request_is_settled_into_history():
    led = SourceLedger()
    _ingest(led, openai_request_events([SYS, {"role": "user", "content": "step one"}], ledger=led, first_turn=True))
    _ingest(led, openai_request_events([SYS, {"role": "user", "content": "step one"},
                                        {"role": "user", "content": "step two"}], ledger=led, first_turn=False))
    third = openai_request_events([SYS, {"role": "user", "content": "step one"}, {"role": "user", "content": "step two"},
                                   {"role": "user", "content": "step three"}], ledger=led, first_turn=False)
    settled = [e for e in third if e[3].get("settled_from") == "user_request"]
    assert [e[2] for e in settled] == ["step two"]
    assert settled[0][1] == message_source_id("user", "step two")  # same source: a new revision of it


def test_tool_ids_are_content_derived():
    a = tool_call_event("c1", "run", '{"cmd": "ls", "cwd": "/"}', ingress="t")
    b = tool_call_event("c2", "run", '{"cwd": "/", "cmd": "ls"}', ingress="t")
    assert a[1] == b[1] and a[2] == b[2] and a[3]["tool_call_id"] == "c1"
    defs = tool_definition_events([TOOLS[0], {"type": "function", "function": {"name": "run", "x": 1}}])
    assert defs[0][1] != defs[1][1] and all(d[1].startswith("tool-schema:run#") for d in defs)
    led = SourceLedger()
    _ingest(led, tool_definition_events(TOOLS))
    changed = [{"type": "function", "function": {"name": "run", "parameters": {"type": "object", "x": 1}}}]
    evs = openai_request_events([{"role": "user", "content": "q"}], tools=changed, ledger=led, first_turn=False)
    assert evs[0][0] == EventType.TOOL_DEFINITION and evs[0][1] == "tool-schema:run"  # a revision of the same source


def test_assistant_tool_calls_and_results():
    led = SourceLedger()
    msgs = [{"role": "user", "content": "go"},
            {"role": "assistant", "content": None, "tool_calls": [{"id": "c9", "function": {"name": "run",
                                                                                           "arguments": "{}"}}]},
            {"role": "tool", "tool_call_id": "c9", "content": "total 0"}, {"role": "user", "content": "and?"}]
    ev = openai_request_events(msgs, ledger=led, first_turn=False)
    kinds = [e[0] for e in ev]
    assert kinds == [EventType.CONVERSATION_MESSAGE, EventType.TOOL_CALL, EventType.TOOL_OUTPUT,
                     EventType.USER_REQUEST]
    assert ev[2][3]["tool_name"] == "run" and ev[2][2] == "total 0"


def test_declared_prompt_parts_and_the_registry():
    prompt = "Output:\nls -la\ntotal 4\nWhat next?"
    parts = split_around(prompt, "ls -la\ntotal 4")
    assert [p.kind for p in parts] == [KIND_AGENT_DIRECTIVE, KIND_TOOL_OUTPUT, KIND_AGENT_DIRECTIVE]
    assert verified_parts(prompt, parts) == parts
    assert verified_parts(prompt, parts[:2]) is None  # does not join to the prompt
    assert verified_parts(prompt, (PromptPart("secret", prompt),)) is None
    led, reg = SourceLedger(), PromptRegistry()
    ev, st = terminus_turn_events(prompt, [{"role": "user", "content": "Task: list files"},
                                           {"role": "assistant", "content": "{}"}], ledger=led, registry=reg,
                                  declared=parts, first_turn=False)
    assert st == {"declared": True, "verified": True, "parts": [KIND_AGENT_DIRECTIVE, KIND_TOOL_OUTPUT,
                                                                KIND_AGENT_DIRECTIVE]}
    kinds = [e[0] for e in ev]
    assert kinds[-3:] == [EventType.CONVERSATION_MESSAGE, EventType.TOOL_OUTPUT, EventType.USER_REQUEST]
    led.record(ev)
    # next call: the prompt is one history message now; its directive is settled, not ingested again
    ev2, _ = terminus_turn_events("next prompt", [{"role": "user", "content": prompt}], ledger=led, registry=reg,
                                  declared=None, first_turn=False)
    assert all(e[2] != prompt for e in ev2)
    assert any(e[3].get("prompt_part") == KIND_AGENT_DIRECTIVE and e[0] == EventType.CONVERSATION_MESSAGE
               for e in ev2)
    ev3, st3 = terminus_turn_events("p", [], ledger=SourceLedger(), registry=reg, declared=parts, first_turn=True)
    assert ev3[0][0] == EventType.TASK_INSTRUCTION and not st3["verified"]


# ------------------------------------------------------------------- agents
def test_split_text_and_response_parsing():
    chunks = split_text("a" * 10 + "\n\n" + "b" * 10 + "\n" + "c" * 30, 25)
    assert all(len(c) <= 25 for c in chunks) and "".join(chunks).replace("\n", "") == "a" * 10 + "b" * 10 + "c" * 30
    r = parse_agent_response('sure:\n```json\n{"commands": [{"keystrokes": "ls\\n"}], "is_task_complete": true}\n```')
    assert r.is_task_complete and r.commands[0].keystrokes == "ls\n"
    for bad in ("no json", '{"commands": [{"x": 1}]}', '{"commands": "ls"}'):
        with pytest.raises(ValueError):
            parse_agent_response(bad)


def test_pic_llm_compiles_each_block_once_and_links():
    calls = []

    def transport(body):
        calls.append(body)
        return {"choices": [{"message": {"content": "ok"}}], "usage": {"prompt_tokens": 7, "completion_tokens": 1}}

    llm = PICLLM(transport, model="m", legolink_k=32, block_chars=60)
    llm.set_task_context("task-1")
    assert llm.call("first prompt that is long enough to cut in two") == "ok"
    first = [c for c in calls if "sub_context" in c]
    link = [c for c in calls if "pic_link" in c][0]["pic_link"]
    assert len(first) == 1 and link["cache_keys"] == [first[0]["sub_context"]["cache_key"]]
    assert link["block_ids"][0].startswith("agent::task-1::") and link["recompute_initial_tokens"] == 32
    calls.clear()
    llm.call("second", [{"role": "user", "content": "first prompt that is long enough to cut in two"},
                        {"role": "assistant", "content": "ok " * 40}])
    compiles = [c for c in calls if "sub_context" in c]
    link = [c for c in calls if "pic_link" in c][0]["pic_link"]
    assert len(link["cache_keys"]) >= 3 and len(compiles) == len(link["cache_keys"]) - 1  # the prompt's half is reused
    with pytest.raises(ValueError):
        PICLLM(transport, model="m", recompute_mode="tokenwise")


def test_pic_llm_against_the_cpu_runtime():
    from sglang_legolink_b200.server.http_server import build_service

    svc = build_service("tiny-qwen2", device="cpu", max_context=4096, legolink_only=True)
    try:
        llm = PICLLM(svc.complete, model="tiny", legolink_k=8, block_chars=200, max_tokens=3)
        out1 = llm.call("Task: count the files in the repository and report the number.")
        out2 = llm.call("What is next?", [{"role": "user", "content": "Task: count the files in the repository and "
                                                                      "report the number."},
                                          {"role": "assistant", "content": out1 or "done"}])
        assert isinstance(out1, str) and isinstance(out2, str)
        assert svc.scheduler.engine.stats["links"] == 2
    finally:
        svc.scheduler.stop()


class ScriptedLLM:
    def __init__(self, answers):
        self.answers, self.prompts, self.declared = list(answers), [], []

    def call(self, prompt, history):
        self.prompts.append(prompt)
        return self.answers.pop(0)

    def declare_prompt_structure(self, parts):
        self.declared.append(parts)


class FakeTerminal:
    def __init__(self):
        self.sent, self.screen = [], "$ "

    def send_keys(self, keys, *, block=False, timeout_sec=180.0):
        self.sent.append(keys)
        self.screen += f"{keys.strip()}\nout-of-{keys.strip()}\n$ "

    def capture(self):
        return self.screen


def _cmd(*ks, done=False):
    return json.dumps({"commands": [{"keystrokes": k + "\n", "is_blocking": True} for k in ks],
                       "is_task_complete": done})


def test_terminal_agent_loop_outcomes():
    llm = ScriptedLLM(["garbage", _cmd("ls"), _cmd("make", done=True)])
    term = FakeTerminal()
    res = TerminalAgent(llm).perform_task("build it", term)
    assert res.is_task_complete and res.failure_mode == "none" and res.invalid_responses == 1
    assert term.sent == ["ls\n", "make\n"] and "out-of-ls" in llm.prompts[-1]
    rep = TerminalAgent(ScriptedLLM([_cmd("ls")] * 5), max_repeats=2).perform_task("x", FakeTerminal())
    assert rep.failure_mode == "repeated_actions"
    assert TerminalAgent(ScriptedLLM([_cmd("a"), _cmd("b")]), max_steps=2).perform_task(
        "x", FakeTerminal()).failure_mode == "max_steps"
    assert TerminalAgent(ScriptedLLM(["x"] * 9), max_invalid=2).perform_task(
        "x", FakeTerminal()).failure_mode == "invalid_responses"


def test_terminus2_declares_terminal_output_as_a_tool_result():
    llm = ScriptedLLM([_cmd("ls"), _cmd("pwd", done=True)])
    NOCTerminus2Agent(llm).perform_task("where am I", FakeTerminal())
    assert llm.declared and [p.kind for p in llm.declared[0]] == [KIND_AGENT_DIRECTIVE, KIND_TOOL_OUTPUT,
                                                                  KIND_AGENT_DIRECTIVE]
    assert "out-of-ls" in llm.declared[0][1].text


def test_noc_llm_turns_through_the_pipeline(tmp_path):
    tok = HashTokenizer(vocab_size=4096)
    fake = StrictFakeRuntime()
    ad = RuntimeAdapter(fake, model="legolink", tokenizer=tok,
                        repair_planner=RepairWindowPlanner(UniformRepairWindow(8)),
                        generation={"max_tokens": 4, "temperature": 0.0})
    llm = NOCLLM(RequestPipeline(ContextManager("noc-agent", tokenizer=tok), ad),
                 recorder=MetricsRecorder(tmp_path / "m.jsonl"))
    task = "Task: repair the failing unit tests in the payments module. " * 12
    answer = llm.call(task)
    assert isinstance(answer, str)
    out = "FAILED tests/test_pay.py::test_refund - AssertionError " * 20
    prompt = "Output of your last commands:\n" + out + "\n\nWhat next?"
    llm.declare_prompt_structure(split_around(prompt, out))
    llm.call(prompt, [{"role": "user", "content": task}, {"role": "assistant", "content": answer}])
    rows = read_jsonl(tmp_path / "m.jsonl")
    assert len(rows) == 2 and rows[1]["ingress_structure"]["verified"] is True
    fields = {v.context_field for v in llm.pipeline.manager.contexts()}
    assert "tool_history_output" in fields  # the terminal output is a tool result, not the user's request
    assert not fake.plain_generation_requests()


def test_subprocess_terminal_and_tmux_adapter(tmp_path):
    t = SubprocessTerminal(cwd=str(tmp_path))
    t.send_keys("echo hello-agent\n", block=True, timeout_sec=10)
    assert "hello-agent" in t.capture()

    class Pane:
        def __init__(self):
            self.keys = []

        def send_keys(self, keys, block=False, max_timeout_sec=0):
            self.keys.append((keys, block, max_timeout_sec))

        def capture_pane(self):
            return "pane"

    p = Pane()
    a = TmuxSessionAdapter(p)
    a.send_keys("ls", block=True, timeout_sec=5)
    assert p.keys == [("ls", True, 5)] and a.capture() == "pane"
