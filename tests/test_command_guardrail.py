"""Terminal-agent command guardrail: the rule table on the keystrokes a reply
would send, the replan prompt and the parser-safe diagnostic reply, and the
proxy's use of them (re-ask, then block)."""

import json

from sglang_legolink_b200.host import command_guardrail as cg
from sglang_legolink_b200.host.fake_runtime import StrictFakeRuntime
from sglang_legolink_b200.host.tokenizer import HashTokenizer
from sglang_legolink_b200.server.proxy import LegoLinkProxy


def _reply(*keystrokes):
    return json.dumps({"analysis": "a", "plan": "p", "commands": [{"keystrokes": k, "duration": 0.1} for k in keystrokes]})


def test_rules_name_the_first_violation():
    assert cg.command_violation("python3 -c '" + "x" * 950) == cg.MSG_PY_C
    assert cg.command_violation("python3 -c 'items=[]; for row in rows: items.append(row)'") == cg.MSG_PY_C
    assert cg.command_violation(_reply("python3 - <<'PY'\n")) == cg.MSG_HEREDOC_UNCLOSED
    assert cg.command_violation(_reply("cat > /tmp/solve.py <<'PY' && python3 /tmp/solve.py\n")) == cg.MSG_HEREDOC_EMPTY
    assert cg.command_violation(_reply("python3 - <<'PY'\nprint(1)\nPY\n")) == cg.MSG_HEREDOC_INTERACTIVE
    assert cg.command_violation('python3 -c "json.load(open(\\"/app/data/input.csv\\"))"') == cg.MSG_CSV_JSON
    assert cg.command_violation("python3 /app/process_csv.py /app/data/a.csv /tmp/a.json") == cg.MSG_HELPER
    assert cg.command_violation(_reply("ls\n", "python3 /app/transform_csv_to_json.py\n")) == cg.MSG_HELPER


def test_safe_commands_and_analysis_text_pass():
    text = json.dumps({"analysis": "I should not use python3 -c or json.load on a .csv file.", "plan": "Use safe commands.",
                       "commands": [{"keystrokes": "printf '%s\\n' ok\n", "duration": 0.1}]})
    assert cg.command_violation(text) is None
    assert cg.command_violation(_reply("cat > /tmp/solve.py <<'PY'\nimport csv\nprint(1)\nPY\npython3 /tmp/solve.py\n")) is None
    assert cg.command_violation("python3 -c 'print(1)'") is None


def test_replan_prompt_and_diagnostic_reply():
    p = cg.replan_prompt("bad command")
    assert "same parser format" in p and "single commands[i].keystrokes string" in p and "Do not repeat" in p
    r = cg.safe_diagnostic_response("bad command")
    ks = json.loads(r)["commands"][0]["keystrokes"]
    assert "NOC_GUARDRAIL_BLOCKED: bad command" in ks and "NOC_GUARDRAIL_NEXT_ACTION:" in ks
    assert "find /app -maxdepth 2 -type f" in ks and "sed -n '1,8p'" in ks
    assert cg.command_violation(r) is None


def test_proxy_reasks_then_blocks_a_violating_reply(monkeypatch):
    px = LegoLinkProxy(StrictFakeRuntime(), tokenizer=HashTokenizer(vocab_size=4096), repair_tokens=8,
                       json_retries=2, command_guardrail=True)
    bad = "python3 /app/process_csv.py /app/a.csv"
    from sglang_legolink_b200.host import agent as agent_mod

    calls = []

    def fake_call(self, messages, tools=None, **kw):
        calls.append(messages)
        return type("R", (), {"text": bad, "metric": {}, "execution": type("E", (), {
            "result": type("X", (), {"response": {}})(), "compile_requests": 0,
            "route": type("Rt", (), {"value": "fake"})()})()})()

    monkeypatch.setattr(agent_mod.AgentLLM, "call", fake_call)
    out = px.chat_completion({"messages": [{"role": "user", "content": "convert the csv"}], "session_id": "g"})
    text = out["choices"][0]["message"]["content"]
    assert len(calls) == 3 and px.stats["guardrail_replans"] == 2 and px.stats["guardrail_blocked"] == 1
    assert "NOC_GUARDRAIL_BLOCKED" in text and cg.command_violation(text) is None
    assert "Do not repeat" in calls[-1][-1]["content"]
