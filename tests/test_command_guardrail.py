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


def test_verification_probe_targets():
    p = cg.verification_probe("echo 'Hello, world!' > /app/hello.txt\n")
    assert "NOC_VERIFY" in p and "ls -ld '/app/hello.txt'" in p and "head -c 400 '/app/hello.txt'" in p
    assert "NOC_VERIFY_FILE_BYTES" in p and "NOC_VERIFY_FILE_HEAD_BEGIN" in p and "NOC_VERIFY_FILE_HEAD_END" in p
    assert "ls -ld '/app'" in cg.verification_probe("mkdir -p /app\n")
    assert "ls -ld '/app/run.sh'" in cg.verification_probe("chmod 644 /app/run.sh\n")
    assert "'644'" not in cg.verification_probe("chmod 644 /app/f.txt\n")
    cp = cg.verification_probe("cp /app/a.csv /app/b.csv\n")
    assert "head -c 400 '/app/b.csv'" in cp and "head -c 400 '/app/a.csv'" not in cp  # the destination, not the source
    assert "ls -la '/app'" in cg.verification_probe("python3 /tmp/solve.py\n")  # unnamed outputs: the task directory
    for read_only in ("cat /app/schema.json\n", "ls -la /app\n", "grep foo /app/x.txt 2>&1\n", "cmd > /dev/null\n"):
        assert cg.verification_probe(read_only) is None, read_only


def test_inject_verification():
    o = json.dumps({"analysis": "w", "plan": "e",
                    "commands": [{"keystrokes": "echo 'Hello, world!' > /app/hello.txt\n", "duration": 1.0}]})
    i, reason = cg.inject_verification(o)
    c = json.loads(i)["commands"][0]
    assert reason == "/app/hello.txt" and c["duration"] > 1.0
    assert c["keystrokes"].startswith("echo 'Hello, world!' > /app/hello.txt\n") and "NOC_VERIFY" in c["keystrokes"]
    assert cg.command_violation(i) is None  # the probe never trips the guardrail
    once, r1 = cg.inject_verification(json.dumps({"commands": [{"keystrokes": "mkdir -p /app\n", "duration": 1.0}]}))
    twice, r2 = cg.inject_verification(once)
    assert r1 and r2 is None and twice == once  # idempotent
    ro = json.dumps({"commands": [{"keystrokes": "cat /app/schema.json\n", "duration": 1.0}]})
    assert cg.inject_verification(ro) == (ro, None)
