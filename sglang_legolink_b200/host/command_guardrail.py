"""Command guardrail for terminal agents whose replies are JSON objects with
``commands[i].keystrokes`` strings (the Terminus-2 parser format).

Small models driving a terminal repeat a few failure patterns that cost a
whole turn each: a long or compound ``python3 -c`` one-liner that the shell
mangles, a heredoc split across keystroke strings (the shell then waits for
input), an empty heredoc, ``json.load`` on a CSV file, or running a helper
script that nobody created.  :func:`command_violation` checks only the
keystrokes a reply would send (never its free-text analysis or plan) against
an ordered rule table and names the first rule that fires;
:func:`replan_prompt` asks the model to answer again in the same format, and
:func:`safe_diagnostic_response` is a parser-safe reply that inspects the
workspace instead of running the blocked command.

Reference: the Terminal-Bench guardrail of the reference's proxy
(``terminal_bench_integration/noc_openai_proxy.py``; behaviour pinned by
``tests/test_noc_openai_proxy.py:144-270``).  The rules here are this
module's own table; the violation messages are the ones that file's callers
match on.
"""

from __future__ import annotations

import json
import re
from typing import Callable, Optional

PY_C_MAX = 900  # longer python3 -c programs are refused whatever they contain

MSG_PY_C = ("unsafe python3 -c command with multi-statement or compound Python detected; use a heredoc or write a "
            "temporary Python file instead")
MSG_HEREDOC_UNCLOSED = "heredoc opener detected without a standalone closing PY marker in the same keystrokes string"
MSG_HEREDOC_EMPTY = ("empty or malformed heredoc detected; put the script body after the heredoc opener and a "
                     "standalone closing PY marker before running it")
MSG_HEREDOC_INTERACTIVE = ("interactive python heredoc detected; Terminal-Bench JSON commands must put the complete "
                           "heredoc body and closing PY marker inside one keystrokes string")
MSG_CSV_JSON = "CSV input is being parsed with json.load instead of csv.DictReader"
MSG_HELPER = "helper script path is assumed before verifying or creating the file"

_PY_C = re.compile(r"python3?\s+-c\s+(['\"])(?P<body>.*)", re.S)
_OPENER = re.compile(r"<<\s*'?PY'?")
_CLOSER = re.compile(r"(^|\n)PY[ \t]*(\n|$)")
_CSV_JSON = re.compile(r"json\.loads?\(\s*open\([^)]*\.csv", re.S)
_HELPER = re.compile(r"^\s*python3?\s+(/app/[\w./-]+\.py)\b")
_COMPOUND = re.compile(r";|\bfor\b|\bwhile\b|\bif\b|\bwith\b|\btry\b|\bdef\b|\bimport\b.*\n")


def command_strings(reply: str) -> list[str]:
    """The keystrokes a reply would send: ``commands[i].keystrokes`` of a JSON
    reply, else the whole reply taken as one command line."""
    try:
        obj = json.loads(reply)
    except (TypeError, ValueError):
        return [reply]
    if isinstance(obj, dict) and isinstance(obj.get("commands"), list):
        return [c["keystrokes"] for c in obj["commands"] if isinstance(c, dict) and isinstance(c.get("keystrokes"), str)]
    return [reply] if not isinstance(obj, dict) else []


def _py_c(ks: str) -> bool:
    m = _PY_C.search(ks)
    if not m:
        return False
    body = m.group("body")
    return len(ks) > PY_C_MAX or bool(_COMPOUND.search(body))


def _heredoc(ks: str) -> Optional[str]:
    m = _OPENER.search(ks)
    if not m:
        return None
    after = ks[m.end():]
    close = _CLOSER.search(after)
    if close is None:
        # the opener and more shell on the same line ("<<'PY' && python3 x.py") is a heredoc with no body
        first_line = after.split("\n", 1)[0]
        return MSG_HEREDOC_EMPTY if first_line.strip() else MSG_HEREDOC_UNCLOSED
    body = after[: close.start()]
    if not body.strip("\n").strip():
        return MSG_HEREDOC_EMPTY
    if re.search(r"python3?\s+-\s*<<", ks):
        return MSG_HEREDOC_INTERACTIVE  # stdin heredoc into an interpreter: write the file, then run it
    return None


# ordered: the first rule that fires names the violation
RULES: list[tuple[Callable[[str], Optional[str]], str]] = [
    (lambda ks: MSG_CSV_JSON if _CSV_JSON.search(ks) else None, "csv_json"),
    (_heredoc, "heredoc"),
    (lambda ks: MSG_PY_C if _py_c(ks) else None, "python_c"),
    (lambda ks: MSG_HELPER if _HELPER.search(ks) else None, "helper_script"),
]


def command_violation(reply: str) -> Optional[str]:
    """The first rule violated by any keystrokes string of ``reply``, or None."""
    for ks in command_strings(reply):
        for rule, _name in RULES:
            msg = rule(ks)
            if msg:
                return msg
    return None


def replan_prompt(violation: str) -> str:
    return (f"Your previous reply was blocked: {violation}. Answer again in the same parser format. Do not repeat "
            "the blocked command. Write scripts to a file first, e.g. cat > /tmp/solve.py <<'PY' ... PY, with the "
            "whole heredoc (opener, body and closing PY line) inside a single commands[i].keystrokes string, then "
            "run python3 /tmp/solve.py. Return only the JSON object.")


def safe_diagnostic_response(violation: str) -> str:
    """A reply that passes the guardrail and the parser: it reports the block
    and lists the workspace so the next turn starts from facts."""
    ks = (f"printf '%s\\n' 'NOC_GUARDRAIL_BLOCKED: {violation}' "
          "'NOC_GUARDRAIL_NEXT_ACTION: inspect the files, then write any script to a file before running it'; "
          "find /app -maxdepth 2 -type f | head -n 50; for f in $(find /app -maxdepth 2 -name '*.csv' | head -n 3); "
          "do sed -n '1,8p' \"$f\"; done\n")
    return json.dumps({"analysis": "The previous command was blocked by the guardrail.",
                       "plan": "Inspect the workspace before acting.",
                       "commands": [{"keystrokes": ks, "duration": 1.0}], "task_complete": False})


# ------------------------------------------------------------ verification
# A command that changes files silently (a redirect, mkdir, chmod, cp / mv)
# leaves the terminal pane blank, and small models then repeat it or guess.
# The probe appended after such a command prints the evidence: the target's
# listing, its size and its first bytes.  A command whose targets cannot be
# named (a generated script) gets the task directory's listing instead.

PROBE_MARK = "NOC_VERIFY"
WORKDIR = "/app"
PROBE_EXTRA_S = 1.0  # the pane is captured after `duration`: leave the probe time to print

_REDIRECT = re.compile(r"(?<![0-9&])>>?\s*([^\s;&|<>]+)")
_MUTATORS = {"mkdir": "all", "touch": "all", "chmod": "last", "chown": "last", "cp": "last", "mv": "last",
             "ln": "last", "tee": "all"}
_SCRIPT_RUN = re.compile(r"^\s*(python3?|bash|sh|node)\s+\S+")


def _targets(ks: str) -> list[str]:
    """Paths a command line writes: redirect targets, then the operands of
    mutating commands (the destination of cp / mv / ln / chmod, every
    operand of mkdir / touch / tee); options, modes and /dev/* are skipped."""
    out: list[str] = []
    for line in ks.splitlines():
        for m in _REDIRECT.finditer(line):
            out.append(m.group(1).strip("'\""))
        for seg in re.split(r"&&|\|\||;|\|", line):
            words = seg.split()
            if not words or words[0] not in _MUTATORS:
                continue
            ops = [w.strip("'\"") for w in words[1:]
                   if not w.startswith("-") and not re.fullmatch(r"[0-7]{3,4}|[ugoa]*[+-=][rwxXst]+", w)]
            ops = [w for w in ops if not any(c in w for c in "<>")]
            if ops:
                out.extend(ops if _MUTATORS[words[0]] == "all" else ops[-1:])
    seen, res = set(), []
    for t in out:
        if t and not t.startswith("/dev/") and t not in seen:
            seen.add(t)
            res.append(t)
    return res


def verification_probe(keystrokes: str) -> Optional[str]:
    """Shell lines that print what ``keystrokes`` changed, or None for a
    command that changes nothing observable."""
    targets = _targets(keystrokes)
    if not targets:
        if not any(_SCRIPT_RUN.match(line) for line in keystrokes.splitlines()):
            return None
        return f"echo '{PROBE_MARK}: {WORKDIR}'; ls -la '{WORKDIR}'\n"
    parts = []
    for t in targets[:4]:
        parts.append(f"echo '{PROBE_MARK}: {t}'; ls -ld '{t}'; if [ -f '{t}' ]; then "
                     f"echo \"{PROBE_MARK}_FILE_BYTES $(wc -c < '{t}')\"; echo '{PROBE_MARK}_FILE_HEAD_BEGIN'; "
                     f"head -c 400 '{t}'; echo; echo '{PROBE_MARK}_FILE_HEAD_END'; fi")
    return "; ".join(parts) + "\n"


def inject_verification(reply: str) -> tuple[str, Optional[str]]:
    """Appends the probe to each command of a JSON reply that changes files
    and lengthens its duration so the probe's output is on the captured
    pane.  Returns (reply, first probed target or None).  Idempotent: a reply
    that already carries probes, or changes nothing, comes back unchanged."""
    try:
        obj = json.loads(reply)
    except (TypeError, ValueError):
        return reply, None
    if not isinstance(obj, dict) or not isinstance(obj.get("commands"), list):
        return reply, None
    if any(isinstance(c, dict) and PROBE_MARK in str(c.get("keystrokes", "")) for c in obj["commands"]):
        return reply, None
    first = None
    for c in obj["commands"]:
        if not isinstance(c, dict) or not isinstance(c.get("keystrokes"), str):
            continue
        probe = verification_probe(c["keystrokes"])
        if probe is None:
            continue
        ks = c["keystrokes"] if c["keystrokes"].endswith("\n") else c["keystrokes"] + "\n"
        c["keystrokes"] = ks + probe
        c["duration"] = float(c.get("duration") or 0.0) + PROBE_EXTRA_S
        if first is None:
            t = _targets(ks)
            first = t[0] if t else WORKDIR
    return (json.dumps(obj), first) if first is not None else (reply, None)
