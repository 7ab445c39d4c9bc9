"""The server CLI on two GPUs (one process per GPU, spawned by the server):

* ``--tp-size 2`` with the fused NVLink TP boundary: startup warmup, Compile,
  Link (JSON and SSE give the same tokens), a refused Link, and an orderly
  shutdown on SIGTERM;
* ``--dp-size 2``: a block compiled through the router is linked on the other
  replica (read from the owner's pool over NVLink) to the same tokens as on
  the owner.

The test sends SIGTERM to the process group it started; rank 0 turns it into
a shutdown message that the other rank handles between steps.
"""

import json
import os
import signal
import socket
import subprocess
import sys
import time
import urllib.error
import urllib.request

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _post(base, body, stream=False):
    req = urllib.request.Request(base + "/v1/chat/completions", data=json.dumps(body).encode(),
                                 headers={"Content-Type": "application/json"})
    try:
        with urllib.request.urlopen(req, timeout=300) as r:
            raw = r.read().decode()
            return r.status, raw if stream else json.loads(raw)
    except urllib.error.HTTPError as e:
        return e.code, json.loads(e.read().decode())


def _msgs(t):
    return [{"role": "user", "content": t}]


def _start(flags, port):
    env = {**os.environ, "NCCL_NVLS_ENABLE": "0", "TORCH_SYMM_MEM_DISABLE_MULTICAST": "1",
           "PYTHONPATH": ROOT + os.pathsep + os.environ.get("PYTHONPATH", "")}
    p = subprocess.Popen(["timeout", "-k", "90", "600", sys.executable, "-m", "sglang_legolink_b200.server.http_server",
                          "--model", "small-qwen3", "--port", str(port), "--context-length", "4096", *flags],
                         cwd=ROOT, env=env, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True,
                         start_new_session=True)
    lines, t0 = [], time.time()
    while time.time() - t0 < 400:
        line = p.stdout.readline()
        if not line:
            break
        lines.append(line)
        if line.startswith("serving "):
            return p, lines
    _stop(p)
    raise AssertionError("server did not start:\n" + "".join(lines[-60:]))


def _stop(p):
    try:
        os.killpg(p.pid, signal.SIGTERM)
    except ProcessLookupError:
        pass
    try:
        out, _ = p.communicate(timeout=180)
    except subprocess.TimeoutExpired:
        os.killpg(p.pid, signal.SIGKILL)
        out, _ = p.communicate()
    return out


@pytest.mark.gpu
@pytest.mark.multigpu
def test_tp2_server_fused_boundary():
    port = _free_port()
    p, lines = _start(["--tp-size", "2"], port)
    base = f"http://127.0.0.1:{port}"
    try:
        assert any(line.startswith("warmup") for line in lines), lines
        for key, text in (("g-a", "tool output " * 200), ("g-b", "instructions " * 120)):
            code, r = _post(base, {"messages": _msgs(text), "max_tokens": 1, "sub_context": {"cache_key": key}})
            assert code == 200 and r["meta_info"]["compile"]["status"] == "registered", r
        link = {"messages": _msgs("what next?"), "max_tokens": 8, "ignore_eos": True,
                "pic_link": {"cache_keys": ["g-b", "g-a"], "recompute_initial_tokens": 16}}
        code, r = _post(base, link)
        assert code == 200 and len(r["meta_info"]["output_ids"]) == 8, r
        code, raw = _post(base, dict(link, stream=True), stream=True)
        frames = [json.loads(x[6:]) for x in raw.split("\n\n") if x.startswith("data: {")]
        assert [c["meta_info"]["token_id"] for c in frames if "meta_info" in c] == r["meta_info"]["output_ids"]
        code, bad = _post(base, {"messages": _msgs("x"), "max_tokens": 2, "pic_link": {"cache_keys": ["none"]}})
        assert code in (200, 400) and ("error" in json.dumps(bad) or code == 400)
        code, again = _post(base, link)
        assert code == 200 and again["meta_info"]["output_ids"] == r["meta_info"]["output_ids"]
    finally:
        out = _stop(p)
    assert p.returncode == 0, "".join(lines) + out[-3000:]


@pytest.mark.gpu
@pytest.mark.multigpu
def test_dp2_server_cross_replica_link():
    port = _free_port()
    p, lines = _start(["--dp-size", "2", "--skip-warmup"], port)
    base = f"http://127.0.0.1:{port}"
    try:
        code, r = _post(base, {"messages": _msgs("tool output " * 200), "max_tokens": 1,
                               "sub_context": {"cache_key": "d-a"}})
        assert code == 200, r
        assert r["meta_info"]["dp_replica"] == 0  # idle replicas: the first one
        link = {"messages": _msgs("what next?"), "max_tokens": 8, "ignore_eos": True,
                "pic_link": {"cache_keys": ["d-a"], "recompute_initial_tokens": 16}}
        code, local = _post(base, link)
        assert code == 200 and local["meta_info"]["dp_replica"] == 0  # block locality breaks the tie
        # replica 1 links the block out of replica 0's pool over NVLink
        code, peer = _post(f"http://127.0.0.1:{port + 1}", link)
        assert code == 200 and peer["meta_info"]["output_ids"] == local["meta_info"]["output_ids"]
        with urllib.request.urlopen(f"http://127.0.0.1:{port + 1}/model_info", timeout=60) as h:
            assert json.loads(h.read())["engine_stats"]["remote_blocks_linked"] >= 1
    finally:
        out = _stop(p)
    assert p.returncode == 0, "".join(lines) + out[-3000:]
