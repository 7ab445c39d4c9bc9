"""The runtime's HTTP API on CPU (tiny random Qwen2, hash tokenizer):
Compile and Link through /v1/chat/completions (JSON and SSE), refusals
(plain generation in LegoLink-only mode, Compile+Link in one request, Link
input logprobs, runtime-owned fields, a missing block with its recovery
detail), /v1/tokenize, /health, /v1/models, /model_info and the startup
warmup."""

import json
import urllib.error
import urllib.request

import pytest

from sglang_legolink_b200.contract import parse_residency_recovery
from sglang_legolink_b200.server.http_server import build_service, serve


@pytest.fixture(scope="module")
def server():
    svc = build_service("tiny-qwen2", device="cpu", max_context=4096)
    srv = serve(svc, "127.0.0.1", 0)
    yield svc, f"http://127.0.0.1:{srv.server_address[1]}"
    srv.shutdown()
    svc.scheduler.stop()


def _post(base, path, body, stream=False):
    req = urllib.request.Request(base + path, data=json.dumps(body).encode(),
                                 headers={"Content-Type": "application/json"})
    try:
        with urllib.request.urlopen(req, timeout=120) as r:
            raw = r.read().decode()
            return r.status, raw if stream else json.loads(raw)
    except urllib.error.HTTPError as e:  # refusals answer JSON, streaming or not
        return e.code, json.loads(e.read().decode())


def _get(base, path):
    with urllib.request.urlopen(base + path, timeout=30) as r:
        return r.status, json.loads(r.read().decode())


def _msgs(text):
    return [{"role": "user", "content": text}]


def test_compile_link_json_and_sse(server):
    svc, base = server
    code, r = _post(base, "/v1/chat/completions", {"messages": _msgs("tool output " * 60), "max_tokens": 1,
                                                   "sub_context": {"cache_key": "http-a"}})
    assert code == 200 and r["meta_info"]["kind"] == "compile" and r["meta_info"]["compile"]["status"] == "registered"
    _post(base, "/v1/chat/completions", {"messages": _msgs("instructions " * 40), "max_tokens": 1,
                                         "sub_context": {"cache_key": "http-b"}})
    link = {"cache_keys": ["http-b", "http-a"], "recompute_initial_tokens": 8}
    code, r = _post(base, "/v1/chat/completions", {"messages": _msgs("what next?"), "max_tokens": 6,
                                                   "ignore_eos": True, "pic_link": link})
    assert code == 200 and r["meta_info"]["kind"] == "link" and len(r["meta_info"]["output_ids"]) == 6
    assert r["meta_info"]["link"]["recompute_rows"] > 0
    code, raw = _post(base, "/v1/chat/completions", {"messages": _msgs("what next?"), "max_tokens": 6,
                                                     "ignore_eos": True, "pic_link": link, "stream": True},
                      stream=True)
    frames = [x[len("data: "):] for x in raw.split("\n\n") if x.startswith("data: ")]
    assert code == 200 and frames[-1] == "[DONE]"
    chunks = [json.loads(f) for f in frames[:-1]]
    ids = [c["meta_info"]["token_id"] for c in chunks if "meta_info" in c]
    assert ids == r["meta_info"]["output_ids"] and chunks[-1]["choices"][0]["finish_reason"] == "length"


def test_refusals_are_request_scoped(server):
    svc, base = server
    cases = [
        {"messages": _msgs("hello"), "max_tokens": 4},  # plain generation in LegoLink-only mode
        {"messages": _msgs("x"), "sub_context": {"cache_key": "z"}, "pic_link": {"cache_keys": ["z"]}},
        {"messages": _msgs("x"), "pic_link": {"cache_keys": ["http-a"]}, "input_logprobs": True},
        {"messages": _msgs("x"), "pic_link": {"cache_keys": ["http-a"], "imp_indices": [0, 1]}},
        {"messages": _msgs("x"), "pic_link": {"cache_keys": ["http-a"], "not_a_field": 1}},
        {"messages": _msgs("x"), "pic_link": {"cache_keys": "http-a"}},
    ]
    for body in cases:
        code, r = _post(base, "/v1/chat/completions", body)
        assert code == 400 and r["object"] == "error", body
        code, r = _post(base, "/v1/chat/completions", dict(body, stream=True), stream=True)
        assert code == 400, body
    # a missing block: the recovery detail names it
    code, r = _post(base, "/v1/chat/completions", {"messages": _msgs("x"), "max_tokens": 2,
                                                   "pic_link": {"cache_keys": ["never-compiled"]}})
    assert code == 400 and "never-compiled" in parse_residency_recovery(r["message"])["missing"]
    # the server still serves
    assert _get(base, "/health") == (200, {"status": "ok"})


def test_tokenize_models_model_info_and_warmup(server):
    svc, base = server
    code, r = _post(base, "/v1/tokenize", {"messages": _msgs("count these words")})
    assert code == 200 and r["count"] == len(r["tokens"]) > 0
    code, r = _post(base, "/v1/tokenize", {"prompt": "a b c"})
    assert code == 200 and r["count"] == len(r["tokens"])
    code, r = _get(base, "/v1/models")
    assert r["data"][0]["id"] == svc.model_name
    code, info = _get(base, "/model_info")
    assert info["legolink_only"] and info["page_size"] == 16 and "legolink_stats" in info
    w = svc.warmup(block_tokens=64, k=8)
    assert w["compile_s"] > 0 and w["link_s"] > 0
