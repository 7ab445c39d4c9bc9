"""Host token reuse (NOC_HOST_TOKEN_REUSE, off by default): framing answers
block tokenization from ids the stored sub-contexts hold, refuses ids of
another tokenizer, never encodes a text twice in a request, and produces the
same layout as the plain path (reference
``noc_context_manager/authoritative_tokens.py``)."""

from dataclasses import replace

from sglang_legolink_b200.host.adapter import RequestPipeline, RuntimeAdapter
from sglang_legolink_b200.host.events import SourceSpan
from sglang_legolink_b200.host.fake_runtime import StrictFakeRuntime
from sglang_legolink_b200.host.framing import RepairWindowPlanner, UniformRepairWindow
from sglang_legolink_b200.host.manager import ContextManager
from sglang_legolink_b200.host.store import SubContext
from sglang_legolink_b200.host.token_reuse import (CountingTokenizer, RequestTokenSource, SharedTokenCache,
                                                   host_token_reuse_enabled, refusal_reason)
from sglang_legolink_b200.host.tokenizer import HashTokenizer

TOK = HashTokenizer(4096)


def sc(text, tok=TOK, ids=True):
    return SubContext.create(task_id="t", context_field="tool_history_output", source_id="s",
                             spans=[SourceSpan("s", 0, len(text))], raw_text=text, tokenizer=tok, sequence_number=1,
                             source_revision=1, model_fingerprint="m", capture_token_ids=ids)


def test_flag_and_refusals():
    assert not host_token_reuse_enabled({}) and host_token_reuse_enabled({"NOC_HOST_TOKEN_REUSE": "on"})
    v = sc("hello there world")
    assert refusal_reason(v, TOK) is None
    assert refusal_reason(v, HashTokenizer(4096, name="other")) == "tokenizer_fingerprint_mismatch"
    assert refusal_reason(sc("abc", ids=False), TOK) == "no_token_ids"
    assert refusal_reason(replace(v, token_count=v.token_count + 1), TOK) == "token_count_mismatch"
    assert refusal_reason(replace(v, invalidated=True), TOK) == "invalidated"


def test_request_source_reuses_and_counts():
    v = sc("cat main.py\nprint(1)\n")
    src = RequestTokenSource(TOK, shared=SharedTokenCache(4))
    assert src.adopt(v) and not src.adopt(sc("x", tok=HashTokenizer(4096, name="z")))
    assert src.tokenize(v.raw_text) == v.token_ids
    assert src.tokenize("fresh text") == TOK.tokenize("fresh text")
    src.tokenize("fresh text")
    c = src.counts()
    assert c["calls_tokenize"] == 1 and c["reused"] == {"sub_context": 1, "request": 1}
    assert c["refused"] == {"tokenizer_fingerprint_mismatch": 1}
    msgs = [{"role": "user", "content": "hi"}]
    src.tokenize_messages(msgs)
    src.tokenize_messages(msgs)
    assert src.counts()["calls_tokenize_messages"] == 1


def test_shared_cache_is_keyed_by_fingerprint_and_bounded():
    cache = SharedTokenCache(2)
    a = RequestTokenSource(TOK, shared=cache)
    a.mark_immutable("stable block")
    ids = a.tokenize("stable block")
    b = RequestTokenSource(TOK, shared=cache)
    b.mark_immutable("stable block")
    assert b.tokenize("stable block") == ids and b.counts()["tokenizer_calls"] == 0
    other = RequestTokenSource(HashTokenizer(4096, name="other"), shared=cache)
    other.mark_immutable("stable block")
    other.tokenize("stable block")
    assert other.counts()["tokenizer_calls"] == 1  # another tokenizer: a miss, not a stale hit
    a2 = RequestTokenSource(TOK, shared=cache)
    a2.tokenize("mutable question")  # never marked immutable: stays out of the cache
    assert len(cache) == 2 and cache.memory_bytes()["raw_token_id_bytes"] > 0
    for t in ("x1", "x2", "x3"):
        cache.put(TOK.fingerprint, t, [1])
    assert len(cache) == 2 and cache.evictions >= 1


def _pipeline():
    cm = ContextManager("reuse", tokenizer=TOK, capture_token_ids=True)
    ad = RuntimeAdapter(StrictFakeRuntime(), model="m", tokenizer=CountingTokenizer(TOK),
                        repair_planner=RepairWindowPlanner(UniformRepairWindow(8)),
                        generation={"max_tokens": 2, "temperature": 0.0})
    return RequestPipeline(cm, ad)


EVENTS = [("task_instruction", "sys", "You maintain this repository. " * 40, {}),
          ("tool_output", "t1", "pytest output: 3 failed, 17 passed " * 30, {}),
          ("user_request", "q", "which test failed first?", {})]


def test_pipeline_layout_is_the_same_with_reuse(monkeypatch):
    monkeypatch.delenv("NOC_HOST_TOKEN_REUSE", raising=False)
    plain = _pipeline().execute(EVENTS)
    monkeypatch.setenv("NOC_HOST_TOKEN_REUSE", "1")
    p = _pipeline()
    reused = p.execute(EVENTS)
    assert reused.layout.assembled_token_ids == plain.layout.assembled_token_ids
    assert [s.token_ids for s in reused.layout.link_segments] == [s.token_ids for s in plain.layout.link_segments]
    assert "token_reuse" not in plain.timings_ms
    # the next turn re-frames the same blocks: their ids come from the shared cache
    turn2 = p.execute([("user_request", "q2", "and the second one?", {})])
    assert turn2.layout.link_segments[0].token_ids == reused.layout.link_segments[0].token_ids
    tr = turn2.timings_ms["token_reuse"]
    assert tr["reused"].get("shared_immutable", 0) >= 1
