"""Decode under KV pressure (CPU, tiny random Qwen2, a 24-page pool): the
most recently admitted request is retracted so the others keep decoding.  A
plain request is re-queued and resumes from its prompt + generated tokens to
the same tokens it produces alone; a Link fails closed with the retraction
reason (reference ``pic_runtime.py:2978-3007``)."""

import torch

from sglang_legolink_b200.models.config import PRESETS
from sglang_legolink_b200.models.qwen import QwenModel
from sglang_legolink_b200.runtime.engine import Engine
from sglang_legolink_b200.runtime.scheduler import Request, Scheduler


def _engine(pages=24):
    return Engine(QwenModel.random_init(PRESETS["tiny-qwen2"], seed=0), num_pages=pages, page_size=16,
                  max_context=1024)


def _prompts():
    g = torch.Generator().manual_seed(11)
    return [torch.randint(1, 1000, (100,), generator=g).tolist() for _ in range(2)]


def _drain(sch, reqs, limit=2000):
    for _ in range(limit):
        if all(not r.events.empty() and r.events.queue[-1][0] in ("done", "error") for r in reqs):
            return
        sch.step()
    raise AssertionError("requests did not finish")


def _tokens(r):
    return [v for k, v in list(r.events.queue) if k == "token"]


def test_plain_request_is_retracted_and_resumes():
    alone = []
    for ids in _prompts():
        sch = Scheduler(_engine(64), legolink_only=False)
        r = Request("plain", "solo", ids, 120)
        sch.submit(r)
        _drain(sch, [r])
        alone.append(_tokens(r))
    sch = Scheduler(_engine(), legolink_only=False)
    reqs = [Request("plain", f"p{i}", ids, 120) for i, ids in enumerate(_prompts())]
    for r in reqs:
        sch.submit(r)
    _drain(sch, reqs)
    assert sch.stats.get("retracted", 0) >= 1
    assert [r.events.queue[-1][0] for r in reqs] == ["done", "done"]
    assert [_tokens(r) for r in reqs] == alone


def test_link_is_retracted_fail_closed():
    eng = _engine()
    a, b = _prompts()
    eng.compile(b[:64], "blk")
    sch = Scheduler(eng, legolink_only=False)
    plain = Request("plain", "p", a, 120)
    sch.submit(plain)
    sch.step()  # the plain request is admitted first
    link = Request("link", "l", b[64:], 120, pic_link={"cache_keys": ["blk"], "recompute_initial_tokens": 8})
    sch.submit(link)
    _drain(sch, [plain, link])
    assert link.events.queue[-1] == ("error", Scheduler.LINK_RETRACTED)
    assert plain.events.queue[-1][0] == "done" and len(_tokens(plain)) == 120
    # nothing leaked: every page but the scratch page is free or evictable again
    assert sch._pages_free() == eng.kv.num_pages - 1
