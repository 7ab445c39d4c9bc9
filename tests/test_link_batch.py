"""Several Links (and Compiles) in one step: every linked token moves in one
fused KV-link launch per source pool and every repair row goes through ONE
extend forward.  The batched result equals running the Links one by one; an
item that fails fails alone; the scheduler admits the Links of a step
together instead of one Link per forward (the reference admits a Link alone
into an empty engine, ``managers/scheduler.py:2597-2690``)."""

import pytest
import torch

from sglang_legolink_b200.models.config import PRESETS
from sglang_legolink_b200.models.qwen import QwenModel
from sglang_legolink_b200.parallel.dp import LocalDirectory
from sglang_legolink_b200.runtime.engine import Engine, LinkSourceUnavailable


def _toks(n, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.randint(0, 1024, (n,), generator=g).tolist()


@pytest.fixture(scope="module")
def eng():
    e = Engine(QwenModel.random_init(PRESETS["tiny-qwen2"], seed=0), num_pages=1024, page_size=16)
    for i, n in enumerate((70, 33, 128, 9, 64)):
        e.compile(_toks(n, 100 + i), f"b{i}")
    return e


PLANS = [
    ({"cache_keys": ["b2", "b0", "b1"], "recompute_initial_tokens": 8, "recompute_first_block": True}, 11),
    ({"cache_keys": ["b3", "b4"], "recompute_initial_tokens": 4}, 5),
    ({"cache_keys": ["b1", "b1", "b2"], "recompute_tokens_per_block": [33, 2, 7]}, 17),
    ({"cache_keys": ["b4", "b2", "b3", "b0"], "recompute_initial_tokens": 0}, 3),
]


def test_batched_links_equal_serial_links(eng):
    serial = []
    for plan, n in PLANS:
        s = eng.link(dict(plan), _toks(n, n))
        eng.decode([s], 6)
        serial.append((list(s.output_ids), list(s.token_ids)))
        eng.free(s)
    free0 = eng.alloc.num_free
    out = eng.link_batch([(dict(plan), _toks(n, n)) for plan, n in PLANS])
    assert all(not isinstance(s, Exception) for s in out), out
    eng.decode(out, 6)
    for s, (ids, toks) in zip(out, serial):
        assert s.output_ids == ids
        assert s.token_ids == toks
    for s in out:
        eng.free(s)
    assert eng.alloc.num_free == free0
    for k in ("b0", "b1", "b2", "b3", "b4"):
        h = eng.registry.handle(k)
        assert h["pin_count"] == 0 and h["active_refs"] == 0


def test_batched_kv_equals_serial_kv(eng):
    plan, n = PLANS[0]
    s1 = eng.link(dict(plan), _toks(n, n))
    kv1 = [eng.kv.k[:, p].clone() for p in s1.pages], [eng.kv.v[:, p].clone() for p in s1.pages]
    eng.free(s1)
    out = eng.link_batch([(dict(p), _toks(m, m)) for p, m in PLANS[:3]])
    s2 = out[0]
    L = s2.length
    ps = eng.page_size
    for i, p in enumerate(s2.pages):
        rows = min(ps, L - i * ps)
        assert torch.allclose(eng.kv.k[:, p, :, :rows], kv1[0][i][:, :, :rows], atol=1e-5)
        assert torch.allclose(eng.kv.v[:, p, :, :rows], kv1[1][i][:, :, :rows], atol=1e-5)
    for s in out:
        eng.free(s)


def test_a_failing_item_fails_alone(eng):
    items = [(dict(PLANS[0][0]), _toks(11, 11)), ({"cache_keys": ["nope"]}, [1, 2]),
             ({"cache_keys": ["b0"], "recompute_initial_tokens": -3}, [1]), (dict(PLANS[1][0]), _toks(5, 5))]
    free0 = eng.alloc.num_free
    out = eng.link_batch(items)
    assert isinstance(out[1], LinkSourceUnavailable) and isinstance(out[2], ValueError)
    assert not isinstance(out[0], Exception) and not isinstance(out[3], Exception)
    ref = eng.link(dict(PLANS[1][0]), _toks(5, 5))
    assert out[3].output_ids == ref.output_ids
    for s in (out[0], out[3], ref):
        eng.free(s)
    assert eng.alloc.num_free == free0


def test_compiles_and_links_share_one_forward(eng, monkeypatch):
    calls = []
    orig = eng.model.forward

    def spy(fb, kv, *a, **k):
        calls.append(int(fb.q_indptr.numel()) - 1)
        return orig(fb, kv, *a, **k)

    monkeypatch.setattr(eng.model, "forward", spy)
    c, l = eng.extend_step(compiles=[(_toks(40, 7), "new-a", None, None), (_toks(20, 8), "new-b", None, None)],
                           links=[(dict(p), _toks(m, m)) for p, m in PLANS[:2]])
    assert calls == [4]  # two Compiles + two Links: one forward with four requests
    assert [r["status"] for r in c] == ["registered", "registered"]
    monkeypatch.setattr(eng.model, "forward", orig)
    # the batched Compile registered the same block a lone Compile would
    alone = Engine(QwenModel.random_init(PRESETS["tiny-qwen2"], seed=0), num_pages=256, page_size=16)
    r = alone.compile(_toks(40, 7), "new-a")
    assert r["first_token"] == c[0]["first_token"]
    for s in l:
        eng.free(s)


def test_scheduler_admits_links_of_a_step_together(eng, monkeypatch):
    from sglang_legolink_b200.runtime.scheduler import Request, Scheduler

    serial = []
    for plan, n in PLANS:
        s = eng.link(dict(plan), _toks(n, n))
        eng.decode([s], 3)
        serial.append(list(s.output_ids))
        eng.free(s)
    steps = []
    orig = eng.extend_step

    def spy(compiles=(), links=(), timer=None):
        steps.append(len(links))
        return orig(compiles=compiles, links=links, timer=timer)

    monkeypatch.setattr(eng, "extend_step", spy)
    sch = Scheduler(eng, max_prefills_per_step=8)
    reqs = [Request("link", f"l{i}", _toks(n, n), 4, pic_link=dict(plan)) for i, (plan, n) in enumerate(PLANS)]
    for r in reqs:
        sch.submit(r)
    while sch.step():
        pass
    assert steps == [4]
    for r, ref in zip(reqs, serial):
        toks = []
        while not r.events.empty():
            kind, v = r.events.get_nowait()
            if kind == "token":
                toks.append(v)
            assert kind != "error", v
        assert toks == ref


def test_batched_links_reading_a_peer_pool():
    cfg = PRESETS["tiny-qwen2"]
    d = LocalDirectory()
    a = Engine(QwenModel.random_init(cfg, seed=0), num_pages=512, directory=d, replica_rank=0)
    b = Engine(QwenModel.random_init(cfg, seed=0), num_pages=512, directory=d, replica_rank=1)
    b.peer_pools[0] = (a.kv.k, a.kv.v)
    for i, n in enumerate((50, 70)):
        a.compile(_toks(n, i), f"p{i}")
        b.compile(_toks(n + 3, 9 + i), f"q{i}")
    plans = [{"cache_keys": ["p0", "q1"], "recompute_initial_tokens": 4},
             {"cache_keys": ["q0", "p1", "p0"], "recompute_initial_tokens": 2}]
    serial = []
    for p in plans:
        s = b.link(dict(p), [1, 2, 3])
        serial.append(s.output_ids)
        b.free(s)
    out = b.link_batch([(dict(p), [1, 2, 3]) for p in plans])
    assert [s.output_ids for s in out] == serial
    assert d.add("rcu/begun/1", 0) == d.add("rcu/ended/1", 0) == 4


@pytest.mark.gpu
def test_batched_links_on_gpu_match_serial_kv():
    """On the sm_100a kernels: four Links in one step write the same K/V
    (bf16 tolerance) as the same Links run one at a time."""
    cfg = PRESETS["small-qwen2"]
    e = Engine(QwenModel.random_init(cfg, seed=0, device="cuda", dtype=torch.bfloat16), num_pages=2048,
               page_size=16, max_context=4096)
    V = cfg.vocab_size
    for i, n in enumerate((300, 130, 512, 64, 257)):
        e.compile([t % V for t in _toks(n, 100 + i)], f"b{i}")
    plans = [(dict(p), [t % V for t in _toks(n, n)]) for p, n in PLANS]

    def kv_of(seq):
        idx = torch.tensor(seq.pages, device="cuda")
        return e.kv.k[:, idx].float(), e.kv.v[:, idx].float()

    serial = []
    for p, ids in plans:
        s = e.link(dict(p), ids)
        serial.append((kv_of(s), s.output_ids[0]))
        e.free(s)
    out = e.link_batch([(dict(p), ids) for p, ids in plans])
    torch.cuda.synchronize()
    agree = 0
    for s, ((k1, v1), first) in zip(out, serial):
        assert not isinstance(s, Exception), s
        k2, v2 = kv_of(s)
        L, ps = s.length, e.page_size
        for a, b in ((k1, k2), (v1, v2)):
            a = a.transpose(2, 3).reshape(a.shape[0], -1, a.shape[2], a.shape[4])[:, :L]
            b = b.transpose(2, 3).reshape(b.shape[0], -1, b.shape[2], b.shape[4])[:, :L]
            assert ((a - b).norm() / (a.norm() + 1e-6)).item() < 2e-2
        agree += int(s.output_ids[0] == first)
        e.free(s)
    assert agree >= 3


def test_compile_states_refuse_conflicts_and_links_wait_for_compiles(eng):
    """absent -> compiling -> resident; a conflicting Compile of an in-flight
    key is refused at arrival, an agreeing one attaches; a Link queued behind
    the Compile of its key waits for it instead of failing."""
    import gc

    from sglang_legolink_b200.runtime.scheduler import (COMPILE_STATE_ABSENT, COMPILE_STATE_COMPILING,
                                                        COMPILE_STATE_RESIDENT, Request, Scheduler)

    sch = Scheduler(eng, max_prefills_per_step=1)
    toks = _toks(70, 501)
    c1 = Request("compile", "c1", toks, 1, sub_context={"cache_key": "state-k"})
    link = Request("link", "l1", [1, 2, 3], 2, pic_link={"cache_keys": ["state-k"], "recompute_initial_tokens": 4})
    assert sch.compile_states.state("state-k") == COMPILE_STATE_ABSENT
    sch.submit(c1)
    assert sch.compile_states.state("state-k") == COMPILE_STATE_COMPILING
    bad = sch.submit(Request("compile", "c2", _toks(70, 502), 1, sub_context={"cache_key": "state-k"}))
    assert bad.events.get_nowait()[0] == "error"
    same = sch.submit(Request("compile", "c3", list(toks), 1, sub_context={"cache_key": "state-k"}))
    assert sch.compile_states.inflight() == {"state-k": 2}
    sch.waiting.queue.appendleft(link)  # the Link arrives first, its Compile is still queued
    while sch.step():
        pass
    assert sch.compile_states.state("state-k") == COMPILE_STATE_RESIDENT
    kinds = []
    while not link.events.empty():
        kinds.append(link.events.get_nowait()[0])
    assert "error" not in kinds and kinds[-1] == "done"
    assert same.events.get_nowait()[0] == "token"  # the duplicate took the registry's duplicate path
    # a queued Compile whose request vanishes is dropped from the in-flight set
    sch2 = Scheduler(eng)
    r = Request("compile", "c4", _toks(70, 503), 1, sub_context={"cache_key": "ghost"})
    sch2.compile_states.admit(r, "ghost", r.input_ids, "reference")
    assert sch2.compile_states.state("ghost") == COMPILE_STATE_COMPILING
    del r
    gc.collect()
    assert sch2.compile_states.state("ghost") == COMPILE_STATE_ABSENT
