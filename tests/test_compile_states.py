"""Per-key in-flight Compile states (absent -> compiling -> resident) and the
scheduler paths around them, on the CPU engine: agreeing Compiles attach and
finish on their own, a disagreeing one is refused at arrival without
poisoning the first, failures and vanished requests leave no record and no
phantom block, and a Link queued behind its key's Compile waits for it
within a bound (reference ``pic_runtime.py:2270-2361``,
``tests/test_security_l3_inflight_compile.py``)."""

import gc
import threading

import pytest
import torch

from sglang_legolink_b200.models.config import PRESETS
from sglang_legolink_b200.models.qwen import QwenModel
from sglang_legolink_b200.runtime.engine import Engine
from sglang_legolink_b200.runtime.scheduler import (COMPILE_STATE_ABSENT, COMPILE_STATE_COMPILING,
                                                    COMPILE_STATE_RESIDENT, CompileStates, Request, Scheduler)


def _toks(n, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.randint(0, 1024, (n,), generator=g).tolist()


@pytest.fixture(scope="module")
def eng():
    return Engine(QwenModel.random_init(PRESETS["tiny-qwen2"], seed=0), num_pages=512, page_size=16)


def _compile(rid, key, toks, **sc):
    return Request("compile", rid, list(toks), 1, sub_context={"cache_key": key, **sc})


def _drain(req):
    out = []
    while not req.events.empty():
        out.append(req.events.get_nowait())
    return out


def _run(sch):
    while sch.step():
        pass


class _Owner:
    pass


# ------------------------------------------------------- the state table alone
def test_one_compile_moves_absent_compiling_resident():
    resident = set()
    cs = CompileStates(lambda k: k in resident)
    o = _Owner()
    assert cs.state("k") == COMPILE_STATE_ABSENT
    cs.admit(o, "k", [1, 2, 3], "reference")
    assert cs.state("k") == COMPILE_STATE_COMPILING
    resident.add("k")
    assert cs.state("k") == COMPILE_STATE_COMPILING  # resident, but a Compile is still in flight
    cs.finish(o)
    assert cs.state("k") == COMPILE_STATE_RESIDENT and cs.inflight() == {}


def test_identical_in_flight_compiles_attach_and_each_finishes_on_its_own():
    cs = CompileStates(lambda k: False)
    a, b = _Owner(), _Owner()
    cs.admit(a, "k", [5, 6], "reference")
    cs.admit(b, "k", [5, 6], "reference")
    assert cs.inflight() == {"k": 2}
    cs.finish(a)
    assert cs.inflight() == {"k": 1} and cs.state("k") == COMPILE_STATE_COMPILING
    cs.finish(b)
    assert cs.state("k") == COMPILE_STATE_ABSENT


@pytest.mark.parametrize("tokens,mode", [([5, 7], "reference"), ([5, 6], "clone")])
def test_a_disagreeing_compile_is_refused_while_one_is_in_flight(tokens, mode):
    from sglang_legolink_b200.runtime.scheduler import RequestRejected

    cs = CompileStates(lambda k: False)
    first = _Owner()
    cs.admit(first, "k", [5, 6], "reference")
    with pytest.raises(RequestRejected):
        cs.admit(_Owner(), "k", tokens, mode)
    assert cs.inflight() == {"k": 1}  # the first is not poisoned


def test_finishing_an_owner_never_admitted_is_a_no_op_and_finish_is_idempotent():
    cs = CompileStates(lambda k: False)
    o = _Owner()
    cs.finish(o)
    cs.admit(o, "k", [1], "reference")
    cs.finish(o)
    cs.finish(o)
    assert cs.inflight() == {}


def test_readmitting_an_owner_moves_its_record():
    cs = CompileStates(lambda k: False)
    o = _Owner()
    cs.admit(o, "k1", [1], "reference")
    cs.admit(o, "k2", [2], "reference")
    assert cs.inflight() == {"k2": 1}


def test_a_vanished_request_does_not_wedge_its_key():
    cs = CompileStates(lambda k: False)
    o = _Owner()
    cs.admit(o, "k", [1], "reference")
    del o
    gc.collect()
    assert cs.state("k") == COMPILE_STATE_ABSENT


def test_concurrent_admits_and_finishes_keep_the_table_consistent():
    cs = CompileStates(lambda k: False)
    owners = [_Owner() for _ in range(64)]
    errs = []

    def work(i):
        try:
            o = owners[i]
            key = f"k{i % 4}"
            cs.admit(o, key, [i % 4], "reference")
            if i % 2:
                cs.finish(o)
        except Exception as e:  # noqa: BLE001
            errs.append(e)

    ths = [threading.Thread(target=work, args=(i,)) for i in range(64)]
    [t.start() for t in ths]
    [t.join() for t in ths]
    assert not errs
    assert cs.inflight() == {"k0": 16, "k2": 16}  # odd owners (keys k1, k3) finished
    for o in owners:
        cs.finish(o)
    assert cs.inflight() == {}


# ------------------------------------------------------ through the scheduler
def test_a_sequential_same_key_compile_is_a_normal_duplicate(eng):
    sch = Scheduler(eng)
    toks = _toks(40, 1)
    a = sch.submit(_compile("a", "seq-k", toks))
    _run(sch)
    b = sch.submit(_compile("b", "seq-k", toks))
    _run(sch)
    ea, eb = _drain(a), _drain(b)
    assert ea[-1][0] == "done" and ea[-1][1]["compile"]["status"] == "registered"
    assert eb[-1][0] == "done" and eb[-1][1]["compile"]["status"] == "duplicate"
    assert sch.compile_states.state("seq-k") == COMPILE_STATE_RESIDENT


def test_two_same_key_compiles_in_one_step_run_one_per_forward(eng):
    sch = Scheduler(eng, max_prefills_per_step=8)
    toks = _toks(33, 2)
    a = sch.submit(_compile("a", "batch-k", toks))
    b = sch.submit(_compile("b", "batch-k", toks))
    assert sch.compile_states.inflight() == {"batch-k": 2}
    _run(sch)
    sa = _drain(a)[-1][1]["compile"]["status"]
    sb = _drain(b)[-1][1]["compile"]["status"]
    assert sorted([sa, sb]) == ["duplicate", "registered"]
    assert sch.compile_states.inflight() == {}


def test_two_same_key_compiles_with_different_tokens_refuse_the_second_only(eng):
    sch = Scheduler(eng)
    toks = _toks(20, 3)
    a = sch.submit(_compile("a", "diff-k", toks))
    b = sch.submit(_compile("b", "diff-k", _toks(20, 4)))
    assert _drain(b)[0][0] == "error"
    _run(sch)
    assert _drain(a)[-1][0] == "done"
    assert eng.registry.tokens("diff-k") == toks  # the first Compile's tokens, not the refused one's


def test_a_different_content_compile_after_completion_keeps_the_existing_block(eng):
    sch = Scheduler(eng)
    toks = _toks(24, 5)
    sch.submit(_compile("a", "done-k", toks))
    _run(sch)
    free = eng.alloc.num_free
    b = sch.submit(_compile("b", "done-k", _toks(24, 6)))
    _run(sch)
    ev = _drain(b)
    assert ev[-1][0] == "error" and "different content" in ev[-1][1]
    assert eng.registry.tokens("done-k") == toks
    assert eng.alloc.num_free == free  # the refused Compile's pages went back
    assert sch.compile_states.state("done-k") == COMPILE_STATE_RESIDENT


def test_a_failed_compile_leaves_no_record_and_no_phantom_block(eng, monkeypatch):
    sch = Scheduler(eng)
    free = eng.alloc.num_free

    def boom(*a, **k):
        raise RuntimeError("injected forward failure")

    monkeypatch.setattr(eng, "extend_step", boom)
    r = sch.submit(_compile("a", "fail-k", _toks(30, 7)))
    _run(sch)
    monkeypatch.undo()
    assert _drain(r)[-1][0] == "error"
    assert sch.compile_states.state("fail-k") == COMPILE_STATE_ABSENT
    assert not eng.registry.contains("fail-k")
    assert eng.alloc.num_free == free
    ok = sch.submit(_compile("b", "fail-k", _toks(30, 7)))  # a valid Compile after the failure registers
    _run(sch)
    assert _drain(ok)[-1][1]["compile"]["status"] == "registered"


def test_a_failure_with_another_compile_still_in_flight_keeps_the_key_compiling():
    cs = CompileStates(lambda k: False)
    a, b = _Owner(), _Owner()
    cs.admit(a, "k", [9], "reference")
    cs.admit(b, "k", [9], "reference")
    cs.finish(a)  # a failed
    assert cs.state("k") == COMPILE_STATE_COMPILING


def test_a_refused_compile_leaves_no_record(eng):
    sch = Scheduler(eng)
    bad = sch.submit(Request("compile", "x", _toks(8, 8), 1,
                             sub_context={"cache_key": "mode-k", "pic_storage_mode": "mirror"}))
    assert _drain(bad)[0][0] == "error"
    assert sch.compile_states.inflight() == {}


def test_clone_mode_completion_closes_its_record(eng):
    sch = Scheduler(eng)
    r = sch.submit(_compile("a", "clone-k", _toks(40, 9), pic_storage_mode="clone"))
    _run(sch)
    assert _drain(r)[-1][1]["compile"]["status"] == "registered"
    assert sch.compile_states.inflight() == {} and sch.compile_states.state("clone-k") == COMPILE_STATE_RESIDENT


def test_a_link_queued_behind_its_compile_waits_for_it(eng):
    sch = Scheduler(eng, max_prefills_per_step=1)
    c = sch.submit(_compile("c", "wait-k", _toks(50, 10)))
    link = Request("link", "l", [3, 4], 2, pic_link={"cache_keys": ["wait-k"], "recompute_initial_tokens": 2})
    sch.waiting.queue.appendleft(link)
    _run(sch)
    assert _drain(c)[-1][0] == "done"
    ev = _drain(link)
    assert ev[-1][0] == "done" and not any(e[0] == "error" for e in ev)


def test_a_link_waits_for_a_stuck_compile_only_within_its_bound(eng):
    sch = Scheduler(eng, max_prefills_per_step=1)
    sch.max_link_waits = 3
    holder = _Owner()
    sch.compile_states.admit(holder, "stuck-k", [1, 2], "reference")  # a Compile that never finishes
    link = sch.submit(Request("link", "l", [5], 1, pic_link={"cache_keys": ["stuck-k"]}))
    for _ in range(20):
        sch.step()
        if not link.events.empty():
            break
    ev = _drain(link)
    assert ev and ev[-1][0] == "error"  # missing source after the bound, never plain generation
    assert getattr(link, "_compile_waits", 0) <= 3
    sch.compile_states.finish(holder)


def test_no_record_survives_any_completion_path(eng, monkeypatch):
    sch = Scheduler(eng)
    good = sch.submit(_compile("g", "path-ok", _toks(17, 11)))
    conflict = sch.submit(_compile("c", "path-ok", _toks(17, 12)))
    _run(sch)
    monkeypatch.setattr(eng, "extend_step", lambda *a, **k: (_ for _ in ()).throw(RuntimeError("x")))
    fail = sch.submit(_compile("f", "path-fail", _toks(17, 13)))
    _run(sch)
    monkeypatch.undo()
    assert [_drain(r)[-1][0] for r in (good, conflict, fail)] == ["done", "error", "error"]
    assert sch.compile_states.inflight() == {}
