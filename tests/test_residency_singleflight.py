"""Single-flight residency recovery under concurrency: requests that find
the same key evicted compile it once (one owner, the rest wait), different
keys recover in parallel, an owner failure fails its waiters and is not
sticky, waits are bounded, an owner that raises still ends its flight, and
two requests that each own a key the other needs do not deadlock
(reference ``noc_context_manager/residency_recovery.py``,
``tests/test_residency_singleflight.py``)."""

import threading
import time

import pytest

from sglang_legolink_b200.host.adapter import (RequestPipeline, ResidencyRecoveryCoordinator, Role, RuntimeAdapter,
                                               TransportError)
from sglang_legolink_b200.host.fake_runtime import StrictFakeRuntime
from sglang_legolink_b200.host.framing import RepairWindowPlanner, UniformRepairWindow
from sglang_legolink_b200.host.manager import ContextManager
from sglang_legolink_b200.host.planner import CacheCatalog
from sglang_legolink_b200.host.tokenizer import HashTokenizer

TOK = HashTokenizer(vocab_size=4096)
SYS = "You maintain the billing service; every change needs a passing test run. " * 20
TOOL = "pytest output: 4 failed, 31 passed in 12.3s; failures in refunds and invoices " * 25


class SlowCompiles(StrictFakeRuntime):
    """Compiles take a while, so concurrent recoveries overlap."""

    def __init__(self, delay=0.05, fail_keys=()):
        super().__init__()
        self.delay, self.fail_keys = delay, set(fail_keys)

    def __call__(self, payload):
        sc = payload.get("sub_context")
        if sc is not None:
            time.sleep(self.delay)
            if sc.get("cache_key") in self.fail_keys:
                raise TransportError("compile failed (injected)", 500)
        return super().__call__(payload)

    def compiles(self):
        return [r["sub_context"]["cache_key"] for r in self.requests if r.get("sub_context")]


def _adapter(rt, coordinator):
    return RuntimeAdapter(rt, model="m", tokenizer=TOK, catalog=CacheCatalog(), coordinator=coordinator,
                          repair_planner=RepairWindowPlanner(UniformRepairWindow(8)),
                          generation={"max_tokens": 2, "temperature": 0.0})


def _pipelines(rt, n, coordinator=None):
    co = coordinator or ResidencyRecoveryCoordinator(wait_timeout_s=10)
    ad = _adapter(rt, co)
    return [RequestPipeline(ContextManager(f"task-{i}", tokenizer=TOK), ad) for i in range(n)], ad, co


EVENTS = [("task_instruction", "sys", SYS, {}), ("tool_output", "t1", TOOL, {}),
          ("user_request", "q", "which failure comes first?", {})]


def _run_all(pipes, events):
    out, errs = [None] * len(pipes), []
    gate = threading.Barrier(len(pipes))

    def go(i):
        try:
            gate.wait()
            out[i] = pipes[i].execute(events)
        except Exception as e:  # noqa: BLE001
            errs.append(e)

    ths = [threading.Thread(target=go, args=(i,)) for i in range(len(pipes))]
    [t.start() for t in ths]
    [t.join(60) for t in ths]
    return out, errs


@pytest.mark.parametrize("n", [2, 6])
def test_requests_missing_the_same_keys_recompile_each_once(n):
    rt = SlowCompiles()
    pipes, ad, co = _pipelines(rt, n)
    first = pipes[0].execute(EVENTS)  # compiles the blocks once
    for p in pipes[1:]:  # the other sessions hold the same context and link it
        p.execute(EVENTS)
    linked = list(first.layout.link_segments)
    before = len(rt.compiles())
    assert before == len(linked)
    rt.evict_everything()
    out, errs = _run_all(pipes, [("user_request", "q2", "and the next one?", {})])
    assert not errs, errs
    recompiled = rt.compiles()[before:]
    assert sorted(recompiled) == sorted(s.cache_key for s in linked)  # one Compile per key, not per request
    outcomes = [o.result.recovery["outcome"] for o in out]
    assert outcomes.count("recovered_after_source_missing") >= 1
    assert co.counters["owners"] == len(linked) and co.counters["failures"] == 0


def test_different_keys_recover_concurrently_with_their_own_owners():
    co = ResidencyRecoveryCoordinator(wait_timeout_s=5)
    owners, lock = [], threading.Lock()

    def worker(key):
        t = co.claim("rt", key, observed=0)
        with lock:
            owners.append((key, t.role))
        time.sleep(0.05)
        co.complete(t, ok=True)

    ths = [threading.Thread(target=worker, args=(k,)) for k in ("a", "b", "c")]
    t0 = time.perf_counter()
    [t.start() for t in ths]
    [t.join() for t in ths]
    assert all(role == Role.OWNER for _, role in owners) and time.perf_counter() - t0 < 0.14


def test_owner_failure_fails_every_waiter_and_is_not_sticky():
    co = ResidencyRecoveryCoordinator(wait_timeout_s=5)
    owner = co.claim("rt", "k", observed=0)
    waiters = [co.claim("rt", "k", observed=0) for _ in range(3)]
    assert owner.role == Role.OWNER and all(w.role == Role.WAITER for w in waiters)
    res = []
    ths = [threading.Thread(target=lambda w=w: res.append(co.wait(w))) for w in waiters]
    [t.start() for t in ths]
    co.complete(owner, ok=False, error="compile failed")
    [t.join() for t in ths]
    assert res == [False, False, False]
    again = co.claim("rt", "k", observed=co.completions)  # a new request starts a new flight
    assert again.role == Role.OWNER
    co.complete(again, ok=True)
    assert co.claim("rt", "k", observed=0).role == Role.SETTLED


def test_waits_are_bounded():
    co = ResidencyRecoveryCoordinator(wait_timeout_s=0.1)
    co.claim("rt", "k", observed=0)  # an owner that never finishes
    w = co.claim("rt", "k", observed=0)
    with pytest.raises(TimeoutError):
        co.wait(w)


def test_an_owner_whose_compile_raises_still_ends_its_flight():
    rt = SlowCompiles()
    pipes, ad, co = _pipelines(rt, 1)
    first = pipes[0].execute(EVENTS)
    rt.evict_everything()
    rt.fail_keys = {first.layout.link_segments[0].cache_key}
    with pytest.raises(TransportError):
        pipes[0].execute([("user_request", "q2", "again?", {})])
    assert not co._flights  # no flight is left open
    assert co.counters["failures"] == 1
    rt.fail_keys = set()
    ok = pipes[0].execute([("user_request", "q3", "and now?", {})])  # the failure is not remembered
    assert ok.result.text


def test_resident_keys_cost_no_recovery():
    rt = SlowCompiles(delay=0)
    pipes, ad, co = _pipelines(rt, 1)
    pipes[0].execute(EVENTS)
    r = pipes[0].execute([("user_request", "q2", "next?", {})])
    assert r.result.recovery["outcome"] == "not_needed" and co.counters["owners"] == 0


def test_crossing_recoveries_do_not_deadlock():
    """Request A recovers k1 then needs k2; request B recovers k2 then needs
    k1: each owner finishes its own Compile before claiming the next key."""
    co = ResidencyRecoveryCoordinator(wait_timeout_s=5)
    done = []

    def request(mine, theirs):
        t = co.claim("rt", mine, observed=0)
        if t.role == Role.OWNER:
            time.sleep(0.05)
            co.complete(t, ok=True)
        t2 = co.claim("rt", theirs, observed=0)
        if t2.role == Role.OWNER:
            time.sleep(0.05)
            co.complete(t2, ok=True)
        elif t2.role == Role.WAITER:
            assert co.wait(t2)
        done.append(mine)

    a = threading.Thread(target=request, args=("k1", "k2"))
    b = threading.Thread(target=request, args=("k2", "k1"))
    a.start(), b.start()
    a.join(3), b.join(3)
    assert sorted(done) == ["k1", "k2"]


def test_recovery_compiles_carry_no_physical_fields():
    rt = SlowCompiles(delay=0)
    pipes, ad, co = _pipelines(rt, 1)
    pipes[0].execute(EVENTS)
    rt.evict_everything()
    pipes[0].execute([("user_request", "q2", "next?", {})])
    from sglang_legolink_b200.contract import PIC_LINK_RUNTIME_OWNED_FIELDS

    for r in rt.requests:
        body = r.get("sub_context") or r.get("pic_link") or {}
        assert not set(body) & PIC_LINK_RUNTIME_OWNED_FIELDS
