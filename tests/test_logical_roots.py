"""Logical roots end to end: two agent tasks hold the same file, one as
workspace evidence and one as a tool output, and run through the host
pipeline against one runtime per namespace mode.  Checks what each mode
compiles, what the Link requests name, alias invalidation after eviction,
the request summaries, and that nothing namespace-related or runtime-owned
reaches the wire (reference ``tests/test_logical_radix_roots.py``,
``noc_context_manager/cache_namespace.py:502-730``)."""

import pytest

from sglang_legolink_b200.contract import PIC_LINK_RUNTIME_OWNED_FIELDS
from sglang_legolink_b200.host.adapter import RequestPipeline, RuntimeAdapter
from sglang_legolink_b200.host.fake_runtime import StrictFakeRuntime
from sglang_legolink_b200.host.framing import RepairWindowPlanner, UniformRepairWindow
from sglang_legolink_b200.host.manager import ContextManager
from sglang_legolink_b200.host.namespaces import (LOGICAL_ROOTS, PERSISTENT_NAMESPACES, NamespaceMode,
                                                  NamespacePolicy, NamespaceResolver)
from sglang_legolink_b200.host.planner import CacheCatalog, Planner
from sglang_legolink_b200.host.tokenizer import HashTokenizer

TOK = HashTokenizer(vocab_size=4096)
SYS = "You maintain the payments service and answer with a patch. " * 12
FILE = "def charge(order):\n    total = sum(i.price for i in order.items)\n    return gateway.post(total)\n" * 14


def _events(file_kind):
    return [("task_instruction", "sys", SYS, {}), (file_kind, "payments.py", FILE, {}),
            ("user_request", "q", "why does charge double-bill?", {})]


def _turns(pipe, file_kind):
    """Two turns: in the first the newest history (a tool output) is the open
    turn and is recomputed; the second adds the assistant's reply, after
    which the tool output is final and can be linked."""
    pipe.execute(_events(file_kind))
    return pipe.execute([("conversation_message", "a1", "Reading the charge path first.", {}),
                         ("user_request", "q2", "and where is the retry?", {})])


class Rig:
    def __init__(self, mode, pairs=()):
        self.rt = StrictFakeRuntime()
        self.catalog = CacheCatalog()
        self.resolver = NamespaceResolver(mode, NamespacePolicy(cross_namespace_pairs=list(pairs)))
        self.ad = RuntimeAdapter(self.rt, model="m", tokenizer=TOK, catalog=self.catalog,
                                 repair_planner=RepairWindowPlanner(UniformRepairWindow(8)),
                                 generation={"max_tokens": 2, "temperature": 0.0})

    def pipeline(self, task):
        return RequestPipeline(ContextManager(task, tokenizer=TOK, capture_token_ids=True), self.ad,
                               planner=Planner(catalog=self.catalog, resolver=self.resolver))

    def compiles(self):
        return [r["sub_context"]["cache_key"] for r in self.rt.requests if r.get("sub_context")]

    def links(self):
        return [r["pic_link"] for r in self.rt.requests if r.get("pic_link")]


def _file_block(execution, field):
    return [v for v in execution.plan.linked_contexts if v.context_field == field]


def test_there_are_exactly_five_logical_roots_and_they_are_the_persistent_namespaces():
    assert len(LOGICAL_ROOTS) == 5
    assert set(LOGICAL_ROOTS) == {n.value for n in PERSISTENT_NAMESPACES}
    assert NamespaceResolver().describe()["logical_roots"] == list(LOGICAL_ROOTS)


def test_a_misspelled_mode_fails_at_construction():
    with pytest.raises(ValueError):
        NamespaceResolver("globl")
    assert NamespaceMode.parse("Hard_Namespace") is NamespaceMode.HARD


def test_global_mode_serves_the_second_task_from_the_first_tasks_block():
    rig = Rig("global")
    a = _turns(rig.pipeline("task-a"), "workspace_file")
    n_after_a = len(rig.compiles())
    b = _turns(rig.pipeline("task-b"), "tool_output")
    new = rig.compiles()[n_after_a:]
    served = {v.cache_key for v in _file_block(a, "workspace_evidence")}
    assert served and not (set(new) & served)
    b_file_keys = {v.cache_key for v in b.plan.linked_contexts if v.metadata.get("physical_entry")}
    assert b_file_keys and b_file_keys <= served  # the alias views carry the serving block's key
    assert set(rig.links()[-1]["cache_keys"]) >= served
    s = b.metrics_row()["namespace"]["totals"]
    assert s["reused_token_count"] > 0


def test_hard_namespace_mode_compiles_the_twin_and_reports_the_missed_reuse():
    rig = Rig("hard_namespace")
    _turns(rig.pipeline("task-a"), "workspace_file")
    n = len(rig.compiles())
    b = _turns(rig.pipeline("task-b"), "tool_output")
    assert len(rig.compiles()) > n  # the tool-output block is compiled in its own root
    row = b.metrics_row()
    lookups = [lk for lk in b.plan.namespace_lookups if lk.context_field == "tool_history_output"]
    assert lookups and all(not lk.resident and lk.cross_namespace_opportunity for lk in lookups)
    assert row["semantic_cache_namespace_mode"] == "hard_namespace"


def test_logical_mode_reuses_across_roots_only_for_a_named_pair():
    plain = Rig("logical_namespace")
    _turns(plain.pipeline("task-a"), "workspace_file")
    n = len(plain.compiles())
    _turns(plain.pipeline("task-b"), "tool_output")
    assert len(plain.compiles()) > n
    paired = Rig("logical_namespace", pairs=["tool_output->workspace"])
    _turns(paired.pipeline("task-a"), "workspace_file")
    n = len(paired.compiles())
    b = _turns(paired.pipeline("task-b"), "tool_output")
    file_compiles = [k for k in paired.compiles()[n:]]
    hits = [lk for lk in b.plan.namespace_lookups if lk.cross_namespace_hit]
    assert hits and hits[0].cross_namespace_pair == "tool_output->workspace"
    served = {lk.physical_cache_key for lk in hits}
    assert not (set(file_compiles) & served)


def test_evicting_the_physical_block_makes_every_name_miss_and_one_compile_heals_them():
    rig = Rig("global")
    a_pipe, b_pipe = rig.pipeline("task-a"), rig.pipeline("task-b")
    _turns(a_pipe, "workspace_file")
    _turns(b_pipe, "tool_output")
    rig.rt.evict_everything()
    n = len(rig.compiles())
    r = b_pipe.execute([("user_request", "q2", "and the refund path?", {})])
    assert r.result.recovery["outcome"] == "recovered_after_source_missing"
    again = rig.compiles()[n:]
    assert len(again) == len(set(again))  # each evicted key compiled once
    n2 = len(rig.compiles())
    a_pipe.execute([("user_request", "q3", "and the retry path?", {})])
    assert len(rig.compiles()) == n2  # the other task's names resolve to the healed blocks


@pytest.mark.parametrize("mode", list(NamespaceMode))
def test_the_wire_carries_no_runtime_owned_or_namespace_field_in_any_mode(mode):
    rig = Rig(mode, pairs=["tool_output<->workspace"] if mode is NamespaceMode.LOGICAL else ())
    _turns(rig.pipeline("task-a"), "workspace_file")
    _turns(rig.pipeline("task-b"), "tool_output")
    for req in rig.rt.requests:
        body = req.get("pic_link") or req.get("sub_context") or {}
        assert not set(body) & PIC_LINK_RUNTIME_OWNED_FIELDS
        assert not any("namespace" in k for k in body)


def test_a_block_linked_through_an_alias_sends_the_same_key_as_through_its_own_name():
    rig = Rig("global")
    a = _turns(rig.pipeline("task-a"), "workspace_file")
    b = _turns(rig.pipeline("task-b"), "tool_output")
    la, lb = rig.links()[1], rig.links()[3]
    own = [v.cache_key for v in a.plan.linked_contexts]
    via_alias = [v.cache_key for v in b.plan.linked_contexts]
    assert own == via_alias and la["cache_keys"] == lb["cache_keys"]


def test_the_host_keeps_one_physical_cache_and_the_index_is_a_view_over_it():
    rig = Rig("global")
    _turns(rig.pipeline("task-a"), "workspace_file")
    _turns(rig.pipeline("task-b"), "tool_output")
    assert rig.resolver.describe()["physical_cache_instances"] == 1
    snap = rig.catalog.logical_index.snapshot()
    names = [n for root in snap["roots"].values() for n in root]
    primaries = {e["runtime_key"] for root in snap["roots"].values() for e in root.values()
                 if e["alias_kind"] is None}
    assert primaries <= set(rig.compiles())  # every primary name is a compiled block, none is a copy
    assert len(names) >= len(primaries)
    assert snap["aliases_recorded"] >= 1


def test_the_proxy_forwards_the_namespace_mode_and_shares_one_catalog():
    from sglang_legolink_b200.server.proxy import LegoLinkProxy

    with pytest.raises(ValueError):
        LegoLinkProxy(StrictFakeRuntime(), tokenizer=TOK, namespace_mode="hard")
    rt = StrictFakeRuntime()
    proxy = LegoLinkProxy(rt, tokenizer=TOK, namespace_mode="hard_namespace")
    a, _ = proxy.sessions.get("s-a")
    b, _ = proxy.sessions.get("s-b")
    for agent in (a, b):
        planner = agent.pipeline.planner
        assert planner.resolver is proxy.resolver and planner.catalog is proxy.catalog
        assert agent.pipeline.adapter.catalog is proxy.catalog
    msgs = [{"role": "system", "content": SYS}, {"role": "user", "content": "why does charge double-bill?"}]
    r = proxy.chat_completion({"messages": msgs, "session_id": "s-a"})
    assert r["legolink"]["session"] == "s-a"
    row = a.pipeline.planner.resolver.describe()
    assert row["semantic_cache_namespace_mode"] == "hard_namespace"
    n = len([q for q in rt.requests if q.get("sub_context")])
    proxy.chat_completion({"messages": msgs, "session_id": "s-b"})  # the shared instruction is not compiled again
    assert len([q for q in rt.requests if q.get("sub_context")]) == n


def test_make_pipeline_validates_the_mode_and_pairs():
    from sglang_legolink_b200.host.adapter import make_pipeline

    with pytest.raises(ValueError):
        make_pipeline(StrictFakeRuntime(), task_id="t", tokenizer=TOK, namespace_mode="logical")
    with pytest.raises(ValueError):
        make_pipeline(StrictFakeRuntime(), task_id="t", tokenizer=TOK, namespace_mode="logical_namespace",
                      cross_namespace_pairs=["workspace->nowhere"])
    p = make_pipeline(StrictFakeRuntime(), task_id="t", tokenizer=TOK, namespace_mode="logical_namespace",
                      cross_namespace_pairs=["workspace<->tool_output"])
    assert p.planner.resolver.describe()["cross_namespace_pairs"] == ["tool_output->workspace",
                                                                      "workspace->tool_output"]
