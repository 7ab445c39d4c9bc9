"""Host cache namespaces: field -> namespace policy, persistence, the
cross-namespace pair rules, physical KV identity, root-first lookup per mode
(global / hard_namespace / logical_namespace), alias recording and
invalidation, persistence enforcement on the planner's decisions and the
per-request summary (reference ``noc_context_manager/cache_namespace.py``,
``semantic_cache_index.py``)."""

from dataclasses import replace

import pytest

from sglang_legolink_b200.host.events import SourceSpan
from sglang_legolink_b200.host.manager import AgentContextManifest
from sglang_legolink_b200.host.namespaces import (
    ALIAS_CROSS_ROOT, ALIAS_SAME_ROOT, NAMESPACE_NOT_PERSISTENT, NAMESPACE_PROFILES, PERSISTENT_NAMESPACES,
    CacheNamespace, LogicalRootIndex, NamespaceMode, NamespacePolicy, NamespaceResolver, parse_cross_namespace_pairs,
    physical_kv_identity, summarize_namespace_request)
from sglang_legolink_b200.host.planner import CacheCatalog, CompileAction, Planner
from sglang_legolink_b200.host.store import SubContext
from sglang_legolink_b200.host.tokenizer import HashTokenizer

TOK = HashTokenizer(1024)


def sc(field, text, *, sid=None, mutable=False, metadata=None, model="m1", ids=True):
    return SubContext.create(task_id="t", context_field=field, source_id=sid or f"src-{field}-{text[:6]}",
                             spans=[SourceSpan("s", 0, len(text))], raw_text=text, tokenizer=TOK,
                             sequence_number=1, source_revision=1, model_fingerprint=model, is_mutable=mutable,
                             capture_token_ids=ids, metadata=metadata)


TEXT = "cat README.md -> the build uses cmake and ninja " * 8


# ----------------------------------------------------------------- policy
@pytest.mark.parametrize("field,kw,ns", [
    ("user_prompt", {}, CacheNamespace.MUTABLE_CURRENT_TURN),
    ("task_instruction", {}, CacheNamespace.INSTRUCTION),
    ("tool_definitions", {}, CacheNamespace.TOOL_SCHEMA),
    ("tool_history_output", {}, CacheNamespace.TOOL_OUTPUT),
    ("workspace_evidence", {}, CacheNamespace.WORKSPACE),
    ("conversation_history", {}, CacheNamespace.CONVERSATION),
    ("conversation_history", {"finalized": False}, CacheNamespace.MUTABLE_CURRENT_TURN),
    ("task_metadata", {}, CacheNamespace.NO_CACHE),
    ("task_metadata", {"explicitly_cacheable": True}, CacheNamespace.INSTRUCTION),
    ("task_metadata", {"explicitly_cacheable": True, "finalized": False}, CacheNamespace.NO_CACHE),
])
def test_field_to_namespace(field, kw, ns):
    assert NamespacePolicy().namespace_for(field, **kw) is ns


def test_unknown_field_is_refused():
    with pytest.raises(ValueError):
        NamespacePolicy().namespace_for("secret_oracle")


def test_task_metadata_opt_in_needs_all_three_flags():
    p = NamespacePolicy()
    both = {"model_visible": True, "stable": True, "reusable": True}
    assert p.namespace_of(sc("task_metadata", "x y", metadata=both)) is CacheNamespace.INSTRUCTION
    assert p.namespace_of(sc("task_metadata", "x y", metadata=dict(both, stable="yes"))) is CacheNamespace.NO_CACHE


def test_profiles_and_persistence():
    assert {n.value for n in PERSISTENT_NAMESPACES} == {"instruction", "tool_schema", "conversation", "tool_output",
                                                        "workspace"}
    for ns, prof in NAMESPACE_PROFILES.items():
        assert prof.persistent == (ns in PERSISTENT_NAMESPACES)
    assert NAMESPACE_PROFILES[CacheNamespace.TOOL_OUTPUT].expected_reuse == "to_be_measured"


# ------------------------------------------------------------------ pairs
def test_pair_parsing_forms():
    both = parse_cross_namespace_pairs(["workspace<->tool_output"])
    assert both == ((CacheNamespace.WORKSPACE, CacheNamespace.TOOL_OUTPUT),
                    (CacheNamespace.TOOL_OUTPUT, CacheNamespace.WORKSPACE))
    assert parse_cross_namespace_pairs(["instruction->tool_schema", ("conversation", "workspace")]) == (
        (CacheNamespace.INSTRUCTION, CacheNamespace.TOOL_SCHEMA), (CacheNamespace.CONVERSATION, CacheNamespace.WORKSPACE))
    assert len(parse_cross_namespace_pairs(["workspace->tool_output", "workspace<->tool_output"])) == 2


@pytest.mark.parametrize("bad", ["workspace", "workspace->workspace", "no_cache->workspace",
                                 "workspace<->mutable_current_turn", "nonsense->workspace"])
def test_pair_parsing_refusals(bad):
    with pytest.raises(ValueError):
        parse_cross_namespace_pairs([bad])


def test_only_vetted_pairs_when_required():
    parse_cross_namespace_pairs(["workspace<->tool_output"], require_vetted=True)
    with pytest.raises(ValueError):
        parse_cross_namespace_pairs(["instruction->workspace"], require_vetted=True)
    assert NamespaceMode.parse(None) is NamespaceMode.GLOBAL
    assert NamespaceMode.parse(" Logical_Namespace ") is NamespaceMode.LOGICAL
    with pytest.raises(ValueError):
        NamespaceMode.parse("strict")


# --------------------------------------------------------------- identity
def test_physical_identity_ignores_field_and_namespace():
    a, b = sc("tool_history_output", TEXT), sc("workspace_evidence", TEXT)
    assert a.cache_key != b.cache_key  # the field enters the cache key ...
    assert physical_kv_identity(a) == physical_kv_identity(b)  # ... but not the KV
    assert physical_kv_identity(sc("workspace_evidence", TEXT, model="m2")) != physical_kv_identity(a)
    assert physical_kv_identity(sc("workspace_evidence", TEXT, ids=False)) is None  # text alone proves nothing


# ----------------------------------------------------------------- lookup
def _compiled(index, v, root):
    index.register(root, v.cache_key, identity=physical_kv_identity(v), semantic_identity=v.semantic_identity,
                   context_field=v.context_field, token_count=v.token_count)


def test_own_root_hit_in_every_mode():
    v = sc("tool_history_output", TEXT)
    for mode in NamespaceMode:
        idx = LogicalRootIndex()
        _compiled(idx, v, "tool_output")
        r = NamespaceResolver(mode).resolve(v, idx)
        assert r.resident and r.same_namespace_hit and r.alias_kind is None and r.physical_cache_key == v.cache_key


def test_cross_root_twin_per_mode():
    out = sc("tool_history_output", TEXT)  # compiled as a tool output
    ws = sc("workspace_evidence", TEXT)    # the same file as workspace evidence
    idx = LogicalRootIndex()
    _compiled(idx, out, "tool_output")
    g = NamespaceResolver("global").resolve(ws, idx)
    assert g.resident and g.alias_kind == ALIAS_CROSS_ROOT and g.physical_cache_key == out.cache_key
    assert g.fallback_attempted and g.cross_namespace_opportunity
    off = NamespaceResolver("global", global_physical_dedup=False).resolve(ws, idx)
    assert not off.resident and off.missed_reuse_tokens == ws.token_count
    hard = NamespaceResolver("hard_namespace").resolve(ws, idx)
    assert not hard.resident and not hard.fallback_attempted and hard.cross_namespace_opportunity
    plain = NamespaceResolver("logical_namespace").resolve(ws, idx)
    assert not plain.resident and not plain.fallback_attempted
    pol = NamespacePolicy(cross_namespace_pairs=["workspace->tool_output"])
    lg = NamespaceResolver("logical_namespace", pol).resolve(ws, idx)
    assert lg.resident and lg.cross_namespace_pair == "workspace->tool_output" and lg.cross_namespace_hit
    # the pair is directional
    idx2 = LogicalRootIndex()
    _compiled(idx2, ws, "workspace")
    assert not NamespaceResolver("logical_namespace", pol).resolve(out, idx2).resident


def test_logical_mode_never_aliases_a_block_that_is_not_linked():
    out = sc("tool_history_output", TEXT)
    idx = LogicalRootIndex()
    _compiled(idx, out, "tool_output")
    pol = NamespacePolicy(cross_namespace_pairs=["workspace<->tool_output"])
    ws = replace(sc("workspace_evidence", TEXT), reuse_candidate=False)
    r = NamespaceResolver("logical_namespace", pol).resolve(ws, idx)
    assert not r.resident and not r.alias_eligible and not r.cross_namespace_opportunity


def test_same_root_alias_between_two_fields():
    meta = {"model_visible": True, "stable": True, "reusable": True}
    instr = sc("task_instruction", TEXT)
    md = sc("task_metadata", TEXT, metadata=meta)  # opt-in metadata also lands in the instruction root
    idx = LogicalRootIndex()
    _compiled(idx, instr, "instruction")
    r = NamespaceResolver("hard_namespace").resolve(md, idx)
    assert r.resident and r.alias_kind == ALIAS_SAME_ROOT and r.physical_cache_key == instr.cache_key


def test_non_persistent_blocks_outside_global_mode():
    cur = sc("user_prompt", TEXT, mutable=True)
    r = NamespaceResolver("hard_namespace").resolve(cur, LogicalRootIndex())
    assert r.not_persistent and not r.resident and r.logical_root is None
    g = NamespaceResolver("global").resolve(cur, LogicalRootIndex())
    assert not g.not_persistent


def test_alias_views_records_and_invalidation():
    out = sc("tool_history_output", TEXT)
    ws = sc("workspace_evidence", TEXT)
    cat = CacheCatalog()
    _compiled(cat.logical_index, out, "tool_output")
    res = NamespaceResolver("logical_namespace", NamespacePolicy(cross_namespace_pairs=["workspace<->tool_output"]))
    views, lookups = res.apply([ws], cat)
    assert views[0].cache_key == out.cache_key
    assert views[0].metadata["physical_entry"] == {"namespace": "tool_output", "context_field": "tool_history_output"}
    assert lookups[0].physical_alias_count == 2 and not lookups[0].alias_recorded
    assert res.record_aliases(lookups, cat) == 1
    assert res.record_aliases(lookups, cat) == 0  # already recorded
    again = res.resolve(ws, cat)
    assert again.alias_recorded and again.physical_alias_count == 2
    assert cat.logical_index.lookup_alias("workspace", ws.cache_key).runtime_key == out.cache_key
    cat.invalidate(out.cache_key)  # the block is gone: its primary name and the alias miss
    assert cat.logical_index.lookup_alias("workspace", ws.cache_key) is None
    assert not res.resolve(ws, cat).resident


def test_sweep_drops_dangling_aliases():
    idx = LogicalRootIndex()
    out = sc("tool_history_output", TEXT)
    target = idx.register("tool_output", out.cache_key, identity=physical_kv_identity(out))
    idx.record_alias(root="workspace", name="ws-key", target=target, context_field="workspace_evidence",
                     token_count=5)
    idx._entries.pop(("tool_output", out.cache_key))
    assert idx.sweep() == 1 and idx.lookup_alias("workspace", "ws-key") is None


# ------------------------------------------------------------- planner
def _manifest(blocks):
    return AgentContextManifest("t", 1, tuple(b.sub_context_id for b in blocks), (), "what next?")


def test_planner_keeps_non_persistent_blocks_out_of_the_cache():
    instr = sc("task_instruction", TEXT)
    cur = replace(sc("conversation_history", TEXT + " latest", mutable=True), is_mutable=True, reuse_candidate=True)
    tools = sc("tool_definitions", "def run(cmd): ... " * 30)
    hard = Planner(resolver=NamespaceResolver("hard_namespace"))
    plan = hard.plan(_manifest([instr, cur, tools]), [instr, cur, tools])
    by = {r.sub_context_id: r for r in plan.records}
    assert by[cur.sub_context_id].planner_category == "mutable"
    # the block after the non-persistent one is demoted, never the other way round
    assert by[tools.sub_context_id].planner_category == "mutable"
    assert by[instr.sub_context_id].planner_category in ("linked", "compile_on_miss")
    assert plan.namespace_config["semantic_cache_namespace_mode"] == "hard_namespace"
    lk = {r.sub_context_id: r for r in plan.namespace_lookups}
    assert lk[cur.sub_context_id].not_persistent


def test_enforce_persistence_rewrites_compile_decisions():
    from sglang_legolink_b200.host.planner import CompileDecision

    md = sc("task_metadata", TEXT)  # no opt-in: no_cache
    res = NamespaceResolver("logical_namespace")
    lookups = [res.resolve(md, LogicalRootIndex())]
    d = CompileDecision(md.sub_context_id, md.cache_key, CompileAction.COMPILE, "floor", md.token_count)
    (out,) = res.enforce_persistence(lookups, [d])
    assert out.action is CompileAction.KEEP_MUTABLE and out.reason == NAMESPACE_NOT_PERSISTENT
    (same,) = NamespaceResolver("global").enforce_persistence(lookups, [d])
    assert same is d
    assert res.layout_permissions(lookups) == (False,)
    assert NamespaceResolver("global").layout_permissions(lookups) is None


def test_summary_counts_reuse_compile_and_recovery():
    a, b, c = sc("task_instruction", TEXT), sc("tool_definitions", "x " * 80), sc("tool_history_output", "y " * 90)
    idx = LogicalRootIndex()
    _compiled(idx, a, "instruction")
    _compiled(idx, c, "tool_output")
    res = NamespaceResolver("global")
    lookups = [res.resolve(v, idx) for v in (a, b, c)]
    s = summarize_namespace_request(lookups, linked_block_ids=[a.sub_context_id, b.sub_context_id, c.sub_context_id],
                                    link_cache_key_by_block={v.sub_context_id: v.cache_key for v in (a, b, c)},
                                    repair_tokens_by_cache_key={a.cache_key: 16}, recovered_cache_keys=[c.cache_key])
    t = s["totals"]
    assert t["reused_token_count"] == a.token_count
    assert t["compiled_token_count"] == b.token_count + c.token_count
    assert t["residency_recovered_blocks"] == 1 and t["repair_token_count"] == 16
    assert s["by_namespace"]["tool_schema"]["namespace_lookup_miss"] == 1
