"""Field classifiers, model-assisted segmentation guardrails, budgeted and
model-assisted selection, token accounting and the physical-token
equivalence audit (CPU)."""

import pytest

from sglang_legolink_b200.host.audits import (TokenAccountingError, TokenCount, TokenUnit, at_least, audit_layout,
                                              audit_sequences, count_tokens, require_authoritative)
from sglang_legolink_b200.host.classification import (DeterministicFieldClassifier, HybridFieldClassifier,
                                                      ModelFieldClassifier)
from sglang_legolink_b200.host.events import EventCollector, ExtractedSource, FieldClassificationError, FieldExtractor
from sglang_legolink_b200.host.framing import Stitcher, build_layout
from sglang_legolink_b200.host.manager import ContextManager, validate_segments
from sglang_legolink_b200.host.planner import Planner
from sglang_legolink_b200.host.segmentation import (AtomicUnitBuilder, AtomicUnitPolicy, ModelSegmenter,
                                                    UnitGroupingError, validate_split_points)
from sglang_legolink_b200.host.selection import BudgetedSelector, ModelSelector
from sglang_legolink_b200.host.tokenizer import HashTokenizer, RegexTokenizer


def _events(*items):
    c = EventCollector("t")
    return c.add_events(list(items))


def test_classifiers_table_model_and_fallback():
    typed, untyped = _events(("tool_output", "a", "out", {}), ("unclassified", "b", "??", {}))
    assert DeterministicFieldClassifier().classify(typed).field == "tool_history_output"
    assert DeterministicFieldClassifier().classify(untyped) is None
    good = ModelFieldClassifier(lambda req: {"field": "workspace_evidence", "confidence": 0.9})
    assert good.classify(untyped).field == "workspace_evidence"
    with pytest.raises(FieldClassificationError):
        ModelFieldClassifier(lambda req: {"field": "nonsense", "confidence": 0.9}).classify(untyped)
    with pytest.raises(FieldClassificationError):
        ModelFieldClassifier(lambda req: {"field": "workspace_evidence", "confidence": 2}).classify(untyped)
    hy = HybridFieldClassifier(ModelFieldClassifier(lambda req: {"field": "task_metadata", "confidence": 0.2}),
                               fallback_field="conversation_history")
    r = hy.classify(untyped)
    assert r.field == "conversation_history" and r.source == "explicit_fallback"
    assert hy.classify(untyped) is r and hy.model_invocations == 1  # memoised
    with pytest.raises(FieldClassificationError):
        HybridFieldClassifier(None).classify(untyped)
    # plugged into the extractor as a callable
    ext = FieldExtractor(HybridFieldClassifier(good)).extract([typed, untyped])
    assert ext.fields["workspace_evidence"][0].source_id == "b"


def _src(text):
    return ExtractedSource("tool_history_output", "e1", "s1", text, 1, "", {}, 1)


def test_atomic_units_and_split_point_validation():
    text = "\n\n".join(f"paragraph {i} " + "word " * 60 for i in range(6))
    units = AtomicUnitBuilder(RegexTokenizer(), AtomicUnitPolicy(target_max_tokens=150)).build(_src(text))
    assert len(units) == 6 and units[0].start == 0 and units[-1].end == len(text)
    groups = validate_split_points({"split_points": [{"after_unit_id": "u001", "reason": "a"},
                                                     {"after_unit_id": "u001", "reason": "again"},
                                                     {"after_unit_id": "u003", "reason": "b"}]}, units)
    assert [(g[0].unit_id, g[1].unit_id) for g in groups] == [("u000", "u001"), ("u002", "u003"), ("u004", "u005")]
    for bad, code in [({"split_points": [{"after_unit_id": "u005", "reason": ""}]}, "final_unit_split"),
                      ({"split_points": [{"after_unit_id": "u003", "reason": ""},
                                         {"after_unit_id": "u001", "reason": ""}]}, "unsorted_split_ids"),
                      ({"split_points": [{"after_unit_id": "zz", "reason": ""}]}, "unknown_split_id"),
                      ({"segments": []}, "unit_schema")]:
        with pytest.raises(UnitGroupingError) as e:
            validate_split_points(bad, units)
        assert e.value.code == code


def test_model_segmenter_validates_and_falls_back():
    text = "\n\n".join(f"section {i} " + "token " * 60 for i in range(4))
    pol = AtomicUnitPolicy(target_max_tokens=150)
    ok = ModelSegmenter(lambda req: {"split_points": [{"after_unit_id": req["units"][1]["unit_id"], "reason": "x"}]},
                        RegexTokenizer(), policy=pol)
    segs = ok.segment(_src(text))
    validate_segments(text, segs)
    assert len(segs) == 2 and not ok.fallbacks
    bad = ModelSegmenter(lambda req: {"split_points": "everything"}, RegexTokenizer(), policy=pol)
    segs = bad.segment(_src(text))
    validate_segments(text, segs)
    assert bad.fallbacks and bad.fallbacks[0]["code"] == "unit_schema"


def _manager(selector):
    cm = ContextManager("sel", tokenizer=RegexTokenizer(), selector=selector)
    cm.ingest([("task_instruction", "sys", "Fix the bug. " * 20, {}),
               ("tool_output", "t1", "old tool output " * 100, {}),
               ("tool_output", "t2", "newer tool output " * 100, {}),
               ("user_request", "u", "what next?", {})])
    return cm


def test_budgeted_selection_keeps_mandatory_and_newest_history():
    cm = _manager(BudgetedSelector(token_budget=1000))
    man = cm.select("q")
    by_src = {v.sub_context_id: v.source_id for v in cm.contexts()}
    kept = {by_src[i] for i in man.selected_sub_context_ids}
    assert {"sys", "u"} <= kept and "t2" in kept and "t1" not in kept
    assert man.excluded_sub_context_ids and man.token_budget == 1000
    full = _manager(None).select("q")
    assert len(full.selected_sub_context_ids) > len(man.selected_sub_context_ids)


def test_model_selection_subset_and_fallback():
    cm = _manager(None)
    opt = [v for v in cm.ordered_contexts() if v.source_id == "t1"]
    cm.selector = ModelSelector(lambda req: {"keep": [opt[0].sub_context_id]})
    man = cm.select("q")
    srcs = {v.sub_context_id: v.source_id for v in cm.contexts()}
    assert {srcs[i] for i in man.selected_sub_context_ids} == {"sys", "t1", "u"}
    cm.selector = ModelSelector(lambda req: {"keep": ["not-an-id"]}, token_budget=1000)
    man = cm.select("q")
    assert man.selector == "budgeted-rule-v1" and cm.selector.fallbacks


def test_token_accounting_units():
    est, model = RegexTokenizer(), HashTokenizer(vocab_size=512)
    assert count_tokens("a b c", est).unit == TokenUnit.ESTIMATED
    assert count_tokens("a b c", model).unit == TokenUnit.MODEL
    with pytest.raises(TokenAccountingError):
        require_authoritative(est, "compile floor")
    require_authoritative(model, "compile floor")
    with pytest.raises(TokenAccountingError):
        at_least(TokenCount(100, TokenUnit.ESTIMATED), 64, "compile floor")
    assert at_least(TokenCount(100, TokenUnit.MODEL, "h"), 64, "compile floor")


def test_equivalence_audit_on_a_real_layout():
    a = audit_sequences("r", "tok", [1, 2, 3, 4, 5], [1, 2, 9, 4, 5])
    assert not a.token_ids_match and a.first_mismatch_index == 2 and a.common_suffix_tokens == 2
    assert audit_sequences("r", "tok", [1, 2], [1, 2, 3]).first_mismatch_index == 2
    tok = HashTokenizer(vocab_size=4096)
    cm = ContextManager("aud", tokenizer=tok)
    cm.ingest([("task_instruction", "sys", "Instruction text. " * 50, {}),
               ("tool_output", "t1", "tool text " * 80, {}), ("user_request", "u", "go", {})])
    plan = Planner().plan(cm.select("go"), cm.contexts())
    layout = build_layout(Stitcher().stitch(plan), tok)
    aud = audit_layout(layout, "req-1")
    assert aud.status == "exact" and aud.token_delta == 0
    assert aud.baseline.sha256 == aud.assembled.sha256


def _profile(**over):
    from sglang_legolink_b200.host.group_profile import GroupRepairProfile, SCHEMA_VERSION, ShapeBands

    kw = dict(profile_id="p", profile_version="1", schema_version=SCHEMA_VERSION, method="prefix_absorb_refresh_1",
              supported_ordering="in_order_only", context_token_buckets=((100, 5000),), semantic_block_count_min=2,
              semantic_block_count_max=8, execution_group_member_min=2, execution_group_member_max=4,
              reconstruction_policy="prefix_absorb", member0_prefix_refresh_tokens=16, later_member_refresh="full",
              requires_all_members_resident=True, requires_group_absent_for_reconstruction=True,
              promotion="execution_group", fallback_policy="FULL_GROUP_RECOMPILE",
              supported_member_shapes=("balanced", "front_heavy"),
              member_shape_classifier=ShapeBands(1.5, 2.0, 6.0, 1.5),
              compatibility={"model_id": "m", "tokenizer_fingerprint": "t", "adapter_id": "base"})
    kw.update(over)
    return GroupRepairProfile(**kw)


def _greq(**over):
    from sglang_legolink_b200.host.group_profile import GroupRequest

    kw = dict(context_tokens=900, token_unit="model", semantic_block_count=3, request_member_ids=("a", "b"),
              group_member_ids=("a", "b"), member_token_counts=(200, 180), members_resident=(True, True),
              group_present=False, reconstruction_policy="prefix_absorb", member0_prefix_refresh_tokens=16,
              later_member_refresh="full", compatibility={"model_id": "m", "tokenizer_fingerprint": "t",
                                                          "adapter_id": "base"})
    kw.update(over)
    return GroupRequest(**kw)


def test_group_repair_profile_contract_checks_and_routes(tmp_path):
    from sglang_legolink_b200.host import group_profile as gp

    p = _profile()
    with pytest.raises(ValueError):
        _profile(compatibility={"model_id": "m", "logits": "x"})
    with pytest.raises(ValueError):
        _profile(later_member_refresh="partial")
    (tmp_path / "p.json").write_text(__import__("json").dumps(p.to_dict()))
    assert gp.load_profile(tmp_path / "p.json").digest == p.digest
    bad = dict(p.to_dict(), contract_digest="grqp-0")
    with pytest.raises(ValueError):
        gp.GroupRepairProfile.from_dict(bad)
    cases = [({}, "ELIGIBLE"), ({"group_present": True}, "GROUP_ALREADY_PRESENT"),
             ({"requested_profile_version": "2"}, "PROFILE_VERSION_MISMATCH"),
             ({"compatibility": {"model_id": "x", "tokenizer_fingerprint": "t"}}, "MODEL_MISMATCH"),
             ({"compatibility": {"model_id": "m", "tokenizer_fingerprint": "t", "adapter_id": "lora"}},
              "COMPATIBILITY_MISMATCH"),
             ({"token_unit": "estimated"}, "TOKEN_UNIT_NOT_MODEL"), ({"request_member_ids": ("b", "a")}, "REORDERED"),
             ({"semantic_block_count": 9}, "UNSUPPORTED_BLOCK_COUNT"), ({"context_tokens": 9000}, "OUT_OF_CONTEXT_RANGE"),
             ({"member_token_counts": (100, 400)}, "UNSUPPORTED_LAYOUT"),
             ({"member0_prefix_refresh_tokens": 32}, "WRONG_RECONSTRUCTION_POLICY"),
             ({"members_resident": (False, False)}, "MEMBERS_NOT_RESIDENT"),
             ({"members_resident": (True, False)}, "PARTIAL_MEMBER_RESIDENCY")]
    for over, code in cases:
        assert gp.evaluate(_greq(**over), p).reason_code == code, over
    assert gp.ShapeBands(1.5, 2.0, 6.0, 1.5).classify([600, 150, 160]) == "front_heavy"
    r = gp.route(_greq(), p, promotion_feature_enabled=False)
    assert r.route == "FULL_GROUP_RECOMPILE" and r.reason_code == "PROMOTION_FEATURE_DISABLED"
    r = gp.route(_greq(), p, promotion_feature_enabled=True)
    assert r.route == "PREFIX_ABSORB_RECONSTRUCT_AND_PROMOTE" and r.reconstruction_windows == (16, 180)
    assert gp.route(_greq(group_present=True), p, promotion_feature_enabled=True).route == "GROUP_CACHE_HIT"
    rows = gp.trace_rows(r, request_id="q1")
    assert [x["event"] for x in rows] == ["repair_profile_checked", "repair_profile_eligible"]
    with pytest.raises(ValueError):
        gp.trace_rows(r, logits=[1.0])
    gp.append_trace(tmp_path / "t.jsonl", rows)
    assert len((tmp_path / "t.jsonl").read_text().splitlines()) == 2
    assert gp.link_fields(r, "grp")["promote_reconstructed_group"] is True


def test_group_profile_route_drives_engine_promotion(monkeypatch):
    """An eligible route's Link fields make the runtime promote the group."""
    import torch

    from sglang_legolink_b200.host import group_profile as gp
    from sglang_legolink_b200.models.config import PRESETS
    from sglang_legolink_b200.models.qwen import QwenModel
    from sglang_legolink_b200.runtime.engine import Engine

    eng = Engine(QwenModel.random_init(PRESETS["tiny-qwen2"], seed=0), num_pages=256, page_size=16)
    g = torch.Generator().manual_seed(3)
    a, b = (torch.randint(0, 1024, (n,), generator=g).tolist() for n in (200, 180))
    eng.compile(a, "a")
    eng.compile(b, "b")
    r = gp.route(_greq(), _profile(), promotion_feature_enabled=True)
    monkeypatch.setenv("SGLANG_PIC_EXPERIMENTAL_GROUP_PROMOTION", "1")
    seq = eng.link({"cache_keys": ["a", "b"], **gp.link_fields(r, "grp-ab")}, [5, 6, 7])
    assert seq.promotion is not None and eng.registry.contains("grp-ab")


def test_legacy_plan_bridge_is_refused_then_replayed_with_runtime_layout(tmp_path, monkeypatch):
    """A pre-contract plan carries host-estimated layout: refused by default;
    replayed with the legacy flag, the runtime derives its own layout."""
    import torch

    from sglang_legolink_b200.contract import ContractError
    from sglang_legolink_b200.host.legacy_bridge import (LegacyBlock, build_legacy_link_plan, read_plan_file,
                                                         write_plan_file)
    from sglang_legolink_b200.models.config import PRESETS
    from sglang_legolink_b200.models.qwen import QwenModel
    from sglang_legolink_b200.runtime.engine import Engine

    eng = Engine(QwenModel.random_init(PRESETS["tiny-qwen2"], seed=0), num_pages=256, page_size=16)
    g = torch.Generator().manual_seed(5)
    a, b = (torch.randint(0, 1024, (n,), generator=g).tolist() for n in (100, 60))
    eng.compile(a, "la")
    eng.compile(b, "lb")
    query = [3, 4, 5, 6, 7]
    plan = build_legacy_link_plan([LegacyBlock("A", "la", 100), LegacyBlock("B", "lb", 60)], request_id="old",
                                  recompute_initial_tokens=8, mutable_token_estimate=3)  # estimate is off by 2
    plan = read_plan_file(write_plan_file(plan, tmp_path / "plan.json"))
    assert plan["imp_indices"] == list(range(100, 108)) + [160, 161, 162]
    monkeypatch.delenv("SGLANG_PIC_ALLOW_LEGACY_LINK_FIELDS", raising=False)
    with pytest.raises(ContractError):
        eng.link(dict(plan), query)
    monkeypatch.setenv("SGLANG_PIC_ALLOW_LEGACY_LINK_FIELDS", "1")
    seq = eng.link(dict(plan), query)
    assert list(seq.link_plan.recompute_positions) == list(range(100, 108)) + list(range(160, 165))


def _estimated_and_model_contexts():
    text = [("task_instruction", "sys", "Instruction text. " * 50, {}),
            ("tool_output", "t1", "tool text " * 80, {}), ("user_request", "u", "go", {})]
    est = ContextManager("est", tokenizer=RegexTokenizer())
    est.ingest(text)
    mod = ContextManager("mod", tokenizer=HashTokenizer(vocab_size=4096))
    mod.ingest(text)
    return est, mod


def test_compile_floor_refuses_estimated_counts_unless_asked():
    """The compile floor is in model tokens: a plan over blocks counted by the
    regex estimator fails closed, plans over model-token counts are
    unchanged, and estimate-only planning works when the caller asks."""
    from sglang_legolink_b200.host.planner import PolicyContext

    est, mod = _estimated_and_model_contexts()
    assert all(v.token_unit == "estimated" for v in est.contexts())
    with pytest.raises(TokenAccountingError, match="model tokens"):
        Planner().plan(est.select("go"), est.contexts())
    plan = Planner().plan(est.select("go"), est.contexts(), policy_context=PolicyContext(allow_estimated_tokens=True))
    assert plan is not None
    # model-token counts: the policy decides exactly as before (the floor
    # still keeps a short block mutable)
    plan = Planner().plan(mod.select("go"), mod.contexts())
    assert plan is not None


def test_cost_benefit_policy_refuses_estimated_counts():
    from sglang_legolink_b200.host import compile_cost as cc
    from sglang_legolink_b200.host.planner import CostBenefitCompilePolicy, PolicyContext

    est, _ = _estimated_and_model_contexts()
    pol = CostBenefitCompilePolicy(reuse_expectation=cc.FixedReuseExpectation(2.0), fallback="legacy_fixed_64")
    v = next(v for v in est.contexts() if v.reuse_candidate and not v.is_mutable)
    with pytest.raises(TokenAccountingError):
        pol.decide(v, PolicyContext())
    assert pol.decide(v, PolicyContext(allow_estimated_tokens=True)).policy == "cost_benefit"


def test_stored_rows_keep_a_model_unit_only_with_its_provenance():
    """A stored sub-context serializes its unit; on read a model-token claim
    stands only with the fingerprint of a model tokenizer, and a row with no
    unit (an older row) reads as an estimate."""
    from sglang_legolink_b200.host.store import SubContext

    est, mod = _estimated_and_model_contexts()
    v = next(iter(mod.contexts()))
    d = v.to_dict()
    assert d["token_unit"] == "model" and SubContext.from_dict(d).token_unit == "model"
    assert SubContext.from_dict(next(iter(est.contexts())).to_dict()).token_unit == "estimated"
    legacy = dict(d)
    legacy.pop("token_unit")
    assert SubContext.from_dict(legacy).token_unit == "estimated"
    forged = dict(d, metadata={**d["metadata"], "tokenizer_fingerprint": RegexTokenizer.fingerprint})
    assert SubContext.from_dict(forged).token_unit == "estimated"
    bare = dict(d, metadata={k: x for k, x in d["metadata"].items() if k != "tokenizer_fingerprint"})
    assert SubContext.from_dict(bare).token_unit == "estimated"
