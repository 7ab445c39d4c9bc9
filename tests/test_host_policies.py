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
