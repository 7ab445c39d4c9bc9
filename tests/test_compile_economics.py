"""Compile economics from measured latency curves (reference
``noc_context_manager/compile_cost.py``, ``compile_policy.py:386-560``) and
the summarize-then-compile branch (``compile_policy.py:334-350``,
``pruning.py``)."""

import math

import pytest

from sglang_legolink_b200.host import compile_cost as cc
from sglang_legolink_b200.host.events import SourceSpan
from sglang_legolink_b200.host.manager import AgentContextManifest
from sglang_legolink_b200.host.planner import (CompileAction, CompilePolicy, ContextSummarizer,
                                               CostBenefitCompilePolicy, Planner, PolicyContext)
from sglang_legolink_b200.host.store import SubContext
from sglang_legolink_b200.host.tokenizer import HashTokenizer

TOK = HashTokenizer(1024)


def block(n_words, field="tool_history_output", text=None):
    text = text or " ".join("w" + chr(97 + i % 26) + chr(97 + i // 26 % 26) for i in range(n_words))
    return SubContext.create(task_id="t", context_field=field, source_id=f"s-{field}-{n_words}",
                             spans=[SourceSpan("s", 0, len(text))], raw_text=text, tokenizer=TOK, sequence_number=1,
                             source_revision=1, model_fingerprint="m", capture_token_ids=True)


def profile(prefill=((16, 4.0), (8192, 400.0)), compile_=((16, 5.0), (8192, 420.0)), link=((16, 2.0), (8192, 30.0)),
            repair=None, hw="B200", model="qwen2.5-7b"):
    prov = cc.ProfileProvenance("test-v1", hw, model, dtype="bfloat16", source_artifact="hand-built for a test")
    return cc.CompileCostProfile(prov, cc.build_curve(prefill, name="prefill_ms"),
                                 cc.build_curve(compile_, name="compile_ms"), cc.build_curve(link, name="link_ms"),
                                 cc.build_curve(repair, name="repair_ms") if repair else None)


# ------------------------------------------------------------------ curves
def test_curve_interpolates_inside_and_refuses_outside():
    c = cc.build_curve([(100, 10.0), (200, 30.0), (400, 50.0)], name="x")
    assert c.estimate_ms(100) == 10.0 and c.estimate_ms(150) == 20.0 and c.estimate_ms(300) == 40.0
    for n in (99, 401):
        with pytest.raises(cc.CompileCostUnavailable):
            c.estimate_ms(n)
    assert cc.build_curve([(64, 3.0)], name="one").estimate_ms(64) == 3.0


@pytest.mark.parametrize("pts", [[], [(5, 1.0), (5, 2.0)], [(9, 1.0), (4, 2.0)], [(-1, 1.0)], [(4, -1.0)]])
def test_malformed_curves(pts):
    with pytest.raises(cc.CompileCostProfileError):
        cc.build_curve(pts, name="bad")


def test_profile_provenance_compatibility_and_json(tmp_path):
    p = profile()
    assert p.check_compatibility(None) == cc.PROFILE_UNCHECKED
    assert p.check_compatibility(cc.DeploymentIdentity("B200", "qwen2.5-7b", "bfloat16", 1)) == cc.PROFILE_MATCHED
    with pytest.raises(cc.CompileCostUnavailable):
        p.check_compatibility(cc.DeploymentIdentity("H100", "qwen2.5-7b"))
    assert p.check_compatibility(cc.DeploymentIdentity("B200", "qwen2.5-7b", tensor_parallel_size=8),
                                 strict=False) == cc.PROFILE_MISMATCHED
    path = p.write_json(tmp_path / "p.json")
    q = cc.CompileCostProfile.from_json(path)
    assert q.profile_id == p.profile_id and q.to_dict() == p.to_dict()
    assert profile(link=((16, 2.0), (8192, 31.0))).profile_id != p.profile_id
    with pytest.raises(cc.CompileCostProfileError):
        cc.CompileCostProfile.from_payload({"prefill_ms": p.prefill_ms.to_dict()})
    with pytest.raises(cc.CompileCostProfileError):
        cc.ProfileProvenance("v", "", "m")


def test_reuse_expectations_and_residency():
    kw = dict(cache_key="k", context_field="f", planned_future_reuse=6)
    assert cc.FixedReuseExpectation(3).estimate(**kw).effective_reuses == 3
    assert cc.PlannedTurnsReuseExpectation().estimate(**kw).effective_reuses == 3.0
    obs = cc.ObservedReuseExpectation(default=0.5)
    assert obs.estimate(**kw).source == "observed:unseen" and obs.estimate(**kw).effective_reuses == 0.5
    obs.record_reuse("k", 4)
    assert obs.estimate(**kw).effective_reuses == 4
    assert cc.NoReuseExpectation().estimate(**kw).effective_reuses == 0
    with pytest.raises(cc.CompileCostError):
        cc.ReuseEstimate(1, 1.5, "x")
    with pytest.raises(cc.CompileCostError):
        cc.ReuseEstimate(1, 1.0, " ")
    assert cc.DisabledResidencyCost().estimate_ms(model_tokens=100, expected_hold_reuses=2, memory_pressure=1) == 0
    lin = cc.LinearPressureResidencyCost(ms_per_model_token_hold=0.01)
    assert math.isclose(lin.estimate_ms(model_tokens=100, expected_hold_reuses=2, memory_pressure=0.5), 1.0)


def test_the_arithmetic():
    p = profile(prefill=((100, 100.0),), compile_=((100, 50.0),), link=((100, 10.0),))
    cand = cc.CompileCandidate("s", "k", "f", 100)
    b = cc.evaluate_compile_economics(cand, profile=p, reuse=cc.FixedReuseExpectation(2, probability=0.5),
                                      residency=cc.DisabledResidencyCost(), planned_future_reuse=0)
    assert (b.per_reuse_saved_ms, b.expected_saved_ms, b.total_cost_ms, b.net_benefit_ms) == (90.0, 90.0, 50.0, 40.0)
    assert b.is_profitable and b.repair_source == cc.REPAIR_FOLDED_INTO_LINK
    sunk = cc.evaluate_compile_economics(cc.CompileCandidate("s", "k", "f", 100, cache_present=True), profile=p,
                                         reuse=cc.FixedReuseExpectation(0.1), residency=cc.DisabledResidencyCost(),
                                         planned_future_reuse=0)
    assert sunk.estimated_compile_ms == 0.0 and sunk.compile_cost_sunk and sunk.is_profitable
    even = cc.evaluate_compile_economics(cand, profile=p, reuse=cc.FixedReuseExpectation(50 / 90),
                                         residency=cc.DisabledResidencyCost(), planned_future_reuse=0)
    assert abs(even.net_benefit_ms) < 1e-9 and not even.is_profitable  # break-even does not change the plan
    pr = profile(prefill=((100, 100.0),), compile_=((100, 50.0),), link=((100, 10.0),), repair=((0, 0.0), (64, 32.0)))
    with pytest.raises(cc.CompileCostUnavailable):
        cc.evaluate_compile_economics(cand, profile=pr, reuse=cc.FixedReuseExpectation(2),
                                      residency=cc.DisabledResidencyCost(), planned_future_reuse=0)
    r = cc.evaluate_compile_economics(cc.CompileCandidate("s", "k", "f", 100, planned_repair_model_tokens=32,
                                                          repair_window_source=cc.REPAIR_WINDOW_CALLER_SUPPLIED),
                                      profile=pr, reuse=cc.FixedReuseExpectation(2),
                                      residency=cc.DisabledResidencyCost(), planned_future_reuse=0)
    assert r.estimated_repair_ms == 16.0 and r.per_reuse_saved_ms == 74.0
    assert r.repair_window_source == cc.REPAIR_WINDOW_CALLER_SUPPLIED


# ---------------------------------------------------------------- policies
def test_cost_benefit_policy_decides_on_economics_not_size():
    pol = CostBenefitCompilePolicy(reuse_expectation=cc.FixedReuseExpectation(12), profile=profile())
    small = block(20)  # below the legacy floor, but it comes back twelve times
    assert small.token_count < 64
    assert CompilePolicy().decide(small, PolicyContext()).action is CompileAction.KEEP_MUTABLE
    d = pol.decide(small, PolicyContext())
    assert d.action is CompileAction.COMPILE and d.cost["net_benefit_ms"] > 0
    assert d.provenance["profile_id"] == pol.profile.profile_id and d.provenance["profile_compatibility"] == "unchecked"
    never = CostBenefitCompilePolicy(reuse_expectation=cc.NoReuseExpectation(), profile=profile())
    d = never.decide(block(500), PolicyContext())
    assert d.action is CompileAction.KEEP_MUTABLE and d.cost["expected_saved_ms"] == 0.0


def test_cost_benefit_refuses_without_evidence_unless_fallback_is_named():
    with pytest.raises(cc.CompileCostError):
        CostBenefitCompilePolicy(profile=profile())
    with pytest.raises(cc.CompileCostUnavailable):
        CostBenefitCompilePolicy(reuse_expectation=cc.FixedReuseExpectation(2)).decide(block(100), PolicyContext())
    fb = CostBenefitCompilePolicy(reuse_expectation=cc.FixedReuseExpectation(2), fallback="legacy_fixed_64")
    d = fb.decide(block(100), PolicyContext())
    assert d.action is CompileAction.COMPILE and d.provenance["fallback_policy"] == "legacy_fixed_64"
    other_gpu = CostBenefitCompilePolicy(reuse_expectation=cc.FixedReuseExpectation(2), profile=profile(hw="H100"),
                                         deployment=cc.DeploymentIdentity("B200", "qwen2.5-7b"))
    with pytest.raises(cc.CompileCostUnavailable):
        other_gpu.decide(block(100), PolicyContext())
    big = block(20000)  # outside the measured range: no decision, no extrapolation
    with pytest.raises(cc.CompileCostUnavailable):
        CostBenefitCompilePolicy(reuse_expectation=cc.FixedReuseExpectation(2), profile=profile()).decide(
            big, PolicyContext())


def test_legacy_summarize_branch():
    pol = CompilePolicy()
    ctx = PolicyContext(summarize_threshold_tokens=300)
    assert pol.decide(block(400), ctx).action is CompileAction.SUMMARIZE_THEN_COMPILE
    assert pol.decide(block(400, "workspace_evidence"), ctx).action is CompileAction.COMPILE
    assert pol.decide(block(400, "tool_definitions"), ctx).action is CompileAction.COMPILE
    assert block(100).token_count < 300 and pol.decide(block(100), ctx).action is CompileAction.COMPILE


def test_summarizer_rules():
    big = block(400)
    keep, why = ContextSummarizer().apply(big)
    assert keep is big and why == "summarizer unavailable"
    s = ContextSummarizer(lambda text, n: " ".join(text.split()[:n]), tokenizer=TOK)
    out, why = s.apply(big)
    assert why == "summarized" and out.token_count < big.token_count and out.cache_key != big.cache_key
    assert out.token_count == TOK.count(out.raw_text)
    assert out.metadata["derived_from"] == [big.sub_context_id]
    code = block(0, text="run this:\n```\nmake -j\n```\n" + "x " * 300)
    assert s.apply(code) == (code, "verbatim content")
    assert ContextSummarizer(lambda t, n: t + " more", tokenizer=TOK).apply(big)[1] == "summary did not reduce the context"


def test_planner_links_the_summary_in_place_of_a_large_block():
    big, small = block(500), block(80, "task_instruction")
    man = AgentContextManifest("t", 1, (small.sub_context_id, big.sub_context_id), (), "next?")
    s = ContextSummarizer(lambda text, n: " ".join(text.split()[:n]), tokenizer=TOK, target_ratio=0.2)
    plan = Planner(summarizer=s).plan(man, [small, big], policy_context=PolicyContext(summarize_threshold_tokens=300))
    linked = {v.sub_context_id: v for v in plan.linked_contexts}
    assert linked[big.sub_context_id].token_count < big.token_count
    assert linked[big.sub_context_id].cache_key != big.cache_key
    rec = {r.sub_context_id: r for r in plan.records}
    assert rec[big.sub_context_id].policy_action == "summarize_then_compile"


def test_profile_measured_on_the_engine_drives_decisions():
    """A profile timed on this runtime's own engine (CPU here; the same call
    on a B200 gives that deployment's curves)."""
    from sglang_legolink_b200.models.config import PRESETS
    from sglang_legolink_b200.models.qwen import QwenModel
    from sglang_legolink_b200.runtime.engine import Engine

    eng = Engine(QwenModel.random_init(PRESETS["tiny-qwen2"], seed=0), num_pages=512, page_size=16)
    p = eng_profile = cc.measure_engine_profile(eng, [64, 256], hardware_id="cpu", model_id="tiny-qwen2", repeats=1,
                                                repair_window=8)
    assert eng_profile.prefill_ms.measured_range == (64, 256) and p.provenance.tensor_parallel_size == 1
    assert all(y > 0 for _, y in p.prefill_ms.points + p.compile_ms.points + p.link_ms.points)
    assert not eng.registry.keys() or all(not k.startswith("compile-cost-profile") for k in eng.registry.keys())
    pol = CostBenefitCompilePolicy(reuse_expectation=cc.FixedReuseExpectation(4), profile=p,
                                   deployment=cc.DeploymentIdentity("cpu", "tiny-qwen2"))
    d = pol.decide(block(60), PolicyContext())  # ~120 model tokens: inside the measured range
    assert d.cost is not None and d.provenance["profile_compatibility"] == "matched"
