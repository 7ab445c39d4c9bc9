"""Execution governance: a formal request is accepted only when its
FramingSpec, RepairDecision and repair fields agree with each other and with
a passing repair-quality measurement in the deployment profile; each rule is
refused on its own (reference ``pic_runtime.py:1060-1148``,
``execution_governance.py:66``)."""

import copy

import pytest

from sglang_legolink_b200 import contract as C

HEX = "0123456789abcdef" * 4


def _good():
    framing = {"framing_layout_version": C.PHYSICAL_TOKEN_LAYOUT_VERSION, "model_id": "qwen", "tokenizer_fingerprint": "tok",
               "chat_template_sha256": HEX, "profile_id": "prof"}
    decision = {"selected_k": 8, "windows": [8, 4, 0], "policy": "quality_guarded",
                "policy_version": C.REPAIR_DECISION_POLICY_VERSION,
                "framing_layout_version": C.PHYSICAL_TOKEN_LAYOUT_VERSION, "quality_profile_id": "q1",
                "evidence_id": "run-7", "reason": "measured", "workload_class": "agent"}
    wire = {"cache_keys": ["a", "b", "c"], "execution_mode": "formal", "framing_spec": framing,
            "repair_decision": decision, "physical_token_layout_version": C.PHYSICAL_TOKEN_LAYOUT_VERSION,
            "recompute_initial_tokens": 8, "recompute_tokens_per_block": [8, 4, 0],
            "recompute_first_block_tokens": 8, "recompute_first_block": True,
            "expected_complete_token_ids_sha256": "input-hash"}
    quality = {"selected_k": 8, "windows": [8, 4, 0], "workload_class": "agent", "evidence_id": "run-7",
               "framing_spec": copy.deepcopy(framing), "status": "PASS", "profile_id": "q1", "metric": "exact_match",
               "measured_value": 0.99, "required_threshold": 0.95}
    profile = {"framing_spec": copy.deepcopy(framing), "canonical_input_hashes": ["input-hash"],
               "repair_quality_profiles": {"q1": quality}}
    return wire, profile


def _set(d, path, value):
    for k in path[:-1]:
        d = d[k]
    if value is _DEL:
        del d[path[-1]]
    else:
        d[path[-1]] = value


_DEL = object()

# (what is changed, where: "w" = request / "p" = profile, path, new value)
VIOLATIONS = [
    ("unknown mode", "w", ("execution_mode",), "strict"),
    ("framing absent", "w", ("framing_spec",), _DEL),
    ("framing extra field", "w", ("framing_spec", "extra"), "x"),
    ("framing blank identity", "w", ("framing_spec", "model_id"), "  "),
    ("framing non-string identity", "w", ("framing_spec", "profile_id"), 3),
    ("framing legacy layout", "w", ("framing_spec", "framing_layout_version"), "noc-legacy-v0"),
    ("template hash short", "w", ("framing_spec", "chat_template_sha256"), "abc"),
    ("template hash uppercase", "w", ("framing_spec", "chat_template_sha256"), HEX.upper()),
    ("layout version disagrees", "w", ("physical_token_layout_version",), "other"),
    ("decision absent", "w", ("repair_decision",), _DEL),
    ("decision missing field", "w", ("repair_decision", "reason"), _DEL),
    ("k negative", "w", ("repair_decision", "selected_k"), -1),
    ("k bool", "w", ("repair_decision", "selected_k"), True),
    ("window above k", "w", ("repair_decision", "windows"), [9, 4, 0]),
    ("window count", "w", ("repair_decision", "windows"), [8, 4]),
    ("window bool", "w", ("repair_decision", "windows"), [8, True, 0]),
    ("policy version", "w", ("repair_decision", "policy_version"), "repair-decision-v0"),
    ("decision layout", "w", ("repair_decision", "framing_layout_version"), "x"),
    ("unknown policy", "w", ("repair_decision", "policy"), "yolo"),
    ("profile id type", "w", ("repair_decision", "quality_profile_id"), 5),
    ("blank reason", "w", ("repair_decision", "reason"), ""),
    ("blank workload", "w", ("repair_decision", "workload_class"), " "),
    ("K replaced", "w", ("recompute_initial_tokens",), 16),
    ("K defaulted", "w", ("recompute_initial_tokens",), _DEL),
    ("windows replaced", "w", ("recompute_tokens_per_block",), [8, 8, 0]),
    ("first block tokens", "w", ("recompute_first_block_tokens",), 4),
    ("first block flag", "w", ("recompute_first_block",), False),
    ("legacy K alias", "w", ("legolink_k",), 4),
    ("formal needs guarded policy", "w", ("repair_decision", "policy"), "fixed_unvalidated_debug"),
    ("profile framing differs", "p", ("framing_spec", "model_id"), "other"),
    ("input not reviewed", "w", ("expected_complete_token_ids_sha256",), "unknown"),
    ("measurement absent", "p", ("repair_quality_profiles", "q1"), _DEL),
    ("measurement other k", "p", ("repair_quality_profiles", "q1", "selected_k"), 4),
    ("measurement other evidence", "p", ("repair_quality_profiles", "q1", "evidence_id"), "run-8"),
    ("measurement failed", "p", ("repair_quality_profiles", "q1", "status"), "FAIL"),
    ("measurement no metric", "p", ("repair_quality_profiles", "q1", "metric"), ""),
    ("measurement other profile", "p", ("repair_quality_profiles", "q1", "profile_id"), "q2"),
    ("below threshold", "p", ("repair_quality_profiles", "q1", "measured_value"), 0.5),
    ("threshold not finite", "p", ("repair_quality_profiles", "q1", "required_threshold"), float("nan")),
    ("measured is bool", "p", ("repair_quality_profiles", "q1", "measured_value"), True),
    ("hash list is a string", "p", ("canonical_input_hashes",), "input-hash"),
    ("quality table not a mapping", "p", ("repair_quality_profiles",), ["q1"]),
]


def test_the_good_formal_request_is_accepted():
    wire, profile = _good()
    C.validate_execution_intent(wire, profile)
    C.validate_pic_link_request(wire, profile=profile, require_formal=True)


@pytest.mark.parametrize("name,where,path,value", VIOLATIONS, ids=[v[0] for v in VIOLATIONS])
def test_each_governance_rule_refuses_alone(name, where, path, value):
    wire, profile = _good()
    _set(wire if where == "w" else profile, path, value)
    with pytest.raises(C.ContractError):
        C.validate_execution_intent(wire, profile)


def test_legacy_debug_without_governance_is_accepted():
    C.validate_execution_intent({"cache_keys": ["a"]}, None)
    C.validate_execution_intent({"cache_keys": ["a"], "execution_mode": "legacy_debug"}, None)


def test_formal_deployment_refuses_legacy_requests():
    with pytest.raises(C.ContractError):
        C.validate_execution_intent({"cache_keys": ["a"]}, None, require_formal=True)


def test_legacy_debug_with_unvalidated_decision_skips_evidence():
    wire, _ = _good()
    wire["execution_mode"] = "legacy_debug"
    wire["repair_decision"]["policy"] = "fixed_unvalidated_debug"
    C.validate_execution_intent(wire, None)  # no deployment profile needed
    wire["repair_decision"]["policy"] = "quality_guarded"  # a guarded decision always needs its evidence
    with pytest.raises(C.ContractError):
        C.validate_execution_intent(wire, None)


def test_legacy_debug_with_framing_only_still_needs_a_decision():
    wire, _ = _good()
    wire["execution_mode"] = "legacy_debug"
    del wire["repair_decision"]
    with pytest.raises(C.ContractError):
        C.validate_execution_intent(wire, None)


@pytest.mark.parametrize("field,value,ok", [
    ("request_id", 7, True), ("request_id", True, False), ("request_id", 1.5, False), ("task_id", None, True),
    ("variant", None, True), ("variant", 3, False), ("profiling_warmup", 1, False), ("concurrency", None, True),
    ("concurrency", 2 ** 31, False), ("block_ids", None, True), ("block_ids", ["x", 1], False),
    ("recompute_mode", "TOKENWISE", True), ("recompute_mode", None, False), ("recompute_initial_tokens", None, False),
    ("legolink_k", 3, True), ("recompute_first_block_tokens", None, True), ("recompute_first_block_tokens", -2, False),
    ("recompute_tokens_per_block", None, True), ("recompute_tokens_per_block", [1, 2], False),
    ("recompute_tokens_per_block", [2 ** 31], False), ("adapter_id", 1, False), ("promote_reconstructed_group", None, True),
])
def test_value_rules(field, value, ok):
    plan = {"cache_keys": ["a"], field: value}
    if ok:
        C.validate_pic_link_field_types(plan)
    else:
        with pytest.raises(C.ContractError):
            C.validate_pic_link_field_types(plan)


@pytest.mark.parametrize("keys", [None, "a", [], ["a", 2]])
def test_cache_keys_rule(keys):
    with pytest.raises(C.ContractError):
        C.validate_pic_link_field_types({"cache_keys": keys})
    with pytest.raises(C.ContractError):
        C.validate_pic_link_field_types({})
