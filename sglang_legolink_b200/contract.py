"""The Compile/Link wire contract, shared by the host pipeline and the runtime.

The reference keeps two copies of these lists (host
``noc_context_manager/pic_link_contract.py:49-153`` and runtime
``patched_sglang_files/python/sglang/srt/pic_runtime.py:632-764``) and pins
them equal with a test.  Here both sides import this one module.  Field names,
the runtime-owned refusal, strict type rules, the execution-governance rules
and the token hash are part of the wire format and are kept identical to the
reference so existing hosts interoperate.
"""

from __future__ import annotations

import hashlib
import json
import math
import os
from typing import Any, Mapping, Optional

PHYSICAL_TOKEN_LAYOUT_VERSION = "noc-single-chat-template-split-v1"
REPAIR_DECISION_POLICY_VERSION = "repair-decision-v1"
LEGOLINK_POLICY_VERSION = "legolink-radix-v1"

PIC_LINK_IDENTITY_FIELDS = frozenset({"request_id", "task_id", "variant", "profiling_warmup", "concurrency"})
PIC_LINK_SELECTION_FIELDS = frozenset({"cache_keys", "block_ids"})
PIC_LINK_COMPATIBILITY_FIELDS = frozenset({"adapter_id", "segmentation_policy_version", "legolink_policy_version"})
PIC_LINK_REPAIR_POLICY_FIELDS = frozenset(
    {
        "recompute_mode",
        "recompute_initial_tokens",
        "recompute_first_block",
        "recompute_first_block_tokens",
        "recompute_tokens_per_block",
    }
)
PIC_LINK_TOKEN_LAYOUT_FIELDS = frozenset(
    {
        "physical_token_layout_version",
        "physical_input_ids",
        "physical_token_count",
        "physical_token_ids_sha256",
        "physical_prefix_token_count",
        "physical_block_segments",
        "expected_complete_token_count",
        "expected_complete_token_ids_sha256",
        "physical_interblock_fresh_token_counts",
    }
)
PIC_LINK_DIAGNOSTIC_FIELDS = frozenset(
    {
        "diagnostic_flashinfer_reuse_paged_wrapper_across_plans",
        "diagnostic_flashinfer_skip_exact_paged_metadata_cache",
        "diagnostic_sparse_repair_record_function",
        "diagnostic_sparse_repair_row_batching",
        "diagnostic_sparse_repair_rowwise_ffn",
        "diagnostic_sparse_repair_rowwise_output_projection",
    }
)
PIC_LINK_EXPERIMENTAL_PROMOTION_FIELDS = frozenset({"promote_reconstructed_group", "execution_group_key"})
PIC_LINK_DEPRECATED_ALIASES = frozenset({"legolink_k"})
PIC_LINK_GOVERNANCE_FIELDS = frozenset({"execution_mode", "framing_spec", "repair_decision"})

PIC_LINK_REQUEST_FIELDS = (
    PIC_LINK_GOVERNANCE_FIELDS
    | PIC_LINK_IDENTITY_FIELDS
    | PIC_LINK_SELECTION_FIELDS
    | PIC_LINK_COMPATIBILITY_FIELDS
    | PIC_LINK_REPAIR_POLICY_FIELDS
    | PIC_LINK_TOKEN_LAYOUT_FIELDS
    | PIC_LINK_DIAGNOSTIC_FIELDS
    | PIC_LINK_EXPERIMENTAL_PROMOTION_FIELDS
    | PIC_LINK_DEPRECATED_ALIASES
)

PIC_LINK_RUNTIME_OWNED_FIELDS = frozenset(
    {
        "attention_ranges",
        "block_ranges",
        "imp_indices",
        "kvlink",
        "mutable_start_token",
        "mutable_token_count",
        "recompute_positions",
        "token_layout_source",
        "total_token_count",
    }
)
PIC_LINK_INTERNAL_FIELDS = frozenset({"_scheduler_reserved_cache_keys"})
PIC_LINK_MAX_INTEGER = 2**31 - 1
PIC_LINK_RECOMPUTE_MODES = frozenset({"batched", "tokenwise", "full_causal"})

FRAMING_SPEC_FIELDS = frozenset(
    {"framing_layout_version", "model_id", "tokenizer_fingerprint", "chat_template_sha256", "profile_id"}
)
REPAIR_DECISION_FIELDS = frozenset(
    {
        "selected_k",
        "windows",
        "policy",
        "policy_version",
        "framing_layout_version",
        "quality_profile_id",
        "evidence_id",
        "reason",
        "workload_class",
    }
)


class ContractError(ValueError):
    """A request the runtime refuses (request-scoped; never kills the server)."""


def env_flag(name: str, default: str = "0") -> bool:
    return os.getenv(name, default).lower() in ("1", "true", "yes", "on")


def physical_token_ids_sha256(token_ids) -> str:
    """sha256 of the compact JSON int list (``[1,2,3]``), the wire hash."""
    enc = json.dumps([int(t) for t in token_ids], separators=(",", ":")).encode("utf-8")
    return hashlib.sha256(enc).hexdigest()


# ---------------------------------------------------------------- type rules
# Every host-sendable value has one entry in ``_VALUE_RULES``: the field name,
# the shape it must have, and whether an explicit ``null`` is accepted.  The
# shapes are small predicate objects, so the accepted set of a field reads off
# the table (the refusal set is the reference's, ``pic_runtime.py:845-922``).


def _is_int(v) -> bool:
    return isinstance(v, int) and not isinstance(v, bool)


def _in_range(v) -> bool:
    return _is_int(v) and 0 <= v <= PIC_LINK_MAX_INTEGER


class _Shape:
    """A value shape: ``check(value, keys)`` returns None or a refusal."""

    def check(self, value, keys: list) -> Optional[str]:
        raise NotImplementedError


class _OfType(_Shape):
    def __init__(self, what: str, test):
        self.what, self.test = what, test

    def check(self, value, keys):
        return None if self.test(value) else f"is not {self.what}"


class _Count(_Shape):
    def check(self, value, keys):
        if not _is_int(value):
            return "is not an integer"
        return None if _in_range(value) else f"is outside [0, {PIC_LINK_MAX_INTEGER}]"


class _Names(_Shape):
    """A list of strings, optionally non-empty and bounded by the key count."""

    def __init__(self, nonempty: bool = False, per_key_bound: bool = False):
        self.nonempty, self.per_key_bound = nonempty, per_key_bound

    def check(self, value, keys):
        if not isinstance(value, list):
            return "is not a list of strings"
        if self.nonempty and not value:
            return "is empty"
        if not all(isinstance(x, str) for x in value):
            return "holds a non-string entry"
        if self.per_key_bound and len(value) > len(keys):
            return f"names more entries than the {len(keys)} cache keys"
        return None


class _PerKeyCounts(_Shape):
    def check(self, value, keys):
        if not isinstance(value, list):
            return "is not a list of integers"
        if len(value) != len(keys):
            return f"has {len(value)} entries for {len(keys)} cache keys"
        return None if all(_in_range(x) for x in value) else "holds a value that is not a count"


class _Mode(_Shape):
    def check(self, value, keys):
        if not isinstance(value, str):
            return "is not a string"
        return None if value.lower() in PIC_LINK_RECOMPUTE_MODES else \
            "is not one of " + "/".join(sorted(PIC_LINK_RECOMPUTE_MODES))


_TEXT = _OfType("a string", lambda v: isinstance(v, str))
_FLAG = _OfType("a boolean", lambda v: isinstance(v, bool))
_LABEL = _OfType("a string or an integer", lambda v: isinstance(v, str) or _is_int(v))

# (field, shape, null accepted).  ``cache_keys`` is handled first: it is
# required, and other shapes are judged against its length.
_VALUE_RULES: tuple = (
    ("request_id", _LABEL, True),
    ("task_id", _LABEL, True),
    ("variant", _TEXT, True),
    ("profiling_warmup", _FLAG, True),
    ("concurrency", _Count(), True),
    ("block_ids", _Names(per_key_bound=True), True),
    ("adapter_id", _TEXT, True),
    ("segmentation_policy_version", _TEXT, True),
    ("legolink_policy_version", _TEXT, True),
    ("execution_group_key", _TEXT, True),
    ("promote_reconstructed_group", _FLAG, True),
    ("recompute_mode", _Mode(), False),
    ("recompute_initial_tokens", _Count(), False),
    ("legolink_k", _Count(), False),
    ("recompute_first_block", _FLAG, True),
    ("recompute_first_block_tokens", _Count(), True),
    ("recompute_tokens_per_block", _PerKeyCounts(), True),
)


def validate_pic_link_field_types(plan: Mapping) -> None:
    """Checks the type and range of every host-sendable value in ``plan``
    against ``_VALUE_RULES`` (absent fields pass; ``cache_keys`` is required
    and must be a non-empty list of strings).  Reference refusal set:
    ``pic_runtime.py:845-922``."""
    keys = plan.get("cache_keys")
    problem = "is missing" if "cache_keys" not in plan else \
        ("is null" if keys is None else _Names(nonempty=True).check(keys, []))
    if problem:
        raise ContractError(f"pic_link.cache_keys {problem}.")
    for name, shape, nullable in _VALUE_RULES:
        if name not in plan:
            continue
        value = plan[name]
        if value is None:
            if nullable:
                continue
            problem = "is null"
        else:
            problem = shape.check(value, keys)
        if problem:
            raise ContractError(f"pic_link.{name} {problem}.")


# ---------------------------------------------------------- governance rules
# Execution governance (reference ``pic_runtime.py:1060-1148``, host twin
# ``execution_governance.py:66``) as four ordered tables of named checks over
# one view of the request.  Each table may assume the ones before it passed;
# the request is refused with the first failing check's text.
#
#   framing   -- the FramingSpec is complete and names the supported layout;
#   decision  -- the RepairDecision is complete and well formed;
#   binding   -- the request's repair fields are exactly the decision's;
#   evidence  -- (formal, or a quality-guarded decision) the deployment
#                profile holds a passing, matching quality measurement.

_HEX = frozenset("0123456789abcdef")
_REPAIR_POLICIES = ("quality_guarded", "fixed_unvalidated_debug")


def _nonblank(v) -> bool:
    return isinstance(v, str) and bool(v.strip())


def _exact_int(v) -> bool:
    return type(v) is int


def _finite_number(v) -> bool:
    return type(v) in (int, float) and math.isfinite(v)


class _Intent:
    """Read-only view of one request's governance inputs."""

    def __init__(self, wire: Mapping, profile):
        self.wire = wire
        self.profile = profile
        self.spec = wire.get("framing_spec")
        self.decision = wire.get("repair_decision")

    # framing
    @property
    def layout(self):
        return self.spec["framing_layout_version"]

    # decision
    @property
    def k(self):
        return self.decision["selected_k"]

    @property
    def windows(self):
        return self.decision["windows"]

    # evidence
    def measurement(self):
        table = self.profile.get("repair_quality_profiles", {})
        return table.get(self.decision["quality_profile_id"]) if isinstance(table, Mapping) else None

    def reviewed_inputs(self):
        hashes = self.profile.get("canonical_input_hashes", [])
        return hashes if isinstance(hashes, (list, tuple, set, frozenset)) else ()


def _windows_ok(x: _Intent) -> bool:
    w, k = x.windows, x.k
    return (isinstance(w, list) and bool(w) and len(w) == len(x.wire.get("cache_keys", []))
            and all(_exact_int(v) and 0 <= v <= k for v in w))


def _measurement_matches(x: _Intent) -> bool:
    m = x.measurement()
    return all(m.get(f) == x.decision[f] for f in ("selected_k", "windows", "workload_class", "evidence_id"))


def _measurement_passed(x: _Intent) -> bool:
    m = x.measurement()
    return (m.get("framing_spec") == x.spec and m.get("status") == "PASS"
            and m.get("profile_id") == x.decision["quality_profile_id"]
            and bool(x.decision["evidence_id"]) and bool(m.get("metric")))


def _measurement_meets_threshold(x: _Intent) -> bool:
    m = x.measurement()
    got, need = m.get("measured_value"), m.get("required_threshold")
    return _finite_number(got) and _finite_number(need) and got >= need


_FRAMING_RULES = (
    ("FramingSpec is absent or does not carry exactly its five fields",
     lambda x: isinstance(x.spec, dict) and set(x.spec) == FRAMING_SPEC_FIELDS),
    ("FramingSpec has a blank or non-string identity field",
     lambda x: all(_nonblank(v) for v in x.spec.values())),
    ("FramingSpec names a framing layout this runtime does not implement",
     lambda x: x.layout == PHYSICAL_TOKEN_LAYOUT_VERSION),
    ("FramingSpec.chat_template_sha256 is not 64 lowercase hex digits",
     lambda x: len(x.spec["chat_template_sha256"]) == 64 and set(x.spec["chat_template_sha256"]) <= _HEX),
    ("physical_token_layout_version differs from the FramingSpec layout",
     lambda x: x.wire.get("physical_token_layout_version") == x.layout),
)

_DECISION_RULES = (
    ("RepairDecision is absent or does not carry exactly its nine fields",
     lambda x: isinstance(x.decision, dict) and set(x.decision) == REPAIR_DECISION_FIELDS),
    ("RepairDecision.selected_k is not a non-negative integer",
     lambda x: _exact_int(x.k) and x.k >= 0),
    ("RepairDecision.windows is not one window in [0, selected_k] per cache key", _windows_ok),
    ("RepairDecision.policy_version is not supported",
     lambda x: x.decision["policy_version"] == REPAIR_DECISION_POLICY_VERSION),
    ("RepairDecision was made for another framing layout",
     lambda x: x.decision["framing_layout_version"] == x.layout),
    ("RepairDecision.policy is not a known repair policy",
     lambda x: x.decision["policy"] in _REPAIR_POLICIES),
    ("RepairDecision.quality_profile_id is neither a string nor null",
     lambda x: x.decision["quality_profile_id"] is None or isinstance(x.decision["quality_profile_id"], str)),
    ("RepairDecision lacks its reason or workload class",
     lambda x: _nonblank(x.decision["reason"]) and _nonblank(x.decision["workload_class"])),
)

_BINDING_RULES = (
    ("recompute_initial_tokens is not the decision's selected_k",
     lambda x: _exact_int(x.wire.get("recompute_initial_tokens")) and x.wire["recompute_initial_tokens"] == x.k),
    ("recompute_tokens_per_block is not the decision's windows",
     lambda x: x.wire.get("recompute_tokens_per_block") == x.windows),
    ("first-block repair fields disagree with the decision's first window",
     lambda x: x.wire.get("recompute_first_block_tokens") == x.windows[0]
     and x.wire.get("recompute_first_block") is bool(x.windows[0])),
    ("legacy legolink_k disagrees with the decision's selected_k",
     lambda x: "legolink_k" not in x.wire or x.wire["legolink_k"] == x.k),
)

_EVIDENCE_RULES = (
    ("formal execution needs a quality_guarded repair decision",
     lambda x: x.decision["policy"] == "quality_guarded"),
    ("the deployment profile is absent or was made for another FramingSpec",
     lambda x: isinstance(x.profile, dict) and x.profile.get("framing_spec") == x.spec),
    ("the complete input has no reviewed canonical framing in the deployment profile",
     lambda x: x.wire.get("expected_complete_token_ids_sha256") in x.reviewed_inputs()),
    ("the deployment profile has no repair quality measurement under quality_profile_id",
     lambda x: isinstance(x.measurement(), dict)),
    ("the repair quality measurement was made for another decision", _measurement_matches),
    ("the repair quality measurement did not pass or lacks its provenance", _measurement_passed),
    ("the measured repair quality is below its required threshold", _measurement_meets_threshold),
)


def _enforce(rules, x: _Intent) -> None:
    for why, ok in rules:
        if not ok(x):
            raise ContractError(f"execution governance: {why}.")


def validate_execution_intent(wire: Mapping, profile: Optional[Mapping] = None, *, require_formal=False) -> None:
    """Refuses a request whose declared execution intent is not honoured.

    ``legacy_debug`` requests that carry neither a FramingSpec nor a
    RepairDecision are accepted as they are; anything else must pass the
    framing, decision and binding tables, and formal execution (by request or
    by deployment) or a quality-guarded decision must also pass the evidence
    table against ``profile``."""
    mode = wire.get("execution_mode", "legacy_debug")
    if mode not in ("formal", "legacy_debug"):
        raise ContractError(f"execution governance: execution_mode {mode!r} is neither formal nor legacy_debug.")
    if require_formal and mode != "formal":
        raise ContractError("execution governance: this deployment serves formal execution only.")
    formal = mode == "formal"
    x = _Intent(wire, profile)
    if not formal and x.spec is None and x.decision is None:
        return
    for table in (_FRAMING_RULES, _DECISION_RULES, _BINDING_RULES):
        _enforce(table, x)
    if formal or x.decision["policy"] == "quality_guarded":
        _enforce(_EVIDENCE_RULES, x)


def runtime_execution_profile() -> Optional[dict]:
    path = os.getenv("SGLANG_PIC_EXECUTION_PROFILE")
    if not path:
        return None
    with open(path, encoding="utf-8") as f:
        return json.load(f)


def validate_pic_link_request(plan: Any, *, profile: Optional[Mapping] = None, require_formal: Optional[bool] = None,
                              allow_legacy_fields: Optional[bool] = None) -> None:
    """Refuse what the host is not entitled to send (runtime-owned physical
    fields, unknown fields, malformed values, governance violations)."""
    if not isinstance(plan, dict):
        raise ContractError("pic_link must be an object.")
    validate_pic_link_field_types(plan)
    if require_formal is None:
        require_formal = env_flag("SGLANG_PIC_FORMAL_EXECUTION")
    if profile is None:
        profile = runtime_execution_profile()
    validate_execution_intent(plan, profile, require_formal=require_formal)
    physical = sorted(set(plan) & PIC_LINK_RUNTIME_OWNED_FIELDS)
    if physical:
        if allow_legacy_fields is None:
            allow_legacy_fields = env_flag("SGLANG_PIC_ALLOW_LEGACY_LINK_FIELDS")
        if plan.get("execution_mode") == "formal" or not allow_legacy_fields:
            raise ContractError(
                "pic_link carries fields the runtime derives and the host cannot know: "
                f"{', '.join(physical)}. Send the semantic selection only; set "
                "SGLANG_PIC_ALLOW_LEGACY_LINK_FIELDS=1 to replay a pre-contract plan file."
            )
        for n in physical:
            plan.pop(n, None)
    unknown = sorted(set(plan) - PIC_LINK_REQUEST_FIELDS - PIC_LINK_RUNTIME_OWNED_FIELDS - PIC_LINK_INTERNAL_FIELDS)
    if unknown:
        raise ContractError(
            f"pic_link has unknown fields: {', '.join(unknown)}. Host correctness evidence and repair-window "
            "rationale belong in the host audit record, not in the runtime request."
        )


def validate_physical_token_input(meta: Any, *, label: str) -> Optional[list[int]]:
    """Validates an exact token override (count + sha256) on Compile/Link
    metadata; returns the ids or None when absent."""
    if not isinstance(meta, dict) or "physical_input_ids" not in meta:
        return None
    version = meta.get("physical_token_layout_version")
    if version != PHYSICAL_TOKEN_LAYOUT_VERSION:
        raise ContractError(f"{label} physical token layout version is unsupported: {version!r}")
    raw = meta.get("physical_input_ids")
    if not isinstance(raw, list) or not raw:
        raise ContractError(f"{label}.physical_input_ids must be a non-empty integer list.")
    if any(isinstance(t, bool) or not isinstance(t, int) for t in raw):
        raise ContractError(f"{label}.physical_input_ids contains a non-integer token id.")
    ids = [int(t) for t in raw]
    cnt = meta.get("physical_token_count")
    if isinstance(cnt, bool) or not isinstance(cnt, int) or cnt != len(ids):
        raise ContractError(f"{label} physical token count mismatch: metadata={cnt!r}, actual={len(ids)}")
    h = meta.get("physical_token_ids_sha256")
    actual = physical_token_ids_sha256(ids)
    if not isinstance(h, str) or h != actual:
        raise ContractError(f"{label} physical token hash mismatch: expected={h!r}, actual={actual}")
    return ids


def residency_recovery_message(missing=(), stale=(), incompatible=(),
                               reason: str = "scheduler_source_preflight_failed") -> str:
    """The abort text of a Link whose source blocks are not usable.  A JSON
    object naming the missing / stale / incompatible keys is appended so a host
    can recompile exactly those keys under the same identity and resend
    (wire format of reference ``pic_runtime.py:2889-2912``)."""
    detail = {
        "noc_residency_recovery": {
            "reason": reason,
            "missing_cache_keys": [str(k) for k in missing],
            "stale_cache_keys": [str(k) for k in stale],
            "incompatible_cache_keys": [str(k) for k in incompatible],
        }
    }
    names = [*missing, *stale, *incompatible]
    return ("LegoLink source preflight failed before destination KV allocation: " + ", ".join(map(str, names))
            + " | " + json.dumps(detail, separators=(",", ":")))


def parse_residency_recovery(message: str) -> dict[str, tuple[str, ...]]:
    """Inverse of :func:`residency_recovery_message`; also unwraps an HTTP
    error body whose ``message`` holds the text.  Empty tuples when absent."""
    empty = {"missing": (), "stale": (), "incompatible": ()}
    marker = '{"noc_residency_recovery"'
    start = message.find(marker)
    if start < 0:
        try:
            body = json.loads(message)
        except ValueError:
            return empty
        inner = body.get("message") if isinstance(body, dict) else None
        if isinstance(inner, str) and inner != message:
            return parse_residency_recovery(inner)
        return empty
    try:
        parsed, _ = json.JSONDecoder().raw_decode(message[start:])
    except ValueError:
        return empty
    detail = (parsed or {}).get("noc_residency_recovery") or {}
    return {n: tuple(str(v) for v in (detail.get(f"{n}_cache_keys") or ())) for n in ("missing", "stale", "incompatible")}
