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
def _err(name: str, problem: str) -> ContractError:
    return ContractError(f"pic_link.{name} {problem}.")


def _int_field(plan: Mapping, name: str, *, nullable=False, minimum=0, maximum=PIC_LINK_MAX_INTEGER):
    if name not in plan:
        return None
    v = plan[name]
    if v is None:
        if nullable:
            return None
        raise _err(name, "must not be null")
    if isinstance(v, bool) or not isinstance(v, int):
        raise _err(name, "must be an integer")
    if v < minimum or v > maximum:
        raise _err(name, f"must be between {minimum} and {maximum}")
    return v


def _opt_str(plan: Mapping, name: str) -> None:
    v = plan.get(name)
    if v is not None and not isinstance(v, str):
        raise _err(name, "must be a string when present")


def _opt_bool(plan: Mapping, name: str) -> None:
    v = plan.get(name)
    if v is not None and not isinstance(v, bool):
        raise _err(name, "must be a boolean when present")


def _label(plan: Mapping, name: str) -> None:
    v = plan.get(name)
    if v is None or isinstance(v, str):
        return
    if isinstance(v, bool) or not isinstance(v, int):
        raise _err(name, "must be a string or an integer when present")


def _str_list(plan: Mapping, name: str, *, required=False, at_most: Optional[int] = None):
    if name not in plan:
        if required:
            raise _err(name, "must be non-empty")
        return None
    v = plan[name]
    if v is None:
        if required:
            raise _err(name, "must not be null")
        return None
    if not isinstance(v, list):
        raise _err(name, "must be a list of strings")
    if required and not v:
        raise _err(name, "must be non-empty")
    if any(not isinstance(x, str) for x in v):
        raise _err(name, "must contain only strings")
    if at_most is not None and len(v) > at_most:
        raise _err(name, f"may hold at most {at_most} entries")
    return v


def validate_pic_link_field_types(plan: Mapping) -> None:
    """Type/range checks for every host-sendable value (reference
    ``pic_runtime.py:845-922``)."""
    keys = _str_list(plan, "cache_keys", required=True) or []
    for n in ("request_id", "task_id"):
        _label(plan, n)
    _opt_str(plan, "variant")
    _opt_bool(plan, "profiling_warmup")
    _int_field(plan, "concurrency", nullable=True)
    _str_list(plan, "block_ids", at_most=len(keys))
    for n in ("adapter_id", "segmentation_policy_version", "legolink_policy_version", "execution_group_key"):
        _opt_str(plan, n)
    _opt_bool(plan, "promote_reconstructed_group")
    if "recompute_mode" in plan:
        mode = plan["recompute_mode"]
        if not isinstance(mode, str):
            raise _err("recompute_mode", "must be a string")
        if mode.lower() not in PIC_LINK_RECOMPUTE_MODES:
            raise _err("recompute_mode", "must be one of " + ", ".join(sorted(PIC_LINK_RECOMPUTE_MODES)))
    _int_field(plan, "recompute_initial_tokens")
    _int_field(plan, "legolink_k")
    _opt_bool(plan, "recompute_first_block")
    _int_field(plan, "recompute_first_block_tokens", nullable=True)
    if plan.get("recompute_tokens_per_block") is not None:
        w = plan["recompute_tokens_per_block"]
        if not isinstance(w, list):
            raise _err("recompute_tokens_per_block", "must be a list of integers")
        if len(w) != len(keys):
            raise _err("recompute_tokens_per_block", "must contain one value per cache key")
        for x in w:
            if isinstance(x, bool) or not isinstance(x, int) or x < 0 or x > PIC_LINK_MAX_INTEGER:
                raise _err("recompute_tokens_per_block", "must contain only non-negative integers within range")


def validate_execution_intent(wire: Mapping, profile: Optional[Mapping] = None, *, require_formal=False) -> None:
    """Formal vs legacy_debug governance (reference ``pic_runtime.py:1060-1148``
    and host twin ``execution_governance.py:66``): FramingSpec and
    RepairDecision shape, consistency with the repair fields, and -- for formal
    or quality-guarded execution -- agreement with the deployment profile."""
    mode = wire.get("execution_mode", "legacy_debug")
    if mode not in ("formal", "legacy_debug"):
        raise ContractError("unknown execution_mode")
    if require_formal and mode != "formal":
        raise ContractError("formal deployment rejects legacy_debug execution")
    formal = require_formal or mode == "formal"
    framing, repair = wire.get("framing_spec"), wire.get("repair_decision")
    if not formal and framing is None and repair is None:
        return
    if not isinstance(framing, dict) or set(framing) != FRAMING_SPEC_FIELDS:
        raise ContractError("missing or malformed framing_spec")
    if any(not isinstance(v, str) or not v.strip() for v in framing.values()):
        raise ContractError("framing identity must be nonempty")
    version = framing["framing_layout_version"]
    if version != PHYSICAL_TOKEN_LAYOUT_VERSION:
        raise ContractError("unsupported/legacy framing version")
    th = framing["chat_template_sha256"]
    if len(th) != 64 or any(ch not in "0123456789abcdef" for ch in th):
        raise ContractError("invalid chat template hash")
    if wire.get("physical_token_layout_version") != version:
        raise ContractError("framing and physical layout version disagree")
    if not isinstance(repair, dict) or set(repair) != REPAIR_DECISION_FIELDS:
        raise ContractError("missing or malformed RepairDecision")
    k, windows = repair["selected_k"], repair["windows"]
    if type(k) is not int or k < 0:
        raise ContractError("selected_k must be a nonnegative integer")
    if (not isinstance(windows, list) or len(windows) != len(wire.get("cache_keys", [])) or not windows
            or any(type(v) is not int or v < 0 or v > k for v in windows)):
        raise ContractError("invalid repair window vector")
    if repair["policy_version"] != REPAIR_DECISION_POLICY_VERSION:
        raise ContractError("unsupported repair policy version")
    if repair["framing_layout_version"] != version:
        raise ContractError("repair/framing incompatibility")
    if repair["policy"] not in ("quality_guarded", "fixed_unvalidated_debug"):
        raise ContractError("unknown repair policy")
    if repair["quality_profile_id"] is not None and not isinstance(repair["quality_profile_id"], str):
        raise ContractError("quality_profile_id must be a string or null")
    if not all(isinstance(repair[x], str) and repair[x].strip() for x in ("reason", "workload_class")):
        raise ContractError("missing repair provenance")
    if type(wire.get("recompute_initial_tokens")) is not int or wire["recompute_initial_tokens"] != k:
        raise ContractError("repair K was replaced or defaulted")
    if wire.get("recompute_tokens_per_block") != windows:
        raise ContractError("repair windows were replaced or defaulted")
    if (wire.get("recompute_first_block_tokens") != windows[0]
            or wire.get("recompute_first_block") is not bool(windows[0])):
        raise ContractError("first-block repair disagrees with decision")
    if "legolink_k" in wire and wire["legolink_k"] != k:
        raise ContractError("legacy K alias disagrees with decision")
    if formal or repair["policy"] == "quality_guarded":
        if repair["policy"] != "quality_guarded":
            raise ContractError("formal execution requires measured repair quality")
        if not isinstance(profile, dict) or profile.get("framing_spec") != framing:
            raise ContractError("missing/incompatible deployment framing profile")
        if wire.get("expected_complete_token_ids_sha256") not in profile.get("canonical_input_hashes", []):
            raise ContractError("input has no reviewed canonical framing evidence")
        quality = profile.get("repair_quality_profiles", {}).get(repair["quality_profile_id"])
        if not isinstance(quality, dict):
            raise ContractError("missing repair quality profile")
        for name in ("selected_k", "windows", "workload_class", "evidence_id"):
            if quality.get(name) != repair[name]:
                raise ContractError("incompatible repair quality " + name)
        if (quality.get("framing_spec") != framing or quality.get("status") != "PASS"
                or quality.get("profile_id") != repair["quality_profile_id"]
                or not repair["evidence_id"] or not quality.get("metric")):
            raise ContractError("unvalidated repair quality provenance")
        measured, threshold = quality.get("measured_value"), quality.get("required_threshold")
        if (type(measured) not in (float, int) or type(threshold) not in (float, int)
                or not math.isfinite(measured) or not math.isfinite(threshold) or measured < threshold):
            raise ContractError("repair quality threshold not satisfied")


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
