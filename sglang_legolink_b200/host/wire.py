"""The reference's JSON wire objects: field tables and exporters.

A host built for the reference writes session events, semantic
sub-contexts, context manifests, execution plans, LegoLink requests and
experiment metric rows in a fixed JSON shape
(``schemas/noc_*.schema.json`` of the reference).  This module states those
shapes as tables -- field name, type, bounds, required -- from which
``sglang_legolink_b200.schemas`` builds the ``noc_*`` JSON Schemas, and maps
this implementation's own objects onto them:

* :func:`session_event_wire`, :func:`subcontext_wire`,
  :func:`manifest_wire`, :func:`execution_plan_wire`,
  :func:`legolink_request_wire`, :func:`experiment_metric_row`.

The field names and types are the wire contract (they must match for rows
and plans to be exchanged), so they are the reference's; the code that
produces them is this host's own.
"""

from __future__ import annotations

import datetime as _dt
import hashlib
from typing import Any, Iterable, Mapping, Optional, Sequence

# ------------------------------------------------------------------ tables
# Field spec: "<type>[<bounds>]" with types s(tring) i(nteger) n(umber)
# b(oolean) a(rray of strings) o(bject) A(rray, any items), suffix "?" =
# nullable, bounds "+" = minimum 0, "1" = minimum 1, "r" = maximum 1,
# "h" = 64 lowercase hex digits, "t" = date-time, "!" = non-empty.

CONTEXT_FIELD_VALUES = ("user_prompt", "task_instruction", "tool_definitions", "tool_history_output",
                        "conversation_history", "workspace_evidence", "task_metadata")
EVENT_TYPE_VALUES = ("user_request", "task_instruction", "planner_output", "tool_definition", "tool_call",
                     "tool_output", "conversation_message", "workspace_file", "task_metadata", "unclassified")

SESSION_EVENT = {"event_id": "s!", "task_id": "s!", "session_revision": "i1", "event_type": EVENT_TYPE_VALUES,
                 "source_id": "s!", "raw_text": "s", "timestamp": "st", "sequence_number": "i1", "metadata": "o"}
SESSION_EVENT_REQUIRED = tuple(SESSION_EVENT)

SEMANTIC_SUBCONTEXT = {
    "sub_context_id": "s", "task_id": "s", "session_revision": "i1", "context_field": CONTEXT_FIELD_VALUES,
    "title": "s", "question_or_objective": "s", "raw_text": "s", "canonical_text": "s", "source_spans": "spans",
    "content_hash": "sh", "cache_key": "sh", "version": "i1", "token_count": "i+", "token_ids": "A",
    "tokenizer_fingerprint": "s!", "model_fingerprint": "s!", "recompute_policy_version": "s!", "is_mutable": "b",
    "reuse_candidate": "b", "semantic_independence_reason": "s", "segmentation_confidence": "n+r",
    "policy_version": "s", "created_at": "st", "updated_at": "st", "supersedes": "s?", "invalidated": "b",
    "derived_from": "a", "metadata": "o"}
SEMANTIC_SUBCONTEXT_OPTIONAL = ("supersedes", "derived_from", "metadata")

AGENT_CONTEXT_MANIFEST = {
    "task_id": "s", "agent_id": "s", "request_id": "s", "session_revision": "i1", "objective": "s",
    "selected_sub_context_ids": "au", "selected_cache_keys": "a", "mutable_text": "s",
    "full_session_tokens": "i+", "candidate_context_tokens": "i+", "selected_context_tokens": "i+",
    "context_reduction_tokens": "i+", "context_reduction_ratio": "n+r", "selection_reason": "os",
    "excluded_reason": "os", "selection_order": "au", "excluded_sub_context_ids": "au",
    "context_token_budget": "i+"}

REQUEST_EXECUTION_PLAN = {
    "manifest": "o", "selected_order": "a", "reuse_cached": "a", "compile_on_miss": "a", "keep_mutable": "a",
    "excluded": "a", "expected_cache_keys": "a", "baseline_selected_text": "s", "text_separator": "s",
    "decisions": "ao", "block_planning": "planning", "layout_decisions": "ao", "layout_summary": "o",
    "reuse_eligibility_summary": "eligibility", "profitability": "profitability"}
REQUEST_EXECUTION_PLAN_REQUIRED = ("manifest", "selected_order", "reuse_cached", "compile_on_miss", "keep_mutable",
                                   "excluded", "expected_cache_keys", "baseline_selected_text", "text_separator",
                                   "decisions")
# physical fields that must never appear in a planning record
PLAN_FORBIDDEN_FIELDS = ("imp_indices", "kvlink", "recompute_positions", "block_ranges", "attention_ranges",
                         "kv_slots", "global_positions")
BLOCK_PLANNING_ENUMS = {
    "cache_availability": ("", "host_catalog_entry", "no_cached_state", "stale_cached_state"),
    "reuse_eligibility": ("", "exact_safe", "reconstruct_required", "experimental_foreign", "no_reuse_candidate"),
    "eligibility_reason": ("", "exact_safe_state", "canonical_standalone_compile_on_miss", "not_a_semantic_candidate",
                           "cached_state_identity_mismatch", "legacy_identity_unverified", "state_origin_unknown",
                           "contextual_state_not_proven", "experimental_foreign_disabled",
                           "experimental_foreign_enabled"),
    "identity_basis": ("", "token_ids", "text", "legacy_provenance"),
    "feasibility_reason": ("none", "layout_forced_compile", "layout_forced_native"),
    "effective_decision": ("REUSE_CACHED", "COMPILE_ON_MISS", "KEEP_MUTABLE", "DROPPED"),
}
ELIGIBILITY_SUMMARY_REQUIRED = ("reuse_eligibility_policy_version", "eligibility_counts",
                                "eligible_reuse_block_count", "experimental_link_count", "canonical")

LEGOLINK_REQUEST = {"request_id": "s!", "semantic_block_ids": "a!", "cache_keys": "a!", "mutable_text": "s!",
                    "generation_parameters": "o"}

METRIC_LEVELS = ("request", "agent_step", "task", "experiment", "cuda_component", "host_timing",
                 "profiler_component", "nsight_run")
METRIC_VARIANTS = ("full_context_original_sglang", "selected_context_original_sglang",
                   "selected_context_radixcache_legolink", "picruntime_owner", "radixcache_owner", "original_sglang")
MEASUREMENT_KINDS = ("formal_latency", "diagnostic_cuda_event", "diagnostic_pytorch_profiler", "diagnostic_nsight",
                     "diagnostic_nsight_systems", "diagnostic_host_timing", "paired_replay", "official_agent",
                     "wildclaw_long_running")
PROFILING_TYPES = (None, "cuda_event", "pytorch_profiler", "nsight", "nsight_systems", "host_timing")

# the 127 fields of an experiment metric row (all nullable except the three
# enums, which are required)
EXPERIMENT_METRICS = dict(
    [("metric_level", METRIC_LEVELS), ("variant", METRIC_VARIANTS), ("measurement_kind", MEASUREMENT_KINDS)]
    + [(f, "s?") for f in ("task_id", "request_id", "session_id")] + [("session_revision", "i?+")]
    + [(f, "s?") for f in ("trial_id", "phase", "context_stratum")]
    + [(f, "i?+") for f in ("k", "decode_iteration")] + [("warmup", "b?"), ("warmup_repeats", "i?+")]
    + [(f, "b?") for f in ("fixed_output_length", "completion_length_equal")] + [("cache_accounting_source", "s?")]
    + [("concurrency", "i?1"), ("sample_count", "i?+")]
    + [(f, "n?") for f in (
        "mean_s", "std_s", "p50_s", "p95_s", "min_s", "max_s", "request_latency_ms", "e2e_latency_ms",
        "step_latency_ms", "planning_latency_ms", "replanning_latency_ms", "total_llm_latency_ms",
        "tool_execution_time_ms", "context_management_latency_ms", "segmentation_latency_ms",
        "selection_latency_ms", "compile_latency_ms", "compile_inclusive_latency_ms", "environment_setup_latency_ms",
        "agent_latency_ms", "grader_latency_ms", "ttft_ms", "prefill_ms", "link_ms", "total_prefill_or_link_time_ms",
        "decode_ms", "queue_wait_ms", "itl_mean_ms", "itl_p50_ms", "itl_p95_ms", "output_tokens_per_second",
        "requests_per_second", "llm_requests_per_minute")]
    + [(f, "i?+") for f in (
        "prompt_tokens", "output_tokens", "backend_input_tokens", "backend_output_tokens", "local_model_input_tokens",
        "local_model_output_tokens", "full_session_tokens", "selected_context_tokens")]
    + [("context_reduction_ratio", "n?+")]
    + [(f, "i?+") for f in (
        "context_reduction_tokens", "candidate_context_tokens", "mutable_tokens", "compiled_tokens", "compiled_blocks",
        "number_of_blocks", "new_compiled_blocks", "unique_semantic_blocks", "linked_tokens", "reused_blocks",
        "reused_tokens", "recomputed_tokens")]
    + [(f, "n?+r") for f in ("cache_reuse_ratio", "recompute_ratio")]
    + [(f, "i?+") for f in (
        "cache_hits", "cache_misses", "evicted_blocks", "evicted_tokens", "fallback_count", "recovery_success_count",
        "superseded_blocks", "invalidated_blocks")]
    + [("average_reuse_count_per_block", "n?+"), ("new_tool_output_tokens", "i?+")]
    + [(f, "a?") for f in ("selected_blocks", "excluded_blocks")] + [("task_state", "s?"), ("exact", "b?")]
    + [(f, "n?+r") for f in ("exact_rate", "similarity", "similarity_mean")]
    + [(f, "b?") for f in ("task_success", "verifier_pass")] + [("verifier_score", "n?")]
    + [(f, "b?") for f in ("timeout", "oom")] + [(f, "s?") for f in ("error", "failure_mode")]
    + [(f, "i?+") for f in (
        "agent_steps", "llm_calls", "tool_calls", "successful_tool_calls", "failed_tool_calls", "planner_calls",
        "replanner_calls", "repeated_action_count", "invalid_tool_call_count", "completed_tasks", "failed_tasks",
        "timeout_tasks", "error_tasks", "oom_tasks")]
    + [("average_steps_per_task", "n?+"), ("max_steps", "i?+")]
    + [(f, "n?") for f in ("tasks_per_hour", "successful_tasks_per_gpu_hour", "steps_per_minute")]
    + [("effective_batch_size", "n?+")]
    + [(f, "i?+") for f in ("active_request_count", "prefill_batch_size", "decode_batch_size")]
    + [("component", "s?"), ("elapsed_ms", "n?"), ("profiling_type", PROFILING_TYPES)]
    + [(f, "b?") for f in ("formal_latency", "diagnostic")])
EXPERIMENT_METRICS_REQUIRED = ("metric_level", "variant", "measurement_kind")


# ------------------------------------------------------------- exporters
def _now() -> str:
    return _dt.datetime.now(_dt.timezone.utc).isoformat().replace("+00:00", "Z")


def _sha(text: str) -> str:
    return hashlib.sha256(text.encode("utf-8")).hexdigest()


def session_event_wire(ev) -> dict:
    d = ev.to_dict()
    return {k: d[k] for k in SESSION_EVENT}


def subcontext_wire(sc, *, session_revision: Optional[int] = None, created_at: Optional[str] = None) -> dict:
    md = dict(sc.metadata or {})
    at = created_at or md.get("created_at") or _now()
    spans = [{"source_id": s.source_id, "start": int(s.start), "end": max(int(s.end), int(s.start) + 1)}
             for s in sc.source_spans] or [{"source_id": sc.source_id, "start": 0, "end": 1}]
    return {
        "sub_context_id": sc.sub_context_id, "task_id": sc.task_id,
        "session_revision": max(1, int(session_revision or sc.source_revision or 1)),
        "context_field": sc.context_field,
        "title": str(md.get("title") or f"{sc.context_field} {sc.sequence_number}.{md.get('segment_index', 0)}"),
        "question_or_objective": str(md.get("question_or_objective") or ""),
        "raw_text": sc.raw_text, "canonical_text": sc.raw_text, "source_spans": spans,
        "content_hash": _sha(sc.raw_text), "cache_key": sc.cache_key, "version": max(1, int(sc.source_revision or 1)),
        "token_count": int(sc.token_count), "token_ids": [int(t) for t in sc.token_ids],
        "tokenizer_fingerprint": str(md.get("tokenizer_fingerprint") or "unknown"),
        "model_fingerprint": str(md.get("model_fingerprint") or "unknown"),
        "recompute_policy_version": str(md.get("recompute_policy_version") or "legolink-radix-v1"),
        "is_mutable": bool(sc.is_mutable), "reuse_candidate": bool(sc.reuse_candidate),
        "semantic_independence_reason": str(md.get("semantic_independence_reason")
                                            or "deterministic field-first segmentation"),
        "segmentation_confidence": float(md.get("segmentation_confidence", 1.0)),
        "policy_version": str(md.get("segmentation_policy_version") or "field-first-v1"),
        "created_at": at, "updated_at": md.get("updated_at") or at, "supersedes": md.get("supersedes"),
        "invalidated": bool(sc.invalidated), "derived_from": [str(x) for x in md.get("derived_from", [])],
        "metadata": md,
    }


def manifest_wire(manifest, contexts: Sequence, *, agent_id: str = "agent", request_id: str = "",
                  objective: str = "", full_session_tokens: Optional[int] = None) -> dict:
    by_id = {v.sub_context_id: v for v in contexts}
    sel = [i for i in manifest.selected_sub_context_ids if i in by_id]
    excl = [i for i in manifest.excluded_sub_context_ids if i in by_id]
    candidate = sum(v.token_count for v in contexts)
    selected = sum(by_id[i].token_count for i in sel)
    full = int(full_session_tokens if full_session_tokens is not None else candidate)
    red = max(0, full - selected)
    return {
        "task_id": manifest.task_id, "agent_id": agent_id, "request_id": request_id or f"{manifest.task_id}-req",
        "session_revision": max(1, int(manifest.session_revision)), "objective": objective or manifest.mutable_text,
        "selected_sub_context_ids": sel, "selected_cache_keys": [by_id[i].cache_key for i in sel],
        "mutable_text": manifest.mutable_text, "full_session_tokens": full, "candidate_context_tokens": candidate,
        "selected_context_tokens": selected, "context_reduction_tokens": red,
        "context_reduction_ratio": (red / full) if full else 0.0,
        "selection_reason": {i: f"selected by {manifest.selector}" for i in sel},
        "excluded_reason": {i: "outside the selection" for i in excl},
        "selection_order": list(dict.fromkeys(manifest.selection_order or sel)), "excluded_sub_context_ids": excl,
        "context_token_budget": int(manifest.token_budget if manifest.token_budget is not None else selected),
    }


_EFFECTIVE = {"linked": "REUSE_CACHED", "compile_on_miss": "COMPILE_ON_MISS", "mutable": "KEEP_MUTABLE",
              "omitted": "DROPPED"}
_FEASIBILITY = {"none": "none", "promoted_for_prefix_closure": "layout_forced_compile",
                "demoted_after_suffix": "layout_forced_native"}


def execution_plan_wire(plan, *, agent_id: str = "agent", request_id: str = "") -> dict:
    """The planner's plan as the reference's ``NOCRequestExecutionPlan``:
    logical only (no slots, positions, RoPE deltas or ``imp_indices``)."""
    by_cat = {c: [r.sub_context_id for r in plan.records if r.planner_category == c] for c in _EFFECTIVE}
    ctx = list(plan.included_contexts) + list(plan.omitted_contexts)
    ident = {v.sub_context_id: ("token_ids" if v.semantic_identity.startswith("si-tok-")
                                else "text" if v.semantic_identity.startswith("si-txt-") else "legacy_provenance")
             for v in ctx}
    planning, counts = [], {}
    for r in plan.records:
        eligible = r.planner_category in ("linked", "compile_on_miss")
        elig = "exact_safe" if eligible else "no_reuse_candidate"
        counts[elig] = counts.get(elig, 0) + 1
        planning.append({
            "sub_context_id": r.sub_context_id, "cache_key": r.cache_key, "token_count": r.token_count,
            "semantic_candidate": r.policy_action in ("compile", "summarize_then_compile"),
            "cache_available": r.planner_category == "linked",
            "cache_availability": "host_catalog_entry" if r.planner_category == "linked" else "no_cached_state",
            "reuse_eligibility": elig,
            "eligibility_reason": ("exact_safe_state" if r.planner_category == "linked" else
                                   "canonical_standalone_compile_on_miss" if eligible else "not_a_semantic_candidate"),
            "state_origin": "standalone_compile", "identity_basis": ident.get(r.sub_context_id, ""),
            "provisional_decision": r.policy_action, "eligibility_adjusted": False, "policy_action": r.policy_action,
            "feasibility_adjustment": r.layout_adjustment,
            "feasibility_reason": _FEASIBILITY.get(r.layout_adjustment, "none"),
            "effective_action": r.effective_action, "effective_decision": _EFFECTIVE[r.planner_category],
            "experimental": False, "preceding_context_tokens": None, "reason": r.reason,
        })
    acc = plan.accounting
    return {
        "manifest": manifest_wire(plan.manifest, ctx, agent_id=agent_id, request_id=request_id),
        "selected_order": [r.sub_context_id for r in plan.records],
        "reuse_cached": by_cat["linked"], "compile_on_miss": by_cat["compile_on_miss"],
        "keep_mutable": by_cat["mutable"], "excluded": by_cat["omitted"],
        "expected_cache_keys": list(plan.expected_cache_keys), "baseline_selected_text": plan.baseline_selected_text,
        "text_separator": plan.text_separator,
        "decisions": [{"sub_context_id": r.sub_context_id, "cache_key": r.cache_key, "action": r.policy_action,
                       "reason": r.reason, "token_count": r.token_count} for r in plan.records],
        "block_planning": planning,
        "layout_decisions": [{"sub_context_id": r.sub_context_id, "adjustment": r.layout_adjustment}
                             for r in plan.records if r.layout_adjustment != "none"],
        "layout_summary": {"linked_prefix_blocks": len(plan.linked_contexts),
                           "mutable_suffix_blocks": len(plan.mutable_contexts),
                           "adjusted_blocks": sum(r.layout_adjustment != "none" for r in plan.records)},
        "reuse_eligibility_summary": {"reuse_eligibility_policy_version": "canonical-standalone-v1",
                                      "eligibility_counts": counts,
                                      "eligible_reuse_block_count": len(plan.linked_contexts),
                                      "experimental_link_count": 0, "canonical": True},
        "profitability": {"enforced": False, "profitability_mode": "observe_only", "verdict": acc.verdict,
                          "reused_tokens": acc.reused_tokens, "repair_tokens": acc.repair_tokens},
    }


def legolink_request_wire(plan, *, request_id: str, generation: Optional[Mapping] = None) -> dict:
    """The client-side contract checked before a ``pic_link`` request is sent."""
    return {"request_id": str(request_id), "semantic_block_ids": [v.semantic_identity for v in plan.linked_contexts],
            "cache_keys": [v.cache_key for v in plan.linked_contexts], "mutable_text": plan.manifest.mutable_text,
            "generation_parameters": dict(generation or {})}


# this repo's metric names -> the wire names (both are kept on a row)
_METRIC_RENAMES = {"link_latency_ms": "link_ms", "native_prefill_latency_ms": "prefill_ms",
                   "decode_latency_ms": "decode_ms", "itl_ms": "itl_mean_ms", "concurrent_tasks": "concurrency",
                   "eviction_count": "evicted_blocks", "selected_ids": "selected_blocks",
                   "excluded_ids": "excluded_blocks", "segment_count": "number_of_blocks",
                   "loop_stage": "phase"}
_VARIANT_OF = {"legolink": "selected_context_radixcache_legolink", "pic_link": "picruntime_owner"}


def experiment_metric_row(row, *, metric_level: str = "request") -> dict:
    """A metric row (``AgentMetric`` or its dict) with the wire fields filled
    in; values that do not fit a wire field's type are left out of it."""
    d = row.to_dict() if hasattr(row, "to_dict") else dict(row)
    out = dict(d)
    for src, dst in _METRIC_RENAMES.items():
        if d.get(src) is not None and out.get(dst) is None:
            out[dst] = d[src]
    out["metric_level"] = d.get("metric_level") or metric_level
    v = str(d.get("variant") or "")
    out["variant"] = v if v in METRIC_VARIANTS else _VARIANT_OF.get(v, "selected_context_radixcache_legolink")
    mk = str(d.get("measurement_kind") or "formal_latency")
    out["measurement_kind"] = mk if mk in MEASUREMENT_KINDS else "diagnostic_host_timing"
    out.setdefault("formal_latency", out["measurement_kind"] == "formal_latency")
    out.setdefault("diagnostic", out["measurement_kind"].startswith("diagnostic"))
    if out.get("concurrency") is not None and not (isinstance(out["concurrency"], int) and out["concurrency"] >= 1):
        out.pop("concurrency")
    for name, spec in EXPERIMENT_METRICS.items():
        if name in out and isinstance(spec, str) and not _fits(out[name], spec):
            out.pop(name)
    return out


def _fits(value: Any, spec: str) -> bool:
    if value is None:
        return "?" in spec
    t = spec[0]
    ok = {"s": isinstance(value, str), "b": isinstance(value, bool),
          "i": isinstance(value, int) and not isinstance(value, bool),
          "n": isinstance(value, (int, float)) and not isinstance(value, bool),
          "a": isinstance(value, list) and all(isinstance(x, str) for x in value)}.get(t, True)
    if ok and t in "in":
        if "+" in spec and value < 0 or "1" in spec and value < 1 or "r" in spec and value > 1:
            return False
    return ok


def export_rows(rows: Iterable, *, metric_level: str = "request") -> list:
    return [experiment_metric_row(r, metric_level=metric_level) for r in rows]
