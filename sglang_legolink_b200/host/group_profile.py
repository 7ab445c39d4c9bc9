"""EXPERIMENTAL group repair quality profile: may this execution group be
reconstructed from its cached members and promoted, or must it be compiled
as a whole?

Off by default and not consulted by the default planner.  A profile is a
contract over what a request shows *before* it runs -- token counts, member
order and residency, the declared reconstruction policy and the deployment's
compatibility identity.  It cannot be given an answer, a logit or a margin
(:data:`FORBIDDEN_ONLINE_FIELDS` are refused at construction), and it owns no
physical layout (:data:`RUNTIME_OWNED_FIELDS`).  The certification evidence
is referenced by the profile but never read when deciding.

:func:`evaluate` runs the structural checks in a fixed order and names the
first that fails; :func:`route` turns the decision into one of three routes
(group cache hit, reconstruct-and-promote, full group recompile -- an
ineligible request is always served, by the recompile); the
reconstruct-and-promote route also needs the deployment's promotion flag.
:func:`link_fields` writes a route into a Link request for the runtime
(`Engine._promote_group` does the promotion).

Reference: ``noc_context_manager/group_repair_profile.py:47-515``
(``GroupRepairQualityProfile`` ``:154``, ``route_execution_group`` ``:438``).
"""

from __future__ import annotations

import hashlib
import json
import time
from dataclasses import asdict, dataclass, field
from enum import Enum
from pathlib import Path
from typing import Any, Mapping, Optional, Sequence

SCHEMA_VERSION = "group-repair-quality-profile-v1"
TRACE_SCHEMA_VERSION = 1

FORBIDDEN_ONLINE_FIELDS = frozenset({"answer", "expected", "expected_answer", "target_code", "oracle_id",
                                     "native_answer", "native_margin", "margin", "logits", "logprobs",
                                     "top_logprobs", "correct", "matches_native"})
RUNTIME_OWNED_FIELDS = frozenset({"imp_indices", "kvlink", "recompute_positions", "kv_slots", "block_ranges",
                                  "global_positions"})
PROVENANCE_FIELDS = frozenset({"request_id", "task_id", "agent_id", "session_id"})


class Reason(str, Enum):
    ELIGIBLE = "ELIGIBLE"
    GROUP_ALREADY_PRESENT = "GROUP_ALREADY_PRESENT"
    PROFILE_VERSION_MISMATCH = "PROFILE_VERSION_MISMATCH"
    MODEL_MISMATCH = "MODEL_MISMATCH"
    TOKENIZER_MISMATCH = "TOKENIZER_MISMATCH"
    COMPATIBILITY_MISMATCH = "COMPATIBILITY_MISMATCH"
    TOKEN_UNIT_NOT_MODEL = "TOKEN_UNIT_NOT_MODEL"
    REORDERED = "REORDERED"
    UNSUPPORTED_BLOCK_COUNT = "UNSUPPORTED_BLOCK_COUNT"
    UNSUPPORTED_GROUP_SIZE = "UNSUPPORTED_GROUP_SIZE"
    OUT_OF_CONTEXT_RANGE = "OUT_OF_CONTEXT_RANGE"
    UNSUPPORTED_LAYOUT = "UNSUPPORTED_LAYOUT"
    WRONG_RECONSTRUCTION_POLICY = "WRONG_RECONSTRUCTION_POLICY"
    MEMBERS_NOT_RESIDENT = "MEMBERS_NOT_RESIDENT"
    PARTIAL_MEMBER_RESIDENCY = "PARTIAL_MEMBER_RESIDENCY"


class Route(str, Enum):
    PREFIX_ABSORB_RECONSTRUCT_AND_PROMOTE = "PREFIX_ABSORB_RECONSTRUCT_AND_PROMOTE"
    GROUP_CACHE_HIT = "GROUP_CACHE_HIT"
    FULL_GROUP_RECOMPILE = "FULL_GROUP_RECOMPILE"


@dataclass(frozen=True)
class ShapeBands:
    """Member-length shapes that were characterized: ``balanced`` (every
    member within ``balanced_max_ratio`` of every other), ``front_heavy`` /
    ``back_heavy`` (the largest member first / last, ``heavy_ratio_min..max``
    times the mean of the others, the others within ``others_max_ratio`` of
    each other).  Anything else is unclassified (None)."""

    balanced_max_ratio: float
    heavy_ratio_min: float
    heavy_ratio_max: float
    others_max_ratio: float

    def classify(self, lengths: Sequence[int]) -> Optional[str]:
        ls = [int(v) for v in lengths]
        if len(ls) < 2 or min(ls) <= 0:
            return None
        if max(ls) <= self.balanced_max_ratio * min(ls):
            return "balanced"
        h = ls.index(max(ls))
        rest = ls[:h] + ls[h + 1:]
        if max(rest) > self.others_max_ratio * min(rest):
            return None
        ratio = ls[h] * len(rest) / sum(rest)
        if not self.heavy_ratio_min <= ratio <= self.heavy_ratio_max:
            return None
        return {0: "front_heavy", len(ls) - 1: "back_heavy"}.get(h)


@dataclass(frozen=True)
class GroupRepairProfile:
    profile_id: str
    profile_version: str
    schema_version: str
    method: str
    supported_ordering: str
    context_token_buckets: tuple  # ((low, high), ...) in model tokens of the whole request
    semantic_block_count_min: int
    semantic_block_count_max: int
    execution_group_member_min: int
    execution_group_member_max: int
    reconstruction_policy: str
    member0_prefix_refresh_tokens: int
    later_member_refresh: str
    requires_all_members_resident: bool
    requires_group_absent_for_reconstruction: bool
    promotion: str
    fallback_policy: str
    supported_member_shapes: tuple
    member_shape_classifier: ShapeBands
    compatibility: Mapping[str, str]
    certification: Mapping[str, Any] = field(default_factory=dict)  # evidence pointer; never read to decide

    def __post_init__(self):
        names = set(asdict(self)) | set(self.compatibility)
        bad = names & (RUNTIME_OWNED_FIELDS | PROVENANCE_FIELDS | FORBIDDEN_ONLINE_FIELDS)
        if bad:
            raise ValueError(f"profile carries forbidden fields: {sorted(bad)}")
        rules = [
            (self.supported_ordering == "in_order_only", "v1 profiles are in-order only"),
            (self.later_member_refresh == "full", "later members must be refreshed in full"),
            (type(self.member0_prefix_refresh_tokens) is int and self.member0_prefix_refresh_tokens > 0,
             "member0_prefix_refresh_tokens must be a positive integer"),
            (self.fallback_policy == Route.FULL_GROUP_RECOMPILE.value, "the fallback must be FULL_GROUP_RECOMPILE"),
            (all(0 < lo <= hi for lo, hi in self.context_token_buckets), "invalid context bucket"),
            (2 <= self.execution_group_member_min <= self.execution_group_member_max,
             "a reconstructed group has at least two members"),
        ]
        for ok, msg in rules:
            if not ok:
                raise ValueError(msg)

    def contract(self) -> dict:
        d = asdict(self)
        d.pop("certification")
        d["context_token_buckets"] = [list(b) for b in self.context_token_buckets]
        d["supported_member_shapes"] = list(self.supported_member_shapes)
        d["compatibility"] = dict(sorted(self.compatibility.items()))
        return d

    @property
    def digest(self) -> str:
        blob = json.dumps(self.contract(), sort_keys=True, separators=(",", ":"))
        return "grqp-" + hashlib.sha256(blob.encode()).hexdigest()[:24]

    def to_dict(self) -> dict:
        return {**self.contract(), "certification": dict(self.certification), "contract_digest": self.digest}

    @classmethod
    def from_dict(cls, data: Mapping[str, Any]) -> "GroupRepairProfile":
        d = dict(data)
        declared = d.pop("contract_digest", None)
        if d.get("schema_version") != SCHEMA_VERSION:
            raise ValueError("unsupported group repair profile schema")
        ints = ("semantic_block_count_min", "semantic_block_count_max", "execution_group_member_min",
                "execution_group_member_max")
        p = cls(**{
            **{k: str(d[k]) for k in ("profile_id", "profile_version", "schema_version", "method",
                                      "supported_ordering", "reconstruction_policy", "later_member_refresh",
                                      "promotion", "fallback_policy")},
            **{k: int(d[k]) for k in ints},
            "context_token_buckets": tuple((int(a), int(b)) for a, b in d["context_token_buckets"]),
            "member0_prefix_refresh_tokens": d["member0_prefix_refresh_tokens"],
            "requires_all_members_resident": bool(d["requires_all_members_resident"]),
            "requires_group_absent_for_reconstruction": bool(d["requires_group_absent_for_reconstruction"]),
            "supported_member_shapes": tuple(d["supported_member_shapes"]),
            "member_shape_classifier": ShapeBands(**d["member_shape_classifier"]),
            "compatibility": {str(k): str(v) for k, v in d["compatibility"].items()},
            "certification": dict(d.get("certification") or {}),
        })
        if declared is not None and declared != p.digest:
            raise ValueError("profile contract digest does not match its contents")
        return p


def load_profile(path) -> GroupRepairProfile:
    return GroupRepairProfile.from_dict(json.loads(Path(path).read_text(encoding="utf-8")))


@dataclass(frozen=True)
class GroupRequest:
    """What the planner knows about an execution group before it runs.
    ``request_member_ids``: member order in the request; ``group_member_ids``:
    the grouping order.  Residency and presence are host bookkeeping (the
    runtime stays authoritative and fails closed)."""

    context_tokens: int
    token_unit: str
    semantic_block_count: int
    request_member_ids: tuple
    group_member_ids: tuple
    member_token_counts: tuple
    members_resident: tuple
    group_present: bool
    reconstruction_policy: str
    member0_prefix_refresh_tokens: int
    later_member_refresh: str
    compatibility: Mapping[str, str]
    requested_profile_id: Optional[str] = None
    requested_profile_version: Optional[str] = None

    def __post_init__(self):
        n = len(self.group_member_ids)
        if len(self.member_token_counts) != n or len(self.members_resident) != n:
            raise ValueError("member counts and residency must match the group")


@dataclass(frozen=True)
class Decision:
    eligible: bool
    reason_code: str
    profile_id: str
    profile_version: str
    contract_digest: str
    features: Mapping[str, Any]
    details: str = ""


@dataclass(frozen=True)
class Routing:
    route: str
    reason_code: str
    promote: bool
    reconstruction_windows: Optional[tuple]
    decision: Decision

    def to_dict(self) -> dict:
        d = asdict(self)
        d["reconstruction_windows"] = list(self.reconstruction_windows) if self.reconstruction_windows else None
        return d


def features(req: GroupRequest, profile: GroupRepairProfile) -> dict:
    ls = [int(v) for v in req.member_token_counts]
    total = sum(ls)
    return {
        "context_tokens": int(req.context_tokens), "token_unit": req.token_unit,
        "semantic_block_count": int(req.semantic_block_count),
        "execution_group_member_count": len(req.group_member_ids),
        "ordering": "in_order" if tuple(req.request_member_ids) == tuple(req.group_member_ids) else "reordered",
        "member_token_counts": ls, "member0_tokens": ls[0] if ls else 0,
        "member0_ratio": round(ls[0] / total, 4) if total else None,
        "member_shape": profile.member_shape_classifier.classify(ls),
        "all_members_resident": bool(req.members_resident) and all(req.members_resident),
        "resident_member_count": sum(1 for v in req.members_resident if v),
        "group_present": bool(req.group_present), "reconstruction_policy": req.reconstruction_policy,
        "member0_prefix_refresh_tokens": req.member0_prefix_refresh_tokens,
        "later_member_refresh": req.later_member_refresh,
    }


def evaluate(req: GroupRequest, profile: GroupRepairProfile) -> Decision:
    """Structural, deterministic, answer-free; the first failing check in
    this order names the decision."""
    f = features(req, profile)
    comp, want = dict(req.compatibility), profile.compatibility
    mismatched = sorted(k for k, v in want.items() if comp.get(k) != v)
    n = f["execution_group_member_count"]
    checks = [
        (lambda: req.group_present, Reason.GROUP_ALREADY_PRESENT, ""),
        (lambda: req.requested_profile_id not in (None, profile.profile_id)
         or req.requested_profile_version not in (None, profile.profile_version), Reason.PROFILE_VERSION_MISMATCH, ""),
        (lambda: comp.get("model_id") != want.get("model_id"), Reason.MODEL_MISMATCH, ""),
        (lambda: comp.get("tokenizer_fingerprint") != want.get("tokenizer_fingerprint"), Reason.TOKENIZER_MISMATCH,
         ""),
        (lambda: bool(mismatched), Reason.COMPATIBILITY_MISMATCH, ",".join(mismatched)),
        (lambda: req.token_unit != "model", Reason.TOKEN_UNIT_NOT_MODEL, ""),
        (lambda: f["ordering"] != "in_order", Reason.REORDERED, ""),
        (lambda: not profile.semantic_block_count_min <= f["semantic_block_count"] <= profile.semantic_block_count_max,
         Reason.UNSUPPORTED_BLOCK_COUNT, ""),
        (lambda: not profile.execution_group_member_min <= n <= profile.execution_group_member_max,
         Reason.UNSUPPORTED_GROUP_SIZE, ""),
        (lambda: not any(lo <= f["context_tokens"] <= hi for lo, hi in profile.context_token_buckets),
         Reason.OUT_OF_CONTEXT_RANGE, ""),
        (lambda: f["member_shape"] not in profile.supported_member_shapes, Reason.UNSUPPORTED_LAYOUT, ""),
        (lambda: (req.reconstruction_policy, req.member0_prefix_refresh_tokens, req.later_member_refresh)
         != (profile.reconstruction_policy, profile.member0_prefix_refresh_tokens, profile.later_member_refresh),
         Reason.WRONG_RECONSTRUCTION_POLICY, ""),
        (lambda: f["resident_member_count"] == 0, Reason.MEMBERS_NOT_RESIDENT, ""),
        (lambda: f["resident_member_count"] < n, Reason.PARTIAL_MEMBER_RESIDENCY, ""),
    ]
    reason, details = Reason.ELIGIBLE, ""
    for failed, code, why in checks:
        if failed():
            reason, details = code, why
            break
    return Decision(reason is Reason.ELIGIBLE, reason.value, profile.profile_id, profile.profile_version,
                    profile.digest, f, details)


def windows(member_token_counts: Sequence[int], profile: GroupRepairProfile) -> tuple:
    """Policy-level budget per member: ``(min(K0, L0), L1, ..., L(N-1))``."""
    ls = [int(v) for v in member_token_counts]
    return (min(profile.member0_prefix_refresh_tokens, ls[0]),) + tuple(ls[1:])


def route(req: GroupRequest, profile: GroupRepairProfile, *, promotion_feature_enabled: bool) -> Routing:
    d = evaluate(req, profile)
    if d.reason_code == Reason.GROUP_ALREADY_PRESENT.value:
        return Routing(Route.GROUP_CACHE_HIT.value, d.reason_code, False, None, d)
    if d.eligible and promotion_feature_enabled:
        return Routing(Route.PREFIX_ABSORB_RECONSTRUCT_AND_PROMOTE.value, d.reason_code, True,
                       windows(req.member_token_counts, profile), d)
    return Routing(Route.FULL_GROUP_RECOMPILE.value, d.reason_code if not d.eligible else "PROMOTION_FEATURE_DISABLED",
                   False, None, d)


def link_fields(routing: Routing, group_key: str) -> dict:
    """Link-request fields for a reconstruct-and-promote route (empty for the
    other routes: a cache hit links ``group_key``, a recompile compiles the
    group as one block)."""
    if routing.route != Route.PREFIX_ABSORB_RECONSTRUCT_AND_PROMOTE.value:
        return {}
    return {"recompute_tokens_per_block": list(routing.reconstruction_windows),
            "promote_reconstructed_group": True, "execution_group_key": str(group_key)}


def trace_rows(routing: Routing, **context) -> list:
    bad = set(context) & FORBIDDEN_ONLINE_FIELDS
    if bad:
        raise ValueError(f"trace context carries forbidden fields: {sorted(bad)}")
    d, f = routing.decision, routing.decision.features
    base = {"schema_version": TRACE_SCHEMA_VERSION, "timestamp_unix_s": time.time(), "profile_id": d.profile_id,
            "profile_version": d.profile_version, "contract_digest": d.contract_digest, **context}
    checked = {**base, "event": "repair_profile_checked", "eligible": d.eligible, "reason": d.reason_code,
               "context_tokens": f["context_tokens"], "block_count": f["semantic_block_count"],
               "group_member_count": f["execution_group_member_count"], "member_shape": f["member_shape"],
               "ordering": f["ordering"], "resident_member_count": f["resident_member_count"],
               "group_present": f["group_present"]}
    outcome = {**base, "route": routing.route, "reason": routing.reason_code,
               "event": ("repair_profile_eligible"
                         if routing.route == Route.PREFIX_ABSORB_RECONSTRUCT_AND_PROMOTE.value
                         else "repair_profile_fallback")}
    return [checked, outcome]


def append_trace(path, rows: Sequence[Mapping[str, Any]]) -> None:
    p = Path(path)
    p.parent.mkdir(parents=True, exist_ok=True)
    with p.open("a", encoding="utf-8", newline="\n") as fh:
        for r in rows:
            fh.write(json.dumps(r, ensure_ascii=False, separators=(",", ":")) + "\n")
