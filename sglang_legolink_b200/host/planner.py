"""Reuse planning: namespaces, catalog, compile policy, the three gates and
the planner (host stages 5-6).

Pipeline of :meth:`Planner.plan` (reference ``noc_context_manager/
scheduler.py:919-967``):

1. namespace resolution -- which cache identity each sub-context uses
   (global: content key; hard: key scoped to the task; logical: content key
   with per-namespace aliases, so one physical block serves many tasks);
2. provisional compile decisions (policy);
3. Gate 1, reuse eligibility -- only standalone-compiled canonical state;
4. Gate 2, link-layout feasibility -- the runtime executes
   ``[linked prefix][one mutable suffix]``: reusable blocks before the first
   compiled block are promoted to Compile so the prefix closes, compiled
   blocks after the suffix starts are demoted to fresh text;
5. effective decisions -> ``linked`` / ``compile_on_miss`` / ``mutable`` /
   ``omitted`` sets and per-block planning records;
6. Gate 3 (observe-only) reuse accounting and profitability verdict.
"""

from __future__ import annotations

import hashlib
import json
import os
import threading
from dataclasses import dataclass, field, replace
from enum import Enum
from typing import Iterable, Optional, Sequence

from .manager import AgentContextManifest
from .store import SubContext

LEGACY_COMPILE_POLICY_VERSION = "legacy-fixed-64-v1"
BELOW_COMPILE_FLOOR = "below the compile token floor"
NO_EXPECTED_REUSE = "no expected future reuse"


# ---------------------------------------------------------------- namespaces
# The namespace taxonomy, logical roots and the resolver live in
# ``host/namespaces.py``; the planner applies them first (stage 1 above).
from .namespaces import (CacheNamespace, LogicalRootIndex, NamespaceLookup, NamespaceMode,  # noqa: E402,F401
                         NamespacePolicy, NamespaceResolver, index_of, physical_kv_identity,
                         summarize_namespace_request)


# ------------------------------------------------------------------ catalog
class CacheCatalog:
    """Host *intent*: which keys the host believes compiled (not residency).
    A per-key lock is held across a Compile so two callers never compile the
    same key at once."""

    def __init__(self):
        self._entries: dict[str, dict] = {}
        self._locks: dict[str, threading.Lock] = {}
        self._guard = threading.Lock()
        self.logical_index = LogicalRootIndex()  # names per namespace root over the compiled blocks

    def lock(self, key: str) -> threading.Lock:
        with self._guard:
            return self._locks.setdefault(key, threading.Lock())

    def is_compiled(self, key: str) -> bool:
        e = self._entries.get(key)
        return bool(e) and not e.get("stale")

    def mark_compiled(self, key: str, **meta) -> None:
        self._entries[key] = {"compiled": True, "stale": False, **meta}

    def invalidate(self, key: str) -> None:
        if key in self._entries:
            self._entries[key]["stale"] = True
        self.logical_index.drop_physical(key)  # its primary name and every alias miss from now on

    def entries(self) -> dict:
        return dict(self._entries)


class PersistentCacheCatalog(CacheCatalog):
    """Append-only JSONL variant shared between processes; the file is read
    by whole lines only (a torn last line is ignored), and deleting it resets
    the catalog."""

    def __init__(self, path: str):
        super().__init__()
        self.path = path
        self._offset = 0
        self._refresh()

    def _refresh(self) -> None:
        if not os.path.exists(self.path):
            return
        with open(self.path, "rb") as f:
            f.seek(self._offset)
            data = f.read()
        end = data.rfind(b"\n")
        if end < 0:
            return
        for line in data[: end + 1].splitlines():
            try:
                rec = json.loads(line)
            except ValueError:
                continue
            if rec.get("op") == "compiled":
                super().mark_compiled(rec["key"], **rec.get("meta", {}))
            elif rec.get("op") == "invalidate":
                super().invalidate(rec["key"])
        self._offset += end + 1

    def _append(self, rec: dict) -> None:
        line = (json.dumps(rec, separators=(",", ":")) + "\n").encode()
        fd = os.open(self.path, os.O_RDWR | os.O_CREAT | os.O_APPEND, 0o644)
        try:
            # A torn last line (a writer died mid-record) would swallow this
            # record; terminate it first so only the torn record is lost.
            size = os.fstat(fd).st_size
            if size and os.pread(fd, 1, size - 1) != b"\n":
                line = b"\n" + line
            os.write(fd, line)
        finally:
            os.close(fd)

    def is_compiled(self, key: str) -> bool:
        self._refresh()
        return super().is_compiled(key)

    def mark_compiled(self, key: str, **meta) -> None:
        super().mark_compiled(key, **meta)
        self._append({"op": "compiled", "key": key, "meta": meta})

    def invalidate(self, key: str) -> None:
        super().invalidate(key)
        self._append({"op": "invalidate", "key": key})


# ----------------------------------------------------------- compile policy
class CompileAction(str, Enum):
    COMPILE = "compile"
    KEEP_MUTABLE = "keep_mutable"
    DO_NOT_INCLUDE = "do_not_include"
    SUMMARIZE_THEN_COMPILE = "summarize_then_compile"


# actions that place the block's state through a Link (Gate 1 input)
LINK_ACTIONS = frozenset({CompileAction.COMPILE, CompileAction.SUMMARIZE_THEN_COMPILE})
SUMMARIZE_EXEMPT_FIELDS = frozenset({"workspace_evidence", "tool_definitions"})  # verbatim by nature


@dataclass(frozen=True)
class CompileDecision:
    sub_context_id: str
    cache_key: str
    action: CompileAction
    reason: str
    token_count: int = 0
    policy: str = "legacy_fixed_64"
    # why: policy + version, and for an economic decision the profile id,
    # hardware, model, compatibility verdict and the full cost breakdown
    provenance: dict = field(default_factory=dict)
    cost: Optional[dict] = None

    def to_dict(self) -> dict:
        d = dict(self.__dict__)
        d["action"] = self.action.value
        return d


@dataclass(frozen=True)
class PolicyContext:
    expected_future_reuse: int = 1
    memory_pressure: float = 0.0
    cache_present: bool = False
    min_compile_model_tokens: int = 64
    summarize_threshold_tokens: int = 8192
    preceding_model_tokens: int = 0
    planned_repair_model_tokens: Optional[int] = None
    repair_window_source: str = "unspecified"
    # The compile floor is defined in model tokens: a block counted by an
    # estimating tokenizer cannot be compared with it unless the caller asks
    # for estimate-only planning (reference token_accounting.py:44-187).
    allow_estimated_tokens: bool = False


def _require_model_tokens(v: SubContext, ctx: PolicyContext, what: str) -> None:
    """Compile decisions compare token counts with quantities defined in
    model tokens; a count from an estimating tokenizer may take part only
    when the caller asked for estimate-only planning."""
    if getattr(v, "token_unit", "model") != "model" and not ctx.allow_estimated_tokens:
        from .audits import TokenAccountingError

        raise TokenAccountingError(
            f"sub-context {v.sub_context_id}: its {v.token_count} tokens are an estimate ({v.token_unit}); "
            f"{what} is in model tokens (count with the model's tokenizer, or plan with "
            "allow_estimated_tokens=True)")


class CompilePolicy:
    """Legacy fixed floor: compile an immutable reuse candidate iff it has at
    least ``min_compile_model_tokens`` tokens; a very large compressible block
    (``summarize_threshold_tokens``, not workspace evidence or tool schemas)
    is summarized first (reference ``compile_policy.py:234-350``)."""

    name = "legacy_fixed_64"
    version = LEGACY_COMPILE_POLICY_VERSION

    def decide(self, v: SubContext, ctx: PolicyContext = PolicyContext()) -> CompileDecision:
        D = self._maker(v)
        if v.invalidated:
            return D(CompileAction.DO_NOT_INCLUDE, "invalidated version")
        if v.is_mutable:
            return D(CompileAction.KEEP_MUTABLE, "content is mutable")
        if not v.reuse_candidate:
            return D(CompileAction.KEEP_MUTABLE, "not a reuse candidate")
        if ctx.cache_present:
            return D(CompileAction.COMPILE, "already compiled; reuse catalog entry", v.token_count)
        return self._decide(v, ctx, D)

    def _maker(self, v: SubContext, **extra):
        prov = {"compile_policy": self.name, "compile_policy_version": self.version, **extra.pop("provenance", {})}
        return lambda a, r, n=0, **kw: CompileDecision(v.sub_context_id, v.cache_key, a, r, n, self.name,
                                                       {**prov, **kw.pop("provenance", {})}, kw.get("cost"))

    def _decide(self, v, ctx, D):
        _require_model_tokens(v, ctx, f"the compile floor of {ctx.min_compile_model_tokens}")
        if v.token_count < ctx.min_compile_model_tokens:
            return D(CompileAction.KEEP_MUTABLE, BELOW_COMPILE_FLOOR)
        if ctx.expected_future_reuse < 1:
            return D(CompileAction.KEEP_MUTABLE, NO_EXPECTED_REUSE)
        if ctx.memory_pressure >= 0.9:
            return D(CompileAction.KEEP_MUTABLE, "high KV memory pressure")
        if v.token_count >= ctx.summarize_threshold_tokens and v.context_field not in SUMMARIZE_EXEMPT_FIELDS:
            return D(CompileAction.SUMMARIZE_THEN_COMPILE, "large compressible stable context")
        return D(CompileAction.COMPILE, "immutable reuse candidate above the floor",
                 v.token_count * ctx.expected_future_reuse)


class CompileAllImmutablePolicy(CompilePolicy):
    name = "compile_all_immutable"
    version = "compile-all-immutable-v1"

    def _decide(self, v, ctx, D):
        return D(CompileAction.COMPILE, "ablation: every immutable block", v.token_count)


class CostBenefitCompilePolicy(CompilePolicy):
    """Compile iff the expected reuse savings exceed the Compile cost, from a
    measured :class:`~.compile_cost.CompileCostProfile` of this deployment
    and a :class:`~.compile_cost.ReuseExpectation` (required: assuming one
    reuse is exactly the hidden guess this policy replaces).  The eligibility
    checks before the floor are the legacy policy's; the floor itself is
    replaced by the arithmetic.  Without a usable profile there is no
    decision -- unless the caller named ``fallback="legacy_fixed_64"``, which
    every decision it produces records.  Memory pressure >= 0.9 stays a hard
    stop (residency cost is unmeasured, see ``DisabledResidencyCost``).
    Reference: ``compile_policy.py:386-560``."""

    name = "cost_benefit"
    memory_pressure_stop = 0.9

    def __init__(self, *, reuse_expectation=None, profile=None, residency_cost_model=None, deployment=None,
                 strict_profile_compatibility: bool = True, fallback: Optional[str] = None):
        from . import compile_cost as cc

        if reuse_expectation is None:
            raise cc.CompileCostError("a cost-benefit policy needs a ReuseExpectation; there is no safe default")
        if fallback not in (None, "legacy_fixed_64"):
            raise cc.CompileCostError("the only supported fallback is legacy_fixed_64")
        self.version = cc.COMPILE_COST_POLICY_VERSION
        self.reuse = reuse_expectation
        self.profile = profile
        self.residency = residency_cost_model or cc.DisabledResidencyCost()
        self.deployment = deployment
        self.strict = strict_profile_compatibility
        self.fallback = fallback
        self._legacy = CompilePolicy()

    def _decide(self, v, ctx, D):
        from . import compile_cost as cc

        _require_model_tokens(v, ctx, "the measured compile-cost curve")
        if ctx.memory_pressure >= self.memory_pressure_stop:
            return D(CompileAction.KEEP_MUTABLE, "high KV memory pressure")
        try:
            if self.profile is None:
                raise cc.CompileCostUnavailable("no CompileCostProfile was supplied")
            compat = self.profile.check_compatibility(self.deployment, strict=self.strict)
            cand = cc.CompileCandidate(v.sub_context_id, v.cache_key, v.context_field, v.token_count,
                                       not v.is_mutable, v.reuse_candidate, v.invalidated,
                                       ctx.preceding_model_tokens, ctx.planned_repair_model_tokens,
                                       ctx.repair_window_source, ctx.cache_present)
            b = cc.evaluate_compile_economics(cand, profile=self.profile, reuse=self.reuse, residency=self.residency,
                                              planned_future_reuse=ctx.expected_future_reuse,
                                              memory_pressure=ctx.memory_pressure)
        except cc.CompileCostUnavailable as e:
            if self.fallback is None:
                raise
            d = self._legacy.decide(v, ctx)
            return replace(d, policy=self.name, provenance={**d.provenance, "compile_policy": self.name,
                                                            "fallback_policy": self.fallback,
                                                            "fallback_reason": str(e)})
        prov = {"profile_id": self.profile.profile_id, "profile_hardware": self.profile.provenance.hardware_id,
                "profile_model": self.profile.provenance.model_id, "profile_compatibility": compat,
                "reuse_expectation": self.reuse.name}
        if not b.is_profitable:
            return D(CompileAction.KEEP_MUTABLE, "expected reuse savings do not exceed the compile cost",
                     provenance=prov, cost=b.to_dict())
        return D(CompileAction.COMPILE, "expected reuse savings exceed the compile cost", v.token_count,
                 provenance=prov, cost=b.to_dict())


def build_compile_policy(mode: str = "legacy_fixed_64", **kw) -> CompilePolicy:
    return {"legacy_fixed_64": CompilePolicy, "compile_all_immutable": CompileAllImmutablePolicy,
            "cost_benefit": CostBenefitCompilePolicy}[mode](**kw)


class ContextSummarizer:
    """Turns a SUMMARIZE_THEN_COMPILE block into a derived summary block
    (same field and spans, ``derived_from`` provenance, its own identity and
    cache key) through a caller's ``summarize(text, target_tokens)``.  The
    original is kept when there is no summarizer, when the text must stay
    verbatim (code fences, JSON, tracebacks, shell prompts, error lines), or
    when the summary does not reduce the token count.  Counting uses the
    same tokenizer as the original.  Reference: ``pruning.py:22-80``."""

    VERBATIM = __import__("re").compile(r"```|\{\s*[\"']|Traceback|(?:^|\n)\s*[$>]\s|(?:error|exception):",
                                        __import__("re").IGNORECASE)

    def __init__(self, summarize=None, *, tokenizer=None, target_ratio: float = 0.25):
        self.summarize, self.tokenizer, self.target_ratio = summarize, tokenizer, target_ratio

    def apply(self, v: SubContext) -> tuple[SubContext, str]:
        if self.summarize is None or self.tokenizer is None:
            return v, "summarizer unavailable"
        if self.VERBATIM.search(v.raw_text):
            return v, "verbatim content"
        target = max(1, int(v.token_count * self.target_ratio))
        try:
            text = str(self.summarize(v.raw_text, target) or "").strip()
        except Exception as e:  # noqa: BLE001 - a failed summary keeps the original
            return v, f"summarizer failed: {e}"[:200]
        n = self.tokenizer.count(text) if hasattr(self.tokenizer, "count") else len(self.tokenizer.tokenize(text))
        if not text or n >= v.token_count:
            return v, "summary did not reduce the context"
        md = dict(v.metadata or {})
        derived = SubContext.create(task_id=v.task_id, context_field=v.context_field, source_id=v.source_id,
                                    spans=list(v.source_spans), raw_text=text, tokenizer=self.tokenizer,
                                    sequence_number=v.sequence_number, source_revision=v.source_revision,
                                    model_fingerprint=md.get("model_fingerprint", "runtime-local"),
                                    segmentation_policy_version=str(md.get("segmentation_policy_version",
                                                                           "field-first-v1")) + "+summary-v1",
                                    capture_token_ids=bool(v.token_ids),
                                    metadata={**md, "derived_from": [v.sub_context_id],
                                              "semantic_independence_reason":
                                                  "derived compression of a source-backed block"})
        return derived, "summarized"


# --------------------------------------------------------------------- gates
class ReuseEligibility:
    """Gate 1: only canonical, standalone-compiled state may be linked."""

    def __init__(self, allow_foreign: bool = False):
        self.allow_foreign = allow_foreign

    def gate(self, v: SubContext, decision: CompileDecision) -> tuple[bool, str]:
        if decision.action not in LINK_ACTIONS:
            return False, "not compiled"
        if v.metadata.get("foreign_state") and not self.allow_foreign:
            return False, "foreign state (experimental) is off"
        return True, "canonical standalone compile"


@dataclass(frozen=True)
class LayoutAdjustment:
    sub_context_id: str
    adjustment: str  # "none" | "promoted_for_prefix_closure" | "demoted_after_suffix"
    reason: str = ""


class LinkLayoutFeasibility:
    """Gate 2: force ``[linked prefix][mutable suffix]``."""

    def apply(self, ordered: Sequence[SubContext], link_ok: dict[str, bool],
              promotable: dict[str, bool]) -> tuple[dict[str, bool], list[LayoutAdjustment]]:
        eff = dict(link_ok)
        adj = []
        last_linked = max((i for i, v in enumerate(ordered) if link_ok.get(v.sub_context_id)), default=-1)
        # promote reusable (immutable) blocks that sit before a linked block
        for i, v in enumerate(ordered[: last_linked + 1]):
            if not eff.get(v.sub_context_id):
                if promotable.get(v.sub_context_id):
                    eff[v.sub_context_id] = True
                    adj.append(LayoutAdjustment(v.sub_context_id, "promoted_for_prefix_closure",
                                                "reusable block inside the linked prefix"))
                else:
                    break
        # everything after the first non-linked block is the mutable suffix
        in_suffix = False
        for v in ordered:
            if not eff.get(v.sub_context_id):
                in_suffix = True
            elif in_suffix:
                eff[v.sub_context_id] = False
                adj.append(LayoutAdjustment(v.sub_context_id, "demoted_after_suffix",
                                            "compiled block after the mutable suffix starts"))
        return eff, adj


@dataclass(frozen=True)
class ReuseAccounting:
    reused_tokens: int
    compiled_tokens: int
    recompute_tokens: int
    repair_tokens: int
    total_tokens: int
    verdict: str  # observe-only profitability

    def to_dict(self) -> dict:
        return dict(self.__dict__)


# ------------------------------------------------------------------ planner
@dataclass(frozen=True)
class BlockPlanningRecord:
    sub_context_id: str
    block_id: str
    cache_key: str
    token_count: int
    policy_action: str
    layout_adjustment: str
    effective_action: str
    planner_category: str  # linked | compile_on_miss | mutable | omitted
    reason: str = ""

    def to_dict(self) -> dict:
        return dict(self.__dict__)


@dataclass(frozen=True)
class ExecutionPlan:
    manifest: AgentContextManifest
    included_contexts: tuple
    linked_contexts: tuple
    compile_on_miss_contexts: tuple
    mutable_contexts: tuple
    omitted_contexts: tuple
    records: tuple
    accounting: ReuseAccounting
    text_separator: str = "\n\n"
    namespace_lookups: tuple = ()
    namespace_config: dict = field(default_factory=dict)

    @property
    def expected_cache_keys(self) -> tuple:
        return tuple(v.cache_key for v in self.linked_contexts)

    @property
    def baseline_selected_text(self) -> str:
        parts = [v.raw_text for v in self.included_contexts]
        if self.manifest.mutable_text:
            parts.append(self.manifest.mutable_text)
        return self.text_separator.join(parts)

    def to_dict(self) -> dict:
        return {"manifest": self.manifest.to_dict(), "linked": [v.sub_context_id for v in self.linked_contexts],
                "compile_on_miss": [v.sub_context_id for v in self.compile_on_miss_contexts],
                "mutable": [v.sub_context_id for v in self.mutable_contexts],
                "omitted": [v.sub_context_id for v in self.omitted_contexts],
                "block_planning": [r.to_dict() for r in self.records], "reuse_accounting": self.accounting.to_dict(),
                "namespace_lookups": [r.to_dict() for r in self.namespace_lookups],
                "namespace_config": dict(self.namespace_config)}

    def namespace_summary(self, recovered_cache_keys=(), repair_tokens_by_cache_key=None) -> dict:
        return summarize_namespace_request(
            self.namespace_lookups, linked_block_ids=[v.sub_context_id for v in self.linked_contexts],
            link_cache_key_by_block={v.sub_context_id: v.cache_key for v in self.linked_contexts},
            repair_tokens_by_cache_key=repair_tokens_by_cache_key, recovered_cache_keys=recovered_cache_keys)


class Planner:
    def __init__(self, policy: Optional[CompilePolicy] = None, catalog: Optional[CacheCatalog] = None,
                 resolver: Optional[NamespaceResolver] = None, eligibility: Optional[ReuseEligibility] = None,
                 feasibility: Optional[LinkLayoutFeasibility] = None, repair_window: int = 16,
                 separator: str = "\n\n", summarizer: Optional[ContextSummarizer] = None):
        self.summarizer = summarizer or ContextSummarizer()
        self.policy = policy or CompilePolicy()
        self.catalog = catalog or CacheCatalog()
        self.resolver = resolver or NamespaceResolver()
        self.eligibility = eligibility or ReuseEligibility()
        self.feasibility = feasibility or LinkLayoutFeasibility()
        self.repair_window = repair_window
        self.separator = separator

    def plan(self, manifest: AgentContextManifest, contexts: Iterable[SubContext], *,
             policy_context: PolicyContext = PolicyContext(), namespace: Optional[str] = None) -> ExecutionPlan:
        """``namespace`` is accepted for older callers and ignored: a block's
        namespace follows from its field (``host/namespaces.py``)."""
        by_id = {v.sub_context_id: v for v in contexts}
        selected = [by_id[i] for i in manifest.selected_sub_context_ids if i in by_id]
        ordered, lookups = self.resolver.apply(selected, self.catalog)
        ordered = list(ordered)
        provisional = []
        for v, r in zip(ordered, lookups):
            ctx = replace(policy_context, cache_present=r.resident or self.catalog.is_compiled(v.cache_key))
            provisional.append(self.policy.decide(v, ctx))
        decisions = dict(zip((v.sub_context_id for v in ordered),
                             self.resolver.enforce_persistence(lookups, provisional)))
        # SUMMARIZE_THEN_COMPILE: the derived summary block takes the place
        # of the original (same position, id kept so the manifest still names it)
        for i, v in enumerate(ordered):
            d = decisions[v.sub_context_id]
            if d.action is not CompileAction.SUMMARIZE_THEN_COMPILE:
                continue
            derived, why = self.summarizer.apply(v)
            if derived is not v:
                ordered[i] = replace(derived, sub_context_id=v.sub_context_id)
            decisions[v.sub_context_id] = replace(d, cache_key=ordered[i].cache_key,
                                                  token_count=ordered[i].token_count,
                                                  provenance={**d.provenance, "summary": why})
        perms = self.resolver.layout_permissions(lookups)
        may_link = {v.sub_context_id: (True if perms is None else perms[i]) for i, v in enumerate(ordered)}
        included = [v for v in ordered if decisions[v.sub_context_id].action != CompileAction.DO_NOT_INCLUDE]
        omitted = [v for v in ordered if decisions[v.sub_context_id].action == CompileAction.DO_NOT_INCLUDE]
        link_ok = {v.sub_context_id: self.eligibility.gate(v, decisions[v.sub_context_id])[0] for v in included}
        promotable = {v.sub_context_id: (not v.is_mutable and v.reuse_candidate and not v.invalidated
                                         and may_link[v.sub_context_id]) for v in included}
        eff, adj = self.feasibility.apply(included, link_ok, promotable)
        adj_of = {a.sub_context_id: a.adjustment for a in adj}
        linked = [v for v in included if eff.get(v.sub_context_id)]
        mutable = [v for v in included if not eff.get(v.sub_context_id)]
        com = [v for v in linked if not self.catalog.is_compiled(v.cache_key)]
        records = []
        for v in ordered:
            d = decisions[v.sub_context_id]
            if v in omitted:
                cat, ea = "omitted", "do_not_include"
            elif eff.get(v.sub_context_id):
                cat = "compile_on_miss" if v in com else "linked"
                ea = "link"
            else:
                cat, ea = "mutable", "recompute"
            records.append(BlockPlanningRecord(v.sub_context_id, v.semantic_identity, v.cache_key, v.token_count,
                                               d.action.value, adj_of.get(v.sub_context_id, "none"), ea, cat,
                                               d.reason))
        reused = sum(v.token_count for v in linked if v not in com)
        compiled = sum(v.token_count for v in com)
        recompute = sum(v.token_count for v in mutable)
        repair = sum(min(self.repair_window, v.token_count) for v in linked)
        total = sum(v.token_count for v in included)
        verdict = "observe_only:" + ("profitable" if reused > repair else "not_profitable")
        acc = ReuseAccounting(reused, compiled, recompute, repair, total, verdict)
        return ExecutionPlan(manifest, tuple(included), tuple(linked), tuple(com), tuple(mutable), tuple(omitted),
                             tuple(records), acc, self.separator, tuple(lookups), self.resolver.describe())

    def after_compile(self, plan: ExecutionPlan) -> int:
        """The blocks a plan's Compiles made resident become primary names in
        their roots."""
        keys = [v.cache_key for v in plan.linked_contexts if self.catalog.is_compiled(v.cache_key)]
        idx = index_of(self.catalog)
        fresh = [k for v, k in zip(plan.linked_contexts, keys)
                 if idx.lookup(self._root_of(plan, v), k) is None]
        by_id = {r.sub_context_id: r for r in plan.namespace_lookups}
        views = [v for v in plan.linked_contexts if v.sub_context_id in by_id]
        return self.resolver.register_compiled(views, [by_id[v.sub_context_id] for v in views], self.catalog, fresh)

    @staticmethod
    def _root_of(plan: ExecutionPlan, v) -> str:
        owner = (v.metadata or {}).get("physical_entry") or {}
        for r in plan.namespace_lookups:
            if r.sub_context_id == v.sub_context_id:
                return owner.get("namespace") or r.logical_root or r.namespace
        return ""

    def after_link(self, plan: ExecutionPlan) -> int:
        """A successful Link: record the names it served through other blocks."""
        return self.resolver.record_aliases(plan.namespace_lookups, self.catalog,
                                            linked_block_ids=[v.sub_context_id for v in plan.linked_contexts])
