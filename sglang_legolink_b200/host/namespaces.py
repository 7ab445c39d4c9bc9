"""Host-side cache namespaces over the one runtime block registry.

A namespace is bookkeeping on the host: where a block is looked up and
whether it may be kept.  The runtime still has one registry, one allocator
and one KV pool and owns every physical field (slots, ranges, positions,
``imp_indices``); nothing here reaches it.  Three notions stay apart:

* the *functional field* of a block (``host/events.py`` CONTEXT_FIELDS);
* its *namespace* -- a function of the field, whether the block can still
  change, and an explicit opt-in for task metadata (:class:`NamespacePolicy`);
* its *physical KV identity* -- whether one compiled KV may stand in for
  another block: exact token ids, source bytes, model, tokenizer and the
  policy versions the KV was compiled under (:func:`physical_kv_identity`).
  Field, namespace, task and session do not enter the KV, so they are not
  part of it.

Each persistent namespace is a *logical root* of :class:`LogicalRootIndex`:
its entries are names (cache keys) for compiled blocks, and a name may be an
alias of a block another name compiled.  Lookup is root first:

1. the block's own name in its own root (``global`` mode: in any root);
2. another name in the same root whose block has the same physical identity;
3. a same-identity block of another root, if the mode allows it: ``global``
   always (unless physical dedup is switched off), ``logical_namespace`` only
   for a (block namespace, entry namespace) pair the policy lists,
   ``hard_namespace`` never.

Outside ``global`` mode a block of a non-persistent namespace
(``mutable_current_turn``, ``no_cache``) is never compiled by any stage: the
resolver tells the layout gate it may not be linked and turns a Compile
decision for it into ``keep_mutable``.

Reference behaviour: ``noc_context_manager/cache_namespace.py:61-127``
(namespaces, profiles, modes), ``:166-211`` (pairs), ``:214-291`` (policy),
``:294-326`` (identity), ``:502-730`` (resolver), ``:733-823`` (summary);
``semantic_cache_index.py:171-354`` (roots and aliases).
"""

from __future__ import annotations

import hashlib
import json
import threading
import time
from dataclasses import dataclass, field, replace
from enum import Enum
from typing import Any, Iterable, Mapping, Optional, Sequence


class CacheNamespace(str, Enum):
    INSTRUCTION = "instruction"
    TOOL_SCHEMA = "tool_schema"
    CONVERSATION = "conversation"
    TOOL_OUTPUT = "tool_output"
    WORKSPACE = "workspace"
    MUTABLE_CURRENT_TURN = "mutable_current_turn"  # changes every turn: never kept
    NO_CACHE = "no_cache"  # never enters the persistent cache


PERSISTENT_NAMESPACES = frozenset({CacheNamespace.INSTRUCTION, CacheNamespace.TOOL_SCHEMA,
                                   CacheNamespace.CONVERSATION, CacheNamespace.TOOL_OUTPUT,
                                   CacheNamespace.WORKSPACE})
LOGICAL_ROOTS = tuple(sorted(n.value for n in PERSISTENT_NAMESPACES))


@dataclass(frozen=True)
class NamespaceProfile:
    """Retention metadata of a namespace, recorded with experiment rows for a
    later residency policy to read (nothing acts on it yet)."""
    namespace: CacheNamespace
    persistent: bool
    expected_reuse: str
    lifecycle: str


NAMESPACE_PROFILES: dict = {p.namespace: p for p in (
    NamespaceProfile(CacheNamespace.INSTRUCTION, True, "high", "stable"),
    NamespaceProfile(CacheNamespace.TOOL_SCHEMA, True, "high", "stable"),
    NamespaceProfile(CacheNamespace.CONVERSATION, True, "medium", "append_heavy_reusable_after_finalized"),
    NamespaceProfile(CacheNamespace.WORKSPACE, True, "medium", "task_or_cross_task_evidence"),
    NamespaceProfile(CacheNamespace.TOOL_OUTPUT, True, "to_be_measured", "often_request_specific"),
    NamespaceProfile(CacheNamespace.MUTABLE_CURRENT_TURN, False, "none", "current_turn_only"),
    NamespaceProfile(CacheNamespace.NO_CACHE, False, "none", "never_persisted"),
)}

NAMESPACE_NOT_PERSISTENT = "namespace is not persistent"
PHYSICAL_ENTRY_METADATA_KEY = "physical_entry"
ALIAS_SAME_ROOT = "same_root"
ALIAS_CROSS_ROOT = "cross_root"


class NamespaceMode(str, Enum):
    GLOBAL = "global"                       # one registry, no namespace restriction
    HARD = "hard_namespace"                 # a block is served only through its own namespace
    LOGICAL = "logical_namespace"           # own root first, then policy-listed cross-root aliases

    @classmethod
    def parse(cls, value) -> "NamespaceMode":
        if value is None:
            return cls.GLOBAL
        if isinstance(value, cls):
            return value
        text = str(value).strip().lower()
        for m in cls:
            if m.value == text:
                return m
        raise ValueError(f"unknown semantic_cache_namespace_mode {value!r}; expected one of "
                         + ", ".join(m.value for m in cls))


# ------------------------------------------------------ cross-namespace pairs
CROSS_NAMESPACE_PAIR_POLICY_VERSION = "cross-namespace-pairs-q1-v1"
# The same bytes can reach the context through two channels only here: a file
# read by a tool (tool_output) and the same file shown as workspace evidence.
VETTED_CROSS_NAMESPACE_PAIRS = frozenset({("workspace", "tool_output"), ("tool_output", "workspace")})


def _pair_items(item) -> list:
    if not isinstance(item, str):
        a, b = item
        return [(a, b)]
    text = item.strip()
    for arrow, both in (("<->", True), ("->", False)):
        if arrow in text:
            a, b = (p.strip() for p in text.split(arrow, 1))
            return [(a, b), (b, a)] if both else [(a, b)]
    raise ValueError(f"cross-namespace pair {item!r} must look like 'a<->b' or 'a->b'")


def parse_cross_namespace_pairs(spec: Optional[Iterable[Any]], *, require_vetted: bool = False) -> tuple:
    """Ordered (block namespace, entry namespace) pairs from config: ``"a<->b"``
    (both directions), ``"a->b"`` (a block of ``a`` may be served by an entry
    of ``b``) or a 2-sequence.  Both namespaces must be persistent and differ;
    with ``require_vetted`` anything outside the vetted set is refused, so a
    configuration typo cannot widen reuse."""
    out: list = []
    for item in spec or ():
        for a, b in _pair_items(item):
            pair = (CacheNamespace(a), CacheNamespace(b))
            if pair[0] is pair[1]:
                raise ValueError(f"cross-namespace pair {item!r} names one namespace twice")
            bad = [n.value for n in pair if n not in PERSISTENT_NAMESPACES]
            if bad:
                raise ValueError(f"cross-namespace pair {pair[0].value}->{pair[1].value} names {bad[0]!r}, which "
                                 "is not persistent; a non-persistent namespace never aliases")
            if require_vetted and (pair[0].value, pair[1].value) not in VETTED_CROSS_NAMESPACE_PAIRS:
                raise ValueError(f"cross-namespace pair {pair[0].value}->{pair[1].value} is not vetted; vetted: "
                                 + ", ".join(sorted(f"{x}->{y}" for x, y in VETTED_CROSS_NAMESPACE_PAIRS)))
            if pair not in out:
                out.append(pair)
    return tuple(out)


class NamespacePolicy:
    """field -> namespace, persistence, and the cross-namespace pairs (empty
    by default: no cross-namespace fallback)."""

    version = "cache-namespace-policy-v1"
    FIXED = {
        "user_prompt": CacheNamespace.MUTABLE_CURRENT_TURN,
        "task_instruction": CacheNamespace.INSTRUCTION,
        "tool_definitions": CacheNamespace.TOOL_SCHEMA,
        "tool_history_output": CacheNamespace.TOOL_OUTPUT,
        "workspace_evidence": CacheNamespace.WORKSPACE,
    }

    def __init__(self, *, cross_namespace_pairs: Iterable = (), require_vetted_pairs: bool = False):
        self.cross_namespace_pairs = frozenset(parse_cross_namespace_pairs(cross_namespace_pairs,
                                                                           require_vetted=require_vetted_pairs))

    def namespace_for(self, context_field: str, *, finalized: bool = True,
                      explicitly_cacheable: bool = False) -> CacheNamespace:
        """``finalized``: the block can no longer change.  ``explicitly_cacheable``:
        task metadata declared model-visible, stable and reusable."""
        if context_field == "conversation_history":
            return CacheNamespace.CONVERSATION if finalized else CacheNamespace.MUTABLE_CURRENT_TURN
        if context_field == "task_metadata":
            return CacheNamespace.INSTRUCTION if (finalized and explicitly_cacheable) else CacheNamespace.NO_CACHE
        ns = self.FIXED.get(context_field)
        if ns is None:
            raise ValueError(f"unknown functional field {context_field!r}")
        return ns

    def namespace_of(self, sc) -> CacheNamespace:
        md = sc.metadata or {}
        opt_in = all(md.get(k) is True for k in ("model_visible", "stable", "reusable"))
        return self.namespace_for(sc.context_field, finalized=not sc.is_mutable, explicitly_cacheable=opt_in)

    @staticmethod
    def profile(ns) -> NamespaceProfile:
        return NAMESPACE_PROFILES[CacheNamespace(ns)]

    @staticmethod
    def is_persistent(ns) -> bool:
        return CacheNamespace(ns) in PERSISTENT_NAMESPACES

    def permits_fallback(self, block_ns, entry_ns) -> bool:
        return (CacheNamespace(block_ns), CacheNamespace(entry_ns)) in self.cross_namespace_pairs


# ------------------------------------------------------------- identity
PHYSICAL_KV_IDENTITY_VERSION = "physical-kv-identity-v1"


def physical_kv_identity(sc) -> Optional[str]:
    """Digest of what decides whether one compiled KV can serve another
    block, or None when the block has no recorded token ids (equal text is
    not equal tokens, so text alone never licenses sharing).  Runtime-side
    fingerprints (kv dtype, rope, backend, TP size, adapter) are checked by
    the runtime's own registry key and are not host knowledge."""
    if not sc.token_ids:
        return None
    md = sc.metadata or {}
    payload = {
        "version": PHYSICAL_KV_IDENTITY_VERSION,
        "token_ids": [int(t) for t in sc.token_ids],
        "content_hash": hashlib.sha256(sc.raw_text.encode("utf-8")).hexdigest(),
        "model_fingerprint": md.get("model_fingerprint"),
        "tokenizer_fingerprint": md.get("tokenizer_fingerprint"),
        "segmentation_policy_version": md.get("segmentation_policy_version"),
        "recompute_policy_version": md.get("recompute_policy_version"),
    }
    return hashlib.sha256(json.dumps(payload, sort_keys=True, separators=(",", ":"), default=str)
                          .encode("utf-8")).hexdigest()


# ------------------------------------------------------- logical roots
@dataclass(frozen=True)
class RootEntry:
    """One name in a logical root.  ``runtime_key`` is the cache key the
    runtime knows the physical block by; for an alias it is another name's."""
    root: str
    name: str
    runtime_key: str
    identity: Optional[str]
    semantic_identity: str
    context_field: str
    token_count: int
    compiled_at: Optional[float]
    alias_kind: Optional[str] = None

    @property
    def is_alias(self) -> bool:
        return self.alias_kind is not None


class LogicalRootIndex:
    """Names per persistent namespace over one set of physical blocks.

    * :meth:`register` -- a Compile made ``name`` the primary name of a block;
    * :meth:`record_alias` -- ``name`` is served by another name's block;
    * :meth:`drop_physical` -- the block is gone: its primary and every alias
      are removed (their next lookup misses);
    * :meth:`sweep` -- drops aliases whose target block no longer exists."""

    def __init__(self):
        self._entries: dict = {}  # (root, name) -> RootEntry
        self._lock = threading.RLock()
        self.aliases_recorded = 0

    def register(self, root: str, name: str, *, identity: Optional[str], semantic_identity: str = "",
                 context_field: str = "", token_count: int = 0, runtime_key: Optional[str] = None) -> RootEntry:
        e = RootEntry(str(root), str(name), str(runtime_key or name), identity, semantic_identity, context_field,
                      int(token_count), time.time())
        with self._lock:
            self._entries[(e.root, e.name)] = e
        return e

    def lookup(self, root: str, name: str, *, any_root: bool = False) -> Optional[RootEntry]:
        """The primary entry (a compiled block) named ``name`` in ``root``;
        ``any_root``: in whichever root holds it.  Aliases are not returned:
        a name served through another block is found again by identity."""
        with self._lock:
            e = self._entries.get((root, name))
            if e is not None and not e.is_alias:
                return e
            if not any_root:
                return None
            hits = [x for (r, n), x in self._entries.items() if n == name and not x.is_alias]
        return sorted(hits, key=lambda x: x.root)[0] if hits else None

    def lookup_alias(self, root: str, name: str) -> Optional[RootEntry]:
        with self._lock:
            e = self._entries.get((root, name))
        return e if e is not None and e.is_alias else None

    def find_by_identity(self, identity: Optional[str]) -> list:
        """Primary entries (compiled blocks) of this physical identity, in
        root order, oldest first within a root."""
        if identity is None:
            return []
        with self._lock:
            hits = [e for e in self._entries.values() if e.identity == identity and not e.is_alias]
        return sorted(hits, key=lambda e: (LOGICAL_ROOTS.index(e.root) if e.root in LOGICAL_ROOTS else 99,
                                           e.compiled_at or 0.0, e.name))

    def record_alias(self, *, root: str, name: str, target: RootEntry, context_field: str,
                     token_count: int) -> bool:
        kind = ALIAS_SAME_ROOT if target.root == root else ALIAS_CROSS_ROOT
        with self._lock:
            cur = self._entries.get((root, name))
            if cur is not None and (not cur.is_alias or cur.runtime_key == target.runtime_key):
                return False
            self._entries[(root, name)] = RootEntry(root, name, target.runtime_key, target.identity,
                                                    target.semantic_identity, context_field, int(token_count),
                                                    target.compiled_at, kind)
            self.aliases_recorded += 1
            return True

    def aliases_of(self, runtime_key: str) -> list:
        with self._lock:
            return [e for e in self._entries.values() if e.is_alias and e.runtime_key == runtime_key]

    def logical_refs(self, runtime_key: str) -> int:
        """Names (primary + aliases) that reference the block."""
        with self._lock:
            return sum(1 for e in self._entries.values() if e.runtime_key == runtime_key)

    def drop_physical(self, runtime_key: str) -> int:
        with self._lock:
            dead = [k for k, e in self._entries.items() if e.runtime_key == runtime_key]
            for k in dead:
                del self._entries[k]
            return len(dead)

    def sweep(self) -> int:
        with self._lock:
            live = {e.runtime_key for e in self._entries.values() if not e.is_alias}
            dead = [k for k, e in self._entries.items() if e.is_alias and e.runtime_key not in live]
            for k in dead:
                del self._entries[k]
            return len(dead)

    def snapshot(self) -> dict:
        with self._lock:
            roots: dict = {r: {} for r in LOGICAL_ROOTS}
            for (r, n), e in sorted(self._entries.items()):
                roots.setdefault(r, {})[n] = {"runtime_key": e.runtime_key, "alias_kind": e.alias_kind,
                                             "context_field": e.context_field, "token_count": e.token_count}
            return {"roots": roots, "aliases_recorded": self.aliases_recorded}


def index_of(catalog) -> LogicalRootIndex:
    """The logical index that travels with a host catalog."""
    idx = getattr(catalog, "logical_index", None)
    if idx is None:
        idx = LogicalRootIndex()
        catalog.logical_index = idx
    return idx


# ------------------------------------------------------------- lookups
@dataclass(frozen=True)
class NamespaceLookup:
    sub_context_id: str
    context_field: str
    namespace: str
    mode: str
    token_count: int
    resident: bool
    same_namespace_hit: bool = False
    fallback_attempted: bool = False
    cross_namespace_hit: bool = False
    physical_cache_key: Optional[str] = None
    physical_semantic_identity: Optional[str] = None
    missed_reuse_tokens: int = 0
    alias_eligible: bool = True
    cross_namespace_opportunity: bool = False
    cross_namespace_pair: Optional[str] = None
    not_persistent: bool = False
    lookup_latency_s: float = 0.0
    entry_age_s: Optional[float] = None
    logical_root: Optional[str] = None
    logical_entry_key: Optional[str] = None
    physical_kv_identity: Optional[str] = None
    alias_kind: Optional[str] = None
    alias_recorded: bool = False
    physical_alias_count: int = 0
    physical_namespace: Optional[str] = None
    physical_context_field: Optional[str] = None

    @property
    def second_compile_avoided(self) -> bool:
        return self.alias_kind is not None

    def to_dict(self) -> dict:
        """Metric-row fields of this lookup."""
        logical_hit = self.same_namespace_hit or self.alias_recorded
        return {
            "sub_context_id": self.sub_context_id, "context_field": self.context_field,
            "namespace": self.namespace, "cache_namespace": self.namespace, "mode": self.mode,
            "token_count": self.token_count, "resident": self.resident,
            "namespace_lookup_hit": self.same_namespace_hit,
            "namespace_lookup_miss": not self.resident and not self.not_persistent,
            "logical_root": self.logical_root, "logical_entry_key": self.logical_entry_key,
            "logical_lookup_hit": logical_hit, "logical_lookup_miss": not logical_hit and not self.not_persistent,
            "cross_namespace_fallback_attempted": self.fallback_attempted,
            "cross_namespace_attempt": self.fallback_attempted, "cross_namespace_hit": self.cross_namespace_hit,
            "alias_kind": self.alias_kind, "alias_recorded": self.alias_recorded,
            "physical_alias_count": self.physical_alias_count, "physical_namespace": self.physical_namespace,
            "physical_context_field": self.physical_context_field,
            "physical_kv_identity": self.physical_kv_identity, "physical_kv_reused": self.resident,
            "second_compile_avoided": self.second_compile_avoided,
            "cross_namespace_second_compile_avoided": self.alias_kind == ALIAS_CROSS_ROOT,
            "physical_cache_key": self.physical_cache_key,
            "cross_namespace_missed_reuse_tokens": self.missed_reuse_tokens,
            "cross_namespace_opportunity": self.cross_namespace_opportunity,
            "cross_namespace_opportunity_tokens": self.token_count if self.cross_namespace_opportunity else 0,
            "cross_namespace_pair": self.cross_namespace_pair, "alias_eligible": self.alias_eligible,
            "not_persistent": self.not_persistent, "lookup_latency_s": self.lookup_latency_s,
            "entry_age_s": self.entry_age_s, "physical_block_residency_age_s": self.entry_age_s,
        }


class NamespaceResolver:
    """Root-first lookup per mode (module docstring).  It rewrites only how
    a block is *presented* to the rest of the host (an alias view carries the
    serving block's cache key, as a repeated occurrence of one block does)
    and never decides compile economics, layout or repair.

    ``hard_persistence_constraint`` (default on): outside ``global`` mode a
    non-persistent block may not be compiled by any later stage, the layout's
    prefix closure included.  ``global_physical_dedup`` (default on): in
    ``global`` mode an exact-identity block of any root may serve a block."""

    def __init__(self, mode=NamespaceMode.GLOBAL, policy: Optional[NamespacePolicy] = None, *,
                 hard_persistence_constraint: bool = True, global_physical_dedup: bool = True):
        self.mode = NamespaceMode.parse(mode)
        self.policy = policy or NamespacePolicy()
        self.hard_persistence_constraint = bool(hard_persistence_constraint)
        self.global_physical_dedup = bool(global_physical_dedup)

    @property
    def enforces_persistence(self) -> bool:
        return self.mode is not NamespaceMode.GLOBAL

    def describe(self) -> dict:
        return {
            "semantic_cache_namespace_mode": self.mode.value,
            "cache_namespace_policy_version": self.policy.version,
            "cross_namespace_pair_policy_version": CROSS_NAMESPACE_PAIR_POLICY_VERSION,
            "cross_namespace_pairs": sorted(f"{a.value}->{b.value}" for a, b in self.policy.cross_namespace_pairs),
            "global_physical_dedup": self.global_physical_dedup,
            "logical_roots": list(LOGICAL_ROOTS),
            "physical_cache_instances": 1,
        }

    def _crossing_allowed(self, ns: CacheNamespace, entry_root: str) -> bool:
        if self.mode is NamespaceMode.GLOBAL:
            return self.global_physical_dedup
        if self.mode is NamespaceMode.LOGICAL:
            return self.policy.permits_fallback(ns, entry_root)
        return False

    def _attempts_crossing(self) -> bool:
        return ((self.mode is NamespaceMode.GLOBAL and self.global_physical_dedup)
                or (self.mode is NamespaceMode.LOGICAL and bool(self.policy.cross_namespace_pairs)))

    def resolve(self, sc, catalog_or_index) -> NamespaceLookup:
        t0 = time.perf_counter()
        index = catalog_or_index if isinstance(catalog_or_index, LogicalRootIndex) else index_of(catalog_or_index)
        ns = self.policy.namespace_of(sc)
        persistent = self.policy.is_persistent(ns)
        ident = physical_kv_identity(sc)
        common = dict(sub_context_id=sc.sub_context_id, context_field=sc.context_field, namespace=ns.value,
                      mode=self.mode.value, token_count=int(sc.token_count),
                      logical_root=ns.value if persistent else None,
                      logical_entry_key=sc.cache_key if persistent else None, physical_kv_identity=ident)
        if self.enforces_persistence and not persistent:
            return NamespaceLookup(resident=False, not_persistent=True,
                                   lookup_latency_s=time.perf_counter() - t0, **common)
        own = index.lookup(ns.value, sc.cache_key, any_root=self.mode is NamespaceMode.GLOBAL)
        serving: Optional[RootEntry] = None
        kind: Optional[str] = None
        pair: Optional[str] = None
        attempted = opportunity = False
        eligible = True
        twins: list = []
        if own is None:
            twins = [e for e in index.find_by_identity(ident) if e.name != sc.cache_key]
            same_root = [e for e in twins if e.root == ns.value]
            if same_root:
                serving, kind = same_root[0], ALIAS_SAME_ROOT
            else:
                foreign = [e for e in twins if e.root != ns.value]
                eligible = not sc.is_mutable and not sc.invalidated and bool(sc.reuse_candidate)
                opportunity = bool(foreign) and eligible
                if self.mode is NamespaceMode.LOGICAL and not eligible:
                    foreign = []  # a block that is never linked gains nothing from an alias
                attempted = bool(foreign) and self._attempts_crossing()
                allowed = [e for e in foreign if self._crossing_allowed(ns, e.root)]
                if allowed:
                    serving, kind = allowed[0], ALIAS_CROSS_ROOT
                    pair = f"{ns.value}->{serving.root}"
        anchor = serving if serving is not None else own
        age = max(time.time() - anchor.compiled_at, 0.0) if anchor is not None and anchor.compiled_at else None
        key = serving.runtime_key if serving is not None else (sc.cache_key if own is not None else None)
        recorded = serving is not None and any(a.root == ns.value and a.name == sc.cache_key
                                               for a in index.aliases_of(serving.runtime_key))
        refs = 0
        if key is not None:
            refs = index.logical_refs(key) + (1 if serving is not None and not recorded else 0)
        return NamespaceLookup(
            resident=own is not None or serving is not None,
            same_namespace_hit=own is not None and own.root == ns.value,
            fallback_attempted=attempted, cross_namespace_hit=kind == ALIAS_CROSS_ROOT,
            physical_cache_key=key,
            physical_semantic_identity=serving.semantic_identity if serving is not None else None,
            missed_reuse_tokens=int(sc.token_count) if (twins and serving is None and own is None) else 0,
            lookup_latency_s=time.perf_counter() - t0, entry_age_s=age, alias_kind=kind,
            alias_recorded=recorded, physical_alias_count=refs,
            physical_namespace=serving.root if serving is not None else None,
            physical_context_field=serving.context_field if serving is not None else None,
            alias_eligible=eligible, cross_namespace_opportunity=opportunity, cross_namespace_pair=pair, **common)

    def apply(self, ordered: Sequence, catalog) -> tuple:
        """(views, lookups): a block served through another name is presented
        as that block (its cache key and semantic identity), remembering the
        owner so a recovery Compile registers the owner's block."""
        views, lookups = [], []
        for sc in ordered:
            r = self.resolve(sc, catalog)
            lookups.append(r)
            if r.alias_kind is None:
                views.append(sc)
                continue
            md = dict(sc.metadata or {})
            md[PHYSICAL_ENTRY_METADATA_KEY] = {"namespace": r.physical_namespace,
                                               "context_field": r.physical_context_field}
            views.append(replace(sc, cache_key=str(r.physical_cache_key),
                                 semantic_identity=str(r.physical_semantic_identity), metadata=md))
        return tuple(views), tuple(lookups)

    def record_aliases(self, lookups: Sequence[NamespaceLookup], catalog, *,
                       linked_block_ids: Optional[Iterable[str]] = None) -> int:
        """After a Link succeeded: record each name it served through another
        name's block (the planner itself has no side effects)."""
        index = index_of(catalog)
        only = None if linked_block_ids is None else set(linked_block_ids)
        n = 0
        for r in lookups:
            if r.alias_kind is None or r.logical_root is None:
                continue
            if only is not None and r.sub_context_id not in only:
                continue
            target = index.lookup(r.physical_namespace or r.namespace, str(r.physical_cache_key), any_root=True)
            if target is None:
                continue
            n += int(index.record_alias(root=r.logical_root, name=str(r.logical_entry_key), target=target,
                                        context_field=r.context_field, token_count=r.token_count))
        return n

    def register_compiled(self, views: Sequence, lookups: Sequence[NamespaceLookup], catalog,
                          compiled_cache_keys: Iterable[str]) -> int:
        """After Compiles: each newly compiled block becomes the primary name
        in the root of the block it was compiled for (an alias view's owner)."""
        index = index_of(catalog)
        keys = set(compiled_cache_keys)
        n = 0
        for v, r in zip(views, lookups):
            if v.cache_key not in keys:
                continue
            owner = (v.metadata or {}).get(PHYSICAL_ENTRY_METADATA_KEY) or {}
            root = owner.get("namespace") or r.logical_root or r.namespace
            index.register(root, v.cache_key, identity=r.physical_kv_identity, semantic_identity=v.semantic_identity,
                           context_field=owner.get("context_field") or v.context_field, token_count=v.token_count)
            n += 1
        return n

    def layout_permissions(self, lookups: Sequence[NamespaceLookup]) -> Optional[tuple]:
        """Per block: may the layout gate link (compile) it?  None: no
        restriction.  A non-persistent block is told it may not, so the
        prefix closure demotes later blocks instead of promoting it."""
        if not (self.enforces_persistence and self.hard_persistence_constraint):
            return None
        return tuple(not r.not_persistent for r in lookups)

    def enforce_persistence(self, lookups: Sequence[NamespaceLookup], decisions: Sequence) -> tuple:
        """A Compile decision of a non-persistent block becomes keep_mutable
        with reason :data:`NAMESPACE_NOT_PERSISTENT` (no-op in global mode)."""
        if not self.enforces_persistence:
            return tuple(decisions)
        from .planner import CompileAction

        out = []
        for r, d in zip(lookups, decisions):
            if r.not_persistent and d.action is CompileAction.COMPILE:
                d = replace(d, action=CompileAction.KEEP_MUTABLE, reason=NAMESPACE_NOT_PERSISTENT, token_count=0)
            out.append(d)
        return tuple(out)


# ------------------------------------------------------------- summary
_SUMMARY_COUNTERS = (
    "namespace_lookup_hit", "namespace_lookup_miss", "cross_namespace_fallback_attempted", "cross_namespace_hit",
    "cross_namespace_missed_reuse_tokens", "cross_namespace_opportunity", "cross_namespace_opportunity_tokens",
    "reused_token_count", "compiled_token_count", "repair_token_count", "logical_lookup_hit", "logical_lookup_miss",
    "cross_namespace_attempt", "physical_kv_reused", "physical_kv_dedup_count",
    "cross_namespace_second_compile_avoided", "alias_count", "residency_recovered_blocks",
    "residency_recovered_token_count",
)


def summarize_namespace_request(lookups: Sequence[NamespaceLookup], *, linked_block_ids: Iterable[str],
                                link_cache_key_by_block: Mapping[str, str],
                                repair_tokens_by_cache_key: Optional[Mapping[str, int]] = None,
                                recovered_cache_keys: Optional[Iterable[str]] = None) -> dict:
    """Per-namespace and total counters of one request.  A linked block that
    was resident at planning counts as reused, otherwise as compiled; a key
    the runtime reported gone and the host compiled again counts as compiled
    (never reused) and is named in ``residency_recovered_*``."""
    linked = set(linked_block_ids)
    recovered = {str(k) for k in (recovered_cache_keys or ())}
    repair = dict(repair_tokens_by_cache_key or {})
    per: dict = {}
    for r in lookups:
        row = per.setdefault(r.namespace, {"blocks": 0, "functional_fields": [], **dict.fromkeys(_SUMMARY_COUNTERS, 0)})
        d = r.to_dict()
        row["blocks"] += 1
        if r.context_field not in row["functional_fields"]:
            row["functional_fields"].append(r.context_field)
        for k in ("namespace_lookup_miss", "cross_namespace_fallback_attempted", "cross_namespace_hit",
                  "cross_namespace_opportunity", "logical_lookup_miss", "cross_namespace_attempt"):
            row[k] += int(bool(d[k]))
        row["namespace_lookup_hit"] += int(r.resident)
        row["logical_lookup_hit"] += int(r.resident)
        row["cross_namespace_missed_reuse_tokens"] += r.missed_reuse_tokens
        row["cross_namespace_opportunity_tokens"] += d["cross_namespace_opportunity_tokens"]
        if r.sub_context_id not in linked:
            continue
        key = str(link_cache_key_by_block.get(r.sub_context_id))
        rep = min(int(repair.get(key, 0)), r.token_count)
        if key in recovered:
            row["residency_recovered_blocks"] += 1
            row["residency_recovered_token_count"] += r.token_count
            row["compiled_token_count"] += r.token_count
            row["repair_token_count"] += rep
        elif r.resident:
            row["physical_kv_reused"] += 1
            row["physical_kv_dedup_count"] += int(r.second_compile_avoided)
            row["cross_namespace_second_compile_avoided"] += int(r.alias_kind == ALIAS_CROSS_ROOT)
            row["alias_count"] += int(r.alias_kind is not None)
            row["reused_token_count"] += r.token_count
            row["repair_token_count"] += rep
        else:
            row["compiled_token_count"] += r.token_count
    totals = {k: sum(row[k] for row in per.values()) for k in _SUMMARY_COUNTERS}
    totals["namespace_lookup_latency_s"] = sum(r.lookup_latency_s for r in lookups)
    ages = [r.entry_age_s for r in lookups if r.entry_age_s is not None]
    totals["physical_block_residency_age_s_max"] = max(ages) if ages else None
    return {"by_namespace": per, "totals": totals, "blocks": len(lookups)}
