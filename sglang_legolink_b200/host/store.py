"""Semantic sub-contexts: identity, cache keys and a transactional store.

* ``semantic_block_id`` -- provenance (task, field, source spans).
* ``semantic_identity`` -- *what* the KV is of: field + token ids (or text when
  no ids were captured), no task / agent / revision, so byte-identical blocks
  from different agents share one identity.
* ``semantic_cache_key`` -- identity qualified by model / tokenizer /
  segmentation / recompute-policy fingerprints: what makes a compiled block
  *usable*, not merely equal.

Formulas follow reference ``noc_context_manager/subcontext_store.py:52-141``
(the keys are a wire-visible identity, so they are kept the same); the store
is a SQLite table replaced per source revision inside one transaction.
"""

from __future__ import annotations

import hashlib
import json
import sqlite3
import threading
from dataclasses import asdict, dataclass, field, replace
from typing import Any, Iterable, Optional, Sequence

from .events import SourceSpan

SEMANTIC_IDENTITY_VERSION = "semantic-identity-v2"
DEFAULT_SEGMENTATION_POLICY_VERSION = "field-first-v1"
DEFAULT_RECOMPUTE_POLICY_VERSION = "legolink-radix-v1"
STABLE_FIELDS = frozenset({"task_instruction", "tool_definitions", "workspace_evidence", "task_metadata"})
HISTORY_FIELDS = frozenset({"conversation_history", "tool_history_output"})


def semantic_content_hash(text: str) -> str:
    return hashlib.sha256(text.encode("utf-8")).hexdigest()


def semantic_block_id(*, task_id: str, context_field: str, source_spans: Sequence[SourceSpan]) -> str:
    enc = json.dumps({"task_id": task_id, "context_field": context_field,
                      "source_spans": [s.to_dict() for s in source_spans]}, sort_keys=True, separators=(",", ":"))
    return "sc-" + hashlib.sha256(enc.encode()).hexdigest()[:24]


def semantic_identity(*, context_field: str, raw_text: str, token_ids: Sequence[Any] = ()) -> str:
    if token_ids:
        basis, payload = "tok", json.dumps(list(token_ids), separators=(",", ":"), default=str)
    else:
        basis, payload = "txt", raw_text
    enc = json.dumps({"identity_version": SEMANTIC_IDENTITY_VERSION, "basis": basis, "context_field": context_field,
                      "payload": payload}, sort_keys=True, separators=(",", ":"))
    return f"si-{basis}-" + hashlib.sha256(enc.encode()).hexdigest()[:32]


def semantic_cache_key(*, semantic_identity: str, context_field: str, model_fingerprint: str,
                       tokenizer_fingerprint: str, segmentation_policy_version: str,
                       recompute_policy_version: str) -> str:
    v = {"identity_version": SEMANTIC_IDENTITY_VERSION, "semantic_identity": semantic_identity,
         "context_field": context_field, "model_fingerprint": model_fingerprint,
         "tokenizer_fingerprint": tokenizer_fingerprint, "segmentation_policy_version": segmentation_policy_version,
         "recompute_policy_version": recompute_policy_version}
    return hashlib.sha256(json.dumps(v, sort_keys=True, separators=(",", ":")).encode()).hexdigest()


@dataclass(frozen=True)
class SubContext:
    sub_context_id: str
    task_id: str
    context_field: str
    source_id: str
    source_spans: tuple
    raw_text: str
    token_count: int
    token_unit: str
    semantic_identity: str
    cache_key: str
    sequence_number: int
    source_revision: int
    is_mutable: bool = False
    reuse_candidate: bool = True
    invalidated: bool = False
    token_ids: tuple = ()
    metadata: dict = field(default_factory=dict)

    def to_dict(self) -> dict:
        d = asdict(self)
        d["source_spans"] = [s.to_dict() if isinstance(s, SourceSpan) else s for s in self.source_spans]
        return d

    @classmethod
    def from_dict(cls, d: dict) -> "SubContext":
        """A stored row's token unit is not taken on its word: the count is
        a model-token count only if the row says so AND names the tokenizer
        that produced it, and that tokenizer is not an estimator.  A row
        without that provenance (older rows have no unit) reads as an
        estimate, which the compile policies refuse to compare with their
        model-token floors (reference token_accounting.py:44-187)."""
        from .tokenizer import RegexTokenizer

        d = dict(d)
        d["source_spans"] = tuple(SourceSpan(**s) for s in d["source_spans"])
        d["token_ids"] = tuple(d.get("token_ids") or ())
        fp = (d.get("metadata") or {}).get("tokenizer_fingerprint")
        model = d.get("token_unit") == "model" and bool(fp) and fp != RegexTokenizer.fingerprint
        d["token_unit"] = "model" if model else "estimated"
        return cls(**d)

    @classmethod
    def create(cls, *, task_id: str, context_field: str, source_id: str, spans: Sequence[SourceSpan], raw_text: str,
               tokenizer, sequence_number: int, source_revision: int, model_fingerprint: str,
               segmentation_policy_version: str = DEFAULT_SEGMENTATION_POLICY_VERSION,
               recompute_policy_version: str = DEFAULT_RECOMPUTE_POLICY_VERSION, is_mutable: bool = False,
               capture_token_ids: bool = False, metadata: Optional[dict] = None) -> "SubContext":
        toks = tokenizer.tokenize(raw_text)
        ids = tuple(int(t) for t in toks) if capture_token_ids and toks and isinstance(toks[0], int) else ()
        ident = semantic_identity(context_field=context_field, raw_text=raw_text, token_ids=ids)
        key = semantic_cache_key(semantic_identity=ident, context_field=context_field,
                                 model_fingerprint=model_fingerprint, tokenizer_fingerprint=tokenizer.fingerprint,
                                 segmentation_policy_version=segmentation_policy_version,
                                 recompute_policy_version=recompute_policy_version)
        md = dict(metadata or {})
        # what the compiled KV depends on besides its tokens (physical KV identity)
        md.setdefault("model_fingerprint", model_fingerprint)
        md.setdefault("tokenizer_fingerprint", tokenizer.fingerprint)
        md.setdefault("segmentation_policy_version", segmentation_policy_version)
        md.setdefault("recompute_policy_version", recompute_policy_version)
        return cls(semantic_block_id(task_id=task_id, context_field=context_field, source_spans=spans), task_id,
                   context_field, source_id, tuple(spans), raw_text, len(toks),
                   getattr(tokenizer, "token_unit", "estimated"), ident, key, sequence_number, source_revision,
                   is_mutable, True, False, ids, md)


class SubContextStore:
    """SQLite-backed store.  :meth:`replace_source_revisions` swaps every
    sub-context of the given sources in one transaction, so a failed ingest
    leaves the previous revision intact."""

    def __init__(self, path: str = ":memory:"):
        self._db = sqlite3.connect(path, check_same_thread=False, isolation_level=None)
        self._lock = threading.Lock()
        self._db.execute("CREATE TABLE IF NOT EXISTS subctx (id TEXT PRIMARY KEY, task_id TEXT, source_id TEXT, "
                         "seq INTEGER, ord INTEGER, body TEXT)")
        self._db.execute("CREATE INDEX IF NOT EXISTS subctx_task ON subctx(task_id, source_id)")

    def replace_source_revisions(self, task_id: str, by_source: dict[str, list[SubContext]]) -> None:
        with self._lock:
            cur = self._db.cursor()
            cur.execute("BEGIN IMMEDIATE")
            try:
                for sid, values in by_source.items():
                    cur.execute("DELETE FROM subctx WHERE task_id=? AND source_id=?", (task_id, sid))
                    for i, v in enumerate(values):
                        cur.execute("INSERT OR REPLACE INTO subctx VALUES (?,?,?,?,?,?)",
                                    (v.sub_context_id, task_id, sid, v.sequence_number, i, json.dumps(v.to_dict())))
                cur.execute("COMMIT")
            except Exception:
                cur.execute("ROLLBACK")
                raise

    def all(self, task_id: str) -> list[SubContext]:
        with self._lock:
            rows = self._db.execute("SELECT body FROM subctx WHERE task_id=? ORDER BY seq, ord", (task_id,)).fetchall()
        return [SubContext.from_dict(json.loads(r[0])) for r in rows]

    def get(self, sub_context_id: str) -> Optional[SubContext]:
        with self._lock:
            r = self._db.execute("SELECT body FROM subctx WHERE id=?", (sub_context_id,)).fetchone()
        return SubContext.from_dict(json.loads(r[0])) if r else None

    def count(self) -> int:
        return int(self._db.execute("SELECT COUNT(*) FROM subctx").fetchone()[0])
