"""Token accounting units and physical-token equivalence audits.

Token counts are tagged with their unit: ``model`` counts come from the
serving model's tokenizer (or the runtime's ``/v1/tokenize``), ``estimated``
counts from the regex estimator.  Estimated counts may size budgets but may
never be compared against a floor that is defined in model tokens (the
compile floor, repair windows): :func:`require_authoritative` refuses.

:func:`audit_layout` compares, token by token, the sequence a Link will make
the runtime assemble (chat prefix + linked blocks + fresh runs + mutable body
+ chat suffix) with the single-prompt tokenization the baseline request
would send, and reports digests, the first mismatch, the common prefix and
suffix and the length delta.  Exact equality is what exact-repair output
equivalence rests on.

Reference: ``noc_context_manager/token_accounting.py:44-187`` and
``token_equivalence.py:53-246``.
"""

from __future__ import annotations

import hashlib
import json
from dataclasses import asdict, dataclass
from enum import Enum
from typing import Optional, Sequence


class TokenUnit(str, Enum):
    MODEL = "model"
    ESTIMATED = "estimated"


@dataclass(frozen=True)
class TokenCount:
    count: int
    unit: TokenUnit
    tokenizer_fingerprint: str = ""

    def comparable_to(self, other: "TokenCount") -> bool:
        return self.unit == other.unit and (self.unit == TokenUnit.ESTIMATED or
                                            self.tokenizer_fingerprint == other.tokenizer_fingerprint)


class TokenAccountingError(ValueError):
    pass


def count_tokens(text: str, tokenizer) -> TokenCount:
    unit = TokenUnit(getattr(tokenizer, "token_unit", "estimated"))
    n = tokenizer.count(text) if hasattr(tokenizer, "count") else len(tokenizer.tokenize(text))
    return TokenCount(int(n), unit, str(getattr(tokenizer, "fingerprint", "")))


def require_authoritative(tokenizer, purpose: str) -> None:
    if getattr(tokenizer, "token_unit", "estimated") != TokenUnit.MODEL.value:
        raise TokenAccountingError(f"{purpose} is defined in model tokens; an estimating tokenizer "
                                   f"({type(tokenizer).__name__}) cannot decide it")


def at_least(count: TokenCount, floor: int, purpose: str) -> bool:
    """``count >= floor`` for a floor defined in model tokens."""
    if count.unit != TokenUnit.MODEL:
        raise TokenAccountingError(f"{purpose}: an estimated count is not comparable with a model-token floor")
    return count.count >= floor


@dataclass(frozen=True)
class SequenceDigest:
    token_count: int
    sha256: str

    @classmethod
    def of(cls, ids: Sequence) -> "SequenceDigest":
        blob = json.dumps([int(t) for t in ids], separators=(",", ":"))
        return cls(len(ids), hashlib.sha256(blob.encode()).hexdigest())


def first_mismatch(a: Sequence, b: Sequence) -> Optional[int]:
    for i, (x, y) in enumerate(zip(a, b)):
        if x != y:
            return i
    return None if len(a) == len(b) else min(len(a), len(b))


def common_suffix(a: Sequence, b: Sequence, prefix: int) -> int:
    n = 0
    limit = min(len(a), len(b)) - prefix
    while n < limit and a[len(a) - 1 - n] == b[len(b) - 1 - n]:
        n += 1
    return n


@dataclass(frozen=True)
class EquivalenceAudit:
    request_id: str
    tokenizer_fingerprint: str
    baseline: SequenceDigest
    assembled: SequenceDigest
    link_input: SequenceDigest
    block_digests: tuple
    token_ids_match: bool
    first_mismatch_index: Optional[int]
    common_prefix_tokens: int
    common_suffix_tokens: int
    token_delta: int
    framing_path: str
    layout_version: str

    @property
    def status(self) -> str:
        return "exact" if self.token_ids_match else "mismatch"

    def to_dict(self) -> dict:
        d = asdict(self)
        d["status"] = self.status
        return d


def audit_sequences(request_id: str, tokenizer_fingerprint: str, baseline_ids: Sequence, assembled_ids: Sequence,
                    link_input_ids: Sequence = (), block_ids: Sequence[Sequence] = (), framing_path: str = "",
                    layout_version: str = "") -> EquivalenceAudit:
    base, asm = tuple(baseline_ids), tuple(assembled_ids)
    mm = first_mismatch(base, asm)
    prefix = len(base) if mm is None else mm
    return EquivalenceAudit(
        request_id, tokenizer_fingerprint, SequenceDigest.of(base), SequenceDigest.of(asm),
        SequenceDigest.of(tuple(link_input_ids)), tuple(SequenceDigest.of(tuple(b)) for b in block_ids),
        base == asm, mm, prefix, common_suffix(base, asm, prefix), len(asm) - len(base), framing_path, layout_version)


def audit_layout(layout, request_id: str = "") -> EquivalenceAudit:
    """Audit a :class:`~.framing.ChatTokenLayout`."""
    return audit_sequences(request_id, layout.tokenizer_fingerprint, layout.baseline_token_ids,
                           layout.assembled_token_ids, layout.link_input_token_ids,
                           [s.token_ids for s in layout.link_segments], layout.framing_path, layout.version)
