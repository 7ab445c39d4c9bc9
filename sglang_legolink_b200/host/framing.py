"""Stitching, physical token framing, repair windows and the Link request
(host stages 7-8).

* :class:`Stitcher` -- one execution plan -> the baseline text and the
  LegoLink view of the *same* prompt.  Sub-contexts are joined with the
  separator ``"\\n\\n"`` at source boundaries and with nothing between
  segments of one source; a linked block's compiled text is its raw text plus
  the boundary that follows it (reference ``stitch.py:189-351``).
* :func:`build_layout` -- tokenizes the single chat-template prompt and
  splits it into chat prefix + block segments (``tokenize(view_i)``, a
  function of the block alone) + mutable body + chat suffix.  When a token
  crosses a block boundary (tokenizers do not compose) the blocks that no
  longer sit exactly where their compiled tokens say are demoted to fresh
  text (or, with ``interblock=True``, sent as fresh gaps between linked
  blocks).  The assembly always equals the authoritative prompt token for
  token (reference ``physical_framing.py:322-587``).
* Repair windows: uniform / block-length-capped / context-gain policies and a
  :class:`RepairDecision` record (``repair_window.py:209-454``).
* :class:`LinkRequest` / :func:`frame_link` -- the ``pic_link`` object and the
  chat payload; everything the runtime derives is absent by construction and
  :func:`~sglang_legolink_b200.contract.validate_pic_link_request` is run on
  the wire form before it leaves the host.
"""

from __future__ import annotations

import hashlib
import json
import math
from dataclasses import dataclass, field, replace
from typing import Any, Optional, Sequence

from ..contract import (PHYSICAL_TOKEN_LAYOUT_VERSION, REPAIR_DECISION_POLICY_VERSION, ContractError,
                        physical_token_ids_sha256, validate_pic_link_request)
from .planner import ExecutionPlan
from .store import SubContext


class PhysicalTokenLayoutError(ValueError):
    pass


# -------------------------------------------------------------------- stitch
def source_boundary(a: SubContext, b: Optional[SubContext], sep: str) -> str:
    """Separator between two consecutive sub-contexts: none inside one source."""
    if b is None:
        return ""
    return "" if a.source_id == b.source_id else sep


def compose_source_text(values: Sequence[SubContext], *, separator: str, trailing_text: str = "") -> str:
    parts = []
    for i, v in enumerate(values):
        parts.append(v.raw_text)
        nxt = values[i + 1] if i + 1 < len(values) else None
        parts.append(source_boundary(v, nxt, separator) if nxt is not None else "")
    text = "".join(parts)
    if trailing_text:
        text = text + separator + trailing_text if text else trailing_text
    return text


@dataclass(frozen=True)
class StitchedContext:
    selected_text: str
    mutable_text: str
    linked_views: tuple  # SubContext with raw_text = compiled text (block + following boundary)
    mutable_contexts: tuple
    separator: str
    generation_parameters: dict
    generation_parameters_sha256: str
    selected_content_sha256: str
    equivalence: dict

    @property
    def cache_keys(self) -> tuple:
        return tuple(v.cache_key for v in self.linked_views)

    @property
    def block_ids(self) -> tuple:
        return tuple(v.semantic_identity or v.sub_context_id for v in self.linked_views)


class Stitcher:
    def __init__(self, separator: str = "\n\n", tokenizer=None):
        self.separator = separator
        self.tokenizer = tokenizer

    def baseline_text(self, plan: ExecutionPlan) -> str:
        return compose_source_text(list(plan.included_contexts), separator=self.separator,
                                   trailing_text=plan.manifest.mutable_text)

    def stitch(self, plan: ExecutionPlan, generation_parameters: Optional[dict] = None) -> StitchedContext:
        if plan.text_separator != self.separator:
            raise ValueError("execution plan and stitcher separators differ")
        linked, mutable = list(plan.linked_contexts), list(plan.mutable_contexts)
        selected = self.baseline_text(plan)
        views = []
        for i, v in enumerate(linked):
            nxt = linked[i + 1] if i + 1 < len(linked) else (mutable[0] if mutable else None)
            if nxt is None:
                tail = self.separator if plan.manifest.mutable_text else ""
            else:
                tail = source_boundary(v, nxt, self.separator)
            views.append(replace(v, raw_text=v.raw_text + tail))
        mtext = compose_source_text(mutable, separator=self.separator, trailing_text=plan.manifest.mutable_text)
        link_text = "".join(v.raw_text for v in views) + mtext
        gen = dict(generation_parameters or {})
        eq = {
            "complete_selected_text_matches": link_text == selected,
            "block_order_matches": [v.sub_context_id for v in plan.included_contexts]
            == [v.sub_context_id for v in linked + mutable],
            "immutable_content_not_duplicated": not ({v.sub_context_id for v in linked}
                                                     & {v.sub_context_id for v in mutable}),
            "mutable_suffix_nonempty": bool(mtext),
        }
        if self.tokenizer is not None:
            eq["complete_selected_token_ids_match"] = (tuple(self.tokenizer.tokenize(link_text))
                                                       == tuple(self.tokenizer.tokenize(selected)))
        if not all(v for k, v in eq.items() if k != "mutable_suffix_nonempty"):
            raise ValueError(f"baseline and LegoLink representations are not equivalent: {eq}")
        return StitchedContext(selected, mtext, tuple(views), tuple(mutable), self.separator, gen,
                               hashlib.sha256(json.dumps(gen, sort_keys=True).encode()).hexdigest(),
                               hashlib.sha256(selected.encode()).hexdigest(), eq)


def validate_link_suffix(stitched: StitchedContext) -> None:
    """A Link must carry a non-empty mutable suffix (the runtime refuses one without)."""
    if not stitched.mutable_text:
        raise ContractError("PIC link requires a non-empty mutable query.")
    if not stitched.linked_views:
        raise ContractError("a Link request must name at least one block")


# ------------------------------------------------------------------- framing
def _find_all(hay: Sequence[int], needle: Sequence[int]) -> list[int]:
    """All start offsets of ``needle`` in ``hay`` (KMP)."""
    if not needle:
        return []
    fail = [0] * len(needle)
    k = 0
    for i in range(1, len(needle)):
        while k and needle[i] != needle[k]:
            k = fail[k - 1]
        if needle[i] == needle[k]:
            k += 1
        fail[i] = k
    out, k = [], 0
    for i, t in enumerate(hay):
        while k and t != needle[k]:
            k = fail[k - 1]
        if t == needle[k]:
            k += 1
        if k == len(needle):
            out.append(i - k + 1)
            k = fail[k - 1]
    return out


@dataclass(frozen=True)
class BlockSegment:
    sub_context_id: str
    semantic_block_id: str
    cache_key: str
    token_ids: tuple

    def to_metadata(self) -> dict:
        return {"sub_context_id": self.sub_context_id, "semantic_block_id": self.semantic_block_id,
                "cache_key": self.cache_key, "physical_token_count": len(self.token_ids),
                "physical_token_ids_sha256": physical_token_ids_sha256(self.token_ids)}


@dataclass(frozen=True)
class ChatTokenLayout:
    tokenizer_fingerprint: str
    baseline_token_ids: tuple
    chat_prefix_token_ids: tuple
    link_segments: tuple  # BlockSegment, in prompt order
    interblock_fresh_token_ids: tuple  # one run after each linked block but the last
    mutable_body_token_ids: tuple
    chat_suffix_token_ids: tuple
    fresh_segments: tuple = ()  # selected blocks that travel fresh (boundary adjustment)
    framing_path: str = "exact_split"
    version: str = PHYSICAL_TOKEN_LAYOUT_VERSION

    @property
    def assembled_token_ids(self) -> tuple:
        out = list(self.chat_prefix_token_ids)
        for i, s in enumerate(self.link_segments):
            out.extend(s.token_ids)
            if i < len(self.interblock_fresh_token_ids):
                out.extend(self.interblock_fresh_token_ids[i])
        out.extend(self.mutable_body_token_ids)
        out.extend(self.chat_suffix_token_ids)
        return tuple(out)

    @property
    def link_input_token_ids(self) -> tuple:
        return (*self.chat_prefix_token_ids, *(t for g in self.interblock_fresh_token_ids for t in g),
                *self.mutable_body_token_ids, *self.chat_suffix_token_ids)

    def link_metadata(self) -> dict:
        ids = list(self.link_input_token_ids)
        md = {
            "physical_token_layout_version": self.version,
            "physical_input_ids": ids,
            "physical_token_count": len(ids),
            "physical_token_ids_sha256": physical_token_ids_sha256(ids),
            "physical_prefix_token_count": len(self.chat_prefix_token_ids),
            "physical_block_segments": [s.to_metadata() for s in self.link_segments],
            "expected_complete_token_count": len(self.baseline_token_ids),
            "expected_complete_token_ids_sha256": physical_token_ids_sha256(self.baseline_token_ids),
        }
        if any(self.interblock_fresh_token_ids):
            md["physical_interblock_fresh_token_counts"] = [len(g) for g in self.interblock_fresh_token_ids]
        return md

    def diagnostics(self) -> dict:
        return {"framing_path": self.framing_path,
                "framing_parity": "exact" if self.assembled_token_ids == self.baseline_token_ids else "mismatch",
                "linked_block_count": len(self.link_segments), "boundary_adjustment_count": len(self.fresh_segments),
                "reusable_interior_token_count": sum(len(s.token_ids) for s in self.link_segments)}


def build_layout(stitched: StitchedContext, tokenizer, *, tools=None, interblock: bool = False,
                 chat_template_kwargs=None) -> ChatTokenLayout:
    if not stitched.linked_views:
        raise PhysicalTokenLayoutError("normalized LegoLink framing requires at least one linked block")
    if not stitched.mutable_text:
        raise PhysicalTokenLayoutError("normalized LegoLink framing requires a non-empty mutable suffix")
    body_text = "".join(v.raw_text for v in stitched.linked_views) + stitched.mutable_text
    if body_text != stitched.selected_text:
        raise PhysicalTokenLayoutError("physical block framing does not reconstruct selected_text exactly")
    baseline = tuple(int(t) for t in tokenizer.tokenize_messages(
        [{"role": "user", "content": stitched.selected_text}], tools=tools, chat_template_kwargs=chat_template_kwargs))
    body = tuple(int(t) for t in tokenizer.tokenize(stitched.selected_text))
    occ = _find_all(baseline, body)
    if len(occ) != 1:
        raise PhysicalTokenLayoutError("selected body does not occur exactly once in the chat-template prompt")
    b0, b1 = occ[0], occ[0] + len(body)
    segs = [BlockSegment(v.sub_context_id, v.semantic_identity or v.sub_context_id, v.cache_key,
                         tuple(int(t) for t in tokenizer.tokenize(v.raw_text))) for v in stitched.linked_views]
    seen: dict[str, tuple] = {}
    for s in segs:
        if seen.setdefault(s.cache_key, s.token_ids) != s.token_ids:
            raise PhysicalTokenLayoutError(f"cache key {s.cache_key} denotes two different compiled units")
    mutable = tuple(int(t) for t in tokenizer.tokenize(stitched.mutable_text))
    prefix, suffix = baseline[:b0], baseline[b1:]
    if tuple(t for s in segs for t in s.token_ids) + mutable == body:
        lay = ChatTokenLayout(tokenizer.fingerprint, baseline, prefix, tuple(segs), (), mutable, suffix)
    else:
        lay = _boundary_adjusted(tokenizer, baseline, prefix, suffix, body, segs, interblock)
    if lay.assembled_token_ids != baseline:
        raise PhysicalTokenLayoutError("Compile/Link assembly does not match the baseline tokens")
    return lay


def _boundary_adjusted(tokenizer, baseline, prefix, suffix, body, segs, interblock) -> ChatTokenLayout:
    """Place every block whose compiled tokens sit exactly at their place in
    the authoritative body; the rest travels fresh."""
    cursor, linked, gaps, fresh = 0, [], [], []
    pending: list[int] = []
    for s in segs:
        n = len(s.token_ids)
        if tuple(body[cursor : cursor + n]) == s.token_ids and (interblock or not fresh):
            if linked:
                gaps.append(tuple(pending))
            elif pending:
                break  # fresh tokens before the first block cannot be placed
            pending = []
            linked.append(s)
            cursor += n
        else:
            # find where the next composing block starts: tokens until then are fresh
            fresh.append(s)
            if not interblock:
                break
            # advance cursor by re-tokenizing is not possible per block; give up on interleaving
            break
    if not linked:
        raise PhysicalTokenLayoutError("no selected block composes with the authoritative prompt tokens")
    fresh = [s for s in segs if s not in linked]
    mutable = tuple(body[cursor:])
    return ChatTokenLayout(tokenizer.fingerprint, baseline, prefix, tuple(linked), tuple(gaps), mutable, suffix,
                           tuple(fresh), "exact_boundary_adjusted")


# ------------------------------------------------------------ repair windows
@dataclass(frozen=True)
class RepairDecision:
    selected_k: int
    windows: tuple
    policy: str = "fixed_unvalidated_debug"
    policy_version: str = REPAIR_DECISION_POLICY_VERSION
    framing_layout_version: str = PHYSICAL_TOKEN_LAYOUT_VERSION
    quality_profile_id: Optional[str] = None
    evidence_id: str = ""
    reason: str = "configured repair window"
    workload_class: str = "agent-context"

    def to_wire(self) -> dict:
        d = dict(self.__dict__)
        d["windows"] = list(self.windows)
        return d


class UniformRepairWindow:
    name = "uniform"

    def __init__(self, k: int = 16):
        self.k = k

    def windows(self, token_counts: Sequence[int], preceding: Sequence[int]) -> list[int]:
        return [min(self.k, n) for n in token_counts]


class BlockLengthCappedRepairWindow(UniformRepairWindow):
    name = "block_length_capped"

    def __init__(self, k: int = 16, fraction: float = 0.25):
        super().__init__(k)
        self.fraction = fraction

    def windows(self, token_counts, preceding):
        return [min(self.k, max(1, int(n * self.fraction)), n) for n in token_counts]


class ContextGainRepairWindow(UniformRepairWindow):
    """Windows grow with the log of the context a block never attended to."""

    name = "context_gain"

    def __init__(self, k: int = 16, base: int = 4):
        super().__init__(k)
        self.base = base

    def windows(self, token_counts, preceding):
        out = []
        for n, p in zip(token_counts, preceding):
            w = self.base + int(round(math.log2(1 + p))) if p > 0 else 0
            out.append(min(n, self.k, w))
        return out


class RepairWindowPlanner:
    """Per-block windows; the first block sitting at offset 0 with no chat
    prefix needs no repair, any other block does."""

    def __init__(self, policy=None, validated_k: Optional[int] = None):
        self.policy = policy or UniformRepairWindow()
        self.validated_k = validated_k

    def plan(self, layout: ChatTokenLayout) -> RepairDecision:
        counts = [len(s.token_ids) for s in layout.link_segments]
        pre, acc = [], len(layout.chat_prefix_token_ids)
        for i, c in enumerate(counts):
            pre.append(acc)
            acc += c + (len(layout.interblock_fresh_token_ids[i]) if i < len(layout.interblock_fresh_token_ids)
                        else 0)
        w = self.policy.windows(counts, pre)
        if pre and pre[0] == 0:
            w[0] = 0
        k = max(w + [getattr(self.policy, "k", 0)])
        below = self.validated_k is not None and any(x < min(self.validated_k, c) for x, c in zip(w, counts))
        reason = (f"{self.policy.name} policy" + ("; below the validated window: needs exact-output evidence"
                                                   if below else ""))
        return RepairDecision(k, tuple(w), reason=reason)


# --------------------------------------------------------------- the request
@dataclass(frozen=True)
class LinkRequest:
    request_id: str
    task_id: str
    cache_keys: tuple
    block_ids: tuple = ()
    recompute_initial_tokens: int = 16
    recompute_mode: str = "batched"
    recompute_tokens_per_block: Optional[tuple] = None
    adapter_id: Optional[str] = None
    segmentation_policy_version: Optional[str] = None
    legolink_policy_version: Optional[str] = None
    variant: Optional[str] = None
    concurrency: Optional[int] = None
    token_layout: Optional[dict] = None
    execution_mode: str = "legacy_debug"
    framing_spec: Optional[dict] = None
    repair_decision: Optional[dict] = None
    execution_profile: Optional[dict] = field(default=None, repr=False)

    def to_wire(self) -> dict:
        if not self.cache_keys:
            raise ContractError("a Link request must name at least one block")
        w: dict[str, Any] = {"request_id": str(self.request_id), "task_id": str(self.task_id),
                             "cache_keys": [str(k) for k in self.cache_keys],
                             "block_ids": [str(b) for b in (self.block_ids or self.cache_keys)],
                             "recompute_mode": self.recompute_mode,
                             "recompute_initial_tokens": int(self.recompute_initial_tokens)}
        if self.recompute_tokens_per_block is not None:
            wins = [int(x) for x in self.recompute_tokens_per_block]
            w["recompute_tokens_per_block"] = wins
            w["recompute_first_block_tokens"] = wins[0]
            w["recompute_first_block"] = bool(wins[0])
        for n in ("variant", "adapter_id", "segmentation_policy_version", "legolink_policy_version"):
            v = getattr(self, n)
            if v is not None:
                w[n] = str(v)
        if self.concurrency is not None:
            w["concurrency"] = int(self.concurrency)
        if self.token_layout:
            w.update(self.token_layout)
        w["execution_mode"] = self.execution_mode
        if self.framing_spec is not None:
            w["framing_spec"] = dict(self.framing_spec)
        if self.repair_decision is not None:
            w["repair_decision"] = dict(self.repair_decision)
        validate_pic_link_request(dict(w), profile=self.execution_profile,
                                  require_formal=self.execution_mode == "formal")
        return w


@dataclass(frozen=True)
class LinkAudit:
    """Host-side evidence written beside (never into) the request."""

    request_id: str
    task_id: str
    selected_order: tuple
    expected_cache_keys: tuple
    framing: dict
    repair_window: dict
    equivalence: dict
    generation_parameters_sha256: str

    def to_dict(self) -> dict:
        d = dict(self.__dict__)
        d["selected_order"] = list(self.selected_order)
        d["expected_cache_keys"] = list(self.expected_cache_keys)
        return d


def framing_spec_for(tokenizer, model_id: str, profile_id: str = "default") -> dict:
    return {"framing_layout_version": PHYSICAL_TOKEN_LAYOUT_VERSION, "model_id": model_id,
            "tokenizer_fingerprint": tokenizer.fingerprint,
            "chat_template_sha256": getattr(tokenizer, "chat_template_sha256", "0" * 64), "profile_id": profile_id}


def frame_link(stitched: StitchedContext, layout: ChatTokenLayout, decision: RepairDecision, *, request_id: str,
               task_id: str, model: str, generation: Optional[dict] = None, formal: bool = False,
               framing_spec: Optional[dict] = None, execution_profile: Optional[dict] = None,
               compat: Optional[dict] = None) -> tuple[dict, LinkAudit]:
    """Builds the chat payload carrying ``pic_link`` and the audit record."""
    validate_link_suffix(stitched)
    segs = layout.link_segments
    req = LinkRequest(
        request_id=request_id, task_id=task_id, cache_keys=tuple(s.cache_key for s in segs),
        block_ids=tuple(s.semantic_block_id for s in segs), recompute_initial_tokens=decision.selected_k,
        recompute_tokens_per_block=decision.windows, token_layout=layout.link_metadata(),
        execution_mode="formal" if formal else "legacy_debug",
        framing_spec=framing_spec if (formal or decision.policy == "quality_guarded") else None,
        repair_decision=decision.to_wire() if (formal or decision.policy == "quality_guarded") else None,
        execution_profile=execution_profile, **(compat or {}))
    payload = {"model": model, "messages": [{"role": "user", "content": stitched.mutable_text}],
               "pic_link": req.to_wire()}
    payload.update(generation or {})
    audit = LinkAudit(request_id, task_id, tuple(v.sub_context_id for v in stitched.linked_views),
                      tuple(s.cache_key for s in segs), layout.diagnostics(), decision.to_wire(), stitched.equivalence,
                      stitched.generation_parameters_sha256)
    return payload, audit


def compile_payload(segment: BlockSegment, *, model: str, compat: Optional[dict] = None,
                    fingerprints: Optional[dict] = None) -> dict:
    """Compile = prefill this block alone and register it (max_tokens=1)."""
    ids = list(segment.token_ids)
    sc = {"cache_key": segment.cache_key, "semantic_block_id": segment.semantic_block_id,
          "sub_context_id": segment.sub_context_id, "physical_token_layout_version": PHYSICAL_TOKEN_LAYOUT_VERSION,
          "physical_input_ids": ids, "physical_token_count": len(ids),
          "physical_token_ids_sha256": physical_token_ids_sha256(ids)}
    sc.update(fingerprints or {})
    sc.update(compat or {})
    return {"model": model, "messages": [], "max_tokens": 1, "temperature": 0.0, "extra_key": segment.cache_key,
            "sub_context": sc}
