"""Segmentation, incremental ingest and context selection (host stages 3-4).

* :class:`DeterministicSegmenter` -- one segment per source; a source above
  ``max_segment_tokens`` is cut at line boundaries found by binary search on
  the token budget (reference ``semantic_segmentation.py:151-260``).  An
  optional ``proposer(text) -> split offsets`` (e.g. an LLM asked for split
  points only) is validated and falls back to the deterministic cut, with the
  fallback recorded.
* :func:`validate_segments` -- spans must cover the source exactly, in order,
  and the text is rebuilt by slicing (never by the segmenter's own copy).
* :class:`ContextManager` -- ingest transaction: checkpoint -> extract ->
  segment -> store; any failure rolls the collector back.  :meth:`select`
  returns an :class:`AgentContextManifest` (a logical selection: which
  sub-contexts, in what order, plus the mutable query text).

Mutability rule: stable fields (task instruction, tool definitions, workspace
evidence, task metadata) are immutable at once; conversation / tool-history
sources are immutable once a later ingest added newer history (the entries of
the newest batch stay in the mutable suffix); the user prompt is always
mutable.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Callable, Iterable, Optional, Sequence

from .events import (CONTEXT_FIELDS, EventCollector, ExtractedSource, FieldExtractor, SessionEvent, SourceSpan)
from .store import (DEFAULT_RECOMPUTE_POLICY_VERSION, DEFAULT_SEGMENTATION_POLICY_VERSION, HISTORY_FIELDS,
                    STABLE_FIELDS, SubContext, SubContextStore)
from .tokenizer import RegexTokenizer


class SegmentationError(ValueError):
    pass


@dataclass(frozen=True)
class Segment:
    start: int
    end: int


def validate_segments(text: str, segs: Sequence[Segment]) -> None:
    if not text:
        if segs:
            raise SegmentationError("empty source must have no segments")
        return
    if not segs:
        raise SegmentationError("segments must cover the source")
    pos = 0
    for s in segs:
        if s.start != pos or s.end <= s.start:
            raise SegmentationError(f"segments must tile the source exactly (gap/overlap at {pos})")
        pos = s.end
    if pos != len(text):
        raise SegmentationError("segments do not reach the end of the source")
    if "".join(text[s.start:s.end] for s in segs) != text:
        raise SegmentationError("segment text does not reconstruct the source")


class DeterministicSegmenter:
    policy_version = DEFAULT_SEGMENTATION_POLICY_VERSION

    def __init__(self, tokenizer=None, max_segment_tokens: int = 4096,
                 proposer: Optional[Callable[[str], Sequence[int]]] = None):
        self.tokenizer = tokenizer or RegexTokenizer()
        self.max_tokens = max_segment_tokens
        self.proposer = proposer
        self.fallbacks: list[dict] = []

    def _cut_points(self, text: str) -> list[int]:
        """Line-boundary offsets; binary search the longest prefix whose token
        count fits the budget, repeatedly."""
        bounds = [i + 1 for i, ch in enumerate(text) if ch == "\n" and i + 1 < len(text)]
        cuts, start = [], 0
        while self.tokenizer.count(text[start:]) > self.max_tokens:
            cands = [b for b in bounds if b > start]
            lo, hi, best = 0, len(cands) - 1, None
            while lo <= hi:
                mid = (lo + hi) // 2
                if self.tokenizer.count(text[start:cands[mid]]) <= self.max_tokens:
                    best, lo = cands[mid], mid + 1
                else:
                    hi = mid - 1
            if best is None:  # a single line above budget: cut by characters
                lo, hi, best = start + 1, len(text) - 1, start + 1
                while lo <= hi:
                    mid = (lo + hi) // 2
                    if self.tokenizer.count(text[start:mid]) <= self.max_tokens:
                        best, lo = mid, mid + 1
                    else:
                        hi = mid - 1
            cuts.append(best)
            start = best
        return cuts

    def segment(self, src: ExtractedSource) -> list[Segment]:
        text = src.raw_text
        if not text:
            return []
        if self.proposer is not None:
            try:
                pts = sorted(set(int(p) for p in self.proposer(text)))
                segs = [Segment(a, b) for a, b in zip([0] + pts, pts + [len(text)]) if b > a]
                validate_segments(text, segs)
                if all(self.tokenizer.count(text[s.start:s.end]) <= self.max_tokens for s in segs):
                    return segs
                reason = "proposed segment above token budget"
            except Exception as e:  # fall back, recorded
                reason = f"invalid proposal: {e}"
            self.fallbacks.append({"source_id": src.source_id, "reason": reason})
        pts = self._cut_points(text)
        segs = [Segment(a, b) for a, b in zip([0] + pts, pts + [len(text)])]
        validate_segments(text, segs)
        return segs


@dataclass(frozen=True)
class FrozenSourcePrefix:
    """The finalized leading blocks of a source's stored revision, whose
    boundaries must not move when the source grows.

    When the new revision of a source starts with exactly the text these
    blocks cover (it was appended to, not edited), they are replayed as they
    were stored -- same spans, same text, hence the same identity, id and
    cache key -- and only the appended remainder is segmented.  A later
    segmentation (possibly a model, nondeterministic across a context change)
    therefore never re-cuts a block a Link may already depend on.  Blocks are
    frozen from offset 0 while each is a reuse candidate, not invalidated,
    owns exactly one span of this source and starts where the previous one
    ended.  Reference: ``segmentation_validation.py:316-395``,
    ``manager.py:309-341``."""

    source_id: str
    end: int
    text: str
    spans: tuple  # (start, end) of each frozen block, in order

    @classmethod
    def from_blocks(cls, source_id: str, blocks: Sequence[SubContext]) -> Optional["FrozenSourcePrefix"]:
        owned = []
        for b in blocks:
            spans = list(b.source_spans)
            if len(spans) != 1 or spans[0].source_id != source_id:
                return None
            owned.append((spans[0].start, spans[0].end, b))
        owned.sort(key=lambda t: (t[0], t[1], t[2].sub_context_id))
        cur, spans, text = 0, [], []
        for start, end, b in owned:
            if start != cur or b.invalidated or not b.reuse_candidate or b.context_field == "user_prompt":
                break
            spans.append((start, end))
            text.append(b.raw_text)
            cur = end
        if not spans:
            return None
        return cls(source_id, cur, "".join(text), tuple(spans))

    def applies_to(self, new_text: str) -> bool:
        return len(new_text) > self.end and new_text.startswith(self.text)


@dataclass(frozen=True)
class AgentContextManifest:
    task_id: str
    session_revision: int
    selected_sub_context_ids: tuple
    mutable_sub_context_ids: tuple
    mutable_text: str
    selection_order: tuple = ()
    selector: str = "rule-based-v1"
    excluded_sub_context_ids: tuple = ()
    token_budget: Optional[int] = None

    def to_dict(self) -> dict:
        return {"task_id": self.task_id, "session_revision": self.session_revision,
                "selected_sub_context_ids": list(self.selected_sub_context_ids),
                "mutable_sub_context_ids": list(self.mutable_sub_context_ids), "mutable_text": self.mutable_text,
                "selection_order": list(self.selection_order), "selector": self.selector,
                "excluded_sub_context_ids": list(self.excluded_sub_context_ids), "token_budget": self.token_budget}


FIELD_ORDER = {f: i for i, f in enumerate(("task_instruction", "tool_definitions", "task_metadata",
                                           "workspace_evidence"))}


class ContextManager:
    def __init__(self, task_id: str, *, tokenizer=None, store: Optional[SubContextStore] = None,
                 segmenter: Optional[DeterministicSegmenter] = None, model_fingerprint: str = "runtime-local",
                 recompute_policy_version: str = DEFAULT_RECOMPUTE_POLICY_VERSION, classifier=None,
                 capture_token_ids: bool = False, selector=None, boundary_locking: bool = True):
        self.task_id = task_id
        self.tokenizer = tokenizer or RegexTokenizer()
        self.collector = EventCollector(task_id)
        self.extractor = FieldExtractor(classifier)
        self.store = store or SubContextStore()
        self.segmenter = segmenter or DeterministicSegmenter(self.tokenizer)
        self.model_fingerprint = model_fingerprint
        self.recompute_policy_version = recompute_policy_version
        self.capture_token_ids = capture_token_ids
        self.selector = selector  # host.selection selector; None = keep every active sub-context
        self._stored_revision: dict[str, str] = {}
        self.boundary_locking = boundary_locking
        self.frozen_log: list[dict] = []  # one record per source revision segmented after a frozen prefix

    def ingest(self, values: Iterable[tuple], *, fail_after_extract: bool = False) -> list[SessionEvent]:
        cp = self.collector.checkpoint()
        try:
            events = self.collector.add_events(list(values))
            ext = self.extractor.extract(self.collector.events())
            if fail_after_extract:
                raise RuntimeError("injected ingest failure")
            self._store_changed(ext.sources(), ext.session_revision)
            return events
        except Exception:
            self.collector.rollback(cp)
            raise

    def _store_changed(self, sources: list[ExtractedSource], revision: int) -> None:
        changed: dict[str, list[SubContext]] = {}
        for src in sources:
            if self._stored_revision.get(src.source_id) == src.event_id:
                continue
            segs = self._segment_with_frozen_prefix(src)
            values = []
            for i, sg in enumerate(segs):
                span = SourceSpan(src.source_id, sg.start, sg.end, src.source_path)
                values.append(SubContext.create(
                    task_id=self.task_id, context_field=src.context_field, source_id=src.source_id, spans=[span],
                    raw_text=src.raw_text[sg.start:sg.end], tokenizer=self.tokenizer,
                    sequence_number=src.sequence_number, source_revision=src.revision,
                    model_fingerprint=self.model_fingerprint, recompute_policy_version=self.recompute_policy_version,
                    capture_token_ids=self.capture_token_ids,
                    metadata={"segment_index": i, "segment_count": len(segs), "event_id": src.event_id}))
            changed[src.source_id] = values
        if changed:
            self.store.replace_source_revisions(self.task_id, changed)
            for src in sources:
                if src.source_id in changed:
                    self._stored_revision[src.source_id] = src.event_id

    def _segment_with_frozen_prefix(self, src: ExtractedSource) -> list:
        """Segments of ``src``; a source that only grew keeps its stored
        finalized leading blocks (:class:`FrozenSourcePrefix`)."""
        prefix = None
        if self.boundary_locking and src.source_id in self._stored_revision:
            prev = [v for v in self.store.all(self.task_id) if v.source_id == src.source_id]
            prefix = FrozenSourcePrefix.from_blocks(src.source_id, prev) if prev else None
        if prefix is None or not prefix.applies_to(src.raw_text):
            return self.segmenter.segment(src)
        from dataclasses import replace as _replace

        tail = self.segmenter.segment(_replace(src, raw_text=src.raw_text[prefix.end:]))
        segs = [Segment(a, b) for a, b in prefix.spans] + [Segment(prefix.end + t.start, prefix.end + t.end)
                                                            for t in tail]
        validate_segments(src.raw_text, segs)
        self.frozen_log.append({"source_id": src.source_id, "frozen_blocks": len(prefix.spans),
                                "frozen_chars": prefix.end, "appended_chars": len(src.raw_text) - prefix.end})
        return segs

    def contexts(self) -> list[SubContext]:
        ext = self.extractor.extract(self.collector.events())
        active = {s.source_id: s.event_id for s in ext.sources()}
        out = [v for v in self.store.all(self.task_id) if active.get(v.source_id) == v.metadata.get("event_id")]
        newest_hist = max((v.source_revision for v in out if v.context_field in HISTORY_FIELDS), default=-1)
        res = []
        for v in out:
            if v.context_field == "user_prompt":
                mut = True
            elif v.context_field in STABLE_FIELDS:
                mut = False
            else:
                mut = v.source_revision >= newest_hist
            res.append(v if v.is_mutable == mut else _with(v, is_mutable=mut))
        return res

    def select(self, query_text: str = "") -> AgentContextManifest:
        if self.selector is not None:
            return self.selector.select(self, query_text)
        ctx = self.ordered_contexts()
        sel = tuple(v.sub_context_id for v in ctx)
        mut = tuple(v.sub_context_id for v in ctx if v.is_mutable)
        return AgentContextManifest(self.task_id, self.collector.revision, sel, mut, query_text, sel)

    def ordered_contexts(self) -> list[SubContext]:
        """Active sub-contexts in prompt order: stable fields, then history by
        sequence, then the user prompt."""
        ctx = self.contexts()

        def order(v: SubContext):
            stable = FIELD_ORDER.get(v.context_field)
            if v.context_field == "user_prompt":
                return (3, v.sequence_number, v.metadata.get("segment_index", 0))
            if stable is not None:
                return (0, stable, v.sequence_number, v.metadata.get("segment_index", 0))
            return (1, 0, v.sequence_number, v.metadata.get("segment_index", 0))

        ctx.sort(key=order)
        return ctx


def _with(v: SubContext, **kw) -> SubContext:
    from dataclasses import replace

    return replace(v, **kw)
