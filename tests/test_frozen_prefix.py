"""Boundary locking: when a source grows by appending, its stored finalized
leading blocks keep their spans, ids and cache keys and only the appended
text is segmented; an edited source is segmented again as a whole
(reference ``segmentation_validation.py:316``, ``manager.py:309-341``)."""

from sglang_legolink_b200.host.events import SourceSpan
from sglang_legolink_b200.host.manager import ContextManager, DeterministicSegmenter, FrozenSourcePrefix
from sglang_legolink_b200.host.store import SubContext
from sglang_legolink_b200.host.tokenizer import HashTokenizer

TOK = HashTokenizer(4096)


def _lines(tag, n):
    return "".join(f"{tag} line {i}: value = compute({i}) and store it\n" for i in range(n))


def _manager(locking=True):
    return ContextManager("t", tokenizer=TOK, segmenter=DeterministicSegmenter(TOK, max_segment_tokens=120),
                          boundary_locking=locking)


def _blocks(cm, source_id):
    return sorted((v for v in cm.contexts() if v.source_id == source_id), key=lambda v: v.source_spans[0].start)


def test_appended_source_keeps_its_finalized_blocks():
    a = _lines("first", 43)
    cm = _manager()
    cm.ingest([("workspace_file", "ws:log", a, {})])
    before = _blocks(cm, "ws:log")
    assert len(before) >= 3
    cm.ingest([("workspace_file", "ws:log", a + _lines("more", 25), {})])
    after = _blocks(cm, "ws:log")
    for old, new in zip(before, after):
        assert (new.sub_context_id, new.cache_key, new.raw_text) == (old.sub_context_id, old.cache_key, old.raw_text)
    assert len(after) > len(before)
    assert "".join(v.raw_text for v in after) == a + _lines("more", 25)
    assert cm.frozen_log == [{"source_id": "ws:log", "frozen_blocks": len(before), "frozen_chars": len(a),
                              "appended_chars": len(_lines("more", 25))}]


def test_without_locking_the_last_block_is_recut():
    a = _lines("first", 43)
    grown = a + _lines("more", 25)
    locked, free = _manager(True), _manager(False)
    for cm in (locked, free):
        cm.ingest([("workspace_file", "ws:log", a, {})])
        cm.ingest([("workspace_file", "ws:log", grown, {})])
    keys_locked = {v.cache_key for v in _blocks(locked, "ws:log")}
    keys_free = {v.cache_key for v in _blocks(free, "ws:log")}
    first = {v.cache_key for v in _blocks(_manager_with(a), "ws:log")}
    assert first <= keys_locked  # every block of the first revision is still linkable
    assert not first <= keys_free  # re-cutting the grown source moved a boundary


def _manager_with(text):
    cm = _manager()
    cm.ingest([("workspace_file", "ws:log", text, {})])
    return cm


def test_edited_source_is_segmented_again():
    a = _lines("first", 43)
    cm = _manager()
    cm.ingest([("workspace_file", "ws:log", a, {})])
    edited = "EDIT " + a + _lines("more", 5)
    cm.ingest([("workspace_file", "ws:log", edited, {})])
    assert cm.frozen_log == []
    assert "".join(v.raw_text for v in _blocks(cm, "ws:log")) == edited


def test_from_blocks_stops_at_the_first_unusable_block():
    def blk(start, end, text, **kw):
        v = SubContext.create(task_id="t", context_field="workspace_evidence", source_id="s",
                              spans=[SourceSpan("s", start, end)], raw_text=text, tokenizer=TOK, sequence_number=1,
                              source_revision=1, model_fingerprint="m")
        from dataclasses import replace

        return replace(v, **kw)

    a, b, c = blk(0, 3, "abc"), blk(3, 6, "def"), blk(6, 9, "ghi")
    p = FrozenSourcePrefix.from_blocks("s", [c, a, b])
    assert (p.end, p.text, p.spans) == (9, "abcdefghi", ((0, 3), (3, 6), (6, 9)))
    p = FrozenSourcePrefix.from_blocks("s", [a, blk(3, 6, "def", reuse_candidate=False), c])
    assert p.spans == ((0, 3),)
    assert FrozenSourcePrefix.from_blocks("s", [blk(1, 3, "bc")]) is None  # not from offset 0
    assert FrozenSourcePrefix.from_blocks("other", [a]) is None
    assert p.applies_to("abcX") and not p.applies_to("abc") and not p.applies_to("xbcd")
