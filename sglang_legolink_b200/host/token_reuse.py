"""Host token reuse: framing consumes token ids the host already owns instead
of encoding the same text again.  EXPERIMENTAL, opt-in
(``NOC_HOST_TOKEN_REUSE=1``), off by default.

Ownership does not change: a stored sub-context owns its ids (written once
when it was created with ``capture_token_ids``); a request's layout owns its
prefix / block / mutable / prompt ids; the runtime owns every physical
field.  :class:`RequestTokenSource` is a tokenizer for ONE request that
answers ``tokenize(text)`` from ids a sub-context holds for exactly that
text under the same tokenizer fingerprint, and otherwise encodes once and
remembers.  Tokenization is a pure function of (text, tokenizer), so the
answer is what the tokenizer would give -- and framing still checks that the
block ids plus the mutable ids equal a fresh encoding of the whole body,
which catches a store that lies.

:class:`SharedTokenCache` keeps ids of exact immutable texts that no object
owns, keyed by (tokenizer fingerprint, text): a tokenizer change is a miss,
never a stale hit.  Mutable text never enters it.

Reference: ``noc_context_manager/authoritative_tokens.py:44-286``.
"""

from __future__ import annotations

import os
import sys
import threading
import time
from collections import Counter, OrderedDict
from typing import Any, Mapping, Optional, Sequence

FEATURE_FLAG_ENV = "NOC_HOST_TOKEN_REUSE"


def host_token_reuse_enabled(environ: Optional[Mapping[str, str]] = None) -> bool:
    v = (os.environ if environ is None else environ).get(FEATURE_FLAG_ENV, "")
    return v.strip().lower() in ("1", "true", "yes", "on")


def refusal_reason(sc, tokenizer) -> Optional[str]:
    """Why ``sc.token_ids`` may not answer for ``tokenizer`` (None: they may).
    Ids are valid only in the namespace that produced them: the same
    tokenizer fingerprint, model tokens, one id per counted token."""
    if sc.invalidated:
        return "invalidated"
    if not sc.token_ids:
        return "no_token_ids"
    if len(sc.token_ids) != sc.token_count:
        return "token_count_mismatch"
    fp = str(getattr(tokenizer, "fingerprint", "") or "")
    if not fp or (sc.metadata or {}).get("tokenizer_fingerprint") != fp:
        return "tokenizer_fingerprint_mismatch"
    if sc.token_unit != "model":
        return "not_model_tokens"
    if any(type(t) is not int for t in sc.token_ids):
        return "non_integer_token_ids"
    return None


class SharedTokenCache:
    """Bounded LRU, process-wide: (tokenizer fingerprint, exact immutable
    text) -> ids (tuples of ints, shared read-only)."""

    def __init__(self, max_entries: int = 4096):
        if max_entries < 1:
            raise ValueError("max_entries must be positive")
        self.max_entries = max_entries
        self._d: OrderedDict = OrderedDict()
        self._lock = threading.Lock()
        self.hits = self.misses = self.evictions = 0

    def get(self, fingerprint: str, text: str) -> Optional[tuple]:
        with self._lock:
            ids = self._d.get((fingerprint, text))
            if ids is None:
                self.misses += 1
                return None
            self._d.move_to_end((fingerprint, text))
            self.hits += 1
            return ids

    def put(self, fingerprint: str, text: str, token_ids: Sequence[int]) -> tuple:
        ids = tuple(int(t) for t in token_ids)
        with self._lock:
            self._d[(fingerprint, text)] = ids
            self._d.move_to_end((fingerprint, text))
            while len(self._d) > self.max_entries:
                self._d.popitem(last=False)
                self.evictions += 1
        return ids

    def __len__(self) -> int:
        return len(self._d)

    def memory_bytes(self) -> dict:
        """Raw id payload (4 B per id, as an int32 array) and the Python
        objects held (tuples, ints outside the small-int cache, key strings)."""
        with self._lock:
            items = list(self._d.items())
        raw = sum(4 * len(ids) for _, ids in items)
        py = sum(sys.getsizeof(ids) + sys.getsizeof(k[1]) + sys.getsizeof(k) for k, ids in items)
        py += sum(sys.getsizeof(t) for _, ids in items for t in ids if not -5 <= t <= 256)
        return {"entries": len(items), "raw_token_id_bytes": raw, "python_object_bytes": py}


class _Counting:
    def __init__(self, inner):
        self._inner = inner
        self.inner_calls: Counter = Counter()
        self.inner_chars = self.inner_tokens = 0
        self.inner_ms = 0.0

    def __getattr__(self, name: str):
        return getattr(self._inner, name)

    @property
    def fingerprint(self) -> str:
        return self._inner.fingerprint

    def _call(self, method: str, fn, chars: int) -> tuple:
        t0 = time.perf_counter_ns()
        ids = tuple(fn())
        self.inner_ms += (time.perf_counter_ns() - t0) / 1e6
        self.inner_calls[method] += 1
        self.inner_chars += chars
        self.inner_tokens += len(ids)
        return ids

    def counts(self) -> dict:
        return {"tokenizer_calls": sum(self.inner_calls.values()),
                **{f"calls_{k}": v for k, v in self.inner_calls.items()}, "tokenizer_chars": self.inner_chars,
                "tokenizer_tokens": self.inner_tokens, "tokenizer_ms": round(self.inner_ms, 4)}


class CountingTokenizer(_Counting):
    """Counts what reaches the real tokenizer (the baseline path, measured
    the same way as :class:`RequestTokenSource`)."""

    def tokenize(self, text: str):
        return self._call("tokenize", lambda: self._inner.tokenize(text), len(text))

    def tokenize_messages(self, messages, **kw):
        return self._call("tokenize_messages", lambda: self._inner.tokenize_messages(messages, **kw),
                          sum(len(str(m.get("content", ""))) for m in messages))


def _messages_key(messages: Sequence[Mapping], kw: Mapping) -> Optional[tuple]:
    extra = tuple(sorted((k, repr(v)) for k, v in kw.items() if v is not None and v is not False))
    key = []
    for m in messages:
        if set(m) - {"role", "content"} or not isinstance(m.get("content"), str):
            return None  # unusual messages are not memoized
        key.append((m.get("role"), m["content"]))
    return tuple(key), extra


class RequestTokenSource(_Counting):
    """A tokenizer for one request that never encodes a text twice; build one
    per request and drop it (never shared between requests)."""

    def __init__(self, inner, *, shared: Optional[SharedTokenCache] = None):
        super().__init__(inner)
        self._shared = shared
        self._texts: dict = {}
        self._origin: dict = {}
        self._messages: dict = {}
        self._immutable: set = set()
        self.hits: Counter = Counter()
        self.refusals: Counter = Counter()

    def adopt(self, sc) -> bool:
        why = refusal_reason(sc, self._inner)
        if why is not None:
            self.refusals[why] += 1
            return False
        self._texts[sc.raw_text] = tuple(sc.token_ids)
        self._origin[sc.raw_text] = "sub_context"
        return True

    def mark_immutable(self, text: str) -> None:
        self._immutable.add(text)

    def tokenize(self, text: str) -> tuple:
        ids = self._texts.get(text)
        if ids is not None:
            self.hits[self._origin[text]] += 1
            return ids
        shared = self._shared is not None and text in self._immutable
        if shared:
            ids = self._shared.get(self._inner.fingerprint, text)
            if ids is not None:
                self.hits["shared_immutable"] += 1
                self._texts[text], self._origin[text] = ids, "request"
                return ids
        ids = self._call("tokenize", lambda: self._inner.tokenize(text), len(text))
        if shared:
            ids = self._shared.put(self._inner.fingerprint, text, ids)
        self._texts[text], self._origin[text] = ids, "request"
        return ids

    def tokenize_messages(self, messages, **kw) -> tuple:
        key = _messages_key(messages, kw)
        if key is not None and key in self._messages:
            self.hits["request_messages"] += 1
            return self._messages[key]
        ids = self._call("tokenize_messages", lambda: self._inner.tokenize_messages(messages, **kw),
                         sum(len(str(m.get("content", ""))) for m in messages))
        if key is not None:
            self._messages[key] = ids
        return ids

    def counts(self) -> dict:
        return {**super().counts(), "reused": dict(self.hits), "refused": dict(self.refusals)}
