"""Request scheduler: admission of Compile / Link / plain prefills and
continuous batching of decode.

The reference admits a Link only into an empty engine (a batch of one that
waits for every running decode to finish; its own trace attributes 97.8 % of
TTFT at concurrency 8 to that wait, reference ``pic_runtime.py:2023-2026``,
``managers/scheduler.py:2597-2690``).  Here one loop thread alternates:

1. admit: pop up to ``max_prefills_per_step`` queued requests; their
   Compiles and Links run as ONE extend forward (every Link's KV link in one
   fused launch per source pool, every repair row and Compile row in one
   pass), plain prefills one by one -- a Link never waits for the running
   decodes to drain;
2. decode: one batched greedy step for every running sequence (CUDA graph per
   batch bucket on GPU), streaming each new token to its request.

Arrival checks (reference ``managers/scheduler.py:1915-2057``): a request is a
Compile (``sub_context``) XOR a Link (``pic_link``); in LegoLink-only mode
plain generation is refused; a Link may not ask for input logprobs; an
overlength Link is rejected, never truncated.  The Compiles admitted in one
step share one extend forward; a second Compile of a key already in that
batch is deferred to the next one (where the registry keeps the resident copy
on the duplicate).  When nothing is waiting, greedy decode runs
``decode_chunk`` steps back to back on the device (no host read between
them); a Compile or Link is admitted only between chunks.  Every failure is
request-scoped.
"""

from __future__ import annotations

import queue
import threading
import time
import traceback
from dataclasses import dataclass, field
from typing import Any, Callable, Optional

from ..contract import ContractError
from ..utils.trace import emit_trace
from .engine import Engine, RuntimeErrorAbort, Sequence_
from .sampling import GREEDY, SamplingParams


class RequestRejected(ValueError):
    pass


COMPILE_STATE_ABSENT = "absent"
COMPILE_STATE_COMPILING = "compiling"
COMPILE_STATE_RESIDENT = "resident"


class CompileStates:
    """Per cache key: ``absent`` -> ``compiling`` (one or more admitted
    Compiles not yet finished) -> ``resident`` (registered in the engine).

    All in-flight Compiles of a key carry the same tokens and storage mode:
    one that disagrees is refused at arrival instead of racing the first; one
    that agrees is attached as its own record (duplicate work stays harmless:
    the registry keeps the first block and releases the second).  A Compile
    that ends without registering drops its record; a request that vanishes
    without finishing (collected while queued) is dropped by a weak-reference
    finalizer.  Nothing is written for a key before its Compile succeeds, so
    a failure needs no rollback here.
    Reference: ``pic_runtime.py:2270-2361`` (token registry states)."""

    def __init__(self, resident: Callable[[str], bool]):
        self._resident = resident
        self._records: dict = {}  # owner id -> (key, tokens hash, storage mode)
        self._owners: dict = {}   # key -> [owner ids]
        self._lock = threading.Lock()

    def state(self, key: str) -> str:
        with self._lock:
            if self._owners.get(key):
                return COMPILE_STATE_COMPILING
        return COMPILE_STATE_RESIDENT if self._resident(key) else COMPILE_STATE_ABSENT

    def admit(self, owner, key: str, tokens, storage_mode: str) -> None:
        import hashlib
        import weakref

        digest = hashlib.sha256(",".join(str(int(t)) for t in tokens).encode()).hexdigest()
        with self._lock:
            owners = self._owners.get(key)
            if owners:
                _, first_digest, first_mode = self._records[owners[0]]
                if (first_digest, first_mode) != (digest, storage_mode):
                    raise RequestRejected(
                        f"a Compile of cache_key {key} with other tokens or storage mode is already in flight; a "
                        "cache key names one block: wait for the first Compile or use another key")
            oid = id(owner)
            if oid in self._records:
                self._drop_locked(oid)
            self._owners.setdefault(key, []).append(oid)
            self._records[oid] = (key, digest, storage_mode)
        try:
            fin = weakref.finalize(owner, self.finish, oid)
            fin.atexit = False
        except TypeError:
            pass

    def finish(self, owner) -> None:
        """The Compile ended (registered or failed); idempotent."""
        with self._lock:
            self._drop_locked(owner if isinstance(owner, int) else id(owner))

    def _drop_locked(self, oid: int) -> None:
        rec = self._records.pop(oid, None)
        if rec is None:
            return
        owners = self._owners.get(rec[0], [])
        if oid in owners:
            owners.remove(oid)
        if not owners:
            self._owners.pop(rec[0], None)

    def inflight(self) -> dict:
        with self._lock:
            return {k: len(v) for k, v in self._owners.items()}


@dataclass
class Request:
    kind: str  # "compile" | "link" | "plain"
    rid: str
    input_ids: list
    max_new_tokens: int
    stop_ids: tuple = ()
    sub_context: Optional[dict] = None
    pic_link: Optional[dict] = None
    created: float = field(default_factory=time.perf_counter)
    events: "queue.Queue" = field(default_factory=queue.Queue)  # ("token", id) | ("done", info) | ("error", msg)
    seq: Optional[Sequence_] = None
    ttft_s: Optional[float] = None
    sampling: SamplingParams = GREEDY
    resume: Optional[list] = None  # tokens generated before a retraction (plain requests)


class Scheduler:
    def __init__(self, engine: Engine, *, legolink_only: Optional[bool] = None, max_running: int = 64,
                 max_prefills_per_step: int = 8, max_context: Optional[int] = None, decode_chunk: int = 8):
        self.engine = engine
        self._legolink_only = legolink_only  # None: SGLANG_PIC_LEGOLINK_ONLY (default on), read per request
        self.max_running = max_running
        self.max_prefills_per_step = max_prefills_per_step
        self.decode_chunk = decode_chunk
        self._deferred: list = []  # Compiles pushed to the next batch (same key already in this one)
        self._parked: list = []  # Links waiting for an in-flight Compile of one of their keys
        self.max_context = max_context or engine.max_context
        self.waiting: "queue.Queue[Request]" = queue.Queue()
        self.running: list[Request] = []
        self._stop = threading.Event()
        self._thread: Optional[threading.Thread] = None
        self.stats = {"admitted": 0, "rejected": 0, "finished": 0, "decode_steps": 0}
        self.compile_states = CompileStates(lambda k: bool(engine.registry.contains(k)))
        self.max_link_waits = 64  # scheduler steps a Link waits for a Compile of one of its keys

    @property
    def legolink_only(self) -> bool:
        """Plain generation is refused unless the deployment allows it: an
        explicit setting wins, else ``SGLANG_PIC_LEGOLINK_ONLY`` (default on)
        at the time of each request (reference ``pic_runtime.py:1326``)."""
        if self._legolink_only is not None:
            return bool(self._legolink_only)
        from ..contract import env_flag

        return env_flag("SGLANG_PIC_LEGOLINK_ONLY", "1")

    @legolink_only.setter
    def legolink_only(self, value: Optional[bool]) -> None:
        self._legolink_only = value

    # ------------------------------------------------------------ arrival
    def check(self, req: Request) -> None:
        if req.sub_context is not None and req.pic_link is not None:
            raise RequestRejected("a request is either a Compile (sub_context) or a Link (pic_link), not both")
        if req.kind == "plain" and self.legolink_only:
            raise RequestRejected("LegoLink-only runtime: plain generation is refused; send a Compile or a Link")
        if req.kind == "link" and not isinstance(req.pic_link, dict):
            raise RequestRejected("pic_link must be an object.")
        if len(req.input_ids) + req.max_new_tokens > self.max_context and req.kind != "link":
            raise RequestRejected(f"request of {len(req.input_ids)} tokens exceeds the context window")

    def submit(self, req: Request) -> Request:
        try:
            self.check(req)
            if req.kind == "compile":
                sc = req.sub_context or {}
                key = sc.get("cache_key")
                if key:
                    from .engine import Engine as _E

                    self.compile_states.admit(req, str(key), req.input_ids, _E.storage_mode(sc))
        except (RequestRejected, ContractError) as e:
            self.stats["rejected"] += 1
            req.events.put(("error", str(e)))
            return req
        self.waiting.put(req)
        return req

    def _link_waits_for_compile(self, req: Request) -> bool:
        """A Link naming a key whose Compile is still in flight waits (up to
        ``max_link_waits`` steps) instead of failing with a missing source."""
        keys = (req.pic_link or {}).get("cache_keys") if isinstance(req.pic_link, dict) else None
        if not isinstance(keys, list):
            return False
        waits = getattr(req, "_compile_waits", 0)
        if waits >= self.max_link_waits:
            return False
        if any(isinstance(k, str) and self.compile_states.state(k) == COMPILE_STATE_COMPILING for k in keys):
            req._compile_waits = waits + 1
            return True
        return False

    # ---------------------------------------------------------------- loop
    def start(self) -> None:
        if self._thread is None:
            self._thread = threading.Thread(target=self._loop, name="legolink-scheduler", daemon=True)
            self._thread.start()

    def stop(self) -> None:
        self._stop.set()
        if self._thread is not None:
            self._thread.join(timeout=30)

    def _loop(self) -> None:
        # the current CUDA device is per thread: this one drives the engine's
        # GPU (graph capture, streams and events use the current device)
        dev = getattr(self.engine, "device", None)
        if dev is not None and dev.type == "cuda":
            import torch

            torch.cuda.set_device(dev)
        while not self._stop.is_set():
            did = self.step()
            if not did:
                try:
                    req = self.waiting.get(timeout=0.01)
                    self.waiting.put(req)
                except queue.Empty:
                    pass

    def _next_waiting(self) -> Optional[Request]:
        """Deferred requests first (retracted, same-key Compiles), then the
        queue, then Links parked behind an in-flight Compile of their keys."""
        if self._deferred:
            return self._deferred.pop(0)
        try:
            return self.waiting.get_nowait()
        except queue.Empty:
            pass
        return self._parked.pop(0) if self._parked else None

    def step(self) -> bool:
        """One scheduling iteration; returns False when idle."""
        batch, later = [], []
        for _ in range(self.max_prefills_per_step):
            if len(self.running) + len(batch) >= self.max_running:
                break
            req = self._next_waiting()
            if req is None:
                break
            if req.resume is not None and self.running and not self._fits(req):
                self._deferred.insert(0, req)  # a retracted request waits for pages
                break
            if req.kind == "link" and self._link_waits_for_compile(req) and (
                    batch or not self.waiting.empty() or self._deferred):
                # its source is compiling in this or a queued step
                later.append(req)
                emit_trace("link_deferred_compile_in_flight", rid=req.rid)
                continue
            batch.append(req)
        self._parked.extend(later)
        did = bool(batch) or bool(later)
        if batch:
            self._admit_batch(batch)
        if self.running:
            did = True
            self._decode()
        return did

    def _admit_batch(self, batch: list) -> None:
        """The Compiles and Links admitted in one step share ONE extend
        forward (and the Links one fused KV-link launch per source pool); a
        Compile whose key is already in the batch waits for the next one
        (where it takes the registry's duplicate path).  Plain prefills run
        one by one.  The reference admits a Link alone into an empty engine
        (``managers/scheduler.py:2597-2690``; its trace attributes 97.8 % of
        TTFT at concurrency 8 to that wait, ``pic_runtime.py:2023-2026``).
        Compile race guard: ``pic_compile_key_in_batch``
        ``pic_runtime.py:1954-1975``, ``managers/scheduler.py:2611-2617``."""
        compiles, links, keys = [], [], set()
        for req in batch:
            if req.kind == "link":
                links.append(req)
                continue
            if req.kind != "compile":
                continue
            key = (req.sub_context or {}).get("cache_key")
            if key and str(key) in keys:
                self._deferred.append(req)
                emit_trace("compile_deferred_same_key_in_batch", rid=req.rid, cache_key=str(key))
                continue
            if key:
                keys.add(str(key))
            compiles.append(req)
        if compiles or links:
            self._admit_extend(compiles, links)
        for req in batch:
            if req.kind == "plain":
                self._admit(req)

    def _admit_extend(self, compiles: list, links: list) -> None:
        items, live = [], []
        for req in compiles:
            key = (req.sub_context or {}).get("cache_key")
            if not key:
                req.events.put(("error", "sub_context.cache_key is required for a Compile"))
                continue
            items.append((req.input_ids, str(key), req.sub_context or {}, None))
            live.append(req)
        link_items = [(r.pic_link, r.input_ids, r.rid, r.sampling) for r in links]
        try:
            c_res, l_res = self.engine.extend_step(compiles=items, links=link_items)
        except Exception as e:  # the whole step failed: each request fails alone
            c_res, l_res = [e] * len(items), [e] * len(link_items)
        if len(links) > 1:
            self.stats["batched_links"] = self.stats.get("batched_links", 0) + len(links)
        for req in compiles:
            self.compile_states.finish(req)
        for req, r in zip(live, c_res):
            if isinstance(r, Exception):
                emit_trace("legolink_request_failed_closed", rid=req.rid, kind="compile", reason=str(r)[:500])
                req.events.put(("error", str(r)))
                continue
            req.ttft_s = time.perf_counter() - req.created
            req.events.put(("token", r["first_token"]))
            req.events.put(("done", {"compile": r, "finish_reason": "length"}))
            self.stats["finished"] += 1
        for req, r in zip(links, l_res):
            if isinstance(r, Exception):
                emit_trace("legolink_request_failed_closed", rid=req.rid, kind="link", reason=str(r)[:500])
                req.events.put(("error", str(r)))
                continue
            if r.length + req.max_new_tokens > self.max_context:
                self.engine.free(r)
                msg = "overlength Link (total tokens + max_tokens exceeds the context window)"
                emit_trace("legolink_request_failed_closed", rid=req.rid, kind="link", reason=msg)
                req.events.put(("error", msg))
                continue
            self._start(req, r)

    def _start(self, req: Request, seq: Sequence_) -> None:
        """A prefilled request emits its first token and joins the decode."""
        req.seq = seq
        if req.ttft_s is None:
            req.ttft_s = time.perf_counter() - req.created
        first = seq.output_ids[-1]
        req.events.put(("token", first))
        self.stats["admitted"] += 1
        if len(seq.output_ids) >= req.max_new_tokens or first in req.stop_ids:
            self._finish(req, "stop" if first in req.stop_ids else "length")
        else:
            self.running.append(req)

    def _admit(self, req: Request) -> None:
        eng = self.engine
        try:
            if req.kind == "compile":
                sc = req.sub_context or {}
                key = sc.get("cache_key")
                if not key:
                    raise ContractError("sub_context.cache_key is required for a Compile")
                r = eng.compile(req.input_ids, str(key), sub_context=sc)
                req.ttft_s = time.perf_counter() - req.created
                req.events.put(("token", r["first_token"]))
                req.events.put(("done", {"compile": r, "finish_reason": "length"}))
                self.stats["finished"] += 1
                return
            if req.kind == "link":
                seq = eng.link(req.pic_link, req.input_ids, rid=req.rid, sampling=req.sampling)
                if seq.length + req.max_new_tokens > self.max_context:
                    eng.free(seq)
                    raise RequestRejected("overlength Link (total tokens + max_tokens exceeds the context window)")
            elif req.resume is not None:  # re-admitted after a retraction
                seq = eng.prefill(list(req.input_ids) + list(req.resume), rid=req.rid, sampling=req.sampling)
                seq.output_ids[:0] = req.resume
            else:
                seq = eng.prefill(req.input_ids, rid=req.rid, sampling=req.sampling)
            self._start(req, seq)
        except (ContractError, RuntimeErrorAbort, RequestRejected, ValueError, KeyError) as e:
            emit_trace("legolink_request_failed_closed", rid=req.rid, kind=req.kind, reason=str(e)[:500])
            req.events.put(("error", str(e)))
        except Exception as e:  # keep the loop alive: this request fails, the runtime continues
            emit_trace("legolink_request_failed_closed", rid=req.rid, kind=req.kind, reason=repr(e)[:500])
            req.events.put(("error", f"internal error: {e!r}\n{traceback.format_exc(limit=3)}"))

    LINK_RETRACTED = ("LegoLink request was retracted under KV pressure; its linked KV layout cannot be "
                      "replayed, so it fails closed instead of being re-queued.")

    def _pages_free(self) -> int:
        eng = self.engine
        return (eng.alloc.num_free + eng.radix.evictable_pages() + eng.registry.capacity_evictable_pages())

    def _retract_for(self, steps: int) -> None:
        """Before a decode of ``steps`` tokens: while the running sequences
        need more new pages than the pool can give, retract the most recently
        admitted one.  A Link fails closed (its re-prefill could not rebuild
        the linked layout); a plain request is re-queued and resumes from its
        prompt + generated tokens (reference ``pic_runtime.py:2978-3007``)."""
        ps = self.engine.page_size

        def need():
            return sum(max(0, -(-(r.seq.length + steps) // ps) - len(r.seq.pages)) for r in self.running)

        while len(self.running) > 1 and need() > self._pages_free():
            r = self.running.pop()
            out = list(r.seq.output_ids)
            self.engine.free(r.seq)
            self.stats["retracted"] = self.stats.get("retracted", 0) + 1
            if r.kind == "link":
                emit_trace("legolink_request_failed_closed", rid=r.rid, kind="link", reason="link_request_retracted")
                r.events.put(("error", self.LINK_RETRACTED))
            else:
                emit_trace("request_retracted", rid=r.rid, generated=len(out))
                r.resume, r.seq = out, None
                self._deferred.insert(0, r)

    def _fits(self, req: Request) -> bool:
        n = len(req.input_ids) + len(req.resume or ()) + 1
        return -(-n // self.engine.page_size) <= self._pages_free()

    def _decode(self) -> None:
        eng = self.engine
        k = 1
        if (self.decode_chunk > 1 and self.waiting.empty() and not self._deferred and not self._parked
                and eng.use_cuda_graphs
                and all(r.sampling.greedy for r in self.running)):
            k = min(self.decode_chunk, min(r.max_new_tokens - len(r.seq.output_ids) for r in self.running))
        self._retract_for(max(1, k))
        seqs = [r.seq for r in self.running]
        if k >= 2:
            # nothing is waiting: k steps back to back on the device, tokens
            # streamed when the chunk returns
            before = [len(r.seq.output_ids) for r in self.running]
            try:
                eng.decode_chained(seqs, k, [set(int(t) for t in r.stop_ids) for r in self.running])
            except Exception as e:
                for r in self.running:
                    r.events.put(("error", f"decode failed: {e!r}"))
                    self.engine.free(r.seq)
                self.running = []
                return
            self.stats["decode_steps"] += k
            still = []
            for r, b0 in zip(self.running, before):
                for t in r.seq.output_ids[b0:]:
                    r.events.put(("token", int(t)))
                if r.seq.finished:
                    self._finish(r, "stop")
                elif len(r.seq.output_ids) >= r.max_new_tokens:
                    self._finish(r, "length")
                else:
                    still.append(r)
            self.running = still
            return
        try:
            toks = self.engine.decode_step(seqs)
        except Exception as e:
            for r in self.running:
                r.events.put(("error", f"decode failed: {e!r}"))
                self.engine.free(r.seq)
            self.running = []
            return
        self.stats["decode_steps"] += 1
        still = []
        for r, t in zip(self.running, toks):
            r.seq.output_ids.append(int(t))
            r.events.put(("token", int(t)))
            n = len(r.seq.output_ids)
            if int(t) in r.stop_ids:
                self._finish(r, "stop")
            elif n >= r.max_new_tokens:
                self._finish(r, "length")
            else:
                still.append(r)
        self.running = still

    def _finish(self, req: Request, reason: str) -> None:
        info = {"finish_reason": reason, "completion_tokens": len(req.seq.output_ids) if req.seq else 0,
                "prompt_tokens": req.seq.length - len(req.seq.output_ids) + 1 if req.seq else len(req.input_ids)}
        if req.seq is not None:
            if req.seq.link_plan is not None:
                info["link"] = {"total_token_count": req.seq.link_plan.total_token_count,
                                "recompute_rows": len(req.seq.link_plan.recompute_positions)}
            self.engine.free(req.seq)
        req.events.put(("done", info))
        self.stats["finished"] += 1

    # ------------------------------------------------------------ helpers
    def run_sync(self, req: Request, timeout: float = 600.0) -> dict:
        """Submits and drains one request (for in-process callers/tests)."""
        self.submit(req)
        toks = []
        while True:
            if self._thread is None:
                self.step()
                try:
                    kind, val = req.events.get_nowait()
                except queue.Empty:
                    continue
            else:
                kind, val = req.events.get(timeout=timeout)
            if kind == "token":
                toks.append(val)
            elif kind == "done":
                return {"tokens": toks, **val, "ttft_s": req.ttft_s}
            else:
                raise RequestRejected(val)
