"""Tensor-parallel serving: rank 0 drives the engine, the other ranks replay.

Every TP rank holds one shard of the model, and each forward carries
collectives, so every rank must run the same engine steps in the same order.
Rank 0 runs the HTTP server and the scheduler; its engine is wrapped in
:class:`SPMDEngine`, which sends each state-changing call (Compile, Link,
prefill, decode, free) to the other ranks over a CPU (gloo) group before
running it itself.  The other ranks sit in :func:`worker_loop` and make the
same call on their own engine.  Sequences cross the wire as integer handles;
token ids, ``pic_link`` payloads and sampling parameters travel as they are
(sent before rank 0 runs the call, so the engine's in-place publication of the
resolved plan never reaches the workers).

After each call every rank contributes whether the call raised; ranks that
disagree (one raised, another did not) leave the group in different states,
so rank 0 raises :class:`TPDivergence` and the server stops taking requests.
With ``SGLANG_PIC_VALIDATE_TP=1`` each Link also all-gathers the per-rank
manifests and checks them (keys, block lengths, offsets, recompute rows,
local lookup).

A sampled request without a seed gets one drawn on rank 0, so every rank
draws the same token from the same (all-gathered) logits.

Reference: upstream SGLang runs one scheduler per TP rank on a CPU group next
to the device group (``RT/managers/scheduler.py:935,1077``); the TP manifest
check is ``pic_runtime.py:1223-1242,3709-3740``.
"""

from __future__ import annotations

import dataclasses
import os
import random
import threading
from datetime import timedelta
from typing import Optional

import torch
import torch.distributed as dist

from .tp import link_manifest, validate_tp_manifests

_SEQ_OPS = ("decode", "decode_chained", "decode_step")


class TPDivergence(RuntimeError):
    """TP ranks finished an engine call differently; their states differ."""


def control_group(timeout_s: float = 365 * 86400.0):
    """A gloo group over all ranks for the control plane.  Workers wait in a
    broadcast while the server is idle, hence the long timeout."""
    return dist.new_group(backend="gloo", timeout=timedelta(seconds=timeout_s))


def _pin_seed(sampling):
    if sampling is None or sampling.greedy or sampling.seed is not None:
        return sampling
    return dataclasses.replace(sampling, seed=random.getrandbits(62))


def _agree(ok: bool, group) -> tuple[bool, bool]:
    """(all ranks ok, all ranks failed)."""
    t = torch.tensor([1 if ok else 0, 0 if ok else 1], dtype=torch.int32)
    dist.all_reduce(t, op=dist.ReduceOp.MIN, group=group)
    return bool(t[0]), bool(t[1])


def _agree_items(oks: list, group) -> bool:
    """True when every rank has the same per-item outcomes."""
    t = torch.tensor([1 if ok else 0 for ok in oks] or [1], dtype=torch.int32)
    lo, hi = t.clone(), t.clone()
    dist.all_reduce(lo, op=dist.ReduceOp.MIN, group=group)
    dist.all_reduce(hi, op=dist.ReduceOp.MAX, group=group)
    return bool(torch.equal(lo, hi))


def _step_oks(out) -> list:
    c_out, l_out = out
    return [not isinstance(r, Exception) for r in list(c_out) + list(l_out)]


def _validate_tp() -> bool:
    return os.getenv("SGLANG_PIC_VALIDATE_TP", "0") == "1"


def check_manifest(seq, group) -> None:
    """All-gathers every rank's manifest of a resolved Link and validates the
    set (every rank sees the same list, so all raise or none does)."""
    out = [None] * dist.get_world_size(group)
    dist.all_gather_object(out, link_manifest(seq.link_plan, seq.link_plan is not None), group=group)
    validate_tp_manifests(out)


class SPMDEngine:
    """Rank 0's engine: forwards state-changing calls to the worker ranks.
    Every other attribute reads the local engine."""

    def __init__(self, engine, group):
        self._engine = engine
        self._group = group
        self._lock = threading.Lock()
        self._next = 0
        self.broken: Optional[str] = None

    def __getattr__(self, name):
        return getattr(self._engine, name)

    def _call(self, op: str, args: tuple, kw: dict, wire_args: Optional[tuple] = None, handle=None):
        with self._lock:
            if self.broken:
                raise TPDivergence(self.broken)
            msg = (op, wire_args if wire_args is not None else args, dict(kw, _handle=handle))
            dist.broadcast_object_list([msg], src=0, group=self._group)
            ok, err, out = True, None, None
            try:
                if op == "check_manifest":
                    check_manifest(args[0], self._group)
                else:
                    out = getattr(self._engine, op)(*args, **kw)
            except Exception as e:  # every rank reports before anyone raises
                ok, err = False, e
            all_ok, all_failed = _agree(ok, self._group)
            if not (all_ok or all_failed):
                self.broken = f"TP ranks diverged on {op}: rank 0 {'ok' if ok else 'raised ' + repr(err)}"
                raise TPDivergence(self.broken)
            if err is not None:
                raise err
            return out

    def _seq_call(self, op, args, kw):
        self._next += 1
        h = self._next
        if kw.get("sampling") is not None:
            kw = dict(kw, sampling=_pin_seed(kw["sampling"]))
        seq = self._call(op, args, kw, handle=h)
        seq._spmd_handle = h
        if op == "link" and _validate_tp():
            try:
                self._call("check_manifest", (seq,), {}, wire_args=(h,))
            except Exception:
                self.free(seq)
                raise
        return seq

    def link(self, pic_link, mutable_input_ids, **kw):
        return self._seq_call("link", (pic_link, list(mutable_input_ids)), kw)

    def prefill(self, token_ids, **kw):
        return self._seq_call("prefill", (list(token_ids),), kw)

    def compile(self, token_ids, cache_key, **kw):
        return self._call("compile", (list(token_ids), cache_key), kw)

    def compile_batch(self, items):
        return self._call("compile_batch", (list(items),), {})

    def extend_step(self, compiles=(), links=(), timer=None):
        """One batched Compile + Link step on every rank.  Items fail alone,
        so the ranks agree item by item; a Link that succeeded everywhere
        gets a handle the workers know it by."""
        with self._lock:
            if self.broken:
                raise TPDivergence(self.broken)
            compiles = [tuple(c) for c in compiles]
            items, handles = [], []
            for it in links:
                pic_link, ids, rid, sampling = (tuple(it) + (None, None))[:4]
                self._next += 1
                handles.append(self._next)
                items.append((pic_link, list(ids), rid, _pin_seed(sampling)))
            wire = (compiles, [(dict(p), i, r, sp) for p, i, r, sp in items])
            dist.broadcast_object_list([("extend_step", wire, {"_handles": handles})], src=0, group=self._group)
            try:
                out = self._engine.extend_step(compiles=compiles, links=items)
            except Exception as e:  # noqa: BLE001 - the whole step failed alone on this rank
                out = ([e] * len(compiles), [e] * len(items))
            if not _agree_items(_step_oks(out), self._group):
                self.broken = "TP ranks diverged on extend_step"
                raise TPDivergence(self.broken)
            for h, seq in zip(handles, out[1]):
                if not isinstance(seq, Exception):
                    seq._spmd_handle = h
        if _validate_tp():
            for i, seq in enumerate(out[1]):
                if isinstance(seq, Exception):
                    continue
                try:
                    self._call("check_manifest", (seq,), {}, wire_args=(seq._spmd_handle,))
                except Exception as e:  # noqa: BLE001
                    self.free(seq)
                    out[1][i] = e
        return out

    def free(self, seq):
        return self._call("free", (seq,), {}, wire_args=(seq._spmd_handle,))

    def _seqs(self, op, seqs, *rest):
        return self._call(op, (seqs, *rest), {}, wire_args=([s._spmd_handle for s in seqs], *rest))

    def decode(self, seqs, steps, stop_ids=()):
        return self._seqs("decode", seqs, steps, stop_ids)

    def decode_chained(self, seqs, steps, stop=frozenset()):
        return self._seqs("decode_chained", seqs, steps, stop)

    def decode_step(self, seqs):
        return self._seqs("decode_step", seqs)

    def shutdown(self) -> None:
        with self._lock:
            dist.broadcast_object_list([("shutdown", (), {})], src=0, group=self._group)


def worker_loop(engine, group) -> int:
    """Replays rank 0's engine calls until it sends ``shutdown``; returns the
    number of calls replayed."""
    live: dict = {}
    n = 0
    while True:
        box = [None]
        dist.broadcast_object_list(box, src=0, group=group)
        op, args, kw = box[0]
        if op == "shutdown":
            return n
        n += 1
        if op == "extend_step":
            compiles, links = args
            try:
                out = engine.extend_step(compiles=compiles, links=links)
            except Exception as e:  # noqa: BLE001
                out = ([e] * len(compiles), [e] * len(links))
            for h, seq in zip(kw.get("_handles", ()), out[1]):
                if not isinstance(seq, Exception):
                    live[h] = seq
            _agree_items(_step_oks(out), group)
            continue
        handle = kw.pop("_handle", None)
        ok = True
        try:
            if op in _SEQ_OPS:
                args = ([live[h] for h in args[0]], *args[1:])
            elif op == "free":
                args = (live.pop(args[0]),)
            elif op == "check_manifest":
                args = (live[args[0]],)
            if op == "check_manifest":
                check_manifest(args[0], group)
            else:
                out = getattr(engine, op)(*args, **kw)
                if handle is not None:
                    live[handle] = out
                if op == "decode_step":  # rank 0's caller appends the tokens it returns
                    for s, t in zip(args[0], out):
                        s.output_ids.append(int(t))
        except Exception:
            ok = False
        _agree(ok, group)
