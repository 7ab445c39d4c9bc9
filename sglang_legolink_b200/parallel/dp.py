"""Data-parallel replicas that share one block registry, and the
cross-replica KV link.

The reference keeps one RadixCache per scheduler, so replicas never share
compiled blocks (reference ``docs/ARCHITECTURE.md:74-75``,
``docs/KNOWN_LIMITATIONS.md:18-21``).  Here every replica (one process per
GPU) publishes its compiled blocks in a :class:`BlockDirectory`; a Link on
replica ``r`` that names a block compiled on replica ``p`` reads it straight
out of ``p``'s KV pool over NVLink inside the fused link kernel (gather +
RoPE delta + scatter into ``r``'s request pages in one pass), so a block is
compiled once for the whole node.

* :class:`BlockDirectory` -- ``cache_key -> owner, pages, token ids,
  compatibility`` in the c10d store every rank already has (TCPStore).
  :class:`LocalDirectory` is the same API over a dict, for several engines
  in one process (CPU tests).
* :class:`DirectoryClient` -- one replica's view of the directory: entries
  are cached and re-validated once per owner per Link, so a Link costs a
  fixed three store round trips per peer owner whatever its block count.
* :class:`SharedKVPool` -- the KV pool in symmetric memory
  (``torch.distributed._symmetric_memory``): each rank's pool is mapped into
  every peer's address space, so a peer pool is just a base pointer for the
  link kernel.  Peer reads are plain loads over NVLink (no TMA multicast).

Eviction of a published block (the reference's capacity eviction,
``radix_cache.py:1937-1989``, extended across replicas) is a grace period in
the manner of read-copy-update:

1. every reader counts the Links it *began* and *ended* (two counters per
   reader rank); a Link increments ``begun`` before it reads the owner's
   generation and ``ended`` after its link kernel has finished reading;
2. the owner withdraws a block by deleting its entry and bumping its own
   generation, then snapshots every reader's ``begun`` and waits (bounded)
   until each reader's ``ended`` has caught up with the snapshot;
3. a Link that began after the withdrawal sees the new generation, re-reads
   its cached entries and finds the block gone: it aborts with the
   residency-recovery refusal (``missing``), never with stale KV.

A Link that began before the withdrawal holds the grace period open until
it ends, so the owner frees the pages only after every peer read of them has
completed.  If the grace period does not close in time (a reader died in
the middle of a Link) the owner publishes the block again and keeps it.
"""

from __future__ import annotations

import json
import threading
import time
from dataclasses import dataclass
from typing import Iterable, Optional

import torch


@dataclass(frozen=True)
class RemoteBlock:
    owner: int
    cache_key: str
    pages: tuple
    first_page_offset: int
    token_ids: tuple
    compat_key: str
    token_hash: str
    page_size: int

    def to_json(self) -> str:
        d = dict(self.__dict__)
        d["pages"], d["token_ids"] = list(self.pages), list(self.token_ids)
        return json.dumps(d, separators=(",", ":"))

    @classmethod
    def from_json(cls, s) -> "RemoteBlock":
        d = json.loads(s)
        d["pages"], d["token_ids"] = tuple(d["pages"]), tuple(d["token_ids"])
        return cls(**d)


class LocalDirectory:
    """In-process directory (several engines in one process).  Replica ranks
    are registered by their :class:`DirectoryClient`."""

    def __init__(self):
        self._blocks: dict[str, str] = {}
        self._counters: dict[str, int] = {}
        self._replicas: set[int] = set()
        self._lock = threading.Lock()

    # ----------------------------------------------------------- entries
    def publish(self, b: RemoteBlock) -> bool:
        """Publishes ``b``; the first publisher of a key keeps it.  Returns
        whether ``b`` is the published entry now."""
        s = b.to_json()
        with self._lock:
            return self._blocks.setdefault(b.cache_key, s) == s

    def lookup(self, key: str) -> Optional[RemoteBlock]:
        with self._lock:
            s = self._blocks.get(key)
        return RemoteBlock.from_json(s) if s is not None else None

    def unpublish(self, key: str, owner: int) -> None:
        """Removes the entry and moves the owner's generation (readers with a
        cached entry of that owner re-validate at their next Link)."""
        with self._lock:
            self._blocks.pop(key, None)
        self.add(f"gen/{owner}", 1)

    # ----------------------------------------------------------- counters
    def add(self, name: str, delta: int) -> int:
        with self._lock:
            v = self._counters.get(name, 0) + int(delta)
            self._counters[name] = v
            return v

    def generation(self, owner: int) -> int:
        return self.add(f"gen/{owner}", 0)

    def register_replica(self, rank: int) -> None:
        with self._lock:
            self._replicas.add(int(rank))

    def replicas(self) -> list[int]:
        with self._lock:
            return sorted(self._replicas)


class BlockDirectory(LocalDirectory):
    """Directory in a ``torch.distributed`` store (shared by all ranks).
    ``world``: the replica ranks are ``0 .. world-1``."""

    def __init__(self, store, prefix: str = "legolink/blocks/", world: Optional[int] = None):
        super().__init__()
        self.store = store
        self.prefix = prefix
        self.world = world

    def publish(self, b: RemoteBlock) -> bool:
        s = b.to_json()
        # compare_set keeps the first publisher: a block compiled on two
        # replicas at once is served by the one that registered first.
        now = self.store.compare_set(self.prefix + b.cache_key, "", s)
        return (now.decode() if isinstance(now, bytes) else now) == s

    def lookup(self, key: str) -> Optional[RemoteBlock]:
        k = self.prefix + key
        if not self.store.check([k]):
            return None
        raw = self.store.get(k)
        return RemoteBlock.from_json(raw.decode() if isinstance(raw, bytes) else raw) if raw else None

    def unpublish(self, key: str, owner: int) -> None:
        self.store.delete_key(self.prefix + key)
        self.add(f"gen/{owner}", 1)

    def add(self, name: str, delta: int) -> int:
        return int(self.store.add(self.prefix + name, int(delta)))

    def register_replica(self, rank: int) -> None:
        if self.world is None:
            self.add(f"replica/{int(rank)}", 1)

    def replicas(self) -> list[int]:
        if self.world is not None:
            return list(range(self.world))
        return self._scan_replicas()

    def _scan_replicas(self) -> list[int]:
        out, r, misses = [], 0, 0
        while misses < 8:  # ranks register densely from 0
            if self.store.check([self.prefix + f"replica/{r}"]):
                out.append(r)
                misses = 0
            else:
                misses += 1
            r += 1
        return out


class DirectoryClient:
    """One replica's view of a (Local|Block)Directory.

    * :meth:`find` -- cached lookup (a store round trip only on a miss);
    * :meth:`begin` / :meth:`end` -- bracket one Link that reads peer blocks:
      ``begin`` counts the Link, reads each peer owner's generation once and
      re-reads the cached entries of owners whose generation moved; blocks
      that are gone or changed come back as ``missing`` / ``stale``;
    * :meth:`withdraw` -- the owner's side of eviction (the grace period in
      the module docstring).
    """

    def __init__(self, directory, rank: int, grace_timeout_s: float = 5.0):
        self.d = directory
        self.rank = int(rank)
        self.grace_timeout_s = grace_timeout_s
        self._cache: dict[str, tuple[RemoteBlock, Optional[int]]] = {}
        self._open = 0
        directory.register_replica(self.rank)

    # ------------------------------------------------------------ reader
    def find(self, key: str) -> Optional[RemoteBlock]:
        hit = self._cache.get(key)
        if hit is not None:
            return hit[0]
        rb = self.d.lookup(key)
        if rb is not None:
            self._cache[key] = (rb, None)  # validated at the next begin()
        return rb

    def forget(self, key: str) -> None:
        self._cache.pop(key, None)

    def begin(self, blocks: dict) -> tuple[dict, list, list]:
        """Opens a Link over ``blocks`` (key -> RemoteBlock from :meth:`find`).
        Returns (validated blocks, missing keys, stale keys); with any missing
        or stale key the Link is already closed again (:meth:`end` is not
        needed)."""
        self.d.add(f"rcu/begun/{self.rank}", 1)
        self._open += 1
        gens: dict[int, int] = {}
        out, missing, stale = {}, [], []
        for key, rb in blocks.items():
            g = gens.get(rb.owner)
            if g is None:
                g = gens[rb.owner] = self.d.generation(rb.owner)
            cached = self._cache.get(key)
            if cached is None or cached[1] != g:
                fresh = self.d.lookup(key)
                if fresh is None:
                    self._cache.pop(key, None)
                    missing.append(key)
                    continue
                self._cache[key] = (fresh, g)
                if (fresh.token_hash, fresh.compat_key) != (rb.token_hash, rb.compat_key):
                    stale.append(key)  # same key, other content: the plan was resolved on the old tokens
                    continue
                rb = fresh  # same content, maybe other pages (withdrawn and compiled again)
            out[key] = rb
        if missing or stale:
            self.end()
        return out, missing, stale

    def end(self) -> None:
        """Closes a Link opened by :meth:`begin` (after its kernel finished)."""
        if self._open > 0:
            self._open -= 1
            self.d.add(f"rcu/ended/{self.rank}", 1)

    # ------------------------------------------------------------- owner
    def publish(self, b: RemoteBlock) -> bool:
        return self.d.publish(b)

    def withdraw(self, b: RemoteBlock, readers: Optional[Iterable[int]] = None) -> bool:
        """Unpublishes ``b`` (owned here) and waits until every Link that may
        have found it has ended.  True: no reader can touch its pages any
        more.  False: the grace period did not close within the timeout; the
        block is published again and must be kept."""
        self.d.unpublish(b.cache_key, b.owner)
        ranks = [r for r in (readers if readers is not None else self.d.replicas())]
        # this replica's own Links are serialised with this call by the
        # engine's lock; only peers can be in flight
        snap = {r: self.d.add(f"rcu/begun/{r}", 0) for r in ranks if r != self.rank}
        deadline = time.monotonic() + self.grace_timeout_s
        pending = dict(snap)
        sleep = 0.0002
        while pending:
            for r in list(pending):
                if self.d.add(f"rcu/ended/{r}", 0) >= pending[r]:
                    del pending[r]
            if not pending:
                break
            if time.monotonic() > deadline:
                self.d.publish(b)
                return False
            time.sleep(sleep)
            sleep = min(sleep * 2, 0.01)
        return True


class SharedKVPool:
    """A KV pool in symmetric memory; interface of ``runtime.engine.KVPool``
    plus :meth:`peer` (the base pointers of another rank's pool)."""

    def __init__(self, num_layers: int, num_pages: int, num_kv_heads: int, page_size: int, head_dim: int,
                 dtype: torch.dtype, device: torch.device, group=None):
        import torch.distributed as dist
        import torch.distributed._symmetric_memory as symm_mem

        from ..ops import _ext

        self.num_pages, self.page_size = num_pages, page_size
        shape = (num_layers, num_pages, num_kv_heads, page_size, head_dim)
        group = group or dist.group.WORLD
        self.k = symm_mem.empty(shape, dtype=dtype, device=device)
        self.v = symm_mem.empty(shape, dtype=dtype, device=device)
        self.k.zero_()
        self.v.zero_()
        gname = group.group_name if hasattr(group, "group_name") else dist.group.WORLD.group_name
        self._hk = symm_mem.rendezvous(self.k, gname)
        self._hv = symm_mem.rendezvous(self.v, gname)
        self.alloc = _ext.host().PageAllocator(num_pages)
        # held for the pool's lifetime, as in KVPool: padded decode rows write here
        self.scratch_page = int(self.alloc.alloc(1)[0])
        self.layer_stride = num_pages * num_kv_heads * page_size * head_dim

    @property
    def bytes(self) -> int:
        return 2 * self.k.numel() * self.k.element_size()

    def peer(self, rank: int) -> tuple[int, int, int, int]:
        return int(self._hk.buffer_ptrs[rank]), int(self._hv.buffer_ptrs[rank]), self.page_size, self.layer_stride
