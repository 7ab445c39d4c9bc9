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
  compatibility`` in the c10d store every rank already has (TCPStore), with a
  cross-replica pin counter.  :class:`LocalDirectory` is the same API over a
  dict, for several engines in one process (CPU tests).
* :class:`SharedKVPool` -- the KV pool in symmetric memory
  (``torch.distributed._symmetric_memory``): each rank's pool is mapped into
  every peer's address space, so a peer pool is just a base pointer for the
  link kernel.  Peer reads are plain loads over NVLink (no TMA multicast).

Published blocks stay pinned on their owner (a peer may be reading them at
any time), so the owner never evicts a block another replica can link.
"""

from __future__ import annotations

import json
import threading
from dataclasses import dataclass, field
from typing import Optional

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
    """In-process directory (several engines in one process)."""

    def __init__(self):
        self._blocks: dict[str, str] = {}
        self._pins: dict[str, int] = {}
        self._lock = threading.Lock()

    def publish(self, b: RemoteBlock) -> None:
        with self._lock:
            self._blocks.setdefault(b.cache_key, b.to_json())

    def lookup(self, key: str) -> Optional[RemoteBlock]:
        with self._lock:
            s = self._blocks.get(key)
        return RemoteBlock.from_json(s) if s is not None else None

    def unpublish(self, key: str) -> None:
        with self._lock:
            self._blocks.pop(key, None)

    def pin(self, key: str, delta: int = 1) -> int:
        with self._lock:
            self._pins[key] = self._pins.get(key, 0) + delta
            return self._pins[key]

    def pins(self, key: str) -> int:
        with self._lock:
            return self._pins.get(key, 0)


class BlockDirectory(LocalDirectory):
    """Directory in a ``torch.distributed`` store (shared by all ranks)."""

    def __init__(self, store, prefix: str = "legolink/blocks/"):
        super().__init__()
        self.store = store
        self.prefix = prefix

    def publish(self, b: RemoteBlock) -> None:
        k = self.prefix + b.cache_key
        # compare_set keeps the first publisher: a block compiled on two
        # replicas at once is served by the one that registered first.
        self.store.compare_set(k, "", b.to_json())

    def lookup(self, key: str) -> Optional[RemoteBlock]:
        k = self.prefix + key
        if not self.store.check([k]):
            return None
        raw = self.store.get(k)
        return RemoteBlock.from_json(raw.decode() if isinstance(raw, bytes) else raw) if raw else None

    def unpublish(self, key: str) -> None:
        self.store.delete_key(self.prefix + key)

    def pin(self, key: str, delta: int = 1) -> int:
        return int(self.store.add(self.prefix + "pins/" + key, delta))

    def pins(self, key: str) -> int:
        return int(self.store.add(self.prefix + "pins/" + key, 0))


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
