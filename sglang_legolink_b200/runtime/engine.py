"""Single-GPU (or CPU-oracle) execution engine.

Operations (reference call stacks: Compile ``pic_runtime.py:2578-2718,3485``,
Link ``pic_runtime.py:2790-2961,3742-4121``, decode ``model_runner.py:2955``):

* :meth:`Engine.compile`  -- prefill a sub-context alone from position 0 into
  fresh pages and register those pages as a LegoLink block (ownership moves
  to the registry; no copy).
* :meth:`Engine.link`     -- resolve the plan, reserve sources (lookup ->
  pin -> capacity check) *before* allocating request-private pages, gather
  every linked token of every layer with its RoPE delta rotation in one
  kernel launch, recompute all ``imp_indices`` rows in ONE layer-outer
  forward (each layer writes the repaired K/V before its attention, which is
  causal by position over the request's pages), return the first token.
  Sources are unpinned in ``finally``.
* :meth:`Engine.prefill`  -- full prefill (the baseline a Link is compared to).
* :meth:`Engine.decode`   -- batched greedy decode; on CUDA the step is a
  captured CUDA graph per batch-size bucket.
"""

from __future__ import annotations

import math
import threading
import time
from dataclasses import dataclass, field
from typing import Any, Callable, Optional, Sequence

import numpy as np
import torch

from .. import ops
from ..contract import ContractError, physical_token_ids_sha256, residency_recovery_message, \
    validate_physical_token_input, LEGOLINK_POLICY_VERSION
from ..models.qwen import ForwardBatch, QwenModel
from ..ops import _ext
from ..utils import launch_count
from ..utils.trace import emit_trace, CudaTimer
from .link_plan import ResolvedLinkPlan, resolve_link_plan
from .repair_diagnostics import compare_enabled, compare_kv_link
from .sampling import GREEDY, SamplingParams, make_generator, sample_rows


class RuntimeErrorAbort(RuntimeError):
    """A request-scoped failure: the request is aborted, the engine lives on."""


class KernelFault(RuntimeErrorAbort):
    """A kernel recorded an error in the device error word (a bounded wait
    gave up, or an index past its bound was refused): the request that ran
    it fails; the word is cleared, so later requests start clean."""


class LinkSourceUnavailable(RuntimeErrorAbort):
    """A Link source is missing / stale / incompatible; the message carries
    the structured residency-recovery JSON."""

    def __init__(self, message: str, missing=(), stale=(), incompatible=()):
        super().__init__(message)
        self.missing, self.stale, self.incompatible = tuple(missing), tuple(stale), tuple(incompatible)


class CapacityError(RuntimeErrorAbort):
    pass


@dataclass
class Sequence_:
    rid: str
    token_ids: list[int]  # prompt (+ generated) tokens whose KV is resident
    pages: list[int]
    length: int  # tokens with KV written
    output_ids: list[int] = field(default_factory=list)
    kind: str = "plain"
    link_plan: Optional[ResolvedLinkPlan] = None
    timings: dict = field(default_factory=dict)
    finished: bool = False
    sampling: SamplingParams = GREEDY
    generator: Optional[torch.Generator] = None
    promotion: Optional[dict] = None  # record of an experimental group promotion


@dataclass
class _LinkWork:
    """One Link between its reservation and its first token."""
    plan: dict
    resolved: ResolvedLinkPlan
    keys: list
    remote: dict
    pages: list
    rid: str
    sampling: SamplingParams
    generator: Optional[torch.Generator]
    linked_rows: int = 0


def group_promotion_enabled() -> bool:
    """EXPERIMENTAL, off by default.  A Link's reconstructed execution group
    becomes a cache block only when the deployment sets this flag AND the
    request sets ``promote_reconstructed_group`` (neither alone promotes)."""
    from ..contract import env_flag

    return env_flag("SGLANG_PIC_EXPERIMENTAL_GROUP_PROMOTION")


def _pinned_copy(host: np.ndarray, dev) -> torch.Tensor:
    """One pinned staging buffer per dtype and device (grown on demand);
    the copy is asynchronous, and the staging buffer is reused only after the
    previous copy from it has finished."""
    key = (str(host.dtype), str(dev))
    ent = _PINNED.get(key)
    if ent is None or ent[0].numel() < host.size:
        buf = torch.empty(max(host.size, 1 << 16), dtype=torch.from_numpy(host[:0]).dtype, pin_memory=True)
        ent = [buf, None]
        _PINNED[key] = ent
    buf, ev = ent
    if ev is not None:
        ev.synchronize()
    buf[: host.size].numpy()[:] = host
    out = buf[: host.size].to(dev, non_blocking=True)
    ev = torch.cuda.Event()
    ev.record()
    ent[1] = ev
    return out


_PINNED: dict = {}


class KVPool:
    def __init__(self, num_layers: int, num_pages: int, num_kv_heads: int, page_size: int, head_dim: int,
                 dtype: torch.dtype, device: torch.device):
        self.num_pages, self.page_size = num_pages, page_size
        shape = (num_layers, num_pages, num_kv_heads, page_size, head_dim)
        self.k = torch.zeros(shape, dtype=dtype, device=device)
        self.v = torch.zeros(shape, dtype=dtype, device=device)
        self.alloc = _ext.host().PageAllocator(num_pages)
        # Held for the pool's lifetime: padded rows of a decode bucket write
        # their K/V here (never into a live sequence's slot).
        self.scratch_page = int(self.alloc.alloc(1)[0])

    @property
    def bytes(self) -> int:
        return 2 * self.k.numel() * self.k.element_size()

    def slots(self, pages: Sequence[int], positions: torch.Tensor) -> torch.Tensor:
        pt = torch.as_tensor(list(pages), dtype=torch.int64)
        return pt[positions.long() // self.page_size] * self.page_size + positions.long() % self.page_size


def pages_for(n: int, ps: int) -> int:
    return (n + ps - 1) // ps


class Engine:
    def __init__(self, model: QwenModel, *, num_pages: Optional[int] = None, page_size: int = 16,
                 mem_fraction: float = 0.85, max_blocks: Optional[int] = None, max_context: int = 32768,
                 use_cuda_graphs: bool = True, residency: Optional[int] = None, legolink_only: bool = False,
                 compat_overrides: Optional[dict] = None, kv_pool: Optional[KVPool] = None,
                 directory=None, replica_rank: int = 0, peer_pools: Optional[dict] = None):
        self.model = model
        self.cfg = model.cfg
        self.device = model.device
        self.page_size = page_size
        self.max_context = max_context
        self.is_cuda = self.device.type == "cuda"
        model.ensure_rope_positions(max_context + 64)
        if kv_pool is None:
            if num_pages is None:
                num_pages = self._auto_pages(mem_fraction)
            kv_pool = KVPool(self.cfg.num_layers, num_pages, model.hkv, page_size, self.cfg.head_dim, model.dtype,
                             self.device)
        self.kv = kv_pool
        self.alloc = kv_pool.alloc
        h = _ext.host()
        self.residency = residency if residency is not None else (self.device.index or 0)
        if max_blocks is None:  # deployment cap on registered blocks (LRU beyond it)
            import os

            max_blocks = int(os.getenv("SGLANG_PIC_MAX_BLOCKS", "256"))
        self.max_blocks = int(max_blocks)
        self.registry = h.BlockRegistry(self.alloc, self.max_blocks, self.residency)
        self._token_cache: dict = {}  # cache_key -> (content hash, tuple of token ids)
        self._link_side_stream = None  # peer-pool KV links overlap the local one on it
        self.radix = h.RadixIndex(self.alloc, page_size)
        self.legolink_only = legolink_only
        self.compat = self._compat(compat_overrides or {})
        self.use_cuda_graphs = use_cuda_graphs and self.is_cuda
        self.decode_chunk = 64  # greedy steps per chained decode chunk (one host read per chunk)
        self._graphs: dict = {}
        self._graphs_gen = model.buf_generation
        self._lock = threading.RLock()
        self._rid = 0
        self.stats = {"compiles": 0, "links": 0, "prefills": 0, "decode_steps": 0, "remote_blocks_linked": 0}
        # DP replicas sharing compiled blocks: directory of blocks on any
        # replica, and how to reach a peer replica's pool (GPU: base pointers
        # from SharedKVPool.peer; CPU: the peer's (k, v) tensors).
        self.directory = directory
        self.replica_rank = replica_rank
        self.peer_pools = peer_pools if peer_pools is not None else {}
        self._dir = None
        self._published: dict = {}  # cache_key -> RemoteBlock this replica serves to its peers
        if directory is not None:
            from ..parallel.dp import DirectoryClient

            self._dir = DirectoryClient(directory, replica_rank)
        if self.is_cuda:
            ws = ops.workspace(self.device)
            ws.reserve_decode(64 * model.hq, 592, self.cfg.head_dim)
            # split-K partials for M <= 128 rows over the widest weight
            widest = max(2 * model.inter, (model.hq + 2 * model.hkv) * self.cfg.head_dim, self.cfg.hidden_size)
            ws.reserve_gemm(8 * 128 * max(widest, model.lm_head.shape[0]) // 2, 4096)

    def release_graphs(self) -> None:
        """Drops the captured decode graphs.  A TP model's graphs hold NCCL
        calls, which must be released before the process group is destroyed."""
        if self.is_cuda:
            torch.cuda.synchronize(self.device)
        self._graphs.clear()

    # ---------------------------------------------------------------- setup
    def _auto_pages(self, frac: float) -> int:
        c, m = self.cfg, self.model
        per_page = 2 * c.num_layers * m.hkv * self.page_size * c.head_dim * torch.tensor([], dtype=m.dtype).element_size()
        if self.is_cuda:
            free, total = torch.cuda.mem_get_info(self.device)
            budget = int(free * frac) - (2 << 30)
        else:
            budget = 256 << 20
        return max(64, budget // per_page)

    def _compat(self, over: dict) -> dict:
        c = self.cfg
        d = {
            "model_fingerprint": f"{c.name}@{c.fingerprint()}",
            "tokenizer_fingerprint": f"{c.name}:{c.vocab_size}",
            "kv_dtype": str(self.model.dtype),
            "rope_fingerprint": f'{{"max_position_embeddings":{c.max_position_embeddings},"rope_scaling":null,'
                                f'"rope_theta":{c.rope_theta}}}',
            "attention_backend_fingerprint": "sglang_legolink_b200.paged_sm100a",
            "tp_world_size": self.model.tp_size,
            "page_size": self.page_size,
        }
        d.update(over)
        return d

    def compat_key(self, adapter_id=None, segmentation_policy_version=None, legolink_policy_version=None) -> str:
        c = dict(self.compat)
        c["adapter_id"] = str(adapter_id or "none")
        c["segmentation_policy_version"] = str(segmentation_policy_version or "field-first-v1")
        c["legolink_policy_version"] = str(legolink_policy_version or LEGOLINK_POLICY_VERSION)
        return "|".join(f"{k}={c[k]}" for k in sorted(c))

    def next_rid(self, prefix="req") -> str:
        self._rid += 1
        return f"{prefix}-{self._rid}"

    # --------------------------------------------------------------- memory
    def _alloc_pages(self, n: int) -> list[int]:
        if self.alloc.num_free < n:
            self.radix.evict(n - self.alloc.num_free)
        if self.alloc.num_free < n:
            self.registry.evict_for_capacity(n)
        if self.alloc.num_free < n and self._published:
            self._withdraw_published(n)
        if self.alloc.num_free < n:
            raise CapacityError(f"KV pool exhausted: need {n} pages, {self.alloc.num_free} free")
        return list(self.alloc.alloc(n))

    def _published_evictable_pages(self) -> int:
        """Pages of published blocks that only their publication pins."""
        if not self._published:
            return 0
        return sum(p for k, p in self.registry.eviction_candidates(1) if k in self._published)

    def _withdraw_published(self, n: int) -> None:
        """Frees published blocks (lowest keep-value first) until ``n`` pages
        are free: each is withdrawn from the directory and freed only after
        every peer Link that may have found it has ended."""
        for key, _pages in self.registry.eviction_candidates(1):
            if self.alloc.num_free >= n:
                return
            rb = self._published.get(key)
            if rb is None:
                continue
            h = self.registry.handle(key)
            if h["pin_count"] != 1 or h["active_refs"]:
                continue
            if not self._dir.withdraw(rb):
                emit_trace("published_block_withdraw_timeout", cache_key=key)
                continue
            del self._published[key]
            self.registry.unpin([key])
            self.registry.evict_for_capacity(n)
            self.stats["published_blocks_withdrawn"] = self.stats.get("published_blocks_withdrawn", 0) + 1

    def unregister_block(self, cache_key: str) -> bool:
        """Drops a registered block.  A block this replica publishes is first
        withdrawn from the directory (grace period for peer readers); returns
        False when that did not close in time (the block stays)."""
        with self._lock:
            rb = self._published.get(cache_key)
            if rb is not None:
                if not self._dir.withdraw(rb):
                    return False
                del self._published[cache_key]
                self.registry.unpin([cache_key])
            return bool(self.registry.unregister(cache_key))

    def free(self, seq: Sequence_) -> None:
        if seq.pages:
            self.alloc.release(seq.pages)
            seq.pages = []

    def _ensure_capacity(self, seq: Sequence_, new_len: int) -> None:
        need = pages_for(new_len, self.page_size) - len(seq.pages)
        if need > 0:
            seq.pages.extend(self._alloc_pages(need))

    # ----------------------------------------------------------- batch build
    def _extend_batch(self, items: list[tuple[list[int], list[int], list[int], int]],
                      logits_last_only=True) -> ForwardBatch:
        """items: (token_ids_of_rows, positions_of_rows, pages, kv_len).
        The batch's int32 arrays travel in one host->device copy and its
        int64 arrays in another (numpy on the host, views on the device)."""
        ps = self.page_size
        B = len(items)
        max_pages = max(1, max(len(p) for _, _, p, _ in items))
        ids = np.concatenate([np.asarray(t, dtype=np.int32) for t, _, _, _ in items])
        pos = np.concatenate([np.asarray(p, dtype=np.int64) for _, p, _, _ in items])
        counts = np.asarray([len(t) for t, _, _, _ in items], dtype=np.int64)
        qptr = np.concatenate(([0], np.cumsum(counts))).astype(np.int32)
        pt = np.zeros((B, max_pages), dtype=np.int32)
        slots = np.empty(len(pos), dtype=np.int64)
        for b, (_, p, pages, _) in enumerate(items):
            pg = np.asarray(pages, dtype=np.int64)
            pt[b, : len(pg)] = pg
            pp = pos[qptr[b] : qptr[b + 1]]
            slots[qptr[b] : qptr[b + 1]] = pg[pp // ps] * ps + pp % ps
        kvl = np.asarray([kv for _, _, _, kv in items], dtype=np.int32)
        last_rows = (qptr[1:] - 1).astype(np.int64)
        pos32 = pos.astype(np.int32)
        parts32 = [ids, pos32, qptr, pt.reshape(-1), kvl]
        tiles_nsplit = 1
        if self.is_cuda:
            tl = ops.prefill_tiles_np(qptr, pos32, self.model.hq, self.model.hkv, split=True)
            tiles_nsplit = ops.tiles_split_count(tl)
            parts32.append(tl.reshape(-1))
        # every segment starts on a 256-byte boundary: kernels read some of
        # them (the prefill tile list) with 16-byte vector loads
        sizes32 = [a.size for a in parts32]
        starts32 = np.concatenate(([0], np.cumsum([-(-n // 64) * 64 for n in sizes32]))).tolist()
        host32 = np.zeros(starts32[-1], dtype=np.int32)
        for st, a in zip(starts32, parts32):
            host32[st:st + a.size] = a
        n = len(pos)
        off64 = -(-n // 32) * 32
        host64 = np.zeros(off64 + B, dtype=np.int64)
        host64[:n] = slots
        host64[off64:] = last_rows
        dev = self.device
        if self.is_cuda:
            d32 = _pinned_copy(host32, dev)
            d64 = _pinned_copy(host64, dev)
        else:
            d32, d64 = torch.from_numpy(host32), torch.from_numpy(host64)
        view = [d32[st:st + sz] for st, sz in zip(starts32, sizes32)]
        return ForwardBatch(
            mode="extend",
            input_ids=view[0],
            positions=view[1],
            slots=d64[:n],
            q_indptr=view[2],
            page_table=view[3].view(B, max_pages),
            kv_lens=view[4],
            logit_rows=d64[off64:],
            tiles=view[5].view(-1, 4) if self.is_cuda else None,
            tiles_nsplit=tiles_nsplit,
        )

    def _kernel_check(self, what: str) -> None:
        """Reads (and clears) the device error word after a synchronising
        step; a recorded error aborts the request instead of passing silently.
        Kernels that see the word set abandon their work, so an error left
        uncleared would also slow every later kernel down."""
        if not self.is_cuda:
            return
        code = ops.check_errors(self.device)
        if code:
            raise KernelFault(f"{what}: kernel error {code} ({ops.ERROR_NAMES.get(code, 'unknown')})")

    def _sample(self, logits: torch.Tensor, params: Sequence[SamplingParams] = (),
                gens: Sequence[Optional[torch.Generator]] = (), greedy: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Token ids for the rows of ``logits`` (this rank's vocab shard).
        Greedy rows come from the argmax kernel; when any row samples, the
        full-vocab logits are gathered (TP) and those rows are redrawn."""
        with self.model.markers.region("Sampling", logits=logits):
            return self._sample_rows(logits, params, gens, greedy)

    def _sample_rows(self, logits, params, gens, greedy):
        ids = greedy if greedy is not None else self.model.greedy(logits)
        if not any(not p.greedy for p in params):
            return ids
        full = self.model.full_logits(logits[: len(params)])
        drawn = sample_rows(full, list(params), list(gens) or None)
        ids = ids.clone()
        ids[: len(params)] = drawn.to(ids.device)
        return ids

    def _new_sampling(self, sampling: Optional[SamplingParams]):
        sp = sampling or GREEDY
        return sp, make_generator(sp, self.device)

    # --------------------------------------------------------------- compile
    def compile(self, token_ids: Sequence[int], cache_key: str, *, sub_context: Optional[dict] = None,
                block_id: Optional[str] = None) -> dict:
        """Prefill a block alone from position 0 and register it."""
        r = self.compile_batch([(token_ids, cache_key, sub_context, block_id)])[0]
        if isinstance(r, Exception):
            raise r
        return r

    def compile_batch(self, items: Sequence[tuple]) -> list:
        """Several Compiles in one extend forward (each block from position 0
        in its own pages, one logits row per block).  ``items``: (token_ids,
        cache_key, sub_context, block_id).  Returns one result dict or the
        exception per item; an item that fails validation or allocation fails
        alone.  Two Compiles of one key may not share a batch (the scheduler
        defers the second to the next batch, where it takes the duplicate
        path); here that is refused outright.
        Reference: ``pic_compile_key_in_batch``, ``pic_runtime.py:1954-1975``."""
        return self.extend_step(compiles=items)[0]

    @staticmethod
    def storage_mode(sub_context: Optional[dict]) -> str:
        """How a Compile's KV is kept: "reference" (default: the computed
        pages move to the registry) or "clone" (the registry gets a copy in
        fresh pages and the computed pages are released).  Per Compile
        (``pic_storage_mode``) or per deployment (``SGLANG_PIC_STORAGE_MODE``).
        Reference: ``pic_runtime.py:1982-1988`` (mode), ``:3519-3530`` (clone)."""
        import os

        raw = (sub_context or {}).get("pic_storage_mode") or os.getenv("SGLANG_PIC_STORAGE_MODE", "reference")
        mode = str(raw).lower()
        if mode not in ("clone", "reference"):
            raise ContractError("PIC storage mode must be 'clone' or 'reference'.")
        return mode

    def _compile_prepare(self, token_ids, cache_key, sub_context, block_id):
        sc = dict(sub_context or {})
        self.storage_mode(sc)  # validated before any work
        override = validate_physical_token_input(sc, label="sub_context")
        toks = [int(t) for t in (override if override is not None else token_ids)]
        if override is not None and token_ids and list(token_ids) != override:
            raise ContractError("Compile request tokens differ from the validated physical_input_ids override.")
        if not toks:
            raise ContractError("Compile requires a non-empty sub-context.")
        ckey = self.compat_key(sc.get("adapter_id"), sc.get("segmentation_policy_version"),
                               sc.get("legolink_policy_version"))
        return toks, ckey, str(block_id or sc.get("semantic_block_id") or cache_key)

    def _clone_pages(self, pages: list[int]) -> list[int]:
        """Copy whole pages (all layers, K and V) into fresh pages and release
        the originals (checklist K15)."""
        new = self._alloc_pages(len(pages))
        try:
            src = torch.as_tensor(pages, dtype=torch.long, device=self.kv.k.device)
            dst = torch.as_tensor(new, dtype=torch.long, device=self.kv.k.device)
            self.kv.k[:, dst] = self.kv.k[:, src]
            self.kv.v[:, dst] = self.kv.v[:, src]
        except Exception:
            self.alloc.release(new)
            raise
        self.alloc.release(pages)
        return new

    def _compile_register(self, toks, cache_key: str, ckey, bid: str, pages, first: int) -> dict:
        n = len(toks)
        try:
            status = self.registry.register_block(str(cache_key), ckey, physical_token_ids_sha256(toks), toks, pages,
                                                  0, bid)
        except Exception:
            # refused (the key names a block with other content): the
            # registry took nothing, the computed pages go back
            self.alloc.release(pages)
            raise
        self.stats["compiles"] += 1
        if self._dir is not None and status == "registered":
            from ..parallel.dp import RemoteBlock

            rb = RemoteBlock(self.replica_rank, str(cache_key), tuple(int(p) for p in pages), 0,
                             tuple(int(t) for t in toks), ckey, physical_token_ids_sha256(toks), self.page_size)
            if self._dir.publish(rb):
                # a peer may link it at any time: only a withdrawal frees it
                self.registry.pin([str(cache_key)])
                self._published[str(cache_key)] = rb
        emit_trace("compile_registered", cache_key=str(cache_key), token_count=n, status=status)
        return {"cache_key": str(cache_key), "status": status, "token_count": n, "first_token": first}

    def block_tokens(self, cache_key: str, remote: Optional[dict] = None):
        """A registered block's token ids as a tuple of ints.  The converted
        tuple is kept per key with the block's content hash, so a Link over
        blocks it has seen converts no ids (a re-registered key with other
        content has another hash and is fetched again)."""
        h = self.registry.token_hash(cache_key)
        if h is None:
            if remote and cache_key in remote:
                return tuple(remote[cache_key].token_ids)
            return None
        hit = self._token_cache.get(cache_key)
        if hit is not None and hit[0] == h:
            return hit[1]
        t = tuple(int(x) for x in self.registry.tokens(cache_key))
        if len(self._token_cache) >= 4 * max(1, self.max_blocks):
            self._token_cache.pop(next(iter(self._token_cache)))
        self._token_cache[cache_key] = (h, t)
        return t

    # ------------------------------------------------------------------ link
    def resolve(self, pic_link: dict, mutable_input_ids: Sequence[int]) -> ResolvedLinkPlan:
        return resolve_link_plan(pic_link, mutable_input_ids, self.block_tokens)

    def _preflight(self, pic_link: dict) -> dict:
        """Classifies every source before anything is derived from it, so a
        missing / stale / incompatible block aborts with the recovery JSON.
        Returns the sources found on peer replicas (key -> RemoteBlock)."""
        keys = list(dict.fromkeys(str(k) for k in pic_link["cache_keys"]))
        ckey = self.compat_key(pic_link.get("adapter_id"), pic_link.get("segmentation_policy_version"),
                               pic_link.get("legolink_policy_version"))
        res = self.registry.lookup(keys, ckey)
        remote: dict = {}
        if not res["ok"] and self._dir is not None:
            still = []
            for k in res["missing"]:
                rb = self._dir.find(k)
                if rb is not None and rb.owner != self.replica_rank and rb.compat_key == ckey \
                        and (rb.owner in self.peer_pools):
                    remote[k] = rb
                else:
                    still.append(k)
            res["missing"] = still
            res["ok"] = not (still or res["stale"] or res["incompatible"])
        if not res["ok"]:
            emit_trace("legolink_request_failed_closed", reason="scheduler_source_preflight_failed",
                       missing=res["missing"], stale=res["stale"], incompatible=res["incompatible"])
            raise LinkSourceUnavailable(
                residency_recovery_message(res["missing"], res["stale"], res["incompatible"]),
                res["missing"], res["stale"], res["incompatible"])
        return remote

    def reserve_link_sources(self, resolved: ResolvedLinkPlan, pic_link: dict,
                             remote: Optional[dict] = None, extra_pages: int = 0) -> tuple[list[str], dict]:
        """lookup -> pin -> capacity check (reference ``pic_runtime.py:2790-2961``).
        Returns the pinned local keys and the validated peer sources (with a
        grace-period ticket open for them); ``extra_pages`` are pages the same
        batch needs before this Link's own."""
        remote = dict(remote or {})
        keys = [k for k in dict.fromkeys(resolved.cache_keys) if k not in remote]
        ckey = self.compat_key(pic_link.get("adapter_id"), pic_link.get("segmentation_policy_version"),
                               pic_link.get("legolink_policy_version"))
        res = self.registry.lookup(keys, ckey)
        if not res["ok"]:
            emit_trace("legolink_request_failed_closed", reason="scheduler_source_preflight_failed",
                       missing=res["missing"], stale=res["stale"], incompatible=res["incompatible"])
            raise LinkSourceUnavailable(
                residency_recovery_message(res["missing"], res["stale"], res["incompatible"]),
                res["missing"], res["stale"], res["incompatible"])
        self.registry.pin(keys)
        if remote:
            # one grace-period ticket for this Link; entries of owners whose
            # generation moved are re-read (a withdrawn block is missing now)
            valid, missing, stale = self._dir.begin(remote)
            if missing or stale:
                self.registry.unpin(keys)
                emit_trace("legolink_request_failed_closed", reason="scheduler_source_preflight_failed",
                           missing=missing, stale=stale, incompatible=[])
                raise LinkSourceUnavailable(residency_recovery_message(missing, stale, []), missing, stale, ())
            remote = valid
        need = pages_for(resolved.total_token_count, self.page_size) + extra_pages
        allocatable = self.alloc.num_free + self.radix.evictable_pages() + self.registry.capacity_evictable_pages() \
            + self._published_evictable_pages()
        if need > allocatable:
            self.registry.unpin(keys)
            if remote:
                self._dir.end()
            raise CapacityError(
                "LegoLink cannot allocate request-private destination KV without evicting its reserved source "
                f"blocks: required={resolved.total_token_count}, allocatable={allocatable * self.page_size}.")
        return keys, remote

    def _link_rows(self, resolved: ResolvedLinkPlan, dst_pages: list[int], remote: dict) -> dict:
        """(src_slot, dst_slot, local_pos, global_pos) of every linked token
        (recomputed rows are skipped: repair rewrites them), grouped by the
        replica whose pool holds the source block (``None`` = this one)."""
        ps = self.page_size
        groups: dict = {}
        dpg = np.asarray(dst_pages, dtype=np.int64)
        for key, l0, g0, cnt in resolved.linked_rows():
            rb = remote.get(key)
            if rb is None:
                h = self.registry.handle(key)
                pages, off, sps, owner = h["pages"], int(h["first_page_offset"]), ps, None
            else:
                pages, off, sps, owner = rb.pages, rb.first_page_offset, rb.page_size, rb.owner
            spg = np.asarray(pages, dtype=np.int64)
            loc = np.arange(l0, l0 + cnt, dtype=np.int64)
            sl = loc + off
            glob = np.arange(g0, g0 + cnt, dtype=np.int64)
            g = groups.setdefault(owner, ([], [], [], []))
            g[0].append(spg[sl // sps] * sps + sl % sps)
            g[1].append(dpg[glob // ps] * ps + glob % ps)
            g[2].append(loc)
            g[3].append(glob)
        return {o: tuple(np.concatenate(x) for x in g) for o, g in groups.items()}

    def _link_prepare(self, pic_link: dict, mutable_input_ids: Sequence[int], rid: str,
                      sampling: Optional[SamplingParams], extra_pages: int = 0) -> "_LinkWork":
        """Validates, resolves and reserves one Link, then allocates its
        request-private pages.  On failure nothing stays pinned or allocated."""
        from ..contract import validate_pic_link_request

        validate_pic_link_request(pic_link)
        remote = self._preflight(pic_link)
        resolved = resolve_link_plan(pic_link, mutable_input_ids, lambda k: self.block_tokens(k, remote),
                                     validate=False)
        resolved.apply_to(pic_link)
        keys, remote = self.reserve_link_sources(resolved, pic_link, remote, extra_pages)
        try:
            self.registry.acquire(keys)
            try:
                pages = self._alloc_pages(pages_for(resolved.total_token_count, self.page_size))
            except Exception:
                self.registry.release(keys)
                raise
        except Exception:
            self.registry.unpin(keys)
            if remote:
                self._dir.end()
            raise
        sp, gen = self._new_sampling(sampling)
        return _LinkWork(pic_link, resolved, keys, remote, pages, rid, sp, gen)

    def _link_close(self, w: "_LinkWork", ok: bool) -> None:
        """Releases one Link's reservations (after its kernels finished)."""
        self.registry.release(w.keys)
        self.registry.unpin(w.keys)
        if w.remote:
            self._dir.end()  # the link kernel finished reading (the first token is on the host)
            self.stats["remote_blocks_linked"] += len(w.remote)
        if not ok and w.pages:
            self.alloc.release(w.pages)
            w.pages = []

    def _link_account(self, w: "_LinkWork") -> None:
        rec = np.sort(np.asarray(w.resolved.recompute_positions, dtype=np.int64))
        for b in w.resolved.block_ranges:
            recomputed = int(np.searchsorted(rec, b.end_token) - np.searchsorted(rec, b.start_token))
            self.registry.record_execution(b.cache_key, b.token_count - recomputed, recomputed)
        self.stats["links"] += 1

    def link(self, pic_link: dict, mutable_input_ids: Sequence[int], *, rid: Optional[str] = None,
             timer: Optional["CudaTimer"] = None, sampling: Optional[SamplingParams] = None) -> Sequence_:
        """Executes one Link.  Returns a sequence whose KV holds the whole
        linked prompt and whose ``output_ids[0]`` is the first token."""
        out = self.extend_step(links=[(pic_link, mutable_input_ids, rid, sampling)], timer=timer)[1][0]
        if isinstance(out, Exception):
            raise out
        return out

    def link_batch(self, items: Sequence[tuple], timer: Optional["CudaTimer"] = None) -> list:
        """Several Links in one step: every linked token of every Link moves
        in one fused KV-link launch per source pool, and every Link's repair
        rows go through ONE extend forward (per-request pages, positions and
        causal-by-position attention).  ``items``: (pic_link, mutable ids[,
        rid[, sampling]]).  Returns a Sequence_ or the exception per item;
        an item that fails validation, reservation or allocation fails alone."""
        return self.extend_step(links=items, timer=timer)[1]

    def extend_step(self, compiles: Sequence[tuple] = (), links: Sequence[tuple] = (),
                    timer: Optional["CudaTimer"] = None) -> tuple[list, list]:
        """One prefill-type step: the given Compiles and Links share one
        extend forward (one logits row each).  Returns (compile results,
        link results), each a result or the exception per item."""
        with self._lock:
            timer = timer or CudaTimer(enabled=False)
            c_out: list = [None] * len(compiles)
            l_out: list = [None] * len(links)
            # ---- Compiles: validate + allocate
            prepared, seen = [], set()
            for i, it in enumerate(compiles):
                token_ids, cache_key, sub_context, block_id = (tuple(it) + (None, None))[:4]
                try:
                    if str(cache_key) in seen:
                        raise ContractError(f"two Compiles of '{cache_key}' in one batch")
                    seen.add(str(cache_key))
                    toks, ckey, bid = self._compile_prepare(token_ids, cache_key, sub_context, block_id)
                    pages = self._alloc_pages(pages_for(len(toks), self.page_size))
                    prepared.append((i, toks, ckey, bid, str(cache_key), pages))
                except Exception as e:  # noqa: BLE001 - request-scoped
                    c_out[i] = e
            # ---- Links: validate + resolve + reserve + allocate
            works: list = []
            for i, it in enumerate(links):
                pic_link, ids, rid, sampling = (tuple(it) + (None, None))[:4]
                rid = rid or self.next_rid("link")
                try:
                    works.append((i, self._link_prepare(pic_link, ids, rid, sampling)))
                except Exception as e:  # noqa: BLE001 - request-scoped
                    l_out[i] = e
            if not prepared and not works:
                return c_out, l_out
            # ---- device work: fused KV link, then one forward
            try:
                if works:
                    with timer.span("kv_link"):
                        self._run_kv_links([w for _, w in works], timer)
                items, params, gens = [], [], []
                for _, toks, _, _, _, pages in prepared:
                    items.append((toks, list(range(len(toks))), pages, len(toks)))
                    params.append(GREEDY)
                    gens.append(None)
                for _, w in works:
                    rows = list(w.resolved.recompute_positions)
                    items.append(([w.resolved.linked_token_ids[p] for p in rows], rows, w.pages,
                                  w.resolved.total_token_count))
                    params.append(w.sampling)
                    gens.append(w.generator)
                with timer.span("sparse_repair"):
                    fb = self._extend_batch(items)
                    if len(prepared) > 1 and not works:  # grouped execution rows (row-wise compute when enabled)
                        o, ranges = 0, []
                        for _, toks, *_ in prepared:
                            ranges.append({"start": o, "end": o + len(toks)})
                            o += len(toks)
                        fb.repair_meta = {"batch_execution_unit_size": len(prepared), "repair_ranges": ranges}
                    logits = self.model.forward(fb, self.kv)
                    firsts = self._sample(logits, params, gens).tolist()
                self._kernel_check("link" if works else "compile")
            except Exception as e:
                for i, *_rest, pages in prepared:
                    self.alloc.release(pages)
                    c_out[i] = e
                for i, w in works:
                    self._link_close(w, ok=False)
                    l_out[i] = e
                return c_out, l_out
            # ---- Compiles: register
            for (i, toks, ckey, bid, key, pages), first in zip(prepared, firsts):
                try:
                    if self.storage_mode(compiles[i][2] if len(compiles[i]) > 2 else None) == "clone":
                        try:
                            pages = self._clone_pages(pages)
                        except Exception:
                            self.alloc.release(pages)  # no copy: the computed pages go back
                            raise
                    c_out[i] = self._compile_register(toks, key, ckey, bid, pages, int(first))
                except Exception as e:  # noqa: BLE001
                    c_out[i] = e
            # ---- Links: close reservations, account, build sequences
            for (i, w), first in zip(works, firsts[len(prepared):]):
                self._link_close(w, ok=True)
                seq = Sequence_(rid=w.rid, token_ids=list(w.resolved.linked_token_ids), pages=w.pages,
                                length=w.resolved.total_token_count, output_ids=[int(first)], kind="link",
                                link_plan=w.resolved, sampling=w.sampling, generator=w.generator)
                emit_trace("model_link_complete", rid=w.rid, total_token_count=w.resolved.total_token_count,
                           recompute_rows=len(w.resolved.recompute_positions), linked_rows=w.linked_rows,
                           batch_links=len(works))
                # after repair, before decode: a failed promotion costs a
                # trace row, never the answer
                if group_promotion_enabled() and w.plan.get("promote_reconstructed_group"):
                    seq.promotion = self._promote_group(w.resolved, w.pages, w.plan, w.rid)
                w.plan.pop("_scheduler_reserved_cache_keys", None)
                self._link_account(w)
                l_out[i] = seq
            return c_out, l_out

    def _run_kv_links(self, works: list, timer) -> None:
        """One fused KV-link launch per source pool for all ``works``."""
        dev = self.device
        per_owner: dict = {}
        for w in works:
            rows = self._link_rows(w.resolved, w.pages, w.remote)
            w.linked_rows = int(sum(len(g[0]) for g in rows.values()))
            for owner, g in rows.items():
                per_owner.setdefault(owner, []).append(g)
        # Peer pools are read over NVLink and the local pool from HBM: the
        # peer launches go on a side stream so that they overlap the local one
        # (the repair forward after this waits for both).
        side = None
        if self.is_cuda and len(per_owner) > 1:
            if self._link_side_stream is None:
                self._link_side_stream = torch.cuda.Stream(device=dev)
            side = self._link_side_stream
            side.wait_stream(torch.cuda.current_stream(dev))
        for owner, gs in per_owner.items():
            src, dst, lp, gp = (np.concatenate([g[j] for g in gs]) for j in range(4))
            if not src.size:
                continue
            if side is not None and owner is not None:
                with torch.cuda.stream(side):
                    self._launch_kv_link(owner, src, dst, lp, gp, timer)
                continue
            self._launch_kv_link(owner, src, dst, lp, gp, timer)
        if side is not None:
            torch.cuda.current_stream(dev).wait_stream(side)

    def _launch_kv_link(self, owner, src, dst, lp, gp, timer) -> None:
        """One fused KV-link launch for the linked tokens whose source pool
        is ``owner``'s (None: this replica's) on the current stream."""
        dev = self.device
        t = [torch.from_numpy(src), torch.from_numpy(dst), torch.from_numpy(lp.astype(np.int32)),
             torch.from_numpy(gp.astype(np.int32))]
        if self.is_cuda:
            t = [_pinned_copy(x.numpy(), dev) for x in t]
        args = (self.kv.k, self.kv.v, *t, self.model.cos_sin)
        if owner is None:
            with timer.span("kv_link_local"):
                ops.kv_link_rope(*args)
            if compare_enabled("kv_link"):  # diagnostic: fused kernel vs the torch statement
                emit_trace("kv_link_compare", **compare_kv_link(*args))
        elif self.is_cuda:  # peer replica's pool, read over NVLink by the link kernel
            kp, vp, sps, sls = self.peer_pools[owner]
            with timer.span("kv_link_peer"):
                ops.kv_link_rope(*args, src_k_ptr=kp, src_v_ptr=vp, src_page_size=sps, src_layer_stride=sls)
            self.stats["peer_tokens_linked"] = self.stats.get("peer_tokens_linked", 0) + int(src.size)
        else:
            ops.kv_link_rope(*args, src_pools=self.peer_pools[owner])
            self.stats["peer_tokens_linked"] = self.stats.get("peer_tokens_linked", 0) + int(src.size)

    def _promote_group(self, resolved: ResolvedLinkPlan, pages: list[int], plan: dict, rid: str) -> Optional[dict]:
        """EXPERIMENTAL.  Makes a fully reconstructed execution group durable:
        the group's rows (first member's start to last member's end) are
        copied from this request's pages into new cache-owned pages, rotated
        from their global positions back to group-local ones (the inverse of
        the link rotation, done by the same kernel with the two position
        arrays swapped), and registered under ``execution_group_key`` like a
        compiled block, so a later Link of the same members links one block.
        A copy, not a hand-over: the request keeps its own rows and frame.
        Only groups whose members after the first were recomputed in full
        qualify (a partially repaired group is never persisted); an existing
        key wins.  Every refusal or failure is a ``group_promotion_skipped``
        trace row and the request is served regardless.
        Reference: ``pic_runtime.py:5718-6023`` (gate ``:925``)."""

        def skip(reason: str, **details) -> None:
            self.stats["group_promotions_skipped"] = self.stats.get("group_promotions_skipped", 0) + 1
            emit_trace("group_promotion_skipped", rid=rid, reason=reason, **details)
            return None

        key = plan.get("execution_group_key")
        if not isinstance(key, str) or not key.strip():
            return skip("no_execution_group_key")
        key = key.strip()
        ranges = resolved.block_ranges
        if len(ranges) < 2:
            return skip("singleton_group", member_count=len(ranges))
        for i, (b, w) in enumerate(zip(ranges[1:], resolved.recompute_tokens_per_block[1:]), start=1):
            if int(w) < b.token_count:
                return skip("reconstruction_below_promotion_policy", member_index=i, recomputed=int(w),
                            token_count=b.token_count)
        if self.registry.contains(key):
            return skip("already_registered", cache_key=key)
        g0, g1 = ranges[0].start_token, ranges[-1].end_token
        n = g1 - g0
        toks = [int(t) for t in resolved.linked_token_ids[g0:g1]]
        t0 = time.perf_counter()
        try:
            new_pages = self._alloc_pages(pages_for(n, self.page_size))
        except CapacityError:
            return skip("allocation_failed", token_count=n, free_pages=self.alloc.num_free)
        registered = False
        try:
            ps = self.page_size
            glob = np.arange(g0, g1, dtype=np.int64)
            loc = np.arange(n, dtype=np.int64)
            src = np.asarray(pages, dtype=np.int64)[glob // ps] * ps + glob % ps
            dst = np.asarray(new_pages, dtype=np.int64)[loc // ps] * ps + loc % ps
            dev = self.device
            ops.kv_link_rope(self.kv.k, self.kv.v, torch.from_numpy(src).to(dev), torch.from_numpy(dst).to(dev),
                             torch.from_numpy(glob.astype(np.int32)).to(dev),
                             torch.from_numpy(loc.astype(np.int32)).to(dev), self.model.cos_sin)
            ckey = self.compat_key(plan.get("adapter_id"), plan.get("segmentation_policy_version"),
                                   plan.get("legolink_policy_version"))
            status = self.registry.register_block(key, ckey, physical_token_ids_sha256(toks), toks, new_pages, 0,
                                                  key)
            registered = True  # from here the registry owns (or has released) the pages
            if status != "registered":
                return skip("already_registered", cache_key=key)
            self.registry.record_execution(key, 0, n)
        except Exception as e:  # noqa: BLE001 - never fail a served request
            if not registered:
                self.alloc.release(new_pages)
            return skip("promotion_failed", error=str(e)[:300], registered=registered)
        rec = {"cache_key": key, "member_cache_keys": [b.cache_key for b in ranges], "token_count": n,
               "group_start_token": g0, "promotion_elapsed_s": round(time.perf_counter() - t0, 6)}
        self.stats["group_promotions"] = self.stats.get("group_promotions", 0) + 1
        emit_trace("group_promotion_completed", rid=rid, **rec)
        return rec

    # --------------------------------------------------------------- prefill
    def prefill(self, token_ids: Sequence[int], *, rid: Optional[str] = None, namespace: Optional[str] = None,
                use_prefix_cache: bool = False, sampling: Optional[SamplingParams] = None) -> Sequence_:
        """Full prefill of a plain prompt (the baseline of a Link)."""
        with self._lock:
            toks = [int(t) for t in token_ids]
            n = len(toks)
            rid = rid or self.next_rid("prefill")
            cached: list[int] = []
            if use_prefix_cache:
                cached = list(self.radix.match_prefix(namespace or "", toks))
                # keep one token to compute so the last row produces logits
                while cached and len(cached) * self.page_size >= n:
                    cached.pop()
                if cached:
                    self.alloc.incref(cached)
            start = len(cached) * self.page_size
            try:
                pages = cached + self._alloc_pages(pages_for(n, self.page_size) - len(cached))
            except Exception:
                if cached:
                    self.alloc.release(cached)
                raise
            try:
                sp, gen = self._new_sampling(sampling)
                fb = self._extend_batch([(toks[start:], list(range(start, n)), pages, n)])
                logits = self.model.forward(fb, self.kv)
                first = int(self._sample(logits, [sp], [gen])[0].item())
                self._kernel_check("prefill")
            except Exception:
                self.alloc.release(pages)
                raise
            if use_prefix_cache:
                self.radix.insert(namespace or "", toks, pages)
            self.stats["prefills"] += 1
            return Sequence_(rid=rid, token_ids=toks, pages=pages, length=n, output_ids=[first], kind="plain",
                             sampling=sp, generator=gen)

    # ---------------------------------------------------------------- decode
    def decode(self, seqs: list[Sequence_], steps: int, stop_ids: Sequence[int] = ()) -> None:
        """Greedy-decode ``steps`` tokens for every sequence (in place).  The
        last output token of each sequence is fed as the next input."""
        stop = set(int(s) for s in stop_ids)
        done = 0
        while done < steps:
            live = [s for s in seqs if not s.finished]
            if not live:
                break
            if self.use_cuda_graphs and steps - done > 1 and all(s.sampling.greedy for s in live):
                n = min(steps - done, self.decode_chunk if not stop else min(self.decode_chunk, 16))
                self.decode_chained(live, n, stop)
                done += n
                continue
            nxt = self.decode_step(live)
            done += 1
            for s, t in zip(live, nxt):
                s.output_ids.append(int(t))
                if int(t) in stop:
                    s.finished = True

    def warm_decode(self, seqs: list[Sequence_]) -> None:
        """Captures the CUDA graph that a greedy decode of ``seqs`` replays
        (the graph of the bucket of ``len(seqs)`` rows) without generating a
        token, so the first decode of a new batch size does not pay for the
        capture and its two warm-up forwards.  The warm-up writes row 0's
        next KV slot, which the first real step overwrites.  No-op without
        CUDA graphs."""
        if not self.use_cuda_graphs or not seqs:
            return
        with self._lock:
            for s in seqs:
                self._ensure_capacity(s, s.length + 1)
            self._graph(self._bucket(len(seqs)), pages_for(self.max_context, self.page_size), seqs)

    def decode_chained(self, seqs: list[Sequence_], steps: int, stop=frozenset()) -> None:
        """``steps`` greedy decode steps with no host round trip between
        them: capacity for all steps is reserved first, every step's
        positions / slots / lengths are computed on the host and copied to
        the device once, and each step's input ids are the previous step's
        argmax, copied on the device before the graph replays.  The outputs
        are read back once at the end; a sequence that produced a stop token
        keeps the tokens up to it (the rows computed after it are dropped, as
        the per-step loop would never have computed them).  A Compile or Link
        runs only between such chunks: the host waits for the chunk's tokens
        before it returns.  ``stop``: one set of stop ids for all sequences
        or one set per sequence.  Greedy sequences, CUDA graphs only."""
        with self._lock:
            B = len(seqs)
            ps = self.page_size
            for s in seqs:
                self._ensure_capacity(s, s.length + steps)
            bucket = self._bucket(B)
            max_pages = pages_for(self.max_context, ps)
            g = self._graph(bucket, max_pages, seqs)
            ids, _, _, pt, _ = self._decode_inputs(seqs, bucket, max_pages)
            L0 = np.asarray([s.length for s in seqs], dtype=np.int64)
            pos = np.zeros((steps, bucket), dtype=np.int64)
            slots = np.full((steps, bucket), self.kv.scratch_page * ps, dtype=np.int64)
            pos[:, :B] = L0[None, :] + np.arange(steps, dtype=np.int64)[:, None]
            for b, s in enumerate(seqs):
                pg = np.asarray(s.pages, dtype=np.int64)
                pb = pos[:, b]
                slots[:, b] = pg[pb // ps] * ps + pb % ps
            kvl = np.where(np.arange(bucket)[None, :] < B, pos + 1, 1)
            dev = self.device
            d32 = _pinned_copy(np.concatenate([pos.astype(np.int32).reshape(-1), kvl.astype(np.int32).reshape(-1)]),
                               dev)
            d64 = _pinned_copy(slots.reshape(-1), dev)
            dpos = d32[: steps * bucket].view(steps, bucket)
            dkvl = d32[steps * bucket:].view(steps, bucket)
            dslots = d64.view(steps, bucket)
            g["ids"].copy_(ids, non_blocking=True)
            g["pt"].copy_(pt, non_blocking=True)
            hist = torch.empty(steps, bucket, dtype=torch.int32, device=dev)
            for t in range(steps):
                if t > 0:
                    g["ids"].copy_(g["out"])
                g["pos"].copy_(dpos[t])
                g["kvl"].copy_(dkvl[t])
                g["slots"].copy_(dslots[t])
                g["graph"].replay()
                hist[t].copy_(g["out"])
                launch_count.add(g["launches"])
            out = hist[:, :B].t().tolist()
            self._kernel_check("decode")
            stops = stop if isinstance(stop, (list, tuple)) else [stop] * B
            for s, toks, st in zip(seqs, out, stops):
                n = steps
                for j, t in enumerate(toks):
                    if t in st:
                        n = j + 1
                        s.finished = True
                        break
                inputs = [s.output_ids[-1]] + toks[: n - 1]
                s.output_ids.extend(toks[:n])
                s.token_ids.extend(inputs)
                s.length += n
            self.stats["decode_steps"] += steps

    def decode_step(self, seqs: list[Sequence_]) -> list[int]:
        with self._lock:
            B = len(seqs)
            for s in seqs:
                self._ensure_capacity(s, s.length + 1)
            if self.use_cuda_graphs:
                out = self._graph_step(seqs)
            else:
                out = self._eager_step(seqs)
            for s in seqs:
                s.token_ids.append(s.output_ids[-1])
                s.length += 1
            self.stats["decode_steps"] += 1
            return out

    def _decode_inputs(self, seqs, bucket: int, max_pages: int):
        ps = self.page_size
        B = len(seqs)
        ids = torch.zeros(bucket, dtype=torch.int32)
        pos = torch.zeros(bucket, dtype=torch.int32)
        slots = torch.zeros(bucket, dtype=torch.int64)
        pt = torch.zeros(bucket, max_pages, dtype=torch.int32)
        kvl = torch.ones(bucket, dtype=torch.int32)
        for b, s in enumerate(seqs):
            ids[b] = s.output_ids[-1]
            pos[b] = s.length
            slots[b] = s.pages[s.length // ps] * ps + s.length % ps
            pt[b, : len(s.pages)] = torch.as_tensor(s.pages, dtype=torch.int32)
            kvl[b] = s.length + 1
        # padded rows write into the pool's scratch page and attend to 1 key
        # there; no live sequence's slot is touched
        for b in range(B, bucket):
            pt[b, 0] = self.kv.scratch_page
            slots[b] = self.kv.scratch_page * ps
            pos[b] = 0
        return ids, pos, slots, pt, kvl

    def _eager_step(self, seqs) -> list[int]:
        B = len(seqs)
        max_pages = max(len(s.pages) for s in seqs)
        ids, pos, slots, pt, kvl = self._decode_inputs(seqs, B, max_pages)
        dev = self.device
        fb = ForwardBatch(mode="decode", input_ids=ids.to(dev), positions=pos.to(dev), slots=slots.to(dev),
                          q_indptr=torch.arange(B + 1, dtype=torch.int32).to(dev), page_table=pt.to(dev),
                          kv_lens=kvl.to(dev), logit_rows=None)
        logits = self.model.forward(fb, self.kv)
        out = self._sample(logits, [s.sampling for s in seqs], [s.generator for s in seqs]).tolist()
        self._kernel_check("decode")
        return out

    def _bucket(self, B: int) -> int:
        for b in (1, 2, 4, 8, 16, 32, 64):
            if B <= b:
                return b
        return B

    def _graph_step(self, seqs) -> list[int]:
        B = len(seqs)
        bucket = self._bucket(B)
        max_pages = pages_for(self.max_context, self.page_size)
        g = self._graph(bucket, max_pages, seqs)
        ids, pos, slots, pt, kvl = self._decode_inputs(seqs, bucket, max_pages)
        g["ids"].copy_(ids, non_blocking=True)
        g["pos"].copy_(pos, non_blocking=True)
        g["slots"].copy_(slots, non_blocking=True)
        g["pt"].copy_(pt, non_blocking=True)
        g["kvl"].copy_(kvl, non_blocking=True)
        g["graph"].replay()
        launch_count.add(g["launches"])
        if any(not s.sampling.greedy for s in seqs):
            out = self._sample(g["logits"][:B], [s.sampling for s in seqs], [s.generator for s in seqs],
                               greedy=g["out"][:B]).tolist()
        else:
            out = g["out"][:B].tolist()
        self._kernel_check("decode")
        return out

    def _graph(self, bucket: int, max_pages: int, seqs) -> dict:
        """The decode graph of ``bucket`` rows, captured on first use.  The
        graphs point into the model's scratch buffers; when a larger forward
        has since regrown one of them (the old memory is freed), every graph
        is dropped and captured again before it could replay."""
        gen = self.model.buf_generation
        if gen != self._graphs_gen:
            self._graphs.clear()
            self._graphs_gen = gen
        g = self._graphs.get(bucket)
        if g is None:
            g = self._capture(bucket, max_pages, seqs)
            if self.model.buf_generation != gen:  # the capture's warm-up regrew a buffer
                self._graphs.clear()
            self._graphs[bucket] = g
            self._graphs_gen = self.model.buf_generation
        return g

    def _capture(self, bucket: int, max_pages: int, seqs) -> dict:
        dev = self.device
        ids, pos, slots, pt, kvl = self._decode_inputs(seqs, bucket, max_pages)
        st = {"ids": ids.to(dev), "pos": pos.to(dev), "slots": slots.to(dev), "pt": pt.to(dev),
              "kvl": kvl.to(dev)}
        nsplit = ops.decode_splits(bucket, self.model.hkv, self.max_context)
        ops.workspace(dev).reserve_decode(bucket * self.model.hq, nsplit, self.cfg.head_dim)
        fb = ForwardBatch(mode="decode", input_ids=st["ids"], positions=st["pos"], slots=st["slots"],
                          q_indptr=torch.arange(bucket + 1, dtype=torch.int32, device=dev), page_table=st["pt"],
                          kv_lens=st["kvl"], logit_rows=None, decode_nsplit=nsplit)
        out = torch.zeros(bucket, dtype=torch.int32, device=dev)
        # warm-up (allocates the model's scratch buffers outside the graph).
        # Row 0's writes land on the slot it is about to fill, so the real
        # step below overwrites them.
        s = torch.cuda.Stream(device=dev)
        s.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(s):
            for _ in range(2):
                self.model.greedy(self.model.forward(fb, self.kv), out=out)
        torch.cuda.current_stream(dev).wait_stream(s)
        graph = torch.cuda.CUDAGraph()
        # the capture stream belongs to the current device: make it the pool's
        with torch.cuda.device(dev), launch_count.Recorder() as rec, torch.cuda.graph(graph):
            logits = self.model.forward(fb, self.kv)
            self.model.greedy(logits, out=out)
        st.update(graph=graph, out=out, logits=logits, fb=fb, launches=rec.n)
        return st
