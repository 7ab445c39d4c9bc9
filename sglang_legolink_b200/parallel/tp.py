"""Tensor parallelism: process groups and the row-parallel reduction.

The model shards Q/KV heads, the gate/up rows and the down/o_proj columns
across ``tp_size`` ranks (one process per GPU); KV heads are replicated when
``num_kv_heads < tp_size``.  Every rank runs the same engine steps in lockstep
(SPMD), so each rank's KV pool holds only its own heads and the registry's
compatibility key carries ``tp_world_size``.

Communication after o_proj / down_proj (``gemm_allreduce``) and for the
vocab-sharded LM head (``argmax_vocab`` / ``all_gather_vocab``):

* :class:`NcclTPComm` -- local GEMM, then the collective library's
  ``all_reduce`` (the baseline; runs on gloo for CPU tests).

Reference: heads split by ``tp_size`` in ``models/qwen2.py:129-142``, the TP
manifest check ``pic_runtime.py:1223-1242,3709-3740``.
"""

from __future__ import annotations

import os
from dataclasses import dataclass
from typing import Optional

import torch
import torch.distributed as dist

from .. import ops


@dataclass
class TPInfo:
    rank: int = 0
    size: int = 1
    group: Optional[object] = None


def init_from_env(backend: Optional[str] = None, timeout_s: int = 120) -> TPInfo:
    """Initialises the default process group from torchrun's environment."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world == 1:
        return TPInfo()
    if not dist.is_initialized():
        from datetime import timedelta

        be = backend or ("nccl" if torch.cuda.is_available() else "gloo")
        kw = {}
        if be == "nccl":
            kw["device_id"] = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
        dist.init_process_group(be, timeout=timedelta(seconds=timeout_s), **kw)
    return TPInfo(dist.get_rank(), dist.get_world_size(), dist.group.WORLD)


class NcclTPComm:
    """Row-parallel reduction through the collective library (baseline)."""

    name = "nccl"

    def __init__(self, group=None):
        self.group = group
        self.size = dist.get_world_size(group)
        self.rank = dist.get_rank(group)

    def gemm_allreduce(self, x: torch.Tensor, w: torch.Tensor, out: torch.Tensor) -> None:
        ops.linear(x, w, out=out)
        dist.all_reduce(out, group=self.group)

    def all_gather_vocab(self, local: torch.Tensor, vocab: int) -> torch.Tensor:
        parts = [torch.empty_like(local) for _ in range(self.size)]
        dist.all_gather(parts, local.contiguous(), group=self.group)
        return torch.cat(parts, dim=-1)[:, :vocab]

    def argmax_vocab(self, local: torch.Tensor, vocab_start: int) -> torch.Tensor:
        """Greedy token over vocab-sharded logits: each rank contributes its
        local (max, index) pair instead of its logits shard."""
        lf = local.float()
        mx, idx = lf.max(dim=-1)
        pair = torch.stack([mx, (idx + vocab_start).float()], dim=-1)  # [R, 2]
        parts = [torch.empty_like(pair) for _ in range(self.size)]
        dist.all_gather(parts, pair, group=self.group)
        allp = torch.stack(parts, dim=0)  # [tp, R, 2]
        best = allp[:, :, 0].argmax(dim=0)  # the lowest rank wins ties -> smallest token id
        return allp[best, torch.arange(allp.shape[1], device=allp.device), 1].to(torch.int32)

    def barrier(self) -> None:
        dist.barrier(group=self.group)


def validate_tp_manifests(manifests: list[dict]) -> None:
    """Every rank must agree on the logical Link (keys, block lengths, global
    offsets, recompute rows) and resolve every block locally."""
    if not manifests:
        raise RuntimeError("TP validation received no rank manifests.")
    base = manifests[0]
    for r, m in enumerate(manifests):
        for f in ("cache_keys", "block_token_lengths", "destination_global_offsets", "imp_indices"):
            if tuple(m.get(f) or ()) != tuple(base.get(f) or ()):
                raise RuntimeError(f"TP rank {r} disagrees on {f}.")
        if not m.get("local_lookup_success"):
            raise RuntimeError(f"TP rank {r} cannot resolve every local LegoLink block.")


def link_manifest(resolved, lookup_ok: bool) -> dict:
    return {"cache_keys": list(resolved.cache_keys),
            "block_token_lengths": [b.token_count for b in resolved.block_ranges],
            "destination_global_offsets": [b.start_token for b in resolved.block_ranges],
            "imp_indices": list(resolved.recompute_positions), "local_lookup_success": bool(lookup_ok)}


def check_link_across_ranks(resolved, lookup_ok: bool, group=None) -> None:
    """All-gathers the per-rank manifests and validates them
    (``SGLANG_PIC_VALIDATE_TP=1``)."""
    if not dist.is_initialized() or dist.get_world_size(group) == 1:
        return
    out = [None] * dist.get_world_size(group)
    dist.all_gather_object(out, link_manifest(resolved, lookup_ok), group=group)
    validate_tp_manifests(out)
