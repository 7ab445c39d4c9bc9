"""Link plan resolution: the runtime derives every physical consequence of a
host's reuse intent (reference ``pic_runtime.py:3032-3324`` and
``ResolvedLinkPlan`` ``:1163-1220``).

Layout of a resolved Link (token positions)::

    [ chat prefix | block 0 | (fresh gap 0) | block 1 | ... | block n-1 | mutable suffix ]

``recompute_positions`` (= ``imp_indices``) = the whole prefix + the first
``K_i`` tokens of each block + every inter-block fresh gap + the whole mutable
suffix.  Everything else is linked KV, re-rotated from its Compile position
(block-local, starting at 0) to its global position.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any, Callable, Optional, Sequence

import os

from ..contract import (
    PIC_LINK_RECOMPUTE_MODES,
    ContractError,
    env_flag,
    physical_token_ids_sha256,
    validate_physical_token_input,
    validate_pic_link_request,
)


class LinkPlanError(ContractError):
    pass


@dataclass(frozen=True)
class BlockRange:
    block_id: str
    cache_key: str
    start_token: int
    end_token: int

    @property
    def token_count(self) -> int:
        return self.end_token - self.start_token

    def to_dict(self) -> dict:
        return {
            "block_id": self.block_id,
            "cache_key": self.cache_key,
            "start_token": self.start_token,
            "end_token": self.end_token,
            "token_count": self.token_count,
        }


@dataclass(frozen=True)
class ResolvedLinkPlan:
    cache_keys: tuple[str, ...]
    block_ranges: tuple[BlockRange, ...]
    mutable_start_token: int
    mutable_token_count: int
    physical_prefix_token_count: int
    total_token_count: int
    recompute_positions: tuple[int, ...]
    recompute_tokens_per_block: tuple[int, ...]
    recompute_first_block: bool
    recompute_initial_tokens: int
    token_layout_source: str
    linked_token_ids: tuple[int, ...]
    recompute_mode: str = "batched"
    fresh_gap_ranges: tuple[tuple[int, int, int], ...] = ()

    def apply_to(self, plan: dict) -> None:
        """Publishes the resolved fields into the request dict under the keys
        the rest of a runtime reads (``imp_indices`` and ``kvlink`` are both
        names for ``recompute_positions``)."""
        ranges = [b.to_dict() for b in self.block_ranges]
        pos = list(self.recompute_positions)
        plan["block_ranges"] = ranges
        plan["attention_ranges"] = ranges
        plan["mutable_start_token"] = self.mutable_start_token
        plan["mutable_token_count"] = self.mutable_token_count
        plan["physical_prefix_token_count"] = self.physical_prefix_token_count
        plan["total_token_count"] = self.total_token_count
        plan["kvlink"] = pos
        plan["legolink_k"] = self.recompute_initial_tokens
        plan["recompute_first_block"] = self.recompute_first_block
        plan["recompute_first_block_tokens"] = self.recompute_tokens_per_block[0]
        plan["recompute_tokens_per_block"] = list(self.recompute_tokens_per_block)
        plan["imp_indices"] = pos
        plan["recompute_positions"] = pos
        plan["token_layout_source"] = self.token_layout_source

    def linked_rows(self) -> list[tuple[str, int, int]]:
        """(cache_key, local_start, global_start, count) runs of linked (not
        recomputed) tokens; used to build the KV link gather."""
        import numpy as np

        rec = np.zeros(self.total_token_count + 1, dtype=np.bool_)
        if self.recompute_positions:
            rec[np.asarray(self.recompute_positions, dtype=np.int64)] = True
        runs = []
        for b in self.block_ranges:
            linked = ~rec[b.start_token:b.end_token]
            if not linked.any():
                continue
            edges = np.flatnonzero(np.diff(np.concatenate(([False], linked, [False])).astype(np.int8)))
            for i, j in zip(edges[0::2].tolist(), edges[1::2].tolist()):
                runs.append((b.cache_key, i, b.start_token + i, j - i))
        return runs


def indexed_mixed_prefill_enabled() -> bool:
    return env_flag("SGLANG_PIC_EXPERIMENTAL_INDEXED_MIXED_PREFILL")


def _split_fresh_gaps(plan: dict, post_prefix: list[int], nblocks: int):
    raw = plan.get("physical_interblock_fresh_token_counts")
    if raw is None:
        return [[] for _ in range(max(nblocks - 1, 0))], list(post_prefix)
    if not indexed_mixed_prefill_enabled():
        raise LinkPlanError(
            "pic_link.physical_interblock_fresh_token_counts is experimental; set "
            "SGLANG_PIC_EXPERIMENTAL_INDEXED_MIXED_PREFILL=1 to allow fresh tokens between cached blocks."
        )
    if (not isinstance(raw, list) or len(raw) != nblocks - 1
            or any(isinstance(v, bool) or not isinstance(v, int) or v < 0 for v in raw)):
        raise LinkPlanError(
            "pic_link.physical_interblock_fresh_token_counts must hold one non-negative token count between "
            "each pair of consecutive blocks."
        )
    if plan.get("promote_reconstructed_group") and any(raw):
        raise LinkPlanError("A Link with fresh tokens between cached blocks cannot be promoted as a group.")
    runs, cur = [], 0
    for c in raw:
        runs.append(list(post_prefix[cur : cur + c]))
        cur += c
    if cur >= len(post_prefix):
        raise LinkPlanError("pic_link.physical_interblock_fresh_token_counts must leave a non-empty mutable suffix.")
    return runs, list(post_prefix[cur:])


def resolve_link_plan(plan: dict, mutable_input_ids: Sequence[int],
                      block_tokens: Callable[[str], Optional[Sequence[int]]], *, validate: bool = True,
                      profile=None, require_formal=None) -> ResolvedLinkPlan:
    """Builds the authoritative layout.  ``block_tokens(cache_key)`` returns
    the registered token ids of a block (None when not compiled here)."""
    if validate:
        validate_pic_link_request(plan, profile=profile, require_formal=require_formal)
    keys = [str(k) for k in plan["cache_keys"]]
    normalized = plan.get("physical_token_layout_version") is not None
    validated = validate_physical_token_input(plan, label="pic_link")
    ids = list(map(int, mutable_input_ids))
    if normalized:
        if validated is None:
            raise LinkPlanError("normalized pic_link is missing physical_input_ids.")
        if ids != validated:
            raise LinkPlanError("Link request tokens differ from the validated physical_input_ids override.")
        pc = plan.get("physical_prefix_token_count")
        if isinstance(pc, bool) or not isinstance(pc, int) or pc < 0 or pc >= len(ids):
            raise LinkPlanError("pic_link.physical_prefix_token_count must split a non-empty physical Link input.")
        prefix, post = ids[:pc], ids[pc:]
        segs = plan.get("physical_block_segments")
        if not isinstance(segs, list) or len(segs) != len(keys) or any(not isinstance(s, dict) for s in segs):
            raise LinkPlanError("pic_link.physical_block_segments must contain one metadata object per cache key.")
        gaps, suffix = _split_fresh_gaps(plan, post, len(keys))
    else:
        if plan.get("physical_interblock_fresh_token_counts") is not None:
            raise LinkPlanError("Fresh tokens between cached blocks require the normalized physical token layout.")
        prefix, suffix, segs = [], ids, []
        gaps = [[] for _ in range(max(len(keys) - 1, 0))]

    if plan.get("execution_mode") == "formal":
        k_init = int(plan["repair_decision"]["selected_k"])
    else:
        k_init = int(plan.get("recompute_initial_tokens", plan.get("legolink_k", 16)))
    if k_init < 0:
        raise LinkPlanError("recompute_initial_tokens must be non-negative.")
    raw_pb = plan.get("recompute_tokens_per_block")
    if raw_pb is not None:
        if not isinstance(raw_pb, list) or len(raw_pb) != len(keys):
            raise LinkPlanError("pic_link.recompute_tokens_per_block must contain one value per cache key.")
        per_block = [int(v) for v in raw_pb]
        if any(v < 0 for v in per_block):
            raise LinkPlanError("pic_link.recompute_tokens_per_block values must be non-negative.")
    else:
        first = plan.get("recompute_first_block_tokens")
        if first is None:
            first = k_init if bool(plan.get("recompute_first_block", False)) else 0
        first = int(first)
        if first < 0:
            raise LinkPlanError("pic_link.recompute_first_block_tokens must be non-negative.")
        per_block = [first if i == 0 else k_init for i in range(len(keys))]

    full = list(prefix)
    recompute = list(range(len(prefix)))
    block_ids = plan.get("block_ids") or []
    ranges: list[BlockRange] = []
    fresh = []
    for i, key in enumerate(keys):
        toks = block_tokens(key)
        if toks is None:
            raise LinkPlanError(f"PIC block is not compiled in this scheduler: {key}")
        if not isinstance(toks, tuple):  # the engine hands out tuples of ints already
            toks = tuple(map(int, toks))
        if normalized:
            seg = segs[i]
            if str(seg.get("cache_key")) != key:
                raise LinkPlanError(
                    f"physical block segment order/cache key mismatch: expected {key}, got {seg.get('cache_key')!r}")
            ec = seg.get("physical_token_count")
            if isinstance(ec, bool) or not isinstance(ec, int) or ec != len(toks):
                raise LinkPlanError(f"physical block token count mismatch for {key}: expected={ec!r}, "
                                    f"actual={len(toks)}")
            eh = seg.get("physical_token_ids_sha256")
            ah = physical_token_ids_sha256(toks)
            if not isinstance(eh, str) or eh != ah:
                raise LinkPlanError(f"physical block token hash mismatch for {key}: expected={eh!r}, actual={ah}")
        start = len(full)
        full.extend(toks)
        end = len(full)
        ranges.append(BlockRange(str(block_ids[i]) if i < len(block_ids) else key, key, start, end))
        if per_block[i]:
            recompute.extend(range(start, min(start + per_block[i], end)))
        if i < len(gaps) and gaps[i]:
            g0 = len(full)
            full.extend(gaps[i])
            recompute.extend(range(g0, len(full)))
            fresh.append((i, g0, len(full)))
    mstart = len(full)
    full.extend(suffix)
    recompute.extend(range(mstart, len(full)))
    if not suffix:
        raise LinkPlanError("PIC link requires a non-empty mutable query.")
    if normalized:
        ec = plan.get("expected_complete_token_count")
        if isinstance(ec, bool) or not isinstance(ec, int) or ec != len(full):
            raise LinkPlanError(f"normalized Link complete token count mismatch: expected={ec!r}, actual={len(full)}")
        eh = plan.get("expected_complete_token_ids_sha256")
        ah = physical_token_ids_sha256(full)
        if not isinstance(eh, str) or eh != ah:
            raise LinkPlanError(f"normalized Link complete token hash mismatch: expected={eh!r}, actual={ah}")
    mode = str(plan.get("recompute_mode") or os.getenv("SGLANG_PIC_RECOMPUTE_MODE", "batched")).strip().lower()
    if mode not in PIC_LINK_RECOMPUTE_MODES:
        raise LinkPlanError(f"recompute mode {mode!r} (SGLANG_PIC_RECOMPUTE_MODE) is not one of "
                            + ", ".join(sorted(PIC_LINK_RECOMPUTE_MODES)))
    # batched and tokenwise recompute the same rows: one layer-outer pass over
    # them is equal to the row-by-row order; full_causal recomputes every row
    if mode == "full_causal":
        recompute = list(range(len(full)))
    return ResolvedLinkPlan(
        cache_keys=tuple(keys),
        block_ranges=tuple(ranges),
        mutable_start_token=mstart,
        mutable_token_count=len(suffix),
        physical_prefix_token_count=len(prefix),
        total_token_count=len(full),
        recompute_positions=tuple(recompute),
        recompute_tokens_per_block=tuple(per_block),
        recompute_first_block=per_block[0] > 0,
        recompute_initial_tokens=k_init,
        token_layout_source=("single_chat_template_physical_override" if normalized else "sglang_tokenizer_runtime"),
        linked_token_ids=tuple(full),
        recompute_mode=mode,
        fresh_gap_ranges=tuple(fresh),
    )
