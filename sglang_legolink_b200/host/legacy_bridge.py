"""Legacy plan-file bridge (kept for replaying pre-contract plans; off the
serving path).

Before the Link contract, the host wrote a complete plan file: the block
selection *and* the physical layout it could only estimate -- block ranges,
the mutable query's start and (estimated) length, and the recompute
positions (``imp_indices``, with ``kvlink`` as an alias used by an earlier
demo).  :func:`build_legacy_link_plan` reproduces that file from block
token counts.  The runtime does not trust it: the contract refuses those
runtime-owned fields, and with ``SGLANG_PIC_ALLOW_LEGACY_LINK_FIELDS=1`` it
drops them and derives the layout itself from the registered tokens and the
real query (so an estimate that is off changes nothing).

Reference: ``noc_context_manager/sglang_bridge.py:277-400``.
"""

from __future__ import annotations

import json
from dataclasses import dataclass
from pathlib import Path
from typing import Iterable, Optional

LEGACY_PLAN_VERSION = "legacy-host-plan-v1"


@dataclass(frozen=True)
class LegacyBlock:
    block_id: str
    cache_key: str
    token_count: int


def build_legacy_link_plan(blocks: Iterable[LegacyBlock], *, request_id: str, recompute_initial_tokens: int = 16,
                           recompute_first_block: bool = False, mutable_token_estimate: int = 0) -> dict:
    """A pre-contract plan: selection + host-estimated physical layout."""
    if recompute_initial_tokens < 0:
        raise ValueError("recompute_initial_tokens must be non-negative")
    bl = list(blocks)
    ranges, start = [], 0
    for b in bl:
        ranges.append({"block_id": b.block_id, "cache_key": b.cache_key, "start_token": start,
                       "end_token": start + b.token_count})
        start += b.token_count
    positions = []
    for i, r in enumerate(ranges):
        if i == 0 and not recompute_first_block:
            continue
        n = min(recompute_initial_tokens, r["end_token"] - r["start_token"])
        positions.extend(range(r["start_token"], r["start_token"] + n))
    positions.extend(range(start, start + int(mutable_token_estimate)))
    return {
        "request_id": request_id,
        "cache_keys": [b.cache_key for b in bl],
        "block_ids": [b.block_id for b in bl],
        "recompute_initial_tokens": recompute_initial_tokens,
        "recompute_first_block": recompute_first_block,
        # host estimates of runtime-owned layout
        "attention_ranges": ranges,
        "mutable_start_token": start,
        "mutable_token_count": int(mutable_token_estimate),
        "imp_indices": positions,
        "kvlink": list(positions),
        "token_layout_source": LEGACY_PLAN_VERSION,
    }


def write_plan_file(plan: dict, path) -> Path:
    p = Path(path)
    p.parent.mkdir(parents=True, exist_ok=True)
    p.write_text(json.dumps(plan, separators=(",", ":")), encoding="utf-8")
    return p


def read_plan_file(path) -> dict:
    return json.loads(Path(path).read_text(encoding="utf-8"))
