"""Key-range splits of the prefill attention work list, on the host: the
split-count model keeps one CTA per tile when the tiles already fill the
SMs and splits when a tensor-parallel rank's few KV heads leave SMs idle;
the expanded work list carries every (tile, split) once, longest first."""

import numpy as np
import pytest
import torch

from sglang_legolink_b200 import ops


def _rows(n_ctx, tail, windows):
    rows = set(range(n_ctx - tail, n_ctx))
    for w in windows:
        rows |= set(range(w, min(n_ctx, w + 64)))
    return sorted(rows)


def test_many_tiles_keep_one_item_per_tile():
    rows = _rows(16384, 4000, range(0, 16384, 1400))
    qi = torch.tensor([0, len(rows)])
    t = ops.prefill_tiles(qi, torch.tensor(rows), 28, 4, split=True)
    assert ops.tiles_split_count(t) == 1
    assert torch.equal(t, ops.prefill_tiles(qi, torch.tensor(rows), 28, 4))


@pytest.mark.parametrize("Hq,Hkv", [(16, 2), (8, 1)])
def test_few_tiles_over_a_long_context_are_split(Hq, Hkv):
    rows = _rows(32768, 2400, range(0, 32768, 2100))
    qi = torch.tensor([0, len(rows)])
    t = ops.prefill_tiles(qi, torch.tensor(rows), Hq, Hkv, split=True)
    assert ops.tiles_split_count(t) > 1


def test_expanded_items_cover_every_tile_and_split_once_longest_first():
    rows = _rows(9000, 500, (100, 3000, 6000))
    qi, qp = torch.tensor([0, len(rows)]), torch.tensor(rows)
    base = ops.prefill_tiles(qi, qp, 8, 1).numpy()
    S = 3
    t = ops.prefill_tiles(qi, qp, 8, 1, split=S).numpy().astype(np.int64)
    assert len(t) == S * len(base) and ops.tiles_split_count(t) == S
    y = t[:, 1]
    assert ((y >> 16) == S).all()
    got = sorted((int(r[0]), int(r[1] & 0xFF), int(r[2]), int(r[3]), int((r[1] >> 8) & 0xFF)) for r in t)
    want = sorted((int(r[0]), int(r[1]), int(r[2]), int(r[3]), s) for r in base for s in range(S))
    assert got == want
    nb = t[:, 3] // ops.PREFILL_BLOCK_KEYS + 1
    ch = -(-nb // S)
    size = np.clip(nb - ch * ((y >> 8) & 0xFF), 0, ch)
    assert (np.diff(size) <= 0).all()  # longest item first


def test_forced_split_bounds_and_empty_lists():
    qi, qp = torch.tensor([0, 40]), torch.arange(40)
    with pytest.raises(ValueError):
        ops.prefill_tiles(qi, qp, 8, 1, split=300)
    assert ops.tiles_split_count(ops.prefill_tiles(torch.tensor([0, 0]), torch.zeros(0), 8, 1, split=4)) == 1
    assert ops.prefill_split_count([], 0) == 1


def test_the_workspace_cap_limits_the_split():
    nb = np.full(8, 256)  # 8 tiles of 32K keys: S > 1 pays
    assert ops.prefill_split_count(nb, 1000) > 1
    rows_over_cap = ops.PREFILL_SPLIT_MAX_WS_BYTES // (2 * 520) + 1  # even S = 2 would exceed the cap
    assert ops.prefill_split_count(nb, rows_over_cap) == 1


def test_list_schedule_makespan_places_each_item_on_the_first_free_worker():
    from sglang_legolink_b200.ops import _ext

    h = _ext.host()
    assert h.list_schedule_makespan(np.array([3.0, 3.0, 2.0, 2.0, 2.0]), 2) == 7.0
    assert h.list_schedule_makespan(np.array([5.0]), 148) == 5.0
    assert h.list_schedule_makespan(np.zeros(0), 4) == 0.0
    with pytest.raises(ValueError):
        h.list_schedule_makespan(np.array([1.0]), 0)
    # the model of a launch: 74 long tiles leave half of 148 SMs idle and are split; 600 tiles are not
    assert ops.prefill_split_count(np.full(74, 250), 74 * 256) > 1
    assert ops.prefill_split_count(np.full(600, 250), 600 * 256) == 1
