"""CPU fake-runtime config: Compile -> Link (permuted, RoPE remap, repair)
-> greedy decode, compared with full prefill (torch fp32 oracle path)."""

import pytest
import torch

from sglang_legolink_b200.contract import ContractError, physical_token_ids_sha256
from sglang_legolink_b200.models.config import PRESETS
from sglang_legolink_b200.models.qwen import QwenModel
from sglang_legolink_b200.runtime.engine import Engine, LinkSourceUnavailable
from sglang_legolink_b200.contract import parse_residency_recovery


@pytest.fixture(scope="module")
def world():
    cfg = PRESETS["tiny-qwen2"]
    model = QwenModel.random_init(cfg, seed=0)
    eng = Engine(model, num_pages=1024, page_size=16)
    g = torch.Generator().manual_seed(0)
    lens = {"instruction": 128, "tool_schema": 256, "turn": 64, "tool_output": 512}
    subs = {k: torch.randint(0, 1024, (n,), generator=g).tolist() for k, n in lens.items()}
    for k, t in subs.items():
        eng.compile(t, k)
    suffix = torch.randint(0, 1024, (24,), generator=g).tolist()
    return eng, subs, suffix


def test_full_repair_equals_full_prefill(world):
    eng, subs, suffix = world
    order = ["tool_output", "instruction", "turn", "tool_schema"]
    plan = {"cache_keys": order, "recompute_tokens_per_block": [len(subs[k]) for k in order]}
    seq = eng.link(plan, suffix)
    eng.decode([seq], 32)
    full = eng.prefill(sum((subs[k] for k in order), []) + suffix)
    eng.decode([full], 32)
    assert seq.output_ids == full.output_ids
    eng.free(seq), eng.free(full)


def test_sparse_repair_16_per_boundary_runs(world):
    eng, subs, suffix = world
    order = ["turn", "tool_schema", "instruction", "tool_output"]
    plan = {"cache_keys": order, "recompute_initial_tokens": 16, "recompute_first_block": True}
    seq = eng.link(plan, suffix)
    assert len(plan["imp_indices"]) == 16 * 4 + len(suffix)
    assert plan["total_token_count"] == sum(len(subs[k]) for k in order) + len(suffix)
    eng.decode([seq], 8)
    assert len(seq.output_ids) == 9
    eng.free(seq)


def test_linked_kv_equals_compiled_at_global_position(world):
    """Zero-window Link: linked K rows must equal K computed natively at the
    global position (RoPE delta remap by offset, not by block ordinal)."""
    eng, subs, suffix = world
    order = ["instruction", "turn"]
    plan = {"cache_keys": order, "recompute_tokens_per_block": [0, 0]}
    seq = eng.link(plan, suffix)
    full = eng.prefill(subs["instruction"] + subs["turn"] + suffix)
    ps = eng.page_size
    n0 = len(subs["instruction"])
    # block 1 (turn) sits at offset n0: its first layer K must match the native prefill's layer-0 K
    for p in (n0, n0 + 5, n0 + 63):
        a = eng.kv.k[0][seq.pages[p // ps], :, p % ps]
        b = eng.kv.k[0][full.pages[p // ps], :, p % ps]
        assert torch.allclose(a, b, atol=1e-4), p
    eng.free(seq), eng.free(full)


def test_missing_block_raises_recovery_json(world):
    eng, subs, suffix = world
    with pytest.raises(LinkSourceUnavailable) as ei:
        eng.link({"cache_keys": ["instruction", "nope"]}, suffix)
    d = parse_residency_recovery(str(ei.value))
    assert d["missing"] == ("nope",)


def test_runtime_owned_fields_refused(world):
    eng, subs, suffix = world
    with pytest.raises(ContractError):
        eng.link({"cache_keys": ["instruction"], "imp_indices": [0, 1]}, suffix)
    with pytest.raises(ContractError):
        eng.link({"cache_keys": ["instruction"], "bogus_field": 1}, suffix)


def test_duplicate_compile_keeps_resident(world):
    eng, subs, suffix = world
    r = eng.compile(subs["turn"], "turn")
    assert r["status"] == "duplicate"
    with pytest.raises(ValueError):
        eng.compile(subs["instruction"], "turn")


def test_normalized_layout_hashes_checked(world):
    eng, subs, suffix = world
    prefix = [1, 2, 3]
    ids = prefix + suffix
    order = ["turn", "instruction"]
    full = prefix + subs["turn"] + subs["instruction"] + suffix
    plan = {
        "cache_keys": order,
        "physical_token_layout_version": "noc-single-chat-template-split-v1",
        "physical_input_ids": ids,
        "physical_token_count": len(ids),
        "physical_token_ids_sha256": physical_token_ids_sha256(ids),
        "physical_prefix_token_count": 3,
        "physical_block_segments": [
            {"cache_key": k, "physical_token_count": len(subs[k]),
             "physical_token_ids_sha256": physical_token_ids_sha256(subs[k])} for k in order],
        "expected_complete_token_count": len(full),
        "expected_complete_token_ids_sha256": physical_token_ids_sha256(full),
        "recompute_initial_tokens": 8,
    }
    seq = eng.link(dict(plan), ids)
    assert seq.token_ids == full
    # first block sits behind the prefix: it must be remapped (offset 3, not ordinal 0)
    assert seq.link_plan.block_ranges[0].start_token == 3
    eng.free(seq)
    bad = dict(plan)
    bad["expected_complete_token_ids_sha256"] = "0" * 64
    with pytest.raises(ContractError):
        eng.link(bad, ids)


def test_group_promotion_gated_exact_and_fail_closed(world, monkeypatch):
    """EXPERIMENTAL promotion: off unless the deployment flag AND the request
    ask; a fully reconstructed group becomes one block that links to the same
    answer; partial repair and an existing key are refused."""
    eng, subs, suffix = world
    order = ["instruction", "turn", "tool_schema"]
    plan = {"cache_keys": order, "recompute_tokens_per_block": [0] + [len(subs[k]) for k in order[1:]],
            "promote_reconstructed_group": True, "execution_group_key": "grp-a"}
    monkeypatch.delenv("SGLANG_PIC_EXPERIMENTAL_GROUP_PROMOTION", raising=False)
    seq = eng.link(dict(plan), suffix)
    assert seq.promotion is None and not eng.registry.contains("grp-a")
    eng.free(seq)
    monkeypatch.setenv("SGLANG_PIC_EXPERIMENTAL_GROUP_PROMOTION", "1")
    seq = eng.link(dict(plan), suffix)
    assert seq.promotion["cache_key"] == "grp-a" and eng.registry.contains("grp-a")
    assert seq.promotion["token_count"] == sum(len(subs[k]) for k in order)
    one = eng.link({"cache_keys": ["grp-a"], "recompute_tokens_per_block": [0]}, suffix)
    eng.decode([seq], 8)
    eng.decode([one], 8)
    assert one.output_ids == seq.output_ids
    part = dict(plan, execution_group_key="grp-b", recompute_tokens_per_block=[0, 8, 8])
    s2 = eng.link(part, suffix)
    assert s2.promotion is None and not eng.registry.contains("grp-b")
    s3 = eng.link(dict(plan), suffix)  # the key exists: first registration wins
    assert s3.promotion is None
    for s in (seq, one, s2, s3):
        eng.free(s)


def test_scheduler_batches_compiles_and_defers_same_key(world, monkeypatch):
    """Compiles admitted in one step share one forward; a second Compile of a
    key already in that batch waits for the next batch and takes the
    duplicate path; results match one-by-one Compiles."""
    from sglang_legolink_b200.runtime.scheduler import Request, Scheduler

    eng, subs, suffix = world
    g = torch.Generator().manual_seed(11)
    a = torch.randint(0, 1024, (96,), generator=g).tolist()
    b = torch.randint(0, 1024, (40,), generator=g).tolist()
    calls = []
    orig = eng.extend_step

    def spy(compiles=(), links=(), timer=None):
        calls.append([str(it[1]) for it in compiles])
        return orig(compiles=compiles, links=links, timer=timer)

    monkeypatch.setattr(eng, "extend_step", spy)
    sch = Scheduler(eng, max_prefills_per_step=4)
    reqs = [Request("compile", f"c{i}", toks, 1, sub_context={"cache_key": key})
            for i, (key, toks) in enumerate([("sched-a", a), ("sched-a", a), ("sched-b", b)])]
    for r in reqs:
        sch.submit(r)
    while sch.step():
        pass
    assert calls == [["sched-a", "sched-b"], ["sched-a"]]
    done = []
    for r in reqs:
        ev = []
        while not r.events.empty():
            ev.append(r.events.get_nowait())
        done.append([v for k, v in ev if k == "done"][0]["compile"])
    assert [d["status"] for d in done] == ["registered", "duplicate", "registered"]
    solo = Engine(QwenModel.random_init(PRESETS["tiny-qwen2"], seed=0), num_pages=256, page_size=16)
    assert solo.compile(b, "solo-b")["first_token"] == done[2]["first_token"]
    assert solo.compile(a, "solo-a")["first_token"] == done[0]["first_token"]


def test_rowwise_slices_and_state_capture(world, tmp_path, monkeypatch):
    """Row-wise output projection / FFN over grouped Compile rows (validated
    ranges, observation recorded) match the rows compiled alone; the state
    capture writes every layer, the chosen layer's components and the repair
    rows' K/V."""
    from sglang_legolink_b200.runtime.repair_diagnostics import (RepairRowView, RepairStateCapture,
                                                                 SparseRepairComputeError, rowwise_slices)

    meta = {"batch_execution_unit_size": 2, "repair_ranges": [{"start": 0, "end": 5}, {"start": 5, "end": 9}]}
    monkeypatch.delenv("SGLANG_PIC_SPARSE_REPAIR_ROWWISE_FFN", raising=False)
    assert rowwise_slices(dict(meta), 9, "ffn") == ()
    m = dict(meta, rowwise_ffn_enabled=True)
    assert rowwise_slices(m, 9, "ffn") == (slice(0, 5), slice(5, 9))
    assert m["rowwise_ffn_observed"] and m["rowwise_ffn_lengths"] == [5, 4]
    with pytest.raises(SparseRepairComputeError):
        rowwise_slices(dict(m), 10, "ffn")
    with pytest.raises(SparseRepairComputeError):
        rowwise_slices(dict(meta, rowwise_output_projection_enabled="yes"), 9, "output_projection")

    eng, subs, suffix = world
    g = torch.Generator().manual_seed(12)
    a = torch.randint(0, 1024, (70,), generator=g).tolist()
    b = torch.randint(0, 1024, (33,), generator=g).tolist()
    monkeypatch.setenv("SGLANG_PIC_SPARSE_REPAIR_ROWWISE_FFN", "1")
    monkeypatch.setenv("SGLANG_PIC_SPARSE_REPAIR_ROWWISE_OUTPUT_PROJECTION", "1")
    res = eng.compile_batch([(a, "rw-a", None, None), (b, "rw-b", None, None)])
    solo = Engine(QwenModel.random_init(PRESETS["tiny-qwen2"], seed=0), num_pages=256, page_size=16)
    sb = solo.compile(b, "rw-b")
    assert res[1]["first_token"] == sb["first_token"]
    hb, hs = eng.registry.handle("rw-b"), solo.registry.handle("rw-b")
    def block_k(e, h):  # [L, tokens, Hkv * D] of the block's own slots
        k = e.kv.k[:, list(h["pages"])].permute(0, 1, 3, 2, 4)
        return k.reshape(k.shape[0], -1, k.shape[-2] * k.shape[-1])[:, : len(b)]

    assert torch.allclose(block_k(eng, hb), block_k(solo, hs), atol=1e-4, rtol=1e-4)

    cap = RepairStateCapture(tmp_path / "sparse_repair_state.pt", component_layers=[0])
    eng.model.capture = cap
    try:
        order = ["turn", "instruction"]
        seq = eng.link({"cache_keys": order, "recompute_tokens_per_block": [0, 8]}, suffix)
    finally:
        eng.model.capture = None
    rows = list(seq.link_plan.recompute_positions)
    slots = eng.kv.slots(seq.pages, torch.tensor(rows))
    path = cap.save(eng.kv, slots, rows, [rows], None)
    state = torch.load(path)
    L = eng.model.cfg.num_layers
    assert state["diagnostic_only"] and sorted(state["layer_outputs"]) == list(range(L))
    assert set(state["component_outputs"][0]) == {"pre_attention_norm", "qkv_projection", "rope", "attention",
                                                   "output_projection", "post_attention_norm", "mlp"}
    assert state["repaired_kv"][0]["key"].shape[0] == len(rows)
    view = RepairRowView.of("r", slots.tolist(), rows)
    assert view.token_count == len(rows) and len(view.slot_digest) == 64
    eng.free(seq)


def test_layerwise_markers_label_the_profile(world):
    """With markers on, a Link's profiler trace holds the Attention, FFN,
    LMHead and Sampling regions; off, nothing is pushed."""
    from sglang_legolink_b200.utils.layer_markers import LayerMarkers

    eng, subs, suffix = world
    assert not eng.model.markers.enabled
    eng.model.markers = LayerMarkers(True)
    try:
        with torch.profiler.profile() as prof:
            seq = eng.link({"cache_keys": ["turn", "instruction"], "recompute_tokens_per_block": [0, 4]}, suffix)
        names = {e.name for e in prof.events()}
        pushed = eng.model.markers.pushed
    finally:
        eng.model.markers = LayerMarkers(False)
    eng.free(seq)
    L = eng.model.cfg.num_layers
    assert {"LegoLink::Attention", "LegoLink::FFN", "LegoLink::LMHead", "LegoLink::Sampling"} <= names
    assert pushed == 2 * L + 2


def test_debug_compares_kv_link_and_attention(world, monkeypatch, tmp_path):
    """Diagnostic compares (off by default): the link kernel's rows and the
    repair attention rows against the torch fp32 statements, as trace rows."""
    import json

    eng, subs, suffix = world
    path = tmp_path / "trace.jsonl"
    monkeypatch.setenv("SGLANG_PIC_TRACE_PATH", str(path))
    monkeypatch.setenv("SGLANG_PIC_COMPARE_FUSED_TORCH_KV_LINK", "1")
    monkeypatch.setenv("SGLANG_PIC_COMPARE_NATIVE_REFERENCE_ATTENTION", "1")
    seq = eng.link({"cache_keys": ["tool_output", "turn"], "recompute_tokens_per_block": [0, 8]}, suffix)
    eng.free(seq)
    rows = [json.loads(x) for x in path.read_text().splitlines()]
    kv = [r for r in rows if r.get("event") == "kv_link_compare"]
    at = [r for r in rows if r.get("event") == "repair_attention_compare"]
    assert kv and kv[0]["key"]["allclose_bf16"] and kv[0]["value"]["exact"]
    assert len(at) == eng.model.cfg.num_layers and all(r["allclose_bf16"] for r in at)


def test_compile_clone_storage_mode(world):
    """A clone-mode Compile registers a copy in fresh pages; linking it gives
    the reference-mode block's answer; unknown modes are refused."""
    eng, subs, suffix = world
    g = torch.Generator().manual_seed(13)
    t = torch.randint(0, 1024, (50,), generator=g).tolist()
    r1 = eng.compile(t, "clone-ref")
    r2 = eng.compile(t, "clone-copy", sub_context={"pic_storage_mode": "clone"})
    assert r1["first_token"] == r2["first_token"]
    assert set(eng.registry.handle("clone-ref")["pages"]).isdisjoint(eng.registry.handle("clone-copy")["pages"])
    a = eng.link({"cache_keys": ["clone-ref"], "recompute_tokens_per_block": [0]}, suffix)
    b = eng.link({"cache_keys": ["clone-copy"], "recompute_tokens_per_block": [0]}, suffix)
    eng.decode([a], 6)
    eng.decode([b], 6)
    assert a.output_ids == b.output_ids
    with pytest.raises(ContractError):
        eng.compile(t, "clone-bad", sub_context={"pic_storage_mode": "mirror"})
    eng.free(a), eng.free(b)


def test_deployment_flags_are_read_at_call_time(monkeypatch):
    """SGLANG_PIC_LEGOLINK_ONLY (default on) decides per request whether plain
    generation is refused unless the server was given an explicit setting;
    SGLANG_PIC_RECOMPUTE_MODE is the mode of a Link that names none;
    SGLANG_PIC_MAX_BLOCKS caps the registry."""
    from sglang_legolink_b200.runtime.scheduler import Request, RequestRejected, Scheduler

    monkeypatch.setenv("SGLANG_PIC_MAX_BLOCKS", "3")
    e = Engine(QwenModel.random_init(PRESETS["tiny-qwen2"], seed=0), num_pages=256, page_size=16)
    assert e.max_blocks == 3
    for i in range(5):
        e.compile(list(range(10 + i, 40 + i)), f"cap-{i}")
    assert len(e.registry.keys()) == 3  # least recently used beyond the cap are dropped
    sch = Scheduler(e)
    plain = Request("plain", "p", [1, 2, 3], 2)
    monkeypatch.delenv("SGLANG_PIC_LEGOLINK_ONLY", raising=False)
    with pytest.raises(RequestRejected):
        sch.check(plain)
    monkeypatch.setenv("SGLANG_PIC_LEGOLINK_ONLY", "0")
    sch.check(plain)
    with pytest.raises(RequestRejected):
        Scheduler(e, legolink_only=True).check(plain)  # an explicit setting wins
    e.compile(list(range(100, 180)), "rm")
    monkeypatch.setenv("SGLANG_PIC_RECOMPUTE_MODE", "full_causal")
    s = e.link({"cache_keys": ["rm"], "recompute_initial_tokens": 4}, [5, 6])
    assert s.link_plan.recompute_mode == "full_causal" and len(s.link_plan.recompute_positions) == s.length
    e.free(s)
    s = e.link({"cache_keys": ["rm"], "recompute_initial_tokens": 4, "recompute_mode": "batched"}, [5, 6])
    assert s.link_plan.recompute_mode == "batched" and len(s.link_plan.recompute_positions) < s.length
    e.free(s)
    monkeypatch.setenv("SGLANG_PIC_RECOMPUTE_MODE", "sideways")
    with pytest.raises(ContractError):
        e.link({"cache_keys": ["rm"]}, [5, 6])
