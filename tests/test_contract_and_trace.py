"""Request-contract robustness (every malformed ``pic_link`` is refused
before anything runs, and the refusal is request-scoped) and tracing costs
(off: no work and no device read; on: bounded records that never carry
token contents)."""

import json
import time

import pytest
import torch

from sglang_legolink_b200.contract import ContractError, validate_pic_link_request
from sglang_legolink_b200.models.config import PRESETS
from sglang_legolink_b200.models.qwen import QwenModel
from sglang_legolink_b200.runtime.engine import Engine
from sglang_legolink_b200.utils import trace

MALFORMED = {
    "not_an_object": ["a"],
    "keys_not_list": {"cache_keys": "a"},
    "keys_empty": {"cache_keys": []},
    "keys_not_strings": {"cache_keys": [1, 2]},
    "k_negative": {"cache_keys": ["a"], "recompute_initial_tokens": -1},
    "k_bool": {"cache_keys": ["a"], "recompute_initial_tokens": True},
    "k_string": {"cache_keys": ["a"], "recompute_initial_tokens": "8"},
    "k_out_of_range": {"cache_keys": ["a"], "recompute_initial_tokens": 2 ** 40},
    "windows_not_list": {"cache_keys": ["a"], "recompute_tokens_per_block": 3},
    "windows_negative": {"cache_keys": ["a"], "recompute_tokens_per_block": [-1]},
    "mode_unknown": {"cache_keys": ["a"], "recompute_mode": "fancy"},
    "first_block_not_bool": {"cache_keys": ["a"], "recompute_first_block": "yes"},
    "unknown_field": {"cache_keys": ["a"], "foo": 1},
    "runtime_owned_imp_indices": {"cache_keys": ["a"], "imp_indices": [0]},
    "runtime_owned_kvlink": {"cache_keys": ["a"], "kvlink": [1]},
    "formal_without_framing": {"cache_keys": ["a"], "execution_mode": "formal"},
    "more_block_ids_than_keys": {"cache_keys": ["a"], "block_ids": ["x", "y"]},
    "group_key_not_string": {"cache_keys": ["a"], "execution_group_key": 5},
    "promote_not_bool": {"cache_keys": ["a"], "promote_reconstructed_group": "true"},
}


@pytest.mark.parametrize("name", sorted(MALFORMED))
def test_malformed_pic_link_is_refused(name):
    with pytest.raises(ContractError):
        validate_pic_link_request(MALFORMED[name], allow_legacy_fields=False)


@pytest.fixture(scope="module")
def eng():
    e = Engine(QwenModel.random_init(PRESETS["tiny-qwen2"], seed=0), num_pages=256, page_size=16)
    g = torch.Generator().manual_seed(1)
    e.compile(torch.randint(0, 1024, (50,), generator=g).tolist(), "a")
    return e


def test_refusal_is_request_scoped_and_leaves_no_state(eng, monkeypatch):
    monkeypatch.delenv("SGLANG_PIC_ALLOW_LEGACY_LINK_FIELDS", raising=False)
    free0 = eng.alloc.num_free
    for name, plan in MALFORMED.items():
        if not isinstance(plan, dict):
            continue
        with pytest.raises(ContractError):
            eng.link(dict(plan), [1, 2, 3])
        assert eng.alloc.num_free == free0, name  # nothing allocated, nothing pinned
        h = eng.registry.handle("a")
        assert h["active_refs"] == 0 and h["pin_count"] == 0, name
    s = eng.link({"cache_keys": ["a"], "recompute_initial_tokens": 4}, [1, 2, 3])  # still serves
    eng.free(s)


def test_a_block_linked_twice_equals_its_prefill(eng):
    toks = list(eng.block_tokens("a"))
    s = eng.link({"cache_keys": ["a", "a"], "recompute_tokens_per_block": [50, 50]}, [1, 2, 3])
    f = eng.prefill(toks + toks + [1, 2, 3])
    eng.decode([s], 5)
    eng.decode([f], 5)
    assert s.output_ids == f.output_ids and eng.registry.handle("a")["active_refs"] == 0
    eng.free(s), eng.free(f)


def test_tracing_off_does_no_work(monkeypatch):
    monkeypatch.delenv("SGLANG_PIC_TRACE_PATH", raising=False)
    calls = []
    t0 = time.perf_counter()
    for _ in range(20000):
        assert trace.emit_trace("x", lazy=lambda: calls.append(1), big=list(range(1000))) is False
    assert not calls  # lazy values are never evaluated
    assert time.perf_counter() - t0 < 1.0


def test_tracing_on_bounds_records_and_drops_no_fields(monkeypatch, tmp_path):
    path = tmp_path / "t.jsonl"
    monkeypatch.setenv("SGLANG_PIC_TRACE_PATH", str(path))
    monkeypatch.setenv("SGLANG_PIC_TRACE_MAX_ITEMS", "8")
    assert trace.emit_trace("link_done", rows=list(range(1000)), lazy=lambda: 7, t=torch.tensor([1, 2]))
    trace.close_traces()
    rec = json.loads(path.read_text().splitlines()[-1])
    assert rec["event"] == "link_done" and rec["lazy"] == 7 and rec["t"] == [1, 2]
    assert rec["rows"]["count"] == 1000 and len(rec["rows"]["head"]) == 4 and rec["rows"]["tail"][-1] == 999
    assert {"schema_version", "timestamp_unix_s", "timestamp_monotonic_s", "pid", "rank"} <= set(rec)


def test_link_trace_carries_no_token_contents(eng, monkeypatch, tmp_path):
    path = tmp_path / "link.jsonl"
    monkeypatch.setenv("SGLANG_PIC_TRACE_PATH", str(path))
    secret = [1013, 1017, 1019]  # query token ids that must not be written
    s = eng.link({"cache_keys": ["a"], "recompute_initial_tokens": 4}, secret)
    eng.free(s)
    trace.close_traces()
    text = path.read_text()
    assert "model_link_complete" in text
    assert "1013" not in text and "1017" not in text
