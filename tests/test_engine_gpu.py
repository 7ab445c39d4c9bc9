"""End-to-end on the GPU: Compile -> Link (fused KV link + one-pass repair)
-> CUDA-graph decode reproduces full-prefill greedy output."""

import pytest
import torch

from sglang_legolink_b200.models.config import PRESETS
from sglang_legolink_b200.models.qwen import QwenModel
from sglang_legolink_b200.runtime.engine import Engine

pytestmark = pytest.mark.gpu


def _setup(name, seed=0):
    cfg = PRESETS[name]
    model = QwenModel.random_init(cfg, seed=seed, device="cuda", dtype=torch.bfloat16)
    eng = Engine(model, num_pages=2048, page_size=16, max_context=8192)
    g = torch.Generator().manual_seed(seed)
    subs = [torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist() for n in (128, 333, 64, 700)]
    suffix = torch.randint(0, cfg.vocab_size, (21,), generator=g).tolist()
    for i, s in enumerate(subs):
        eng.compile(s, f"k{i}")
    return cfg, eng, subs, suffix


@pytest.mark.parametrize("name", ["small-qwen2", "small-qwen3"])
def test_full_repair_link_equals_full_prefill(name):
    cfg, eng, subs, suffix = _setup(name)
    order = [2, 0, 3, 1]
    plan = {"cache_keys": [f"k{i}" for i in order], "recompute_tokens_per_block": [len(subs[i]) for i in order]}
    seq = eng.link(plan, suffix)
    eng.decode([seq], 16)
    full = eng.prefill(sum((subs[i] for i in order), []) + suffix)
    eng.decode([full], 16)
    assert seq.output_ids == full.output_ids


def test_sparse_link_runs_and_cuda_graph_matches_eager():
    cfg, eng, subs, suffix = _setup("small-qwen2", seed=1)
    order = [3, 1, 0, 2]
    plan = {"cache_keys": [f"k{i}" for i in order], "recompute_initial_tokens": 32, "recompute_first_block": True}
    a = eng.link(dict(plan), suffix)
    b = eng.link(dict(plan), suffix)
    eng.decode([a], 12)
    eng.use_cuda_graphs = False
    eng.decode([b], 12)
    assert a.output_ids == b.output_ids


def test_batched_decode_matches_single():
    cfg, eng, subs, suffix = _setup("small-qwen2", seed=2)
    seqs = [eng.prefill(subs[i] + suffix) for i in range(4)]
    eng.decode(seqs, 8)
    for i in range(4):
        s = eng.prefill(subs[i] + suffix)
        eng.decode([s], 8)
        assert s.output_ids == seqs[i].output_ids
