"""Sampling beyond greedy: seeded reproducibility, top-k / top-p support,
and the engine threading per-request parameters through prefill, Link and
decode (CPU path)."""

import pytest
import torch

from sglang_legolink_b200.models.config import PRESETS
from sglang_legolink_b200.models.qwen import QwenModel
from sglang_legolink_b200.runtime.engine import Engine
from sglang_legolink_b200.runtime.sampling import SamplingParams, make_generator, sample_rows


def test_greedy_params():
    assert SamplingParams().greedy
    assert SamplingParams(temperature=0.7, top_k=1).greedy
    assert not SamplingParams(temperature=0.7).greedy
    p = SamplingParams.from_request({"temperature": 0.5, "top_p": 0.9, "top_k": 20, "seed": 3})
    assert (p.temperature, p.top_p, p.top_k, p.seed) == (0.5, 0.9, 20, 3)


def test_top_k_restricts_support():
    logits = torch.arange(100, dtype=torch.float32)[None].repeat(4, 1)
    p = SamplingParams(temperature=5.0, top_k=3, seed=1)
    g = [make_generator(p, "cpu") for _ in range(4)]
    for _ in range(20):
        ids = sample_rows(logits, [p] * 4, g)
        assert all(int(i) >= 97 for i in ids)


def test_top_p_restricts_support():
    probs = torch.tensor([0.5, 0.3, 0.15, 0.05])
    logits = probs.log()[None]
    p = SamplingParams(temperature=1.0, top_p=0.7, seed=0)
    g = [make_generator(p, "cpu")]
    seen = {int(sample_rows(logits, [p], g)[0]) for _ in range(200)}
    assert seen <= {0, 1} and len(seen) == 2


def test_seed_reproducible_and_greedy_rows_untouched():
    logits = torch.randn(1, 500).repeat(3, 1)
    ps = [SamplingParams(), SamplingParams(temperature=1.0, seed=7), SamplingParams(temperature=1.0, seed=7)]
    a = sample_rows(logits, ps, [make_generator(p, "cpu") for p in ps])
    b = sample_rows(logits, ps, [make_generator(p, "cpu") for p in ps])
    assert torch.equal(a, b)
    assert int(a[0]) == int(torch.argmax(logits[0]))
    assert int(a[1]) == int(a[2])


@pytest.fixture(scope="module")
def eng():
    model = QwenModel.random_init(PRESETS["tiny-qwen2"], seed=0)
    e = Engine(model, num_pages=512, page_size=16, legolink_only=False)
    return e


def test_engine_seeded_decode_reproducible(eng):
    toks = list(range(5, 70))
    p = SamplingParams(temperature=1.0, top_p=0.95, seed=1234)
    outs = []
    for _ in range(2):
        s = eng.prefill(toks, sampling=p)
        eng.decode([s], 12)
        outs.append(list(s.output_ids))
        eng.free(s)
    assert outs[0] == outs[1]
    g = eng.prefill(toks)
    eng.decode([g], 12)
    greedy = list(g.output_ids)
    eng.free(g)
    # a batch mixing a greedy and a sampled sequence keeps the greedy one exact
    s1, s2 = eng.prefill(toks), eng.prefill(toks, sampling=p)
    eng.decode([s1, s2], 12)
    assert s1.output_ids == greedy
    assert s2.output_ids == outs[0]
    eng.free(s1), eng.free(s2)


def test_engine_link_sampling(eng):
    eng.compile(list(range(100, 164)), "blk-a")
    eng.compile(list(range(200, 232)), "blk-b")
    plan = {"cache_keys": ["blk-b", "blk-a"], "recompute_tokens_per_block": [4, 4]}
    p = SamplingParams(temperature=0.8, top_k=50, seed=9)
    a = eng.link(dict(plan), [7, 8, 9], sampling=p)
    eng.decode([a], 6)
    b = eng.link(dict(plan), [7, 8, 9], sampling=p)
    eng.decode([b], 6)
    assert a.output_ids == b.output_ids
    eng.free(a), eng.free(b)
