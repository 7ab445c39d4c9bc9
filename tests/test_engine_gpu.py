"""End-to-end on the GPU: Compile -> Link (fused KV link + one-pass repair)
-> CUDA-graph decode reproduces full-prefill greedy output."""

import pytest
import torch

from sglang_legolink_b200 import ops
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


@pytest.mark.parametrize("name", ["small-qwen2", "small-qwen3"])
def test_fused_decode_step_matches_unfused(name, monkeypatch):
    """The five-kernel decode layer (norms, RoPE and KV write in the GEMV
    stores) gives the logits and the new K/V of the unfused layer."""
    from sglang_legolink_b200.models.qwen import ForwardBatch

    cfg, eng, subs, suffix = _setup(name, seed=3)
    seqs = [eng.prefill(subs[i] + suffix) for i in (0, 1, 2)]
    ids, pos, slots, pt, kvl = eng._decode_inputs(seqs, 4, max(len(s.pages) for s in seqs))
    dev = eng.device
    fb = ForwardBatch(mode="decode", input_ids=ids.to(dev), positions=pos.to(dev), slots=slots.to(dev),
                      q_indptr=torch.arange(5, dtype=torch.int32, device=dev), page_table=pt.to(dev),
                      kv_lens=kvl.to(dev), logit_rows=None,
                      decode_nsplit=ops.decode_splits(4, eng.model.hkv, int(kvl.max())))
    ops.workspace(dev).reserve_decode(4 * eng.model.hq, fb.decode_nsplit)
    assert eng.model._decode_fusable(4)
    fused = eng.model.forward(fb, eng.kv).float()
    kf = eng.kv.k[:, slots[0] // 16].clone()
    monkeypatch.setattr(type(eng.model), "_decode_fusable", lambda self, T: False)
    plain = eng.model.forward(fb, eng.kv).float()
    kp = eng.kv.k[:, slots[0] // 16].clone()
    for r in range(3):
        assert ((fused[r] - plain[r]).norm() / plain[r].norm()).item() < 2e-2
    assert ((kf.float() - kp.float()).norm() / kp.float().norm()).item() < 1e-2


def test_warm_decode_captures_the_graph_and_changes_no_tokens():
    """warm_decode captures the batch's decode graph before any token is
    generated (page boundaries included: one prompt ends on a page edge);
    the decode that follows replays it and gives the tokens of a decode
    without the warm-up."""
    cfg, eng, subs, suffix = _setup("small-qwen2", seed=5)
    prompts = [subs[0] + suffix, subs[2][:32], subs[1] + suffix]
    seqs = [eng.prefill(p) for p in prompts]
    eng.warm_decode(seqs)
    assert eng._bucket(3) in eng._graphs
    g = eng._graphs[eng._bucket(3)]["graph"]
    eng.decode(seqs, 8)
    assert eng._graphs[eng._bucket(3)]["graph"] is g
    for p, ref in zip(prompts, seqs):
        s = eng.prefill(p)
        eng.decode([s], 8)
        assert s.output_ids == ref.output_ids


def test_padded_decode_bucket_keeps_row0_kv():
    """Three sequences in the bucket of four: the padded row writes the
    pool's scratch page, so every sequence decodes as it does alone."""
    cfg, eng, subs, suffix = _setup("small-qwen2", seed=4)
    seqs = [eng.prefill(subs[i] + suffix) for i in range(3)]
    eng.decode(seqs, 8)
    for i in range(3):
        s = eng.prefill(subs[i] + suffix)
        eng.decode([s], 8)
        assert s.output_ids == seqs[i].output_ids


def test_chained_decode_matches_per_step_with_stop_and_continue():
    """Greedy chunks with no host round trip between steps give the eager
    per-step tokens; a stop token ends a sequence at the same token and the
    same length, and decoding it further continues the same stream."""
    cfg, eng, subs, suffix = _setup("small-qwen2", seed=5)
    a = eng.prefill(subs[1] + suffix)
    eng.use_cuda_graphs = False
    eng.decode([a], 12)
    ref_ids, ref_len = list(a.output_ids), a.length
    eng.use_cuda_graphs = True
    b = eng.prefill(subs[1] + suffix)
    eng.decode([b], 12)
    assert b.output_ids == ref_ids and b.length == ref_len
    c = eng.prefill(subs[1] + suffix)
    gen = ref_ids[1:]  # output_ids[0] is the prefill's token
    stop = gen[4]
    j = gen.index(stop)  # decode steps up to and including the first stop
    eng.decode([c], 12, stop_ids=[stop])
    assert c.finished and c.output_ids == ref_ids[: 2 + j] and c.length == ref_len - (12 - (j + 1))
    c.finished = False
    eng.decode([c], 12 - (j + 1))
    assert c.output_ids == ref_ids and c.length == ref_len


def test_scheduler_chunked_decode_streams_the_per_step_tokens():
    """With nothing waiting, the scheduler decodes in chained chunks; the
    streamed tokens, stops and finish reasons are those of per-step decode."""
    from sglang_legolink_b200.runtime.scheduler import Request, Scheduler

    cfg, eng, subs, suffix = _setup("small-qwen2", seed=6)
    prompts = [subs[0] + suffix, subs[2] + suffix]
    eng.use_cuda_graphs = False
    refs = []
    for p in prompts:
        s = eng.prefill(p)
        eng.decode([s], 19)
        refs.append(list(s.output_ids))
        eng.free(s)
    eng.use_cuda_graphs = True
    stop = refs[1][7]
    sch = Scheduler(eng, legolink_only=False, decode_chunk=8)
    reqs = [Request("plain", "p0", prompts[0], 20), Request("plain", "p1", prompts[1], 20, stop_ids=(stop,))]
    for r in reqs:
        sch.submit(r)
    while sch.step():
        pass
    got = []
    for r in reqs:
        ev = []
        while not r.events.empty():
            ev.append(r.events.get_nowait())
        got.append(([v for k, v in ev if k == "token"], [v for k, v in ev if k == "done"][0]["finish_reason"]))
    assert got[0] == (refs[0], "length")
    j = refs[1].index(stop)
    assert got[1] == (refs[1][: j + 1], "stop")


def test_rope_table_covers_the_engine_context_and_kernel_errors_fail_the_request():
    """Positions past the checkpoint's max_position_embeddings stay inside
    the RoPE table (the engine extends it to its context); an error a kernel
    records fails the request that ran it, and the word is cleared."""
    import dataclasses

    from sglang_legolink_b200.runtime.engine import KernelFault

    cfg = dataclasses.replace(PRESETS["small-qwen2"], max_position_embeddings=512)
    model = QwenModel.random_init(cfg, seed=0, device="cuda", dtype=torch.bfloat16)
    eng = Engine(model, num_pages=512, page_size=16, max_context=2048)
    assert model.cos_sin.shape[0] >= 2048
    g = torch.Generator().manual_seed(9)
    prompt = torch.randint(0, cfg.vocab_size, (600,), generator=g).tolist()
    s = eng.prefill(prompt)
    eng.decode([s], 8)  # positions 600..607, past the checkpoint's 512
    assert ops.check_errors(torch.device("cuda")) == 0 and len(s.output_ids) == 9
    # a recorded error fails the step that saw it (a decode step: its
    # kernels are the split-K GEMVs and decode attention, whose early exits
    # on a set error word are bounded waits and a bounded drain)
    ops.workspace(torch.device("cuda")).err.fill_(6)
    with pytest.raises(KernelFault):
        eng.decode_step([s])
    assert ops.check_errors(torch.device("cuda")) == 0
    eng.free(s)


def test_decode_graphs_recaptured_after_scratch_buffers_grow():
    """A decode graph points into the model's scratch buffers.  A later,
    larger prefill replaces them (freeing the old memory); the engine must
    drop and recapture its graphs, so decode after the growth still matches
    eager decode."""
    cfg = PRESETS["small-qwen2"]
    model = QwenModel.random_init(cfg, seed=4, device="cuda", dtype=torch.bfloat16)
    eng = Engine(model, num_pages=4096, page_size=16, max_context=8192)
    g = torch.Generator().manual_seed(4)
    short = torch.randint(0, cfg.vocab_size, (40,), generator=g).tolist()
    long = torch.randint(0, cfg.vocab_size, (3000,), generator=g).tolist()
    s0 = eng.prefill(short)
    eng.decode([s0], 8)  # captures bucket 1 with the short prefill's buffers
    gen0 = model.buf_generation
    eng.free(s0)
    big = eng.prefill(long)  # regrows the scratch buffers
    assert model.buf_generation > gen0
    churn = [torch.full((1 << 20,), 7.0, device="cuda") for _ in range(8)]  # reuse the freed memory
    a = eng.prefill(short)
    eng.decode([a], 12)
    eng.use_cuda_graphs = False
    b = eng.prefill(short)
    eng.decode([b], 12)
    assert a.output_ids == b.output_ids
    assert all(bool((c == 7.0).all()) for c in churn)  # no stale graph wrote into them
    eng.free(big)
