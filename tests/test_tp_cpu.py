"""Tensor parallelism on CPU ranks (gloo, world size 2): the head / MLP /
vocab-sharded model with row-parallel all-reduce reproduces the unsharded
model's Link + greedy decode, and the per-rank Link manifests agree."""

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from sglang_legolink_b200.models.config import PRESETS
from sglang_legolink_b200.models.qwen import QwenModel
from sglang_legolink_b200.runtime.engine import Engine


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _workload():
    g = torch.Generator().manual_seed(3)
    subs = [torch.randint(0, 1000, (n,), generator=g).tolist() for n in (100, 70, 150)]
    suffix = torch.randint(0, 1000, (12,), generator=g).tolist()
    return subs, suffix


def _run(eng, subs, suffix):
    for i, s in enumerate(subs):
        eng.compile(s, f"k{i}")
    plan = {"cache_keys": ["k2", "k0", "k1"], "recompute_initial_tokens": 8, "recompute_first_block": True}
    seq = eng.link(plan, suffix)
    eng.decode([seq], 6)
    return seq


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    import torch.distributed as dist

    from sglang_legolink_b200.parallel.tp import NcclTPComm, check_link_across_ranks

    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        comm = NcclTPComm()
        m = QwenModel.random_init(PRESETS["tiny-qwen2"], seed=0, tp_rank=rank, tp_size=world, comm=comm)
        eng = Engine(m, num_pages=512, page_size=16)
        subs, suffix = _workload()
        seq = _run(eng, subs, suffix)
        check_link_across_ranks(seq.link_plan, True)
        q.put((rank, seq.output_ids))
    finally:
        dist.destroy_process_group()


def test_tp2_matches_single_process():
    ref_model = QwenModel.random_init(PRESETS["tiny-qwen2"], seed=0)
    subs, suffix = _workload()
    ref = _run(Engine(ref_model, num_pages=512, page_size=16), subs, suffix).output_ids
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    [p.start() for p in procs]
    outs = dict(q.get(timeout=300) for _ in procs)
    [p.join(timeout=60) for p in procs]
    assert all(p.exitcode == 0 for p in procs)
    assert outs[0] == outs[1] == ref
