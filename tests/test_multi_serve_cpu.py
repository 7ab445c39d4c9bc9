"""Multi-GPU serving logic on CPU (gloo ranks, tiny random Qwen2, hash
tokenizer):

* a TP=2 server (two processes, rank 0 drives, rank 1 replays) answers
  Compile, Link and a streamed Link with the single-process server's tokens,
  and a refused Link stays request-scoped on both ranks;
* the DP router over in-process replicas sharing one block directory sends a
  Compile of a published key to its owner and other requests by load, then
  locality, and forwards refusals and streams through an HTTP replica;
* pipeline parallelism and mixed TP x DP are refused at launch.
"""

import argparse
import json
import multiprocessing as mp
import os
import socket
import urllib.error
import urllib.request

import pytest

from sglang_legolink_b200.contract import ContractError
from sglang_legolink_b200.server.http_server import build_service, serve
from sglang_legolink_b200.server.launch import HTTPReplica, RouterService, check_parallel_args


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _post(base, body, stream=False):
    req = urllib.request.Request(base + "/v1/chat/completions", data=json.dumps(body).encode(),
                                 headers={"Content-Type": "application/json"})
    try:
        with urllib.request.urlopen(req, timeout=300) as r:
            raw = r.read().decode()
            return r.status, raw if stream else json.loads(raw)
    except urllib.error.HTTPError as e:
        return e.code, json.loads(e.read().decode())


def _frames(raw):
    out = [x[len("data: "):] for x in raw.split("\n\n") if x.startswith("data: ")]
    assert out[-1] == "[DONE]"
    return [json.loads(f) for f in out[:-1]]


def _msgs(t):
    return [{"role": "user", "content": t}]


WORKLOAD = [
    {"messages": _msgs("tool output " * 60), "max_tokens": 1, "sub_context": {"cache_key": "mp-a"}},
    {"messages": _msgs("instructions " * 40), "max_tokens": 1, "sub_context": {"cache_key": "mp-b"}},
    {"messages": _msgs("what next?"), "max_tokens": 6, "ignore_eos": True,
     "pic_link": {"cache_keys": ["mp-b", "mp-a"], "recompute_initial_tokens": 8}},
]


def _run_workload(base):
    outs = []
    for body in WORKLOAD:
        code, r = _post(base, body)
        assert code == 200, r
        outs.append(r["meta_info"]["output_ids"])
    code, raw = _post(base, dict(WORKLOAD[-1], stream=True), stream=True)
    assert code == 200
    outs.append([c["meta_info"]["token_id"] for c in _frames(raw) if "meta_info" in c])
    code, r = _post(base, {"messages": _msgs("x"), "max_tokens": 2, "pic_link": {"cache_keys": ["mp-missing"]}})
    assert code in (200, 400)
    return outs


def _tp_rank(rank, world, port, a, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    from sglang_legolink_b200.server.launch import rank_main

    rank_main(a, rank, world, rank, ready=q if rank == 0 else None)


def test_tp2_server_matches_single_process():
    svc = build_service("tiny-qwen2", device="cpu", max_context=4096)
    srv = serve(svc, "127.0.0.1", 0)
    try:
        ref = _run_workload(f"http://127.0.0.1:{srv.server_address[1]}")
    finally:
        srv.shutdown()
        svc.scheduler.stop()
    ctx = mp.get_context("spawn")
    q, stop = ctx.Queue(), ctx.Event()
    a = argparse.Namespace(model="tiny-qwen2", device="cpu", tokenizer=None, host="127.0.0.1", port=_free_port(),
                           page_size=16, context_length=4096, allow_plain_generation=False, skip_warmup=True,
                           tp_size=2, dp_size=1, pp_size=1, tp_comm="nccl", dp_base_port=0, dist_timeout=120,
                           seed=0, stop_event=stop)
    dport = _free_port()
    procs = [ctx.Process(target=_tp_rank, args=(r, 2, dport, a, q)) for r in range(2)]
    [p.start() for p in procs]
    try:
        port = q.get(timeout=300)
        got = _run_workload(f"http://127.0.0.1:{port}")
        # the server still answers after the refused Link (both ranks agreed on it)
        code, r = _post(f"http://127.0.0.1:{port}", WORKLOAD[-1])
        assert code == 200 and r["meta_info"]["output_ids"] == ref[2]
    finally:
        stop.set()
        [p.join(timeout=120) for p in procs]
        for p in procs:
            if p.is_alive():
                p.kill()
    assert got == ref
    assert all(p.exitcode == 0 for p in procs)


def _replicas():
    import torch

    from sglang_legolink_b200.host.tokenizer import HashTokenizer
    from sglang_legolink_b200.models.config import PRESETS
    from sglang_legolink_b200.models.qwen import QwenModel
    from sglang_legolink_b200.parallel.dp import LocalDirectory
    from sglang_legolink_b200.runtime.engine import Engine
    from sglang_legolink_b200.runtime.scheduler import Scheduler
    from sglang_legolink_b200.server.http_server import RuntimeService

    cfg = PRESETS["tiny-qwen2"]
    d = LocalDirectory()
    engs = [Engine(QwenModel.random_init(cfg, seed=0), num_pages=512, directory=d, replica_rank=r,
                   max_context=4096) for r in range(2)]
    engs[0].peer_pools[1] = (engs[1].kv.k, engs[1].kv.v)
    engs[1].peer_pools[0] = (engs[0].kv.k, engs[0].kv.v)
    svcs = []
    for e in engs:
        s = Scheduler(e)
        s.start()
        svcs.append(RuntimeService(s, HashTokenizer(cfg.vocab_size, name=cfg.name), model_name=cfg.name))
    del torch
    return svcs, d


def test_dp_router_routes_by_owner_load_and_locality():
    svcs, d = _replicas()
    srv = serve(svcs[1], "127.0.0.1", 0)
    try:
        router = RouterService([svcs[0], HTTPReplica("127.0.0.1", srv.server_address[1])], d)
        r = router.complete(WORKLOAD[0])
        first = r["meta_info"]["dp_replica"]
        # a second Compile of the same key goes to the replica that owns it
        assert router.pick(WORKLOAD[0]) == first
        r = router.complete(WORKLOAD[1])
        assert r["meta_info"]["kind"] == "compile"
        # equal load: the Link goes where most of its block tokens are resident
        owners = [d.lookup(k).owner for k in ("mp-a", "mp-b")]
        toks = [len(d.lookup(k).token_ids) for k in ("mp-a", "mp-b")]
        best = owners[0] if toks[0] >= toks[1] or owners[0] == owners[1] else owners[1]
        assert router.pick(WORKLOAD[2]) == best
        # a busy replica loses to an idle one
        router.inflight[best] += 1
        assert router.pick(WORKLOAD[2]) == 1 - best
        router.inflight[best] -= 1
        # both replicas link (one of them reads the other's pool) to the same tokens
        outs = [router.replicas[i].complete(WORKLOAD[2])["meta_info"]["output_ids"] for i in (0, 1)]
        assert outs[0] == outs[1] and len(outs[0]) == 6
        chunks = list(router.stream(dict(WORKLOAD[2], stream=True)))
        assert [c["meta_info"]["token_id"] for c in chunks if "meta_info" in c] == outs[0]
        info = router.model_info()
        assert info["dp_size"] == 2 and sum(info["dp_routed"]) == 3
        # refusals from a remote replica surface as refusals
        from sglang_legolink_b200.runtime.scheduler import RequestRejected

        with pytest.raises((RequestRejected, ContractError)):
            router.replicas[1].complete({"messages": _msgs("hello"), "max_tokens": 2})
    finally:
        srv.shutdown()
        for s in svcs:
            s.scheduler.stop()


def test_parallel_flags_are_checked():
    check_parallel_args(8, 1, 1)
    check_parallel_args(1, 8, 1)
    for tp, dp, pp in ((1, 1, 2), (2, 2, 1), (0, 1, 1)):
        with pytest.raises(ContractError):
            check_parallel_args(tp, dp, pp)


def test_dp2_server_serves_and_shuts_down_cleanly():
    """Two gloo ranks as DP replicas behind rank 0's router: Compile + Link
    through the router, then an orderly shutdown of both ranks."""
    ctx = mp.get_context("spawn")
    q, stop = ctx.Queue(), ctx.Event()
    a = argparse.Namespace(model="tiny-qwen2", device="cpu", tokenizer=None, host="127.0.0.1", port=_free_port(),
                           page_size=16, context_length=4096, allow_plain_generation=False, skip_warmup=True,
                           tp_size=1, dp_size=2, pp_size=1, tp_comm="nccl", dp_base_port=_free_port(),
                           dist_timeout=120, seed=0, stop_event=stop)
    dport = _free_port()
    procs = [ctx.Process(target=_tp_rank, args=(r, 2, dport, a, q)) for r in range(2)]
    [p.start() for p in procs]
    try:
        port = q.get(timeout=300)
        base = f"http://127.0.0.1:{port}"
        code, r = _post(base, {"messages": _msgs("tool output " * 60), "max_tokens": 1,
                               "sub_context": {"cache_key": "dp-a"}})
        assert code == 200, r
        code, r = _post(base, {"messages": _msgs("next?"), "max_tokens": 4, "ignore_eos": True,
                               "pic_link": {"cache_keys": ["dp-a"], "recompute_initial_tokens": 8}})
        assert code == 200 and len(r["meta_info"]["output_ids"]) == 4, r
    finally:
        stop.set()
        [p.join(timeout=120) for p in procs]
        for p in procs:
            if p.is_alive():
                p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
