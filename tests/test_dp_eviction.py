"""Eviction of published blocks across DP replicas: the owner frees a block
a peer may link only after a grace period in which every peer Link that may
have found it has ended; a Link that starts after the withdrawal aborts with
the residency-recovery refusal instead of reading freed pages.

CPU: engines in one process over a :class:`LocalDirectory`, and two gloo
ranks over the TCPStore-backed :class:`BlockDirectory`."""

import json
import os
import threading

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from sglang_legolink_b200.models.config import PRESETS
from sglang_legolink_b200.models.qwen import QwenModel
from sglang_legolink_b200.parallel.dp import BlockDirectory, DirectoryClient, LocalDirectory, RemoteBlock
from sglang_legolink_b200.runtime.engine import Engine, LinkSourceUnavailable


def _pair(pages=512):
    cfg = PRESETS["tiny-qwen2"]
    d = LocalDirectory()
    a = Engine(QwenModel.random_init(cfg, seed=0), num_pages=pages, directory=d, replica_rank=0)
    b = Engine(QwenModel.random_init(cfg, seed=0), num_pages=pages, directory=d, replica_rank=1)
    b.peer_pools[0] = (a.kv.k, a.kv.v)
    a.peer_pools[1] = (b.kv.k, b.kv.v)
    for e in (a, b):
        e._dir.grace_timeout_s = 0.2
    return a, b, d


def _toks(n, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.randint(0, 1000, (n,), generator=g).tolist()


def test_withdraw_waits_for_an_open_peer_link():
    a, b, d = _pair()
    a.compile(_toks(70, 1), "blk")
    rb = b._dir.find("blk")
    valid, missing, stale = b._dir.begin({"blk": rb})  # a peer Link is reading the block
    assert not missing and not stale
    assert not a.unregister_block("blk")  # grace period cannot close: block kept and published again
    assert a.registry.contains("blk") and d.lookup("blk") is not None
    b._dir.end()
    assert a.unregister_block("blk")
    assert not a.registry.contains("blk") and d.lookup("blk") is None


def test_withdraw_closes_when_the_peer_link_ends_during_the_wait():
    a, b, d = _pair()
    a._dir.grace_timeout_s = 5.0
    a.compile(_toks(70, 2), "blk")
    b._dir.begin({"blk": b._dir.find("blk")})
    t = threading.Timer(0.05, b._dir.end)
    t.start()
    assert a.unregister_block("blk")
    t.join()


def test_link_racing_a_withdrawal_gets_the_recovery_refusal():
    a, b, d = _pair()
    blocks = [_toks(n, 10 + n) for n in (64, 80)]
    for i, t in enumerate(blocks):
        a.compile(t, f"k{i}")
    plan = {"cache_keys": ["k1", "k0"], "recompute_initial_tokens": 4, "recompute_first_block": True}
    s = b.link(dict(plan), [5, 6, 7])  # fills b's cached entries for k0, k1
    b.free(s)
    assert b.stats["remote_blocks_linked"] == 2
    assert a.unregister_block("k0")
    # the freed pages are handed to another block on the owner
    a.compile(_toks(64, 99), "other")
    with pytest.raises(LinkSourceUnavailable) as ei:
        b.link(dict(plan), [5, 6, 7])
    assert ei.value.missing == ("k0",)
    detail = json.loads(str(ei.value).split(" | ", 1)[1])["noc_residency_recovery"]
    assert detail["missing_cache_keys"] == ["k0"]
    # recompiling the key on the owner makes the same Link work again
    a.compile(blocks[0], "k0")
    s = b.link(dict(plan), [5, 6, 7])
    assert s.output_ids


def test_republished_block_with_other_content_is_stale():
    a, b, d = _pair()
    a.compile(_toks(64, 3), "k")
    s = b.link({"cache_keys": ["k"], "recompute_initial_tokens": 4}, [1, 2])
    b.free(s)
    assert a.unregister_block("k")
    a.compile(_toks(64, 4), "k")  # same key, other tokens
    with pytest.raises(LinkSourceUnavailable) as ei:
        b.link({"cache_keys": ["k"], "recompute_initial_tokens": 4}, [1, 2])
    assert ei.value.stale == ("k",) or ei.value.missing == ("k",)


def test_owner_under_capacity_pressure_withdraws_published_blocks():
    """Published blocks are no longer pinned forever: a long stream of
    Compiles on a small pool keeps running by withdrawing the coldest."""
    a, b, d = _pair(pages=64)
    for i in range(40):  # 40 blocks x 5 pages >> 63 usable pages
        a.compile(_toks(70, 100 + i), f"t{i}")
    assert a.stats.get("published_blocks_withdrawn", 0) > 20
    live = [k for k in a.registry.keys() if d.lookup(k) is not None]
    assert set(live) == set(a._published)
    assert "t39" in a._published


def test_grace_ticket_counters_balance_after_failures():
    a, b, d = _pair()
    a.compile(_toks(64, 5), "k")
    s = b.link({"cache_keys": ["k"]}, [1, 2, 3])
    b.free(s)
    a.unregister_block("k")
    with pytest.raises(LinkSourceUnavailable):
        b.link({"cache_keys": ["k"]}, [1, 2, 3])
    assert d.add("rcu/begun/1", 0) == d.add("rcu/ended/1", 0) == 2


# ------------------------------------------------------------- gloo ranks
def _rank(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        store = dist.distributed_c10d._get_default_store()
        c = DirectoryClient(BlockDirectory(store, prefix="evict-test/", world=world), rank, grace_timeout_s=0.3)
        rb = RemoteBlock(0, "blk", (3, 4), 0, (1, 2, 3), "ck", "h", 16)
        out = {}
        if rank == 0:
            out["published"] = c.publish(rb)
        dist.barrier()
        if rank == 1:
            found = c.find("blk")
            _, missing, _ = c.begin({"blk": found})
            out["begin_missing"] = missing
        dist.barrier()  # rank 1 holds a ticket
        if rank == 0:
            out["withdraw_while_open"] = c.withdraw(rb)
        dist.barrier()
        if rank == 1:
            c.end()
        dist.barrier()
        if rank == 0:
            out["withdraw_after_end"] = c.withdraw(rb)
        dist.barrier()
        if rank == 1:
            _, missing, _ = c.begin({"blk": c.find("blk") or rb})
            out["after_withdraw_missing"] = missing
        dist.barrier()
        q.put((rank, out))
    finally:
        dist.destroy_process_group()


def test_grace_period_across_gloo_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29000 + os.getpid() % 1000
    ps = [ctx.Process(target=_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = dict(q.get(timeout=120) for _ in ps)
    for p in ps:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert res[0] == {"published": True, "withdraw_while_open": False, "withdraw_after_end": True}
    assert res[1] == {"begin_missing": [], "after_withdraw_missing": ["blk"]}
