"""DP replicas sharing one block directory: a block compiled on one replica
is linked by another straight from the owner's KV pool (CPU: two engines in
one process; the GPU version reads the peer pool over NVLink)."""

import os
import shutil
import subprocess
import sys

import pytest
import torch

from sglang_legolink_b200.models.config import PRESETS
from sglang_legolink_b200.models.qwen import QwenModel
from sglang_legolink_b200.parallel.dp import LocalDirectory, RemoteBlock
from sglang_legolink_b200.runtime.engine import Engine, LinkSourceUnavailable

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _pair():
    cfg = PRESETS["tiny-qwen2"]
    d = LocalDirectory()
    a = Engine(QwenModel.random_init(cfg, seed=0), num_pages=512, directory=d, replica_rank=0)
    b = Engine(QwenModel.random_init(cfg, seed=0), num_pages=512, directory=d, replica_rank=1)
    b.peer_pools[0] = (a.kv.k, a.kv.v)
    a.peer_pools[1] = (b.kv.k, b.kv.v)
    return a, b, d


def test_cross_replica_link_matches_local_link():
    a, b, d = _pair()
    g = torch.Generator().manual_seed(5)
    subs = [torch.randint(0, 1000, (n,), generator=g).tolist() for n in (90, 130, 60)]
    suffix = torch.randint(0, 1000, (10,), generator=g).tolist()
    for i, s in enumerate(subs):
        a.compile(s, f"blk{i}")
    b.compile(subs[2], "blk2")  # one block resident on both replicas
    plan = {"cache_keys": ["blk1", "blk2", "blk0"], "recompute_initial_tokens": 4, "recompute_first_block": True}
    sa = a.link(dict(plan), suffix)
    sb = b.link(dict(plan), suffix)
    a.decode([sa], 5)
    b.decode([sb], 5)
    assert sa.output_ids == sb.output_ids
    assert b.stats["remote_blocks_linked"] == 2
    # the owner keeps published blocks pinned; the pins taken by the link are released
    assert a.registry.handle("blk0")["pin_count"] == 1
    # every Link that read a peer block closed its grace-period ticket
    assert d.add("rcu/begun/1", 0) == d.add("rcu/ended/1", 0) == 1


def test_incompatible_remote_block_is_refused():
    a, b, d = _pair()
    a.compile(list(range(1, 80)), "x")
    with pytest.raises(LinkSourceUnavailable):
        b.link({"cache_keys": ["x"], "adapter_id": "lora-7"}, [3, 4, 5])


@pytest.mark.gpu
@pytest.mark.multigpu
def test_cross_replica_link_over_nvlink_two_gpus():
    """Two ranks with KV pools in symmetric memory: rank 1 links rank 0's
    blocks through peer pointers and must match linking its own copies."""
    runner = shutil.which("torchrun") or None
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr=127.0.0.1", "--master-port=29533", os.path.join(ROOT, "tests", "dp_peer_link_worker.py")]
    env = {**os.environ, "NCCL_NVLS_ENABLE": "0", "TORCH_SYMM_MEM_DISABLE_MULTICAST": "1"}
    r = subprocess.run(["timeout", "-k", "30", "300"] + cmd, capture_output=True, text=True, env=env)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert "PEER_LINK_OK" in r.stdout
