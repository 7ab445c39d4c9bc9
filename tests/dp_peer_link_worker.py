"""Two-rank worker (launched by tests/test_dp_shared_registry.py with torchrun):
rank 0 compiles blocks into its symmetric-memory KV pool; rank 1 links them
through peer pointers (read over NVLink by the fused link kernel) and checks
the tokens against linking its own compiled copies."""

import os
import sys

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from datetime import timedelta  # noqa: E402

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402


def main():
    rank, local = int(os.environ["RANK"]), int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=60), device_id=dev)
    from sglang_legolink_b200.models.config import PRESETS
    from sglang_legolink_b200.models.qwen import QwenModel
    from sglang_legolink_b200.parallel.dp import BlockDirectory, SharedKVPool
    from sglang_legolink_b200.runtime.engine import Engine

    cfg = PRESETS["small-qwen2"]
    model = QwenModel.random_init(cfg, seed=0, device=dev, dtype=torch.bfloat16)
    pool = SharedKVPool(cfg.num_layers, 2048, model.hkv, 16, cfg.head_dim, torch.bfloat16, dev)
    store = dist.distributed_c10d._get_default_store()
    directory = BlockDirectory(store, prefix="peer-link-test/", world=2)
    other = 1 - rank
    eng = Engine(model, kv_pool=pool, max_context=4096, directory=directory, replica_rank=rank,
                 peer_pools={other: pool.peer(other)})
    g = torch.Generator().manual_seed(7)
    subs = [torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist() for n in (200, 96, 333)]
    suffix = torch.randint(0, cfg.vocab_size, (19,), generator=g).tolist()
    ok = True
    if rank == 0:
        for i, s in enumerate(subs):
            eng.compile(s, f"shared-{i}")
        torch.cuda.synchronize()
    dist.barrier()
    if rank == 1:
        plan = {"cache_keys": ["shared-2", "shared-0", "shared-1"], "recompute_initial_tokens": 16,
                "recompute_first_block": True}
        remote = eng.link(dict(plan), suffix)
        eng.decode([remote], 8)
        for i, s in enumerate(subs):
            eng.compile(s, f"own-{i}")
        plan_own = dict(plan, cache_keys=["own-2", "own-0", "own-1"])
        own = eng.link(plan_own, suffix)
        eng.decode([own], 8)
        torch.cuda.synchronize()
        ok = remote.output_ids == own.output_ids and eng.stats["remote_blocks_linked"] == 3
        print("remote", remote.output_ids, "own", own.output_ids, flush=True)
        if ok:
            print("PEER_LINK_OK", flush=True)
    dist.barrier()
    del eng, pool
    dist.destroy_process_group()
    sys.exit(0 if ok else 1)


if __name__ == "__main__":
    main()
