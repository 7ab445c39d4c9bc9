"""KV-link kernel sweep on the Qwen2.5-7B KV layout (28 layers, 4 KV heads,
head_dim 128, bf16): 1-64 registered blocks of 128-8192 tokens, page size
16 or 64, per-block RoPE deltas uniform in +-32K positions, repair density 0
or 10 % (repaired rows are not linked), sources local or resident on a peer
GPU.  Each case is one ``kv_link_rope`` launch over all layers, timed with
CUDA events (median of 10 after 3 warm-ups; inputs larger than L2 except
the smallest cases).  Reported against the roofline:

* local: bytes read + written over the measured HBM copy bandwidth;
* peer: the slower of the K/V bytes read over NVLink (770 GB/s measured per
  direction) and the bytes written to local HBM.

    python -m sglang_legolink_b200.benchmarks.kv_link_sweep            # local, 1 GPU
    torchrun --nproc-per-node N --master-addr 127.0.0.1 -m sglang_legolink_b200.benchmarks.kv_link_sweep --peer

With ``--peer`` on N ranks every rank links, at the same time, blocks that
live in the symmetric-memory pool of rank (r + 1) mod N (P2P loads by the
link kernel, no TMA multicast), so at N = 8 all eight GPUs read over NVSwitch
at once; with N = 2 and ``--one-way`` only rank 1 links (from rank 0).  Every
rank takes the same collective steps; the time is the max over the linking
ranks, and rank 0 prints.
"""

from __future__ import annotations

import argparse
import json
import os
import random
import statistics

import torch

from .. import ops
from ..ops import reference as ref
from .kernels import peaks

L, HKV, D = 28, 4, 128
NVLINK_GBS = 770.0  # measured peer copy, per direction
MAX_TOKENS = 131072  # bound on linked tokens per case (pool memory)


def cases(quick: bool):
    blocks = (1, 8, 64) if not quick else (1, 8)
    toks = (128, 1024, 8192) if not quick else (128, 1024)
    for nb in blocks:
        for bt in toks:
            if nb * bt > MAX_TOKENS:
                continue
            for ps in (16, 64):
                for dens in (0.0, 0.1):
                    yield nb, bt, ps, dens


def build_case(nb, bt, ps, dens, seed=0):
    """Source slots (block-contiguous, block b at pages [b*P, (b+1)*P)),
    destination slots in the second half of the pool (request order); each
    block's rows carry local positions a+t and global positions g+t with a,
    g uniform in [0, 32K] (so the RoPE delta g-a is uniform in +-32K); ``dens``
    of the rows are dropped as repaired."""
    rng = random.Random(seed)
    pages_per_block = (bt + ps - 1) // ps
    half = nb * pages_per_block
    src, dst, lp, gp = [], [], [], []
    for b in range(nb):
        a0, g0 = rng.randint(0, 32768), rng.randint(0, 32768)
        for t in range(bt):
            if dens and rng.random() < dens:
                continue
            src.append(b * pages_per_block * ps + t)
            dst.append(half * ps + b * pages_per_block * ps + t)
            lp.append(a0 + t)
            gp.append(g0 + t)
    return 2 * half, src, dst, lp, gp


def timed(fn, reps=10):
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    ts = []
    for _ in range(reps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        fn()
        e1.record()
        e1.synchronize()
        ts.append(e0.elapsed_time(e1))
    return statistics.median(ts)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--peer", action="store_true", help="sources on a peer GPU (N >= 2 ranks under torchrun)")
    ap.add_argument("--one-way", action="store_true", help="with --peer: only rank 1 links (from rank 0)")
    ap.add_argument("--quick", action="store_true")
    a = ap.parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    pk = peaks()
    cs = ref.rope_cos_sin_table(32768 + 8192 + 64, D, 1e6).to(dev)
    dist = None
    if a.peer:
        if world < 2:
            raise SystemExit("--peer runs on 2 or more ranks")
        from datetime import timedelta

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
        from ..parallel.dp import SharedKVPool
    for nb, bt, ps, dens in cases(a.quick):
        pages, src, dst, lp, gp = build_case(nb, bt, ps, dens)
        n = len(src)
        s = torch.tensor(src, device=dev, dtype=torch.int64)
        d = torch.tensor(dst, device=dev, dtype=torch.int64)
        lpt = torch.tensor(lp, device=dev, dtype=torch.int32)
        gpt = torch.tensor(gp, device=dev, dtype=torch.int32)
        row_bytes = L * HKV * D * 2  # one token's K (or V) over all layers
        moved = 2 * 2 * n * row_bytes  # K and V, read + write
        base = dict(blocks=nb, block_tokens=bt, page_size=ps, repair_density=dens, linked_tokens=n, layers=L)
        if not a.peer:
            kp = torch.randn(L, pages, HKV, ps, D, device=dev, dtype=torch.bfloat16)
            vp = torch.randn_like(kp)
            ms = timed(lambda: ops.kv_link_rope(kp, vp, s, d, lpt, gpt, cs))
            roof_ms = moved / (pk["hbm_gbs"] * 1e6)
            print(json.dumps({**base, "source": "local", "ms": round(ms, 4), "gbs": round(moved / ms / 1e6, 1),
                              "roofline_ms": round(roof_ms, 4), "frac_of_roofline": round(roof_ms / ms, 3),
                              "peaks": pk["src"]}), flush=True)
            del kp, vp
        else:
            pool = SharedKVPool(L, pages, HKV, ps, D, torch.bfloat16, dev)
            pool.k.normal_()
            pool.v.normal_()
            torch.cuda.synchronize()
            dist.barrier()
            ms = 0.0
            linking = rank == 1 if a.one_way else True
            if linking:
                kp_ptr, vp_ptr, sps, sls = pool.peer(0 if a.one_way else (rank + 1) % world)
                ms = timed(lambda: ops.kv_link_rope(pool.k, pool.v, s, d, lpt, gpt, cs, src_k_ptr=kp_ptr,
                                                    src_v_ptr=vp_ptr, src_page_size=sps, src_layer_stride=sls))
            t = torch.tensor([ms], device=dev, dtype=torch.float64)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
            remote = 2 * n * row_bytes
            roof_ms = max(remote / (NVLINK_GBS * 1e6), remote / (pk["hbm_gbs"] * 1e6))
            if rank == 0:
                nlink = 1 if a.one_way else world
                print(json.dumps({**base, "source": "peer_gpu", "world": world, "linking_ranks": nlink, "ms": round(ms, 4),
                                  "nvlink_gbs": round(remote / ms / 1e6, 1),
                                  "aggregate_nvlink_gbs": round(nlink * remote / ms / 1e6, 1),
                                  "roofline_ms": round(roof_ms, 4),
                                  "frac_of_roofline": round(roof_ms / ms, 3), "nvlink_ref_gbs": NVLINK_GBS,
                                  "timing": "max over ranks"}), flush=True)
            dist.barrier()
            del pool
        torch.cuda.empty_cache()
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
