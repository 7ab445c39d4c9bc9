"""Data-parallel replicas sharing one block registry: concurrent synthetic
agent sessions over Qwen2.5-7B-arch (random init, bf16), one replica per GPU
(``torchrun --nproc-per-node N``).

Each session runs ``--turns`` turns.  A turn's prompt is the shared 2K-token
instruction and 4K-token tool schema, the previous turn's tool output and
this turn's new tool output (512-8192 tokens, log-uniform), then a 64-token
user query; the new tool output is compiled that turn (the Compiles of one
round share one forward), the prompt is linked (RoPE remap + 32-row repair
windows), and ``--decode`` tokens are decoded for all of the replica's
sessions together.  Every replica compiles its own copy of the instruction
and tool schema and publishes it in the shared block directory; half of the
sessions link the copies of the next replica, so their reused blocks are read
from a peer GPU's pool over NVLink by the link kernel.  (One turn of tool
history keeps 20 turns inside the context window.)

Two arms for the Links of a round (``--arm``): ``batched`` -- a replica's
Links of the round go through one step (one fused KV-link launch per source
pool, one extend forward for every repair row), each Link's TTFT is that
step; ``serial`` -- one Link per forward, all arriving together, so the k-th
Link's TTFT includes the k - 1 before it (the reference admits a Link alone,
``managers/scheduler.py:2597-2690``).  ``both`` (default) runs both each
round and decodes the batched arm's sequences.

Timed on the device per replica (CUDA events around each Link step and each
decode batch, after a warm-up round), reported as the max over replicas:
Link TTFT p50 / p95 per arm, decode tok/s summed over replicas, and turns/s.

    torchrun --nproc-per-node 8 --master-addr 127.0.0.1 -m sglang_legolink_b200.benchmarks.dp_sessions
"""

from __future__ import annotations

import argparse
import json
import math
import os
import random
import statistics


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="qwen2.5-7b")
    ap.add_argument("--sessions", type=int, default=64)
    ap.add_argument("--turns", type=int, default=20)
    ap.add_argument("--decode", type=int, default=128)
    ap.add_argument("--peer-frac", type=float, default=0.5)
    ap.add_argument("--instruction", type=int, default=2048)
    ap.add_argument("--schema", type=int, default=4096)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--arm", default="both", choices=["batched", "serial", "both"],
                    help="batched: a round's Links of a replica go through one extend forward; serial: one Link "
                         "per forward (a Link waits for the ones before it); both: each round runs both")
    a = ap.parse_args()

    import torch
    import torch.distributed as dist

    from ..models.config import PRESETS
    from ..models.qwen import QwenModel
    from ..runtime.engine import Engine, pages_for

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    cfg = PRESETS[a.model]
    model = QwenModel.random_init(cfg, seed=a.seed, device=dev, dtype=torch.bfloat16)
    mine = [s for s in range(a.sessions) if s % world == rank]
    ps = 16
    max_ctx = a.instruction + a.schema + 2 * 8192 + 64 + a.decode + 64
    pages = len(mine) * pages_for(max_ctx, ps) + 2 * len(mine) * pages_for(8192, ps) + 4096
    kw = {}
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=600), device_id=dev)
        from ..parallel.dp import BlockDirectory, SharedKVPool

        pool = SharedKVPool(cfg.num_layers, pages, model.hkv, ps, cfg.head_dim, torch.bfloat16, dev)
        kw = dict(kv_pool=pool, directory=BlockDirectory(dist.distributed_c10d._get_default_store(),
                                                         prefix="dp-sessions/", world=world),
                  replica_rank=rank, peer_pools={r: pool.peer(r) for r in range(world) if r != rank})
    else:
        kw = dict(num_pages=pages)
    eng = Engine(model, page_size=ps, max_context=max_ctx + 1024, **kw)
    rng = random.Random(a.seed + 17 * rank)
    V = cfg.vocab_size
    shared = random.Random(a.seed)
    instr = [shared.randrange(V) for _ in range(a.instruction)]
    schema = [shared.randrange(V) for _ in range(a.schema)]
    eng.compile(instr, f"instr@{rank}")
    eng.compile(schema, f"schema@{rank}")
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()

    def tool_len():
        return int(math.exp(rng.uniform(math.log(512), math.log(8192))))

    peer = (rank + 1) % world
    owner = {s: (peer if (world > 1 and (s // world) % 2 == 1 and a.peer_frac > 0) else rank) for s in mine}
    prev = {s: None for s in mine}
    links, serial_links, decode_ms, turns_done, peer_links = [], [], 0.0, 0, 0
    tokens_decoded = 0
    for turn in range(a.turns + 1):  # turn 0 is the warm-up round
        timed = turn > 0
        items, keys = [], {}
        for s in mine:
            key = f"tool-{s}-{turn}@{rank}"
            items.append(([rng.randrange(V) for _ in range(tool_len())], key, None, None))
            keys[s] = key
        res = eng.compile_batch(items)
        bad = [r for r in res if isinstance(r, Exception)]
        if bad:
            raise bad[0]
        reqs = []
        for s in mine:
            o = owner[s]
            ck = [f"instr@{o}", f"schema@{o}"] + ([prev[s]] if prev[s] else []) + [keys[s]]
            query = [rng.randrange(V) for _ in range(64)]
            reqs.append(({"cache_keys": ck, "recompute_initial_tokens": 32, "recompute_first_block": True}, query))
            if timed:
                peer_links += int(o != rank)
        seqs = []
        if a.arm in ("serial", "both"):
            # the round's Links arrive together and run one per forward: the
            # k-th one's TTFT includes the k - 1 before it
            waited = 0.0
            for plan, query in reqs:
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                seq = eng.link(dict(plan), query)
                e1.record()
                e1.synchronize()
                waited += e0.elapsed_time(e1)
                if timed:
                    serial_links.append(waited)
                if a.arm == "serial":
                    seqs.append(seq)
                else:
                    eng.free(seq)
        if a.arm in ("batched", "both"):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            out = eng.link_batch([(dict(plan), query) for plan, query in reqs])
            e1.record()
            e1.synchronize()
            bad = [r for r in out if isinstance(r, Exception)]
            if bad:
                raise bad[0]
            if timed:
                links.extend([e0.elapsed_time(e1)] * len(out))
            seqs = list(out)
        d0, d1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        d0.record()
        eng.decode(seqs, a.decode - 1)
        d1.record()
        d1.synchronize()
        if timed:
            decode_ms += d0.elapsed_time(d1)
            tokens_decoded += len(seqs) * (a.decode - 1)
            turns_done += len(seqs)
        for seq in seqs:
            eng.free(seq)
        for s in mine:  # keep one turn of tool history resident
            if prev[s]:
                eng.unregister_block(prev[s])  # published: withdrawn from the directory first
            prev[s] = keys[s]
    primary = links if links else serial_links
    n = max(1, len(mine))
    if links:  # a round's batched step is counted once per Link in it
        link_round_ms = sum(links) / n
    else:  # the last Link of a round waited for the whole round
        link_round_ms = sum(serial_links[n - 1::n])
    total_ms = link_round_ms + decode_ms

    def pct(xs, q):
        return sorted(xs)[int(q * (len(xs) - 1))] if xs else 0.0

    stats = torch.tensor([statistics.median(primary), pct(primary, 0.95), decode_ms, total_ms,
                          statistics.median(serial_links) if serial_links else 0.0, pct(serial_links, 0.95)],
                         dtype=torch.float64, device=dev)
    sums = torch.tensor([tokens_decoded / (decode_ms / 1e3), turns_done, peer_links, len(primary)],
                        dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(stats, op=dist.ReduceOp.MAX)
        dist.all_reduce(sums, op=dist.ReduceOp.SUM)
    p50, p95, dec_ms_max, total_max, s50, s95 = stats.tolist()
    tok_s, turns_all, peers, nlinks = sums.tolist()
    if rank == 0:
        print(json.dumps({
            "metric": "DP replicas sharing one block registry: Link TTFT and decode tok/s",
            "model": f"{a.model} (random init)", "replicas": world, "sessions": a.sessions, "turns": a.turns,
            "decode_tokens": a.decode, "peer_block_fraction": round(peers / max(nlinks, 1), 3),
            "arm": a.arm, "link_ttft_ms_p50": round(p50, 3), "link_ttft_ms_p95": round(p95, 3),
            **({"serial_link_ttft_ms_p50": round(s50, 3), "serial_link_ttft_ms_p95": round(s95, 3)}
               if a.arm == "both" else {}),
            "decode_tok_s": round(tok_s, 1), "turns_per_s": round(turns_all / (total_max / 1e3), 2),
            "timing": "CUDA events per replica, max over replicas (tok/s summed)",
            "history": "one previous tool output per turn",
            "data": "synthetic agent sessions (seeded), random-init weights",
        }), flush=True)
    if world > 1:
        eng._graphs.clear()
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
