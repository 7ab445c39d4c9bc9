"""Qwen3-32B tensor-parallel Link + decode (the TP configuration of the
headline metric): random-init Qwen3-32B-arch bf16 (64 layers, hidden 5120,
64 Q / 8 KV heads, QK-norm), TP = world size, synthetic agent contexts of
``--context`` tokens in ``--subcontexts`` sub-contexts (90 % linked in a
shuffled order, 10 % fresh), repair window ``--repair`` per boundary; then
``--decode`` tokens for ``--batch`` sessions decoded together.

Every session's Link is timed on the device (CUDA events around the API
call, the first token on the host when it returns), max over ranks; the
decode is timed the same way around the whole batch.  Prefill-size steps use
the fused TP path (GEMM epilogue scatter over NVLink -> reduce + RMSNorm +
all-gather -> GEMM waiting on the gather) unless ``--comm nccl``; decode
reduces with NCCL.

    torchrun --nproc-per-node 2 --master-addr 127.0.0.1 -m sglang_legolink_b200.benchmarks.tp_link

Prints one JSON line (rank 0), with the per-rank roofline of the Link and
of a decode step and the achieved fraction of each.

``--shard W`` on ONE process runs one rank's share of TP = W with no
communication (heads, KV heads, intermediate and vocabulary divided by W), to
separate a rank's own kernels from the collectives.  ``--profile`` then
prints, per phase (a Link, eight decode steps), each kernel's share of the
device time and the device idle time between kernels, from the CUDA activity
trace of ``torch.profiler``.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import random
import statistics
import time


NVLINK_GBS = 770.0


def rooflines(cfg, world: int, plan, batch: int, ctx: int, pk: dict) -> dict:
    """Per-rank roofline of one Link and of one batch decode step.

    Link: the slower of (GEMM + attention FLOPs of the repair rows at the
    measured bf16 peak, plus the KV link's HBM bytes at the measured copy
    bandwidth) and (bytes the fused layer boundaries move over NVLink: 2 x
    (W-1)/W x rows x hidden x 2 per boundary, two per layer, at 770 GB/s).
    Decode step: this rank's weight bytes plus the K/V bytes of ``batch``
    contexts of ``ctx`` tokens, at the measured copy bandwidth."""
    L, H, D, I, V = cfg.num_layers, cfg.hidden_size, cfg.head_dim, cfg.intermediate_size, cfg.vocab_size
    hq, hkv = cfg.num_heads // world, max(1, cfg.num_kv_heads // world)
    rows = list(plan.recompute_positions)
    T = len(rows)
    gemm = 2 * T * H * ((hq + 2 * hkv) * D + hq * D + 2 * I // world + I // world) * L
    attn = 4 * D * hq * float(sum(p + 1 for p in rows)) * L
    linked = plan.total_token_count - T
    kv_link_bytes = linked * L * hkv * D * 2 * 2 * 2
    compute_ms = (gemm + attn) / (pk["bf16_tflops"] * 1e9) + kv_link_bytes / (pk["hbm_gbs"] * 1e6)
    nvlink_ms = (2 * 2 * (world - 1) / world * T * H * 2 * L) / (NVLINK_GBS * 1e6) if world > 1 else 0.0
    w_bytes = 2 * L * H * ((hq + 2 * hkv) * D + hq * D + 2 * I // world + I // world) + 2 * H * V // world
    kv_bytes = batch * ctx * L * hkv * D * 2 * 2
    return {"link_roofline_ms": round(max(compute_ms, nvlink_ms), 3),
            "link_roofline_terms_ms": {"compute_and_kv_link": round(compute_ms, 3), "nvlink": round(nvlink_ms, 3)},
            "decode_roofline_ms_per_step": round((w_bytes + kv_bytes) / (pk["hbm_gbs"] * 1e6), 3),
            "peaks": pk["src"]}


def peaks() -> dict:
    from .kernels import peaks as _p

    return _p()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="qwen3-32b")
    ap.add_argument("--context", type=int, default=32768)
    ap.add_argument("--subcontexts", type=int, default=16)
    ap.add_argument("--fresh-frac", type=float, default=0.1)
    ap.add_argument("--repair", type=int, default=64)
    ap.add_argument("--decode", type=int, default=512)
    ap.add_argument("--batch", type=int, default=16)
    ap.add_argument("--comm", default="fused", choices=["fused", "nccl"])
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--shard", type=int, default=1, help="one process: one rank's share of TP = SHARD, no comm")
    ap.add_argument("--profile", action="store_true", help="per-kernel breakdown of a Link and 8 decode steps")
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
    comm = None
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=600), device_id=dev)
        if a.comm == "fused":
            from ..parallel.tp_fused import FusedTPComm

            comm = FusedTPComm(PRESETS[a.model].hidden_size, 16384, dev)
        else:
            from ..parallel.tp import NcclTPComm

            comm = NcclTPComm()
    cfg = PRESETS[a.model]
    if a.shard > 1:
        if world > 1:
            raise SystemExit("--shard runs on one process")
        import dataclasses

        cfg = dataclasses.replace(cfg, num_heads=cfg.num_heads // a.shard,
                                  num_kv_heads=max(1, cfg.num_kv_heads // a.shard),
                                  intermediate_size=cfg.intermediate_size // a.shard,
                                  vocab_size=cfg.vocab_size // a.shard, name=f"{cfg.name}/shard{a.shard}")
    t0 = time.time()
    model = QwenModel.random_init(cfg, seed=a.seed, device=dev, dtype=torch.bfloat16, tp_rank=rank, tp_size=world,
                                  comm=comm)
    rng = random.Random(a.seed)
    # sub-context lengths log-uniform in [64, 4096], rescaled to the context
    raw = [math.exp(rng.uniform(math.log(64), math.log(4096))) for _ in range(a.subcontexts)]
    lens = [max(64, int(r * a.context / sum(raw))) for r in raw]
    lens[-1] += a.context - sum(lens)
    n_fresh = max(1, round(a.subcontexts * a.fresh_frac))
    n_link = a.subcontexts - n_fresh
    ps = 16
    per_seq = pages_for(a.context + 64 + a.decode + 16, ps)
    compiled = sum(pages_for(n, ps) for n in lens[:n_link])
    eng = Engine(model, page_size=ps, max_context=a.context + a.decode + 1024,
                 num_pages=(a.batch + int(a.profile)) * per_seq + compiled + 64)
    init_s = time.time() - t0
    subs = [[rng.randrange(cfg.vocab_size) for _ in range(n)] for n in lens]
    for i in range(n_link):
        eng.compile(subs[i], f"tp-sub-{i}")
    torch.cuda.synchronize()

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def maxr(vals):
        t = torch.tensor(vals, dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return t.tolist()

    def request(i):
        order = list(range(n_link))
        random.Random(1000 + i).shuffle(order)
        fresh = sum((subs[j] for j in range(n_link, a.subcontexts)), [])
        user = [random.Random(2000 + i).randrange(cfg.vocab_size) for _ in range(32)]
        plan = {"cache_keys": [f"tp-sub-{j}" for j in order], "recompute_initial_tokens": a.repair,
                "recompute_first_block": True, "request_id": f"tp-{i}"}
        return plan, fresh + user

    # warm-up: one Link + a short decode (graphs, workspaces)
    plan, suffix = request(-1)
    s = eng.link(plan, suffix)
    eng.decode([s], 4)
    eng.free(s)
    barrier()
    links, seqs, rows = [], [], 0
    for i in range(a.batch):
        plan, suffix = request(i)
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        s = eng.link(plan, suffix)
        e1.record()
        e1.synchronize()
        links.append(e0.elapsed_time(e1))
        rows = len(s.link_plan.recompute_positions)
        seqs.append(s)
    eng.warm_decode(seqs)  # the batch's decode graph is captured before the timed region
    barrier()
    d0, d1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    d0.record()
    eng.decode(seqs, a.decode - 1)
    d1.record()
    d1.synchronize()
    dec_ms = d0.elapsed_time(d1)
    links = maxr(links)
    dec_ms = maxr([dec_ms])[0]
    out = {
        "metric": "Link-request p50 TTFT and decode tok/s, Qwen3-32B TP",
        "model": f"{cfg.name} (random init)", "tp": world, "comm": a.comm if world > 1 else "none",
        "shard": a.shard,
        "context": a.context, "subcontexts": a.subcontexts, "linked": n_link, "repair_window": a.repair,
        "recompute_rows": rows, "batch": a.batch, "decode_tokens": a.decode,
        "link_ttft_ms_p50": round(statistics.median(links), 3), "link_ttft_ms_max": round(max(links), 3),
        "decode_tok_s": round(a.batch * (a.decode - 1) / (dec_ms / 1e3), 1),
        "decode_ms_per_step": round(dec_ms / (a.decode - 1), 3),
        "timing": "CUDA events, max over ranks", "data": "synthetic agent contexts (seeded), random-init weights",
        "init_s": round(init_s, 1),
    }
    out.update(rooflines(cfg, world, seqs[-1].link_plan, a.batch, a.context + 64, peaks()))
    out["link_frac_of_roofline"] = round(out["link_roofline_ms"] / out["link_ttft_ms_p50"], 3)
    out["decode_frac_of_roofline"] = round(out["decode_roofline_ms_per_step"] / out["decode_ms_per_step"], 3)
    if comm is not None and hasattr(comm, "stats"):
        out["fused_stats"] = dict(comm.stats)
    if rank == 0:
        print(json.dumps(out), flush=True)
    if a.profile:
        from torch.profiler import ProfilerActivity, profile, record_function

        from .link_profile import summarize, timeline

        plan, suffix = request(10_000)
        barrier()
        with profile(activities=[ProfilerActivity.CPU, ProfilerActivity.CUDA]) as prof:
            with record_function("link_call"):
                s = eng.link(plan, suffix)
            torch.cuda.synchronize()
        if rank == 0:
            summarize(prof, "link")
            print("   timeline:", timeline(prof, "link_call"), flush=True)
        eng.free(s)
        barrier()
        with profile(activities=[ProfilerActivity.CPU, ProfilerActivity.CUDA]) as prof:
            with record_function("decode_call"):
                eng.decode(seqs, 8)
            torch.cuda.synchronize()
        if rank == 0:
            summarize(prof, f"decode x8, batch {a.batch}")
            print("   timeline:", timeline(prof, "decode_call"), flush=True)
        barrier()
    for s in seqs:
        eng.free(s)
    torch.cuda.synchronize()
    eng._graphs.clear()  # graphs holding NCCL calls are released before the process group
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
