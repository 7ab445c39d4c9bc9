"""Headline benchmark: Link-request p50 TTFT and decode tok/s vs full prefill.

Config: Qwen2.5-7B architecture, bf16, random init,
page size 16.  Synthetic agent context of 12 sub-contexts with lengths
log-uniform in [64, 4096] scaled to 16K tokens in total; 10 are compiled
before timing and linked in a new shuffled order every step, 2 are fresh
(they form the mutable suffix with the user turn).  Repair window 32 tokens
per block boundary; then 256 greedy decode tokens at batch 1.

One step = one Link request (TTFT) + 256 decode tokens + one full prefill of
the same 16K prompt (the baseline the Link is compared to).  With N GPUs
every rank serves its own replica (weak scaling); each per-step time is the
max over ranks.

Reported ``value`` = p50 device-timed Link TTFT in ms (lower is better).
``e2e`` repeats the Link TTFT through the public engine API (plan
resolution, H2D of the step's inputs from pinned host memory, first-token
D2H), host wall clock.

``--impl reference`` runs the unmodified reference.  Its runtime is a patch
series over upstream SGLang that is not vendored and cannot be built offline,
so that arm reports itself unavailable.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import random
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

MEASURED_PEAKS = os.path.join(ROOT, "MEASURED_PEAKS.json")


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=5)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", default="ours", choices=["ours", "reference"])
    p.add_argument("--model", default="qwen2.5-7b")
    p.add_argument("--context", type=int, default=16384)
    p.add_argument("--subcontexts", type=int, default=12)
    p.add_argument("--fresh", type=int, default=2)
    p.add_argument("--repair", type=int, default=32)
    p.add_argument("--decode", type=int, default=256)
    p.add_argument("--page-size", type=int, default=16)
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--no-full-prefill", action="store_true")
    return p.parse_args()


def synthetic_context(n_sub: int, total: int, vocab: int, seed: int):
    """Sub-context lengths log-uniform in [64, 4096], rescaled to ``total``."""
    rng = random.Random(seed)
    raw = [math.exp(rng.uniform(math.log(64), math.log(4096))) for _ in range(n_sub)]
    scale = total / sum(raw)
    lens = [max(64, min(4096, int(round(r * scale)))) for r in raw]
    # fix rounding so the total is exact, respecting the [64, 4096] bounds
    i = 0
    while sum(lens) != total and i < 100000:
        j = i % n_sub
        if sum(lens) < total and lens[j] < 4096:
            lens[j] += 1
        elif sum(lens) > total and lens[j] > 64:
            lens[j] -= 1
        i += 1
    subs = [[rng.randrange(vocab) for _ in range(n)] for n in lens]
    return subs


class ClockSampler:
    """Samples nvidia-smi clocks / throttle reasons during the timed region."""

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.rows = []
        self.proc = None

    def __enter__(self):
        q = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
             "clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.idx), f"--query-gpu={q}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            parts = [x.strip() for x in line.split(",")]
            if len(parts) >= 7:
                self.rows.append(parts)

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        if not self.rows:
            return None
        sm = [float(r[0]) for r in self.rows if r[0].replace(".", "").isdigit()]
        mx = [float(r[1]) for r in self.rows if r[1].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in self.rows for i in range(4) if r[3 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.rows)}


def reference_arm(args):
    why = ("reference runtime is a 28-patch series over upstream SGLang (not vendored; no network to fetch it), "
           "so no Link/decode server can be built offline; only its host package installs")
    print(json.dumps({"impl": "reference", "unavailable": why, "n_gpus": args.gpus}))


def main():
    args = parse()
    if args.impl == "reference":
        if int(os.environ.get("RANK", "0")) == 0:
            reference_arm(args)
        return
    import torch
    import torch.distributed as dist

    from sglang_legolink_b200 import ops
    from sglang_legolink_b200.models.config import PRESETS
    from sglang_legolink_b200.models.qwen import QwenModel
    from sglang_legolink_b200.runtime.engine import Engine
    from sglang_legolink_b200.utils.launch_count import LaunchCounter

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=600), device_id=dev)

    cfg = PRESETS[args.model]
    t0 = time.time()
    model = QwenModel.random_init(cfg, seed=args.seed, device=dev, dtype=torch.bfloat16)
    torch.cuda.synchronize()
    eng = Engine(model, page_size=args.page_size, max_context=args.context + args.decode + 1024,
                 mem_fraction=0.6)
    init_s = time.time() - t0

    subs = synthetic_context(args.subcontexts, args.context, cfg.vocab_size, args.seed)
    n_link = args.subcontexts - args.fresh
    prefix = [151644, 8948, 198]  # chat-template header tokens (system turn start)
    for i in range(n_link):
        eng.compile(subs[i], f"sub-{i}")
    fresh = sum(subs[n_link:], [])
    rng = random.Random(args.seed + 1 + rank)

    def make_request(step):
        order = list(range(n_link))
        rng.shuffle(order)
        user = [rng.randrange(cfg.vocab_size) for _ in range(32)]
        suffix = fresh + user
        plan = {"cache_keys": [f"sub-{i}" for i in order], "recompute_initial_tokens": args.repair,
                "recompute_first_block": True, "request_id": f"bench-{rank}-{step}"}
        full = sum((subs[i] for i in order), []) + suffix
        return plan, suffix, full

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(vals):
        t = torch.tensor(vals, dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return t.tolist()

    def sum_over_ranks(vals):
        t = torch.tensor(vals, dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.SUM)
        return t.tolist()

    counter = LaunchCounter()

    def one_step(step, timed):
        """Full prefill + its decode (the baseline), then Link + its decode.
        Both timed prefills start from the same GPU state -- the end of a
        decode -- so neither inherits the other's power-capped clocks (a
        Link issued right after a 16K-token dense prefill starts at
        ~1.3-1.4 GHz under sw_power_cap instead of 1.97 GHz)."""
        plan, suffix, full = make_request(step)
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(8)]
        fp_ms = float("nan")
        if not args.no_full_prefill:
            # --- full prefill baseline, decoded like the Link
            ev[4].record()
            base = eng.prefill(full)
            ev[5].record()
            eng.decode([base], args.decode - 1)
            ev[6].record()
            eng.free(base)
        # --- Link (device-timed TTFT; e2e measured by the host around the API call)
        torch.cuda.synchronize()
        h0 = time.perf_counter()
        ev[0].record()
        seq = eng.link(plan, suffix)  # returns after the first token reached the host
        ev[1].record()
        h1 = time.perf_counter()
        # --- decode
        ev[2].record()
        eng.decode([seq], args.decode - 1)
        ev[3].record()
        eng.free(seq)
        torch.cuda.synchronize()
        link_ms = ev[0].elapsed_time(ev[1])
        dec_ms = ev[2].elapsed_time(ev[3])
        if not args.no_full_prefill:
            fp_ms = ev[4].elapsed_time(ev[5])
        return link_ms, dec_ms, fp_ms, (h1 - h0) * 1e3, len(plan["imp_indices"])

    for w in range(args.warmup):
        one_step(-1 - w, False)
    barrier()
    links, decs, fps, e2es = [], [], [], []
    rows = 0
    with ClockSampler(local) as clocks:
        counter.start()
        barrier()
        t_start = torch.cuda.Event(enable_timing=True)
        t_end = torch.cuda.Event(enable_timing=True)
        t_start.record()
        for s in range(args.steps):
            l, d, f, e, rows = one_step(s, True)
            links.append(l), decs.append(d), fps.append(f), e2es.append(e)
        t_end.record()
        barrier()
        launches = counter.stop()
    total_ms = t_start.elapsed_time(t_end)
    links = max_over_ranks(links)
    decs = max_over_ranks(decs)
    fps = max_over_ranks(fps)
    e2es = max_over_ranks(e2es)
    total_ms = max_over_ranks([total_ms])[0]
    dec_tok_s_rank = (args.decode - 1) / (statistics.median(decs) / 1e3)
    dec_tok_s = sum_over_ranks([dec_tok_s_rank])[0]
    link_p50 = statistics.median(links)
    fp_p50 = statistics.median(fps) if not args.no_full_prefill else None
    clk = clocks.summary()
    # bytes per step moved by the public API around the Link: token ids of the
    # recomputed rows + positions + slots + page table + link gather lists in,
    # the first token id out (the decode adds 4 B per generated token out).
    n_tot = args.context + 32 + 0
    pages = (n_tot + args.page_size - 1) // args.page_size
    linked = n_tot - rows
    h2d = rows * (4 + 4 + 8) + pages * 4 + linked * (8 + 8 + 4 + 4)
    if rank == 0:
        out = {
            "metric": "Link-request p50 TTFT and decode tok/s vs full prefill, 1/2/4/8 B200",
            "value": round(link_p50, 3),
            "unit": "ms",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(total_ms / args.steps, 3),
            "higher_is_better": False,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic agent context (seeded), random-init weights",
            "config": {
                "model": f"{args.model} (random init)",
                "global_batch": world,
                "seq_len": args.context,
                "parallelism": f"dp{world}" if world > 1 else "single",
                "subcontexts": args.subcontexts,
                "linked": n_link,
                "fresh": args.fresh,
                "repair_window": args.repair,
                "recompute_rows": rows,
                "decode_tokens": args.decode,
                "page_size": args.page_size,
                "l2": "inputs larger than L2: 15.2 GB weights and 0.9 GB of KV per request are streamed each step",
                "step": "full prefill + 255-token decode (baseline), then Link + 255-token decode; each timed "
                        "prefill starts after a decode",
            },
            "link_ttft_ms_p50": round(link_p50, 3),
            "full_prefill_ttft_ms_p50": round(fp_p50, 3) if fp_p50 is not None else None,
            "ttft_speedup_vs_full_prefill": round(fp_p50 / link_p50, 3) if fp_p50 else None,
            "decode_tok_s": round(dec_tok_s, 2),
            "decode_tok_s_per_gpu": round(dec_tok_s_rank, 2),
            "decode_ms_per_token": round(statistics.median(decs) / (args.decode - 1), 4),
            "e2e": {"value": round(statistics.median(e2es), 3), "unit": "ms",
                    "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": 4 * args.decode},
            "gpu_launches": launches,
            "clocks": clk,
            "init_s": round(init_s, 1),
        }
        print(json.dumps(out))
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
