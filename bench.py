"""Headline benchmark: Link-request p50 TTFT and decode tok/s vs full prefill.

Config: Qwen2.5-7B architecture, bf16, random init,
page size 16.  Synthetic agent context of 12 sub-contexts with lengths
log-uniform in [64, 4096] scaled to 16K tokens in total; 10 are compiled
before timing and linked in a new shuffled order every step, 2 are fresh
(they form the mutable suffix with the user turn).  Repair window 32 tokens
per block boundary; then 256 greedy decode tokens at batch 1.

One step = one full prefill of the 16K prompt + its 256-token decode (the
baseline the Link is compared to), then one Link request (TTFT) + its
256-token decode.

With N GPUs (one process per GPU, ``torchrun``) the ranks are DP replicas
that share ONE block directory and map each other's KV pools (symmetric
memory): every rank compiles its own 10 blocks once, and every Link reads a
token-balanced half of its blocks from the next rank's pool over NVLink
inside the fused link kernel (gather + RoPE delta + scatter in one pass),
the other half from its own pool.  Per-GPU work is fixed (weak scaling);
each per-step time is the max over ranks.

Reported ``value`` = p50 over steps of the device-timed Link TTFT in ms
(lower is better), max over ranks.  ``e2e`` is the same Link through the
public engine API timed by the host (plan resolution, directory grace-period
ticket, H2D of the step's inputs from pinned host memory, first-token D2H).
``repair_agreement`` compares each Link's 256 greedy tokens with the full
prefill's (sparse windows are an approximation: reported, not claimed);
``exact_repair_match`` is one Link with full windows checked token for token
against the full prefill during warm-up.

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


def context_lengths(n_sub: int, total: int, seed: int) -> list[int]:
    """Sub-context lengths log-uniform in [64, 4096], rescaled to ``total``
    (the same on every rank, so per-GPU work is identical)."""
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
    return lens


def context_tokens(lens: list[int], vocab: int, seed: int, owner: int) -> list[list[int]]:
    """The token ids of the sub-contexts compiled by replica ``owner``."""
    rng = random.Random(seed * 7919 + 1 + owner)
    return [[rng.randrange(vocab) for _ in range(n)] for n in lens]


def peer_half(lens: list[int]) -> set[int]:
    """Indices of the blocks a Link reads from a peer: a greedy split of the
    linked blocks into two halves of about equal token count."""
    order = sorted(range(len(lens)), key=lambda i: -lens[i])
    a, b, sa, sb = [], [], 0, 0
    for i in order:
        if sa <= sb:
            a.append(i)
            sa += lens[i]
        else:
            b.append(i)
            sb += lens[i]
    return set(b)


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
    # the KV pools are mapped peer to peer; no NVLink multicast object is needed
    os.environ.setdefault("TORCH_SYMM_MEM_DISABLE_MULTICAST", "1")
    import torch
    import torch.distributed as dist

    from sglang_legolink_b200.models.config import PRESETS
    from sglang_legolink_b200.models.qwen import QwenModel
    from sglang_legolink_b200.runtime.engine import Engine, pages_for
    from sglang_legolink_b200.utils.launch_count import LaunchCounter
    from sglang_legolink_b200.utils.trace import CudaTimer

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
    n_tot = args.context + 32
    seq_pages = pages_for(n_tot + args.decode + 64, args.page_size)
    # own compiled blocks + the Link's and the full prefill's sequences (+ the
    # exact-repair check's) + slack; one size on every rank (symmetric memory)
    num_pages = pages_for(args.context, args.page_size) + 3 * seq_pages + 1024
    max_ctx = args.context + args.decode + 1024
    peer = (rank + 1) % world
    if world > 1:
        from sglang_legolink_b200.parallel.dp import BlockDirectory, SharedKVPool

        pool = SharedKVPool(cfg.num_layers, num_pages, model.hkv, args.page_size, cfg.head_dim, torch.bfloat16, dev)
        directory = BlockDirectory(dist.distributed_c10d._get_default_store(), prefix="bench/", world=world)
        eng = Engine(model, page_size=args.page_size, max_context=max_ctx, kv_pool=pool, directory=directory,
                     replica_rank=rank, peer_pools={r: pool.peer(r) for r in range(world) if r != rank})
    else:
        eng = Engine(model, page_size=args.page_size, max_context=max_ctx, num_pages=num_pages)
    init_s = time.time() - t0

    n_link = args.subcontexts - args.fresh
    lens = context_lengths(args.subcontexts, args.context, args.seed)
    own = context_tokens(lens, cfg.vocab_size, args.seed, rank)
    # every block is compiled once on the node: by its owner
    for i in range(n_link):
        eng.compile(own[i], f"sub-{rank}-{i}")
    remote_idx = peer_half(lens[:n_link]) if world > 1 else set()
    nxt = context_tokens(lens, cfg.vocab_size, args.seed, peer) if world > 1 else own
    src_owner = {i: (peer if i in remote_idx else rank) for i in range(n_link)}
    block_toks = {i: (nxt[i] if i in remote_idx else own[i]) for i in range(n_link)}
    fresh = sum(own[n_link:], [])
    peer_tokens = sum(lens[i] for i in remote_idx)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()  # every rank's blocks are published before any Link
    rng = random.Random(args.seed + 1 + rank)

    def make_request(step, exact=False):
        order = list(range(n_link))
        rng.shuffle(order)
        user = [rng.randrange(cfg.vocab_size) for _ in range(32)]
        suffix = fresh + user
        plan = {"cache_keys": [f"sub-{src_owner[i]}-{i}" for i in order], "request_id": f"bench-{rank}-{step}"}
        if exact:
            plan["recompute_tokens_per_block"] = [lens[i] for i in order]
        else:
            plan.update(recompute_initial_tokens=args.repair, recompute_first_block=True)
        full = sum((block_toks[i] for i in order), []) + suffix
        return plan, suffix, full

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def reduce(vals, op):
        t = torch.tensor(vals, dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(t, op=op)
        return t.tolist()

    counter = LaunchCounter()

    def one_step(step, exact=False):
        """Full prefill + its decode (the baseline), then Link + its decode.
        Both timed prefills start from the same GPU state -- the end of a
        decode -- so neither inherits the other's power-capped clocks (a
        Link issued right after a 16K-token dense prefill starts at
        ~1.3-1.4 GHz under sw_power_cap instead of 1.97 GHz)."""
        plan, suffix, full = make_request(step, exact)
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(8)]
        fp_ms, base_out = float("nan"), None
        if not args.no_full_prefill:
            ev[4].record()
            base = eng.prefill(full)
            ev[5].record()
            eng.decode([base], args.decode - 1)
            ev[6].record()
            base_out = list(base.output_ids)
            eng.free(base)
        timer = CudaTimer(enabled=True)
        torch.cuda.synchronize()
        h0 = time.perf_counter()
        ev[0].record()
        seq = eng.link(plan, suffix, timer=timer)  # returns after the first token reached the host
        ev[1].record()
        h1 = time.perf_counter()
        ev[2].record()
        eng.decode([seq], args.decode - 1)
        ev[3].record()
        link_out = list(seq.output_ids)
        eng.free(seq)
        torch.cuda.synchronize()
        spans = timer.finalize()
        r = {"link": ev[0].elapsed_time(ev[1]), "dec": ev[2].elapsed_time(ev[3]), "e2e": (h1 - h0) * 1e3,
             "rows": len(plan["imp_indices"]), "peer_ms": spans.get("kv_link_peer", 0.0),
             "local_ms": spans.get("kv_link_local", 0.0), "fp": float("nan"), "first": float("nan"),
             "prefix": float("nan")}
        if base_out is not None:
            r["fp"] = ev[4].elapsed_time(ev[5])
            r["first"] = float(link_out[0] == base_out[0])
            n = 0
            while n < min(len(link_out), len(base_out)) and link_out[n] == base_out[n]:
                n += 1
            r["prefix"] = float(n)
        return r

    exact_prefix = None
    for w in range(args.warmup):
        r = one_step(-1 - w, exact=(w == 0 and not args.no_full_prefill))
        if w == 0 and not args.no_full_prefill:
            exact_prefix = r["prefix"]
    exact_all = reduce([exact_prefix], dist.ReduceOp.MIN if world > 1 else None)[0] \
        if exact_prefix is not None else None
    barrier()
    res = []
    with ClockSampler(local) as clocks:
        counter.start()
        barrier()
        t_start = torch.cuda.Event(enable_timing=True)
        t_end = torch.cuda.Event(enable_timing=True)
        t_start.record()
        for s in range(args.steps):
            res.append(one_step(s))
        t_end.record()
        barrier()
        launches = counter.stop()
    total_ms = t_start.elapsed_time(t_end)
    MAX = dist.ReduceOp.MAX if world > 1 else None
    SUM = dist.ReduceOp.SUM if world > 1 else None
    col = lambda k: [r[k] for r in res]  # noqa: E731
    links, decs, fps, e2es = (reduce(col(k), MAX) for k in ("link", "dec", "fp", "e2e"))
    peer_ms = reduce(col("peer_ms"), MAX)
    total_ms = reduce([total_ms], MAX)[0]
    firsts = reduce(col("first"), SUM)
    prefixes = reduce(col("prefix"), SUM)
    launches = int(reduce([launches], SUM)[0])
    rows = res[-1]["rows"]
    dec_tok_s_rank = (args.decode - 1) / (statistics.median(col("dec")) / 1e3)
    dec_tok_s = reduce([dec_tok_s_rank], SUM)[0]
    link_p50 = statistics.median(links)
    fp_p50 = statistics.median(fps) if not args.no_full_prefill else None
    clk = clocks.summary()
    # bytes per step moved by the public API around the Link: token ids of the
    # recomputed rows + positions + slots + page table + link gather lists in,
    # the first token id out (the decode adds 4 B per generated token out).
    pages = (n_tot + args.page_size - 1) // args.page_size
    linked = n_tot - rows
    h2d = rows * (4 + 4 + 8) + pages * 4 + linked * (8 + 8 + 4 + 4)
    kv_bytes_per_token = 2 * cfg.num_layers * model.hkv * cfg.head_dim * 2
    peer_link = None
    if world > 1:
        pm = statistics.median(peer_ms)
        gbs = peer_tokens * kv_bytes_per_token / (pm * 1e-3) / 1e9 if pm > 0 else None
        peer_link = {"tokens_per_link": peer_tokens, "bytes_per_link": peer_tokens * kv_bytes_per_token,
                     "kernel_ms_p50": round(pm, 4), "gbs": round(gbs, 1) if gbs else None,
                     "roofline": "NVLink peer read, measured 770 GB/s per direction",
                     "frac_of_measured_nvlink": round(gbs / 770.0, 3) if gbs else None}
    nsteps = args.steps * world
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
                "parallelism": f"dp{world} sharing one block directory" if world > 1 else "single",
                "subcontexts": args.subcontexts,
                "linked": n_link,
                "fresh": args.fresh,
                "repair_window": args.repair,
                "recompute_rows": rows,
                "decode_tokens": args.decode,
                "page_size": args.page_size,
                "peer_blocks_per_link": len(remote_idx),
                "peer_token_fraction": round(peer_tokens / max(1, sum(lens[:n_link])), 3),
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
            "repair_agreement": None if args.no_full_prefill else {
                "first_token_match_frac": round(sum(firsts) / nsteps, 3),
                "greedy_prefix_match_mean": round(sum(prefixes) / nsteps, 2),
                "of_tokens": args.decode, "links": nsteps},
            "exact_repair_match": None if exact_all is None else bool(exact_all >= args.decode),
            "exact_repair_prefix_match": None if exact_all is None else int(exact_all),
            "peer_link": peer_link,
            "e2e": {"value": round(statistics.median(e2es), 3), "unit": "ms",
                    "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": 4 * args.decode},
            "gpu_launches": launches,
            "clocks": clk,
            "init_s": round(init_s, 1),
        }
        print(json.dumps(out), flush=True)
    if world > 1:
        eng.release_graphs()
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
