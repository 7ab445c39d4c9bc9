"""Per-kernel device-time breakdown of one Link, one full prefill and a few
decode steps on the headline configuration (Qwen2.5-7B, 16K context, 12
sub-contexts, 10 linked, repair window 32), from the CUDA activity trace of
``torch.profiler`` (kernel durations as the driver reports them; no replay).

    python -m sglang_legolink_b200.benchmarks.link_profile [--decode 8]

Prints, per phase, each kernel's share of the phase's summed kernel time.
"""

from __future__ import annotations

import argparse
import random
from collections import defaultdict

import torch

from ..models.config import PRESETS
from ..models.qwen import QwenModel
from ..runtime.engine import Engine


def synthetic_context(n_sub: int, total: int, vocab: int, seed: int):
    rng = random.Random(seed)
    raw = [2 ** rng.uniform(6, 12) for _ in range(n_sub)]
    scale = total / sum(raw)
    lens = [max(16, int(x * scale)) for x in raw]
    return [[rng.randrange(vocab) for _ in range(n)] for n in lens]


def summarize(prof, label):
    agg = defaultdict(lambda: [0.0, 0])
    for e in prof.events():
        if e.device_type == torch.autograd.DeviceType.CUDA:
            k = e.name.split("(")[0][:90]
            agg[k][0] += e.device_time_total if hasattr(e, "device_time_total") else e.cuda_time_total
            agg[k][1] += 1
    tot = sum(v[0] for v in agg.values())
    print(f"== {label}: {tot / 1e3:.2f} ms of kernel time, {sum(v[1] for v in agg.values())} launches")
    for k, (us, n) in sorted(agg.items(), key=lambda kv: -kv[1][0])[:14]:
        print(f"  {us / 1e3:8.3f} ms {100 * us / max(tot, 1e-9):5.1f}%  x{n:<5d} {k}")


def timeline(prof, marker: str) -> dict:
    """Where the wall time of the ``marker`` CPU range went: host work before
    the first kernel, device idle gaps between kernels, kernel time, and the
    tail after the last kernel (microseconds, one clock: the profiler's)."""
    mk = [e for e in prof.events() if e.name == marker and e.device_type == torch.autograd.DeviceType.CPU]
    ks = sorted((e.time_range.start, e.time_range.end) for e in prof.events()
                if e.device_type == torch.autograd.DeviceType.CUDA and e.time_range.end > e.time_range.start)
    if not mk or not ks:
        return {}
    t0, t1 = mk[0].time_range.start, mk[0].time_range.end
    busy, gaps, end = 0.0, 0.0, ks[0][0]
    for a, b in ks:
        if a > end:
            gaps += a - end
        busy += max(0.0, b - max(a, end))
        end = max(end, b)
    return {"wall_us": round(t1 - t0, 1), "host_before_first_kernel_us": round(ks[0][0] - t0, 1),
            "device_busy_us": round(busy, 1), "device_idle_gaps_us": round(gaps, 1),
            "after_last_kernel_us": round(t1 - end, 1)}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="qwen2.5-7b")
    ap.add_argument("--context", type=int, default=16384)
    ap.add_argument("--decode", type=int, default=8)
    a = ap.parse_args()
    cfg = PRESETS[a.model]
    model = QwenModel.random_init(cfg, seed=0, device="cuda", dtype=torch.bfloat16)
    eng = Engine(model, page_size=16, max_context=a.context + 2048, mem_fraction=0.6)
    subs = synthetic_context(12, a.context, cfg.vocab_size, 0)
    for i in range(10):
        eng.compile(subs[i], f"sub-{i}")
    suffix = sum(subs[10:], []) + list(range(1000, 1032))
    plan = {"cache_keys": [f"sub-{i}" for i in range(9, -1, -1)], "recompute_initial_tokens": 32,
            "recompute_first_block": True}
    full = sum((subs[i] for i in range(9, -1, -1)), []) + suffix
    # warm-up (graphs, workspaces)
    s = eng.link(dict(plan), suffix)
    eng.decode([s], 2)
    eng.free(s)
    torch.cuda.synchronize()
    acts = [torch.profiler.ProfilerActivity.CUDA]
    acts_cpu = acts + [torch.profiler.ProfilerActivity.CPU]
    with torch.profiler.profile(activities=acts_cpu) as p:
        with torch.profiler.record_function("link_call"):
            s = eng.link(dict(plan), suffix)
            torch.cuda.synchronize()
    summarize(p, "link")
    print("   timeline:", timeline(p, "link_call"))
    with torch.profiler.profile(activities=acts) as p:
        eng.decode([s], a.decode)
        torch.cuda.synchronize()
    summarize(p, f"decode x{a.decode}")
    eng.free(s)
    with torch.profiler.profile(activities=acts) as p:
        b = eng.prefill(full)
        torch.cuda.synchronize()
    summarize(p, "full prefill")
    eng.free(b)


if __name__ == "__main__":
    main()
