"""Prefill attention with key-range splits: time per layer against the split
count S on the repair rows of the Qwen3-32B tensor-parallel Link (32K-token
context in 16 sub-contexts, 14 linked, repair window 64: 3291 rows; the same
synthetic context as ``benchmarks/tp_link.py``), for one rank's heads at
TP = 1/2/4/8 (64/32/16/8 query heads over 8/4/2/1 KV heads).  Each S runs
the tcgen05 kernel on the work list split S ways plus the combine, on 8
layers' K/V pools in turn (inputs larger than L2), timed with CUDA events;
the model's prediction (``ops.prefill_split_time_us``) and its choice are
printed beside the measurement.

    python -m sglang_legolink_b200.benchmarks.attn_split [--shards 8,4,2,1]
"""

from __future__ import annotations

import argparse
import json
import math
import random
import statistics

import torch

from .. import ops
from ..runtime.link_plan import resolve_link_plan


def tp_link_rows(context=32768, subcontexts=16, fresh_frac=0.1, repair=64, seed=0, vocab=151936, request=0):
    """Recompute positions of request ``request`` of the tp_link benchmark."""
    rng = random.Random(seed)
    raw = [math.exp(rng.uniform(math.log(64), math.log(4096))) for _ in range(subcontexts)]
    lens = [max(64, int(r * context / sum(raw))) for r in raw]
    lens[-1] += context - sum(lens)
    n_fresh = max(1, round(subcontexts * fresh_frac))
    n_link = subcontexts - n_fresh
    subs = [[rng.randrange(vocab) for _ in range(n)] for n in lens]
    order = list(range(n_link))
    random.Random(1000 + request).shuffle(order)
    fresh = sum((subs[j] for j in range(n_link, subcontexts)), [])
    user = [random.Random(2000 + request).randrange(vocab) for _ in range(32)]
    plan = {"cache_keys": [f"tp-sub-{j}" for j in order], "recompute_initial_tokens": repair,
            "recompute_first_block": True}
    p = resolve_link_plan(plan, fresh + user, lambda k: subs[int(k.split("-")[2])], validate=False)
    return sorted(p.recompute_positions), p.total_token_count


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--shards", default="8,4,2,1")
    ap.add_argument("--layers", type=int, default=8)
    a = ap.parse_args()
    dev = torch.device("cuda")
    rows, total = tp_link_rows()
    T, D, ps, L = len(rows), 128, 16, a.layers
    pages = (total + ps - 1) // ps
    qi = torch.tensor([0, T], dtype=torch.int32)
    qp = torch.tensor(rows, dtype=torch.int32)
    pt = torch.arange(pages, dtype=torch.int32)[None].to(dev)
    kvl = torch.tensor([total], dtype=torch.int32, device=dev)
    scale = 1 / math.sqrt(D)
    for w in [int(x) for x in a.shards.split(",")]:
        Hq, Hkv = 64 // w, max(1, 8 // w)
        g = torch.Generator(device="cpu").manual_seed(w)
        q = torch.randn(T, Hq, D, generator=g).to(torch.bfloat16).to(dev)
        kp = torch.randn(L, pages, Hkv, ps, D, device=dev, dtype=torch.bfloat16)
        vp = torch.randn_like(kp)
        out = torch.empty(T, Hq * D, device=dev, dtype=torch.bfloat16)
        base = ops.prefill_tiles(qi, qp, Hq, Hkv).numpy()
        nb = base[:, 3] // ops.PREFILL_BLOCK_KEYS + 1
        choice = ops.prefill_split_count(nb, T * Hq)
        ref_out = None
        for S in ops.PREFILL_SPLIT_CHOICES:
            if T * Hq * S * 520 > ops.PREFILL_SPLIT_MAX_WS_BYTES:
                break
            tiles = ops.prefill_tiles(qi, qp, Hq, Hkv, split=S).to(dev)
            qid, posd = qi.to(dev), qp.to(dev)

            def run():
                for li in range(L):
                    ops.attention_prefill(q, kp, vp, li, qid, posd, pt, kvl, scale, tiles=tiles, out=out, nsplit=S)

            run()
            torch.cuda.synchronize()
            if ops.check_errors(dev):
                raise SystemExit(f"device error at S={S}")
            ts = []
            for _ in range(5):
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                run()
                e1.record()
                e1.synchronize()
                ts.append(e0.elapsed_time(e1) * 1e3 / L)
            if ref_out is None:
                ref_out = out.clone()
            err = ((out.float() - ref_out.float()).norm() / ref_out.float().norm()).item()
            print(json.dumps({"tp": w, "q_heads": Hq, "kv_heads": Hkv, "rows": T, "tiles": len(base), "S": S,
                              "us_per_layer": round(statistics.median(ts), 1),
                              "model_us": round(ops.prefill_split_time_us(nb, T * Hq, S), 1),
                              "model_choice": choice, "rel_diff_vs_S1": round(err, 5)}), flush=True)
        del kp, vp
        torch.cuda.empty_cache()


if __name__ == "__main__":
    main()
