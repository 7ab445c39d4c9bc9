"""Decode attention against its split count (split-K over the key axis).

For each (batch, keys) case the kernel runs on 8 layers of a Qwen2.5-7B-shaped
paged pool (32 query heads, 4 KV heads, head_dim 128, page 16), captured in a
CUDA graph so every launch streams its own layer's KV from HBM, and is timed
with CUDA events for the split count ``ops.decode_splits`` picks and for a
fixed set of alternatives.

    python -m sglang_legolink_b200.benchmarks.decode_attn_splits [--quick]

Prints one JSON line per (case, split): microseconds per layer and the share
of the measured HBM copy bandwidth that the K and V bytes take.
"""

from __future__ import annotations

import argparse
import json
import math

import torch

from .. import ops
from .decode_breakdown import graph_time
from .kernels import peaks

CASES = ((1, 32768), (4, 32768), (16, 32768), (16, 8192), (64, 4096))
ALTERNATIVES = (1, 2, 4, 8, 16, 32, 64)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--quick", action="store_true", help="default split only")
    a = ap.parse_args()
    L, Hq, Hkv, D, ps = 8, 32, 4, 128, 16
    dev = torch.device("cuda")
    pk = peaks()
    for B, n in CASES:
        pages = B * ((n + ps - 1) // ps)
        kp = torch.randn(L, pages, Hkv, ps, D, device=dev, dtype=torch.bfloat16)
        vp = torch.randn_like(kp)
        pt = torch.arange(pages, device=dev, dtype=torch.int32).view(B, -1)
        kvl = torch.full((B,), n, device=dev, dtype=torch.int32)
        q = torch.randn(B, Hq, D, device=dev, dtype=torch.bfloat16)
        out = torch.empty(B, Hq * D, device=dev, dtype=torch.bfloat16)
        chosen = ops.decode_splits(B, Hkv, n)
        splits = [chosen] if a.quick else sorted({chosen, *ALTERNATIVES})
        kv_bytes = B * n * Hkv * D * 2 * 2
        for ns in splits:
            ops.workspace(dev).reserve_decode(B * Hq, ns, D)
            ms = graph_time(lambda: [ops.attention_decode(q, kp[i], vp[i], pt, kvl, 1 / math.sqrt(D), nsplit=ns,
                                                          out=out) for i in range(L)])
            us = ms * 1e3 / L
            print(json.dumps({"batch": B, "keys": n, "nsplit": ns, "chosen": ns == chosen,
                              "us_per_layer": round(us, 1),
                              "frac_of_hbm": round(kv_bytes / (us * 1e-6) / (pk["hbm_gbs"] * 1e9), 3),
                              "peaks": pk["src"]}), flush=True)
        del kp, vp
        torch.cuda.empty_cache()


if __name__ == "__main__":
    main()
