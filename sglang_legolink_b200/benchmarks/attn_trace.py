"""Per-block timeline of the tcgen05 repair-attention kernel.

Runs the Link repair case (5087 rows at sorted random positions of a 16K
context, 28 q / 4 kv heads, head_dim 128) with the clock64() trace builds of
the kernel and prints, for CTA 0 (the longest tile), the median cycles of
each hand-off over the steady-state blocks:

* softmax: S seen -> TMEM load done -> row max -> each 32-column P store ->
  p_full arrive, for tile 0 (the chunk events) and tile 1 (totals);
* MMA side: p_full arrive -> the MMA thread sees it, S commit -> the
  softmax sees S (the tensor pipe's PV + S of that tile plus any queue);
* the block period and how long the two tiles' softmax intervals overlap.

    python -m sglang_legolink_b200.benchmarks.attn_trace [--variants 5,9]

Variants are indices of the kernel's build table (trace builds: 5 with one
softmax warpgroup per tile, 6 with two warpgroups of 64 key columns each, 9
with the 8-chain max and P stored after the whole row).
"""

from __future__ import annotations

import argparse
import json
import math
import statistics

import torch

from sglang_legolink_b200 import ops

# event slots written by the kernel (TC_TR)
S_SEEN, LD_DONE, ARRIVE = (0, 3), (1, 4), (2, 5)
MMA_K_SEEN, MMA_P_SEEN, MMA_S_COMMIT = 6, (7, 8), (9, 10)
MAX_DONE, CHUNK, RESCALE_DONE, MASK_DONE = 11, (12, 13, 14, 15), 16, 17


def _case(seed: int = 0):
    torch.manual_seed(seed)
    D, ps, Hq, Hkv, n, qrows = 128, 16, 28, 4, 16384, 5087
    pages = n // ps
    kp = torch.randn(1, pages, Hkv, ps, D, device="cuda", dtype=torch.bfloat16)
    vp = torch.randn_like(kp)
    pt = torch.randperm(pages, device="cuda").to(torch.int32)[None]
    pos = torch.sort(torch.randperm(n)[:qrows]).values.to(torch.int32)
    qi = torch.tensor([0, qrows], dtype=torch.int32)
    tiles = ops.prefill_tiles(qi, pos, Hq, Hkv).cuda()
    q = torch.randn(qrows, Hq, D, device="cuda", dtype=torch.bfloat16)
    kvl = torch.tensor([n], dtype=torch.int32, device="cuda")
    out = torch.empty(qrows, Hq * D, device="cuda", dtype=torch.bfloat16)
    nb = int(tiles[0, 3]) // 128 + 1
    return (lambda: ops.attention_prefill(q, kp, vp, 0, qi.cuda(), pos.cuda(), pt, kvl, 1 / math.sqrt(D),
                                          tiles=tiles, out=out)), nb


def _med(xs):
    xs = [x for x in xs if x is not None]
    return round(statistics.median(xs), 1) if xs else None


def summarize(tr: torch.Tensor, nb: int) -> dict:
    """Median cycle deltas over blocks [4, nb - 4) of one trace [256, 20]."""
    t = tr.tolist()
    js = range(4, max(5, min(nb, 256) - 4))

    def d(j1, e1, j0, e0):
        a, b = t[j1][e1], t[j0][e0]
        return a - b if a and b else None

    r = {"blocks": nb}
    for tile in (0, 1):
        r[f"softmax{tile}_total"] = _med([d(j, ARRIVE[tile], j, S_SEEN[tile]) for j in js])
        r[f"softmax{tile}_tmem_load"] = _med([d(j, LD_DONE[tile], j, S_SEEN[tile]) for j in js])
        r[f"mma_sees_p{tile}"] = _med([d(j + 1, MMA_P_SEEN[tile], j, ARRIVE[tile]) for j in js])
        r[f"s{tile}_commit_to_seen"] = _med([d(j, S_SEEN[tile], j, MMA_S_COMMIT[tile]) for j in js])
        r[f"p{tile}_arrive_to_s_seen"] = _med([d(j + 1, S_SEEN[tile], j, ARRIVE[tile]) for j in js])
    r["t0_max"] = _med([d(j, MAX_DONE, j, LD_DONE[0]) for j in js])
    r["t0_exp_chunks"] = [_med([d(j, CHUNK[c], j, CHUNK[c - 1] if c else MAX_DONE) for j in js]) for c in range(4)]
    r["t0_tail"] = _med([d(j, ARRIVE[0], j, CHUNK[3]) for j in js])
    r["period"] = _med([d(j + 1, S_SEEN[0], j, S_SEEN[0]) for j in js])
    ov = []
    for j in js:
        a0, a1, b0, b1 = t[j][S_SEEN[0]], t[j][ARRIVE[0]], t[j][S_SEEN[1]], t[j][ARRIVE[1]]
        if a0 and a1 and b0 and b1:
            ov.append(max(0, min(a1, b1) - max(a0, b0)))
    r["softmax_overlap"] = _med(ov)
    return r


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--variants", default="5,9")
    a = ap.parse_args()
    ext = ops._cuda()
    fn, nb = _case()
    for v in (int(x) for x in a.variants.split(",")):
        ext.attn_prefill_tc_set_variant(v)
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        r = summarize(ext.attn_prefill_tc_trace(), nb)
        r["variant"] = v
        print(json.dumps(r), flush=True)
    ext.attn_prefill_tc_set_variant(-2)


if __name__ == "__main__":
    main()
