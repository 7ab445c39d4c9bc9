"""Kernel microbenchmarks with roofline fractions.

Each case is timed with CUDA events on the launching stream after warm-up,
with an L2 flush (a 256 MB write) between timed iterations, and reported as
achieved TFLOP/s or GB/s and the fraction of the measured peaks in
``MEASURED_PEAKS.json`` (copy bandwidth, cuBLAS bf16 GEMM), or of the
documented fallback when that file is absent.

Usage: ``python -m sglang_legolink_b200.benchmarks.kernels [--only gemm,attn,...] [--torch]``
(``--torch`` adds the cuBLAS / torch reference of each op on the same shapes).
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics

import torch

from .. import ops
from ..ops import reference as ref

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"], "src": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "src": "fallback"}


_flush = None


def flush_l2():
    global _flush
    if _flush is None:
        _flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    _flush.fill_(1)


def time_fn(fn, iters=10, warmup=3):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    ts = []
    for _ in range(iters):
        flush_l2()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        b.synchronize()
        ts.append(a.elapsed_time(b))
    return statistics.median(ts)


def bench_gemm(pk, with_torch):
    rows = []
    shapes = [  # Qwen2.5-7B linear layers at Link-repair (M=5087) and prefill (16384) row counts
        ("qkv", 5087, 4608, 3584), ("o_proj", 5087, 3584, 3584), ("gate_up", 5087, 37888, 3584),
        ("down", 5087, 3584, 18944), ("gate_up", 16384, 37888, 3584), ("down", 16384, 3584, 18944),
        ("square8k", 8192, 8192, 8192),
    ]
    for name, M, N, K in shapes:
        a = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
        w = torch.randn(N, K, device="cuda", dtype=torch.bfloat16) / math.sqrt(K)
        out = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
        ms = time_fn(lambda: ops.linear(a, w, out=out))
        tf = 2 * M * N * K / ms / 1e9
        r = {"op": f"gemm_tcgen05[{name}]", "M": M, "N": N, "K": K, "ms": round(ms, 4), "tflops": round(tf, 1),
             "frac_of_peak": round(tf / pk["bf16_tflops"], 3)}
        if with_torch:
            mt = time_fn(lambda: torch.matmul(a, w.t(), out=out))
            r["cublas_ms"] = round(mt, 4)
            r["cublas_tflops"] = round(2 * M * N * K / mt / 1e9, 1)
        rows.append(r)
    return rows


def bench_small_m(pk, with_torch):
    rows = []
    for name, M, N, K in [("qkv", 1, 4608, 3584), ("gate_up", 1, 37888, 3584), ("down", 1, 3584, 18944),
                          ("o_proj", 1, 3584, 3584), ("lm_head", 1, 152064, 3584), ("gate_up_b16", 16, 37888, 3584),
                          ("down_b16", 16, 3584, 18944)]:
        a = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
        w = torch.randn(N, K, device="cuda", dtype=torch.bfloat16) / math.sqrt(K)
        out = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
        ms = time_fn(lambda: ops.linear(a, w, out=out))
        gbs = (N * K * 2 + M * K * 2 + M * N * 2) / ms / 1e6
        r = {"op": f"gemm_small_m[{name}]", "M": M, "N": N, "K": K, "ms": round(ms, 4), "gbs": round(gbs, 1),
             "frac_of_hbm": round(gbs / pk["hbm_gbs"], 3)}
        if N % 128 == 0 and K % 64 == 0:
            wt = ops.tile_weight(w)
            ext, wsp = ops._cuda(), ops.workspace("cuda")
            mt = time_fn(lambda: ops._small_m(ext, wsp, a, wt, None, out))
            r["tile_major_ms"] = round(mt, 4)
            r["tile_major_frac_of_hbm"] = round((N * K * 2 + M * K * 2 + M * N * 2) / mt / 1e6 / pk["hbm_gbs"], 3)
        if with_torch:
            mt = time_fn(lambda: torch.matmul(a, w.t(), out=out))
            r["cublas_ms"] = round(mt, 4)
        rows.append(r)
    return rows


def bench_attention(pk, with_torch):
    rows = []
    D, ps = 128, 16
    for (Hq, Hkv, n, qrows, label) in [(28, 4, 16384, 16384, "prefill16k"), (28, 4, 16384, 5087, "repair5k"),
                                        (64, 8, 32768, 4096, "qwen3-32b-repair")]:
        pages = (n + ps - 1) // ps
        kp = torch.randn(1, pages, Hkv, ps, D, device="cuda", dtype=torch.bfloat16)
        vp = torch.randn_like(kp)
        pt = torch.randperm(pages, device="cuda").to(torch.int32)[None]
        pos = torch.sort(torch.randperm(n)[:qrows]).values.to(torch.int32)
        if qrows == n:
            pos = torch.arange(n, dtype=torch.int32)
        qi = torch.tensor([0, qrows], dtype=torch.int32)
        tiles = ops.prefill_tiles(qi, pos, Hq, Hkv).cuda()
        q = torch.randn(qrows, Hq, D, device="cuda", dtype=torch.bfloat16)
        kvl = torch.tensor([n], dtype=torch.int32, device="cuda")
        posd, qid = pos.cuda(), qi.cuda()
        out = torch.empty(qrows, Hq * D, device="cuda", dtype=torch.bfloat16)
        ms = time_fn(lambda: ops.attention_prefill(q, kp, vp, 0, qid, posd, pt, kvl, 1 / math.sqrt(D), tiles=tiles,
                                                   out=out))
        flops = 4 * D * Hq * float((pos.double() + 1).sum())
        tf = flops / ms / 1e9
        r = {"op": f"attn_prefill_tcgen05[{label}]", "q_rows": qrows, "kv": n, "ms": round(ms, 4),
             "tflops": round(tf, 1), "frac_of_peak": round(tf / pk["bf16_tflops"], 3)}
        if with_torch:
            t64 = ops.prefill_tiles(qi, pos, Hq, Hkv, rows_per_tile=64).cuda()
            ml = time_fn(lambda: ops.attention_prefill_mma(q, kp[0], vp[0], qid, posd, pt, 1 / math.sqrt(D),
                                                           tiles=t64, out=out))
            r["mma_sync_baseline_ms"] = round(ml, 4)
            r["mma_sync_baseline_tflops"] = round(flops / ml / 1e9, 1)
        rows.append(r)
    for (B, Hq, Hkv, n, label) in [(1, 28, 4, 16640, "7b-b1-16k"), (16, 64, 8, 33000, "32b-b16-32k")]:
        pages = (n + ps - 1) // ps
        kp = torch.randn(B * pages, Hkv, ps, D, device="cuda", dtype=torch.bfloat16)
        vp = torch.randn_like(kp)
        pt = torch.randperm(B * pages, device="cuda").to(torch.int32).view(B, pages)
        q = torch.randn(B, Hq, D, device="cuda", dtype=torch.bfloat16)
        kvl = torch.full((B,), n, dtype=torch.int32, device="cuda")
        ms = time_fn(lambda: ops.attention_decode(q, kp, vp, pt, kvl, 1 / math.sqrt(D)))
        gbs = B * n * Hkv * D * 2 * 2 / ms / 1e6
        rows.append({"op": f"attn_decode[{label}]", "ms": round(ms, 4), "gbs": round(gbs, 1),
                     "frac_of_hbm": round(gbs / pk["hbm_gbs"], 3)})
    return rows


def bench_attention_variants(pk, with_torch):
    """Every exp2 / bf16-pack variant of the tcgen05 attention kernel on the
    repair case, with its error against the fp32 reference on a small case."""
    rows = []
    ext = ops._cuda()
    nvar = ext.attn_prefill_tc_set_variant(-1)
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
    posd, qid = pos.cuda(), qi.cuda()
    out = torch.empty(qrows, Hq * D, device="cuda", dtype=torch.bfloat16)
    flops = 4 * D * Hq * float((pos.double() + 1).sum())
    # small numerics case: 300 rows over 2000 keys
    sn, sr = 2000, 300
    skp, svp = kp[:, : sn // ps + 1], vp[:, : sn // ps + 1]
    spt = torch.arange(sn // ps + 1, device="cuda", dtype=torch.int32)[None]
    spos = torch.sort(torch.randperm(sn)[:sr]).values.to(torch.int32)
    sqi = torch.tensor([0, sr], dtype=torch.int32)
    sq = q[:sr]
    skvl = torch.tensor([sn], dtype=torch.int32)
    exp = ref.paged_attention(sq.float().cpu(), skp[0].float().cpu(), svp[0].float().cpu(), sqi, spos, spt.cpu(),
                              skvl, 1 / math.sqrt(D))
    for v in range(nvar):
        ext.attn_prefill_tc_set_variant(v)
        ms = time_fn(lambda: ops.attention_prefill(q, kp, vp, 0, qid, posd, pt, kvl, 1 / math.sqrt(D), tiles=tiles,
                                                   out=out))
        so = ops.attention_prefill(sq, skp, svp, 0, sqi.cuda(), spos.cuda(), spt, skvl.cuda(), 1 / math.sqrt(D))
        err = float(((so.float().cpu() - exp).norm() / exp.norm()))
        tf = flops / ms / 1e9
        rows.append({"op": f"attn_prefill_tcgen05[repair5k,variant{v}]", "ms": round(ms, 4), "tflops": round(tf, 1),
                     "frac_of_peak": round(tf / pk["bf16_tflops"], 3), "rel_err_vs_fp32": round(err, 5)})
    ext.attn_prefill_tc_set_variant(-2)
    return rows


def bench_kv_link(pk, with_torch):
    rows = []
    L, Hkv, D, ps = 28, 4, 128, 16
    for n in (2048, 16384):
        pages = 2 * (n + ps - 1) // ps + 8
        k = torch.randn(L, pages, Hkv, ps, D, device="cuda", dtype=torch.bfloat16)
        v = torch.randn_like(k)
        src = torch.arange(n, device="cuda", dtype=torch.int64)
        dst = torch.arange(n, device="cuda", dtype=torch.int64) + (pages // 2) * ps
        lp = torch.arange(n, device="cuda", dtype=torch.int32)
        gp = lp + 4000
        cs = ref.rope_cos_sin_table(32768, D, 1e6).cuda()
        ms = time_fn(lambda: ops.kv_link_rope(k, v, src, dst, lp, gp, cs))
        byts = 2 * 2 * n * L * Hkv * D * 2  # read + write of K and V
        gbs = byts / ms / 1e6
        rows.append({"op": f"kv_link_rope[{n}tok x {L}layers]", "ms": round(ms, 4), "gbs": round(gbs, 1),
                     "frac_of_hbm": round(gbs / pk["hbm_gbs"], 3)})
    return rows


def bench_tp_reduce(pk, with_torch):
    """The fused TP boundary reduction (sum of `world` partial slots +
    residual -> residual, RMSNorm -> every rank's gather buffer) on one GPU
    with all ranks' buffers local: Qwen3-32B hidden 5120, 8192 owned rows.
    Bytes: reads (world slots + residual), writes (residual + world G rows)."""
    rows = []
    ext = ops._cuda()
    err = ops.workspace("cuda").err
    H, R = 5120, 8192
    for W in (2, 4, 8):
        slots = torch.randn(W, R, H, device="cuda").to(torch.bfloat16)
        G = [torch.empty(W * R, H, device="cuda", dtype=torch.bfloat16) for _ in range(W)]
        cnt = torch.zeros(W, 2, device="cuda", dtype=torch.int64)
        res = torch.randn(R, H, device="cuda").to(torch.bfloat16)
        w = torch.ones(H, device="cuda", dtype=torch.bfloat16)
        gp = [x.data_ptr() for x in G]
        gcp = [cnt[i].data_ptr() + 8 for i in range(W)]
        ms = time_fn(lambda: ext.tp_reduce_norm_gather(slots, res, w, 1e-6, R, gp, gcp, 0, 0, 0, W, R, err))
        byts = (W + 1) * R * H * 2 + (1 + W) * R * H * 2
        gbs = byts / ms / 1e6
        rows.append({"op": f"tp_reduce_norm_gather[world{W},rows{R},h{H},1gpu]", "ms": round(ms, 4),
                     "gbs": round(gbs, 1), "frac_of_hbm": round(gbs / pk["hbm_gbs"], 3)})
        del slots, G
    return rows


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--only", default="gemm,small_m,attn,kv_link")
    ap.add_argument("--torch", action="store_true")
    a = ap.parse_args()
    pk = peaks()
    fns = {"gemm": bench_gemm, "small_m": bench_small_m, "attn": bench_attention, "kv_link": bench_kv_link,
           "attn_variants": bench_attention_variants, "tp_reduce": bench_tp_reduce}
    for name in a.only.split(","):
        for r in fns[name](pk, a.torch):
            r["peaks"] = pk["src"]
            print(json.dumps(r), flush=True)


if __name__ == "__main__":
    main()
