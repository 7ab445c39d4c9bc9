"""Per-op device time of one decode step (default: batch 1, Qwen2.5-7B, 16K
context) measured the way the step runs: each op is captured into a CUDA
graph as one launch per layer (on that layer's own weights / KV, so every
launch streams from HBM like the real step), replayed, and timed with CUDA
events.

    python -m sglang_legolink_b200.benchmarks.decode_breakdown [--context 16640]
    python -m sglang_legolink_b200.benchmarks.decode_breakdown --model qwen3-32b --shard 8 --batch 16 --context 32832

``--batch B`` decodes B requests of ``--context`` keys each; ``--shard W``
takes one rank's share of TP = W (heads, KV heads, intermediate size and
vocabulary divided by W) with no communication.  Prints one JSON line per
op: microseconds per layer and the fraction of the measured HBM bandwidth
its bytes (weights, and K/V for attention) would take.
"""

from __future__ import annotations

import argparse
import json
import math

import torch

from .. import ops
from ..models.config import PRESETS
from ..models.qwen import QwenModel
from .kernels import peaks


def graph_time(fn, reps=10) -> float:
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(2):
            fn()
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        fn()
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        g.replay()
    e1.record()
    e1.synchronize()
    return e0.elapsed_time(e1) / reps


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="qwen2.5-7b")
    ap.add_argument("--context", type=int, default=16640)
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--shard", type=int, default=1)
    a = ap.parse_args()
    cfg = PRESETS[a.model]
    if a.shard > 1:
        import dataclasses

        cfg = dataclasses.replace(cfg, num_heads=cfg.num_heads // a.shard,
                                  num_kv_heads=max(1, cfg.num_kv_heads // a.shard),
                                  intermediate_size=cfg.intermediate_size // a.shard,
                                  vocab_size=cfg.vocab_size // a.shard, name=f"{cfg.name}/shard{a.shard}")
    B = a.batch
    dev = torch.device("cuda")
    m = QwenModel.random_init(cfg, seed=0, device=dev, dtype=torch.bfloat16)
    L, H, D = cfg.num_layers, cfg.hidden_size, cfg.head_dim
    hq, hkv, inter = m.hq, m.hkv, m.inter
    n, ps = a.context, 16
    m.ensure_rope_positions(n + 1)  # contexts past the model's table, as the engine does
    pps = (n + ps - 1) // ps  # pages per request
    pages = B * pps
    kpool = torch.randn(L, pages, hkv, ps, D, device=dev, dtype=torch.bfloat16)
    vpool = torch.randn_like(kpool)
    pt = torch.arange(pages, device=dev, dtype=torch.int32).view(B, pps)
    kvl = torch.full((B,), n, device=dev, dtype=torch.int32)
    pos = torch.full((B,), n - 1, device=dev, dtype=torch.int32)
    slot = torch.arange(B, device=dev, dtype=torch.int64) * (pps * ps) + (n - 1)
    x = torch.randn(B, H, device=dev, dtype=torch.bfloat16)
    res = torch.randn(B, H, device=dev, dtype=torch.bfloat16)
    qkv = torch.empty(B, (hq + 2 * hkv) * D, device=dev, dtype=torch.bfloat16)
    q = torch.randn(B, hq, D, device=dev, dtype=torch.bfloat16)
    attn = torch.empty(B, hq * D, device=dev, dtype=torch.bfloat16)
    gu = torch.empty(B, 2 * inter, device=dev, dtype=torch.bfloat16)
    mlp = torch.randn(B, inter, device=dev, dtype=torch.bfloat16)
    nsplit = ops.decode_splits(B, hkv, n)
    ops.workspace(dev).reserve_decode(hq, nsplit, D)
    for lw in m.layers[:1]:  # reserve GEMM workspaces outside capture
        ops.linear(x, lw.gu_w, out=gu)
        ops.linear(x, lw.qkv_w, out=qkv)
    scale = 1.0 / math.sqrt(D)
    pk = peaks()
    kvb = B * n * hkv * D * 2 * 2
    # the five kernels of the fused decode layer (QwenModel._forward_decode_fused)
    eps = cfg.rms_norm_eps
    ss = ops.sumsq_from_values(torch.full((B,), float(H), device=dev))
    sq = ops.sumsq_buffer(B, dev)
    hp = torch.empty(B, H, device=dev, dtype=torch.bfloat16)
    cases = {
        "gemv_qkv_rope": (lambda: [ops.gemv_qkv_rope(x, lw.qkv_w, lw.qkv_b, pos, slot, m.cos_sin, q, kpool[i],
                                                     vpool[i], hq, hkv, lw.q_norm, lw.k_norm, eps, scale_sumsq=ss)
                                   for i, lw in enumerate(m.layers)], m.layers[0].qkv_w.numel() * 2),
        "attn_decode": (lambda: [ops.attention_decode(q, kpool[i], vpool[i], pt, kvl, scale, nsplit=nsplit, out=attn)
                                 for i in range(L)], kvb),
        "gemv_o_proj_residual": (lambda: [ops.gemv_residual(attn, lw.o_w, res, lw.post_norm, hp, sq, eps=eps)
                                          for lw in m.layers], m.layers[0].o_w.numel() * 2),
        "gemv_gate_up_swiglu": (lambda: [ops.gemv_rownorm(hp, lw.gu_w, None, ss, eps, out=mlp, swiglu=True)
                                         for lw in m.layers], m.layers[0].gu_w.numel() * 2),
        "gemv_down_residual": (lambda: [ops.gemv_residual(mlp, lw.down_w, res, lw.in_norm, x, sq, eps=eps)
                                        for lw in m.layers], m.layers[0].down_w.numel() * 2),
    }
    ws = ops.workspace(dev)
    gemv_nk = {"gemv_qkv_rope": ((hq + 2 * hkv) * D, H), "gemv_o_proj_residual": (H, hq * D),
               "gemv_gate_up_swiglu": (2 * inter, H), "gemv_down_residual": (H, inter)}
    total = 0.0
    for name, (fn, bytes_per_layer) in cases.items():
        ms = graph_time(fn)
        err = ops.check_errors(dev)
        if err:
            raise SystemExit(f"{name}: device error {err} (the timing would be of abandoned work)")
        us = ms * 1e3 / L
        total += us
        roof_us = bytes_per_layer / (pk["hbm_gbs"] * 1e3)
        extra = {"gemv_splits": ops._small_m_splits(ws, B, *gemv_nk[name])} if name in gemv_nk else {"nsplit": nsplit}
        print(json.dumps({"op": name, "model": cfg.name, "batch": B, "context": n, **extra,
                          "us_per_layer": round(us, 2), "us_per_step": round(us * L, 1),
                          "roofline_us_per_layer": round(roof_us, 2), "frac_of_hbm": round(roof_us / us, 3),
                          "peaks": pk["src"]}), flush=True)
    print(json.dumps({"op": "sum_of_layer_ops", "ms_per_step": round(total * L / 1e3, 3)}), flush=True)
    lm = graph_time(lambda: ops.linear(x, m.lm_head))
    print(json.dumps({"op": "gemv_lm_head", "us": round(lm * 1e3, 1),
                      "frac_of_hbm": round(m.lm_head.numel() * 2 / (pk["hbm_gbs"] * 1e3) / (lm * 1e3), 3)}))


if __name__ == "__main__":
    main()
