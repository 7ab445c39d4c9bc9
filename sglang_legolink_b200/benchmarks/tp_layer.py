"""Tensor-parallel prefill: fused path vs the NCCL all-reduce path.

Launch one process per GPU::

    python -m torch.distributed.run --nnodes=1 --nproc-per-node N --master-addr 127.0.0.1 \\
        -m sglang_legolink_b200.benchmarks.tp_layer [--model qwen3-32b] [--layers 4] [--rows 8192] [--boundary]

Builds the named architecture with ``--layers`` decoder layers (random init,
bf16, TP = N).  Default mode times an extend forward of ``--rows`` rows (a
prefill from position 0) through both communicators on the same weights: the
fused path (:class:`~sglang_legolink_b200.parallel.tp_fused.FusedTPComm`) and
the NCCL baseline.  ``--boundary`` times only one layer boundary,
o_proj -> reduction -> residual add + RMSNorm -> gate_up, both ways and part
by part.  Device time with CUDA events, max over ranks.

Roofline of the boundary per rank: the slower of its GEMM FLOPs at the
measured bf16 peak and the bytes this rank must send over NVLink
(reduce-scatter of the partial output + all-gather of the normalised input:
2 x (N-1)/N x rows x hidden x 2 bytes) at 770 GB/s per direction.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
from dataclasses import replace
from datetime import timedelta

import torch
import torch.distributed as dist

from ..models.config import PRESETS
from ..models.qwen import QwenModel
from ..parallel.tp import NcclTPComm
from ..parallel.tp_fused import FusedTPComm
from ..runtime.engine import Engine
from .kernels import peaks

NVLINK_GBS = 770.0


def _time(fn, iters, dev):
    for _ in range(2):
        fn()
    torch.cuda.synchronize()
    dist.barrier()
    ts = []
    for _ in range(iters):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        fn()
        e1.record()
        e1.synchronize()
        ts.append(e0.elapsed_time(e1))
        dist.barrier()
    t = torch.tensor([statistics.median(ts)], device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def boundary(a, m, fused, dev, rank, world):
    """o_proj (row-parallel) -> reduction -> residual add + RMSNorm ->
    gate_up (column-parallel, SwiGLU), both ways, and their parts."""
    from .. import ops

    c = m.cfg
    T, H = a.rows, c.hidden_size
    lw = m.layers[0]
    R = fused.rows_per_rank(T)
    Tp = world * R
    g = torch.Generator(device=dev).manual_seed(rank)
    attn = (torch.randn(Tp, m.hq * c.head_dim, device=dev, generator=g) * 0.5).to(torch.bfloat16)
    res_full = torch.randn(Tp, H, device=dev, generator=torch.Generator(device=dev).manual_seed(7)).to(torch.bfloat16)
    res_local = res_full[rank * R : (rank + 1) * R].clone()
    o = torch.empty(Tp, H, device=dev, dtype=torch.bfloat16)
    mlp = torch.empty(Tp, m.inter, device=dev, dtype=torch.bfloat16)
    res_n = res_full.clone()

    def nccl_path():
        ops.linear(attn, lw.o_w, out=o)
        dist.all_reduce(o)
        ops.fused_add_rmsnorm(o, res_n, lw.post_norm, c.rms_norm_eps)
        ops.linear(o, lw.gu_w, out=mlp, swiglu_epilogue=True)

    def fused_path():
        fused.gemm_scatter(attn, lw.o_w, T)
        fused.reduce_norm_gather(res_local, lw.post_norm, c.rms_norm_eps, T)
        fused.gemm_from_gather(lw.gu_w, None, mlp, T, swiglu=True)

    def scatter_and_drain():
        fused.gemm_scatter(attn, lw.o_w, T)
        fused.reduce_norm_gather(res_local, lw.post_norm, c.rms_norm_eps, T)
        fused.wait_gather(dev)

    def reduce_only():
        fused.reduce_norm_gather(res_local, lw.post_norm, c.rms_norm_eps, T)
        fused.wait_gather(dev)

    out = {"bench": "tp_boundary_o_proj_reduce_norm_gate_up", "model": a.model, "rows": T, "tp": world}
    # alternate the two paths and keep each one's best median (clocks drift
    # under the power cap between measurements)
    out["nccl_ms"], out["fused_ms"] = 1e30, 1e30
    for _ in range(3):
        out["nccl_ms"] = min(out["nccl_ms"], _time(nccl_path, a.iters, dev))
        out["fused_ms"] = min(out["fused_ms"], _time(fused_path, a.iters, dev))
    out["gemm_o_proj_ms"] = _time(lambda: ops.linear(attn, lw.o_w, out=o), a.iters, dev)
    out["allreduce_ms"] = _time(lambda: dist.all_reduce(o), a.iters, dev)
    out["add_rmsnorm_ms"] = _time(lambda: ops.fused_add_rmsnorm(o, res_n, lw.post_norm, c.rms_norm_eps), a.iters, dev)
    out["gemm_gate_up_ms"] = _time(lambda: ops.linear(o, lw.gu_w, out=mlp, swiglu_epilogue=True), a.iters, dev)
    out["gemm_scatter_plus_reduce_gather_ms"] = _time(scatter_and_drain, a.iters, dev)
    out["gemm_scatter_ms"] = _time(lambda: fused.gemm_scatter(attn, lw.o_w, T), a.iters, dev)
    out["reduce_norm_gather_ms"] = _time(reduce_only, a.iters, dev)
    out["speedup"] = round(out["nccl_ms"] / out["fused_ms"], 3)
    pk = peaks()
    flops = 2 * Tp * (m.hq * c.head_dim) * H + 2 * Tp * H * 2 * m.inter
    nv = 2 * (world - 1) / world * Tp * H * 2
    t_roof = max(flops / (pk["bf16_tflops"] * 1e12), nv / (NVLINK_GBS * 1e9)) * 1e3
    out["roofline_ms"] = round(t_roof, 4)
    out["fused_frac_of_roofline"] = round(t_roof / out["fused_ms"], 3)
    out["nccl_frac_of_roofline"] = round(t_roof / out["nccl_ms"], 3)
    out["peaks"] = pk["src"]
    out["errors"] = ops.check_errors(dev)
    for k, v in list(out.items()):
        if k.endswith("_ms"):
            out[k] = round(v, 4)
    if rank == 0:
        print(json.dumps(out), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="qwen3-32b")
    ap.add_argument("--layers", type=int, default=4)
    ap.add_argument("--rows", type=int, default=8192)
    ap.add_argument("--iters", type=int, default=5)
    ap.add_argument("--boundary", action="store_true",
                    help="time only the o_proj -> reduce -> norm -> gate_up boundary and its parts")
    a = ap.parse_args()
    rank, local, world = int(os.environ["RANK"]), int(os.environ["LOCAL_RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
    cfg = replace(PRESETS[a.model], num_layers=1 if a.boundary else a.layers)
    T = a.rows
    fused = FusedTPComm(cfg.hidden_size, T, dev)
    nccl = NcclTPComm()
    m = QwenModel.random_init(cfg, seed=0, device=dev, dtype=torch.bfloat16, tp_rank=rank, tp_size=world, comm=fused)
    if a.boundary:
        boundary(a, m, fused, dev, rank, world)
        dist.barrier()
        dist.destroy_process_group()
        return
    eng = Engine(m, page_size=16, max_context=T + 64, mem_fraction=0.5)
    ids = torch.randint(0, cfg.vocab_size, (T,), generator=torch.Generator().manual_seed(0)).tolist()
    pages = eng._alloc_pages((T + 15) // 16)
    fb = eng._extend_batch([(ids, list(range(T)), pages, T)])
    res = {}
    for name, comm in (("nccl", nccl), ("fused", fused), ("nccl", nccl), ("fused", fused)):
        m.comm = comm
        t = _time(lambda: m.forward(fb, eng.kv), a.iters, dev)
        res[name] = min(res.get(name, 1e30), t)
    from .. import ops

    errs = ops.check_errors(dev)
    H, L = cfg.hidden_size, cfg.num_layers
    if rank == 0:
        out = {"bench": "tp_prefill_fused_vs_nccl", "model": a.model, "layers": L, "rows": T, "tp": world,
               "nccl_ms": round(res["nccl"], 3), "fused_ms": round(res["fused"], 3),
               "speedup": round(res["nccl"] / res["fused"], 3),
               "fused_ms_per_layer": round(res["fused"] / L, 4), "nccl_ms_per_layer": round(res["nccl"] / L, 4),
               "errors": errs, "fused_stats": fused.stats}
        print(json.dumps(out), flush=True)
    eng._graphs.clear()
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
