"""Our kernels against the library and reference kernels they replace, on
the headline workload's shapes, on the same B200 (the bars of the native
work-item checklist):

* repair / prefill attention of the Link (Qwen2.5-7B, 16K context, 5087
  recompute rows in 11 contiguous runs): ours vs FlashInfer's paged prefill
  (``fa2`` and ``trtllm-gen`` backends), the runs as FlashInfer requests;
* decode attention (batch 1, 16640 keys): ours vs FlashInfer's decode;
* the KV link with RoPE delta (11329 linked tokens x 28 layers): ours (one
  launch, paged pool) vs the reference's Triton kernel
  (``legolink_triton.py``, loaded by path from ``baseline/_ref`` when the
  reference install put it there; one launch per layer on its token-major
  buffers) vs the torch path (gathers, fp32 rotation, scatters per layer);
* the Link's GEMMs (M = 5087): ours vs cuBLAS through ``torch.matmul``.

Every case times 28 per-layer calls on 28 layers' data (inputs larger than
L2) with CUDA events after warm-up; decode cases are captured in a CUDA
graph.  Each baseline's output is compared with ours.

    python -m sglang_legolink_b200.benchmarks.baselines [--only attn,decode,kv_link,gemm]

Reference kernel: patched_sglang_files/python/sglang/srt/legolink_triton.py:302-647.
"""

from __future__ import annotations

import argparse
import importlib.util
import json
import math
import os
import random

import torch

from .. import ops
from ..ops import reference as ref
from .kernels import peaks

L, HQ, HKV, D, PS = 28, 28, 4, 128, 16


def _time(fn, reps=5, warm=2) -> float:
    for _ in range(warm):
        fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        fn()
    e1.record()
    e1.synchronize()
    return e0.elapsed_time(e1) / reps


def _graph_time(fn, reps=10) -> tuple[float, str]:
    try:
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            fn()
            fn()
        torch.cuda.current_stream().wait_stream(s)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            fn()
        return _time(g.replay, reps=reps, warm=3), "cuda_graph"
    except Exception:  # a library call that cannot be captured is timed eagerly
        torch.cuda.synchronize()
        return _time(fn, reps=reps), "eager"


def _rel(a, b) -> float:
    a, b = a.float(), b.float()
    return ((a - b).norm() / (b.norm() + 1e-12)).item()


def _emit(**kw):
    print(json.dumps(kw), flush=True)


def link_workload():
    """The bench's synthetic Link: 12 sub-contexts (seed 0), 10 linked in a
    shuffled order, 32-row repair windows, the 2 fresh blocks + 32 user
    tokens as the mutable suffix."""
    import importlib

    bench = importlib.import_module("bench")
    from ..runtime.link_plan import resolve_link_plan

    subs = bench.context_tokens(bench.context_lengths(12, 16384, 0), 152064, 0, 0)
    rng = random.Random(1)
    order = list(range(10))
    rng.shuffle(order)
    suffix = sum(subs[10:], []) + [0] * 32
    plan = {"cache_keys": [f"sub-{i}" for i in order], "recompute_initial_tokens": 32,
            "recompute_first_block": True}
    return resolve_link_plan(plan, suffix, lambda k: subs[int(k.split("-")[1])], validate=False)


def _runs(rows):
    out, start, prev = [], rows[0], rows[0]
    for p in rows[1:]:
        if p != prev + 1:
            out.append((start, prev + 1))
            start = p
        prev = p
    out.append((start, prev + 1))
    return out


# ----------------------------------------------------------------- attention
def bench_attention(pk):
    dev = torch.device("cuda")
    r = link_workload()
    rows = list(r.recompute_positions)
    n, T = r.total_token_count, len(rows)
    pages = (n + PS - 1) // PS
    g = torch.Generator(device=dev).manual_seed(0)
    kp = torch.randn(L, pages, HKV, PS, D, device=dev, dtype=torch.bfloat16, generator=g)
    vp = torch.randn(L, pages, HKV, PS, D, device=dev, dtype=torch.bfloat16, generator=g)
    q = torch.randn(T, HQ, D, device=dev, dtype=torch.bfloat16, generator=g)
    scale = 1.0 / math.sqrt(D)
    pt = torch.arange(pages, device=dev, dtype=torch.int32)[None]
    pos = torch.tensor(rows, device=dev, dtype=torch.int32)
    qi = torch.tensor([0, T], device=dev, dtype=torch.int32)
    kvl = torch.tensor([n], device=dev, dtype=torch.int32)
    tiles = ops.prefill_tiles(qi.cpu(), pos.cpu(), HQ, HKV).to(dev)
    out = torch.empty(T, HQ * D, device=dev, dtype=torch.bfloat16)
    flops = sum(p + 1 for p in rows) * 4 * D * HQ
    ours = _time(lambda: [ops.attention_prefill(q, kp, vp, li, qi, pos, pt, kvl, scale, tiles=tiles, out=out)
                          for li in range(L)]) / L
    ops.attention_prefill(q, kp, vp, 0, qi, pos, pt, kvl, scale, tiles=tiles, out=out)
    ref0 = out.clone().view(T, HQ, D)
    base = dict(case="link_attention", rows=T, kv=n, runs=len(_runs(rows)), flop_per_layer=flops)
    _emit(**base, impl="ours_tcgen05", ms_per_layer=round(ours, 4), tflops=round(flops / ours / 1e9, 1),
          frac_of_peak=round(flops / ours / 1e9 / pk["bf16_tflops"], 3), peaks=pk["src"])
    try:
        import flashinfer
    except Exception as e:  # noqa: BLE001
        _emit(**base, impl="flashinfer", unavailable=repr(e)[:200])
        return
    runs = _runs(rows)
    qo = [0]
    kv_ind = [0]
    idx, last = [], []
    for a, b in runs:
        qo.append(qo[-1] + (b - a))
        npg = (b + PS - 1) // PS
        idx.extend(range(npg))
        kv_ind.append(kv_ind[-1] + npg)
        last.append((b - 1) % PS + 1)
    i32 = dict(device=dev, dtype=torch.int32)
    for backend in ("fa2", "trtllm-gen"):
        try:
            ws = torch.zeros(512 << 20, dtype=torch.uint8, device=dev)
            w = flashinfer.BatchPrefillWithPagedKVCacheWrapper(ws, kv_layout="HND", backend=backend)
            w.plan(torch.tensor(qo, **i32), torch.tensor(kv_ind, **i32), torch.tensor(idx, **i32),
                   torch.tensor(last, **i32), HQ, HKV, D, PS, causal=True, sm_scale=scale,
                   q_data_type=torch.bfloat16, kv_data_type=torch.bfloat16)
            o0 = w.run(q, (kp[0], vp[0]))
            t = _time(lambda: [w.run(q, (kp[li], vp[li])) for li in range(L)]) / L
            _emit(**base, impl=f"flashinfer_{backend}", ms_per_layer=round(t, 4),
                  tflops=round(flops / t / 1e9, 1), rel_err_vs_ours=round(_rel(o0, ref0), 5),
                  ours_speedup=round(t / ours, 3))
        except Exception as e:  # noqa: BLE001
            _emit(**base, impl=f"flashinfer_{backend}", unavailable=repr(e)[:300])


def bench_decode(pk):
    dev = torch.device("cuda")
    n = 16640
    pages = n // PS
    g = torch.Generator(device=dev).manual_seed(1)
    kp = torch.randn(L, pages, HKV, PS, D, device=dev, dtype=torch.bfloat16, generator=g)
    vp = torch.randn(L, pages, HKV, PS, D, device=dev, dtype=torch.bfloat16, generator=g)
    q = torch.randn(1, HQ, D, device=dev, dtype=torch.bfloat16, generator=g)
    scale = 1.0 / math.sqrt(D)
    pt = torch.arange(pages, device=dev, dtype=torch.int32)[None]
    kvl = torch.tensor([n], device=dev, dtype=torch.int32)
    nsplit = ops.decode_splits(1, HKV, n)
    ops.workspace(dev).reserve_decode(HQ, nsplit, D)
    out = torch.empty(1, HQ * D, device=dev, dtype=torch.bfloat16)
    kv_bytes = n * HKV * D * 2 * 2
    ours, how = _graph_time(lambda: [ops.attention_decode(q, kp[li], vp[li], pt, kvl, scale, nsplit=nsplit, out=out)
                                     for li in range(L)])
    ours /= L
    ops.attention_decode(q, kp[0], vp[0], pt, kvl, scale, nsplit=nsplit, out=out)
    ref0 = out.clone().view(1, HQ, D)
    base = dict(case="decode_attention", batch=1, kv=n)
    _emit(**base, impl="ours_tma_split_kv", us_per_layer=round(ours * 1e3, 2), timing=how,
          frac_of_hbm=round(kv_bytes / (ours * 1e-3) / 1e9 / pk["hbm_gbs"], 3), peaks=pk["src"])
    try:
        import flashinfer
    except Exception as e:  # noqa: BLE001
        _emit(**base, impl="flashinfer", unavailable=repr(e)[:200])
        return
    i32 = dict(device=dev, dtype=torch.int32)
    for backend, tc in (("fa2", True), ("trtllm-gen", False)):
        name = f"flashinfer_{backend}" + ("_tensor_cores" if tc else "")
        try:
            ws = torch.zeros(256 << 20, dtype=torch.uint8, device=dev)
            w = flashinfer.BatchDecodeWithPagedKVCacheWrapper(ws, kv_layout="HND", use_tensor_cores=tc,
                                                              backend=backend)
            w.plan(torch.tensor([0, pages], **i32), torch.arange(pages, **i32), torch.tensor([PS], **i32), HQ, HKV,
                   D, PS, q_data_type=torch.bfloat16, kv_data_type=torch.bfloat16, sm_scale=scale)
            o0 = w.run(q, (kp[0], vp[0]))
            outs = [torch.empty_like(o0) for _ in range(L)]
            t, how = _graph_time(lambda: [w.run(q, (kp[li], vp[li]), out=outs[li]) for li in range(L)])
            t /= L
            _emit(**base, impl=name, us_per_layer=round(t * 1e3, 2), timing=how,
                  rel_err_vs_ours=round(_rel(o0, ref0), 5), ours_speedup=round(t / ours, 3))
        except Exception as e:  # noqa: BLE001
            _emit(**base, impl=name, unavailable=repr(e)[:300])


# ------------------------------------------------------------------- KV link
def _load_reference_triton():
    here = os.path.dirname(os.path.abspath(__file__))
    path = os.path.join(here, "..", "..", "baseline", "_ref", "legolink_triton.py")
    if not os.path.exists(path):
        return None, f"{os.path.normpath(path)} not present (copied there by the reference install step)"
    import sys

    try:
        spec = importlib.util.spec_from_file_location("legolink_triton_reference", path)
        mod = importlib.util.module_from_spec(spec)
        sys.modules[spec.name] = mod  # its dataclasses look their module up while being created
        spec.loader.exec_module(mod)
    except Exception as e:  # noqa: BLE001
        return None, f"loading {os.path.normpath(path)} failed: {e!r}"[:300]
    return mod, ""


def bench_kv_link(pk):
    dev = torch.device("cuda")
    r = link_workload()
    rec = set(r.recompute_positions)
    loc, glob = [], []
    for b in r.block_ranges:
        for p in range(b.start_token, b.end_token):
            if p not in rec:
                loc.append(p - b.start_token)
                glob.append(p)
    n = len(loc)
    total = r.total_token_count
    pages = 2 * ((total + PS - 1) // PS)
    g = torch.Generator().manual_seed(2)
    perm = torch.randperm(pages * PS, generator=g)
    src = perm[:n].to(dev)
    dst = perm[n : 2 * n].to(dev)
    lp = torch.tensor(loc, device=dev, dtype=torch.int32)
    gp = torch.tensor(glob, device=dev, dtype=torch.int32)
    cs = ref.rope_cos_sin_table(32768, D, 1e6).to(dev)
    bytes_ = 2 * 2 * n * HKV * D * 2 * L  # read + write of K and V
    base = dict(case="kv_link", tokens=n, layers=L)
    kp = torch.randn(L, pages, HKV, PS, D, device=dev, dtype=torch.bfloat16)
    vp = torch.randn_like(kp)
    ours = _time(lambda: ops.kv_link_rope(kp, vp, src, dst, lp, gp, cs))
    _emit(**base, impl="ours_one_launch_all_layers", ms=round(ours, 4),
          gbs=round(bytes_ / ours / 1e6, 1), frac_of_hbm=round(bytes_ / ours / 1e6 / pk["hbm_gbs"], 3),
          peaks=pk["src"])
    # token-major [slots, heads, dim] buffers per layer, as the reference runtime keeps them
    kt = kp.permute(0, 1, 3, 2, 4).reshape(L, pages * PS, HKV, D).contiguous()  # slot = page * PS + offset
    vt = vp.permute(0, 1, 3, 2, 4).reshape(L, pages * PS, HKV, D).contiguous()
    del kp, vp
    src64, dst64 = src.long(), dst.long()
    lp64, gp64 = lp.long(), gp.long()

    def torch_path():
        for li in range(L):
            k = kt[li].index_select(0, src64).float()
            v = vt[li].index_select(0, src64)
            cl, sl = cs[lp64, :64], cs[lp64, 64:]
            cg, sg = cs[gp64, :64], cs[gp64, 64:]
            dc = (cg * cl + sg * sl)[:, None, :]
            ds = (sg * cl - cg * sl)[:, None, :]
            x1, x2 = k[..., :64], k[..., 64:]
            k = torch.cat([x1 * dc - x2 * ds, x2 * dc + x1 * ds], -1).to(kt.dtype)
            kt[li].index_copy_(0, dst64, k)
            vt[li].index_copy_(0, dst64, v)

    t = _time(torch_path, reps=3)
    _emit(**base, impl="torch_path_per_layer", ms=round(t, 4), gbs=round(bytes_ / t / 1e6, 1),
          ours_speedup=round(t / ours, 3))
    mod, why = _load_reference_triton()
    if mod is None:
        _emit(**base, impl="reference_triton", unavailable=why)
        return
    try:
        def ref_path():
            for li in range(L):
                mod.fused_kv_link_inplace(key_buffer=kt[li], value_buffer=vt[li], source_slots=src64,
                                          destination_slots=dst64, local_positions=lp64, global_positions=gp64,
                                          cos_sin_cache=cs, prefix_token_count=0, rotary_dim=D, is_neox_style=True)

        t = _time(ref_path, reps=3)
        _emit(**base, impl="reference_triton_per_layer", ms=round(t, 4), gbs=round(bytes_ / t / 1e6, 1),
              ours_speedup=round(t / ours, 3))
    except Exception as e:  # noqa: BLE001
        _emit(**base, impl="reference_triton", unavailable=repr(e)[:300])


# ---------------------------------------------------------------------- GEMM
def bench_gemm(pk):
    dev = torch.device("cuda")
    M = 5087
    shapes = {"qkv": (4608, 3584), "o_proj": (3584, 3584), "gate_up": (37888, 3584), "down": (3584, 18944)}
    for name, (N, K) in shapes.items():
        x = torch.randn(M, K, device=dev, dtype=torch.bfloat16)
        ws = [torch.randn(N, K, device=dev, dtype=torch.bfloat16) / math.sqrt(K) for _ in range(4)]
        out = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
        fl = 2 * M * N * K
        ours = _time(lambda: [ops.linear(x, w, out=out) for w in ws]) / 4
        y0 = out.clone()
        cub = _time(lambda: [torch.matmul(x, w.t()) for w in ws]) / 4
        err = _rel(y0, torch.matmul(x, ws[-1].t()))
        _emit(case="link_gemm", shape=name, M=M, N=N, K=K, ours_ms=round(ours, 4), cublas_ms=round(cub, 4),
              ours_tflops=round(fl / ours / 1e9, 1), cublas_tflops=round(fl / cub / 1e9, 1),
              ours_speedup=round(cub / ours, 3), rel_err_vs_cublas=round(err, 5), peaks=pk["src"])


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--only", default="attn,decode,kv_link,gemm")
    a = ap.parse_args()
    pk = peaks()
    fns = {"attn": bench_attention, "decode": bench_decode, "kv_link": bench_kv_link, "gemm": bench_gemm}
    for k in a.only.split(","):
        fns[k](pk)
        torch.cuda.empty_cache()


if __name__ == "__main__":
    main()
