"""Small single-kernel cases sized for `ncu --set full` captures (a few
launches, a few hundred MB on the device), one per hot kernel:

    python -m sglang_legolink_b200.benchmarks.ncu_cases {gemm,gemm_link,gemm_link_cublas,attn,gemv,gemv_residual,gemv_qkv_rope,decode,link,rmsnorm,rope_qkv,tp_reduce,tp_scatter,tp_decode}
"""
import sys, os, math

import torch
from sglang_legolink_b200 import ops
from sglang_legolink_b200.ops import reference as ref
case = sys.argv[1]
torch.manual_seed(0)
if case == "gemv":
    for N, K in ((4608, 3584), (3584, 18944)):
        a = torch.randn(1, K, device="cuda", dtype=torch.bfloat16)
        w = torch.randn(N, K, device="cuda", dtype=torch.bfloat16)
        o = torch.empty(1, N, device="cuda", dtype=torch.bfloat16)
        for _ in range(4): ops.linear(a, w, out=o)
elif case == "gemv_residual":  # o_proj GEMV + residual epilogue: 4 launches at M = 16, then 4 at M = 1
    H = 3584
    w = ops.tile_weight((torch.randn(H, H, device="cuda") * 0.02).to(torch.bfloat16))
    nw = torch.ones(H, device="cuda", dtype=torch.bfloat16)
    for M in (16, 1):
        x = torch.randn(M, H, device="cuda", dtype=torch.bfloat16)
        res = torch.randn(M, H, device="cuda", dtype=torch.bfloat16)
        h = torch.empty(M, H, device="cuda", dtype=torch.bfloat16)
        sq = ops.sumsq_buffer(M, "cuda")
        for _ in range(4): ops.gemv_residual(x, w, res, nw, h, sq)
    torch.cuda.synchronize()
elif case == "gemv_qkv_rope":  # one Qwen3-32B TP=8 rank's qkv GEMV + QK-norm + RoPE + KV write: 4 launches at M = 16, then 4 at M = 1
    H, hq, hkv, ctx, ps = 5120, 8, 1, 32832, 16
    w = ops.tile_weight((torch.randn((hq + 2 * hkv) * 128, H, device="cuda") * 0.02).to(torch.bfloat16))
    qn = (torch.rand(128, device="cuda") + 0.5).to(torch.bfloat16)
    kn = (torch.rand(128, device="cuda") + 0.5).to(torch.bfloat16)
    cs = ref.rope_cos_sin_table(ctx + 64, 128, 1e6).to("cuda")
    for M in (16, 1):
        x = torch.randn(M, H, device="cuda", dtype=torch.bfloat16)
        pos = torch.full((M,), ctx - 1, device="cuda", dtype=torch.int32)
        slot = torch.arange(M, device="cuda", dtype=torch.int64) * ps
        kp = torch.zeros(M, hkv, ps, 128, device="cuda", dtype=torch.bfloat16)
        vp = torch.zeros_like(kp)
        q = torch.empty(M, hq, 128, device="cuda", dtype=torch.bfloat16)
        for _ in range(4): ops.gemv_qkv_rope(x, w, None, pos, slot, cs, q, kp, vp, hq, hkv, qn, kn, 1e-6)
    torch.cuda.synchronize()
elif case == "gemm":
    M, N, K = 2048, 37888, 3584
    a = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(N, K, device="cuda", dtype=torch.bfloat16)
    o = torch.empty(M, N // 2, device="cuda", dtype=torch.bfloat16)
    for _ in range(4): ops.linear(a, w, out=o, swiglu_epilogue=True)
elif case in ("gemm_link", "gemm_link_cublas"):  # the Link's gate_up shape: ours vs cuBLAS (torch.matmul)
    M, N, K = 5087, 37888, 3584
    a = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(N, K, device="cuda", dtype=torch.bfloat16) / math.sqrt(K)
    o = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    for _ in range(3):
        if case == "gemm_link":
            ops.linear(a, w, out=o)
        else:
            torch.matmul(a, w.t(), out=o)
    torch.cuda.synchronize()
elif case == "attn":
    D, ps, Hq, Hkv, n, qrows = 128, 16, 28, 4, 8192, 4096
    pages = n // ps
    kp = torch.randn(1, pages, Hkv, ps, D, device="cuda", dtype=torch.bfloat16); vp = torch.randn_like(kp)
    pt = torch.randperm(pages, device="cuda").to(torch.int32)[None]
    pos = torch.sort(torch.randperm(n)[:qrows]).values.to(torch.int32)
    qi = torch.tensor([0, qrows], dtype=torch.int32)
    tiles = ops.prefill_tiles(qi, pos, Hq, Hkv).cuda()
    q = torch.randn(qrows, Hq, D, device="cuda", dtype=torch.bfloat16)
    kvl = torch.tensor([n], dtype=torch.int32, device="cuda")
    for _ in range(4): ops.attention_prefill(q, kp, vp, 0, qi.cuda(), pos.cuda(), pt, kvl, 1/math.sqrt(D), tiles=tiles)
elif case == "decode":
    B, Hq, Hkv, n, D, ps = 1, 28, 4, 16640, 128, 16
    pages = n // ps
    kp = torch.randn(pages, Hkv, ps, D, device="cuda", dtype=torch.bfloat16); vp = torch.randn_like(kp)
    pt = torch.randperm(pages, device="cuda").to(torch.int32)[None]
    q = torch.randn(B, Hq, D, device="cuda", dtype=torch.bfloat16)
    kvl = torch.full((B,), n, dtype=torch.int32, device="cuda")
    for _ in range(4): ops.attention_decode(q, kp, vp, pt, kvl, 1/math.sqrt(D))
elif case == "link":  # fused KV link + RoPE delta: 4096 tokens x 28 layers (Qwen2.5-7B KV layout)
    L, Hkv, D, ps, n = 28, 4, 128, 16, 4096
    pages = 2 * n // ps + 8
    k = torch.randn(L, pages, Hkv, ps, D, device="cuda", dtype=torch.bfloat16); v = torch.randn_like(k)
    src = torch.arange(n, device="cuda", dtype=torch.int64)
    dst = src + (pages // 2) * ps
    lp = torch.arange(n, device="cuda", dtype=torch.int32)
    cs = ref.rope_cos_sin_table(32768, D, 1e6).cuda()
    for _ in range(4): ops.kv_link_rope(k, v, src, dst, lp, lp + 3000, cs)
elif case == "rmsnorm":  # fused residual add + RMSNorm over a Link's rows (8192 x 3584)
    T, H = 8192, 3584
    x = torch.randn(T, H, device="cuda", dtype=torch.bfloat16)
    r = torch.randn(T, H, device="cuda", dtype=torch.bfloat16)
    w = torch.rand(H, device="cuda", dtype=torch.bfloat16) + 0.5
    for _ in range(4): ops.fused_add_rmsnorm(x, r, w, 1e-6)
elif case == "rope_qkv":  # RoPE of q/k + KV write of 8192 rows (Qwen2.5-7B heads) into a paged pool
    T, Hq, Hkv, D, ps = 8192, 28, 4, 128, 16
    pages = T // ps + 8
    qkv = torch.randn(T, (Hq + 2 * Hkv) * D, device="cuda", dtype=torch.bfloat16)
    kp = torch.zeros(pages, Hkv, ps, D, device="cuda", dtype=torch.bfloat16); vp = torch.zeros_like(kp)
    pos = torch.arange(T, device="cuda", dtype=torch.int32)
    slots = torch.arange(T, device="cuda", dtype=torch.int64)
    cs = ref.rope_cos_sin_table(32768, D, 1e6).cuda()
    q = torch.empty(T, Hq, D, device="cuda", dtype=torch.bfloat16)
    for _ in range(4): ops.rope_qkv_write(qkv, pos, slots, cs, q, kp, vp, Hq, Hkv, D)
elif case in ("tp_reduce", "tp_scatter"):  # fused-TP kernels on one GPU: both "ranks'" buffers are local
    W, H, K, T = 2, 5120, 4096, 16384
    R = T // W
    err = ops.workspace("cuda").err
    ext = ops._cuda()
    slots = [torch.zeros(W, R, H, device="cuda", dtype=torch.bfloat16) for _ in range(W)]
    G = [torch.zeros(W * R, H, device="cuda", dtype=torch.bfloat16) for _ in range(W)]
    cnt = [torch.zeros(2, device="cuda", dtype=torch.int64) for _ in range(W)]
    sp, cp = [x.data_ptr() for x in slots], [c.data_ptr() for c in cnt]
    gp, gcp = [x.data_ptr() for x in G], [c.data_ptr() + 8 for c in cnt]
    if case == "tp_reduce":
        res = torch.randn(R, H, device="cuda").to(torch.bfloat16)
        w = torch.ones(H, device="cuda", dtype=torch.bfloat16)
        for _ in range(4): ext.tp_reduce_norm_gather(slots[0], res, w, 1e-6, R, gp, gcp, 0, 0, 0, W, R, err)
    else:
        a = (torch.randn(T, K, device="cuda") * 0.5).to(torch.bfloat16)
        w = (torch.randn(H, K, device="cuda") / 64).to(torch.bfloat16)
        for _ in range(4): ext.gemm_tp(a, w, None, None, 2, H, sp, cp, 0, 0, 0, W, R, err)
elif case == "tp_decode":  # decode TP boundary (one-shot all-reduce + residual + RMSNorm), world 2 on one GPU
    # Both "ranks'" partial rows are local.  This process plays rank 0; before
    # each call the host adds 1 to rank 0's arrival counter for the other
    # rank, so the kernel's own arrival completes its wait (nothing waits on
    # another launch).
    W, rows, H = 2, 16, 5120
    err = ops.workspace("cuda").err
    ext = ops._cuda()
    parts = [torch.randn(rows, H, device="cuda").to(torch.bfloat16) for _ in range(W)]
    res = torch.randn(rows, H, device="cuda").to(torch.bfloat16)
    w = torch.ones(H, device="cuda", dtype=torch.bfloat16)
    out = torch.empty(rows, H, device="cuda", dtype=torch.bfloat16)
    cnt = [torch.zeros(2, device="cuda", dtype=torch.int64) for _ in range(W)]
    epoch = torch.zeros(2, device="cuda", dtype=torch.int64)
    for _ in range(4):
        cnt[0][0] += W - 1
        ext.tp_decode_allreduce_norm(res, w, out, 1e-6, rows, [p.data_ptr() for p in parts],
                                     [c.data_ptr() for c in cnt], epoch, 0, W, err)
elif case == "decode_step":  # Qwen2.5-7B, 16K context, eager decode steps (launch lists only: full size)
    from sglang_legolink_b200.models.config import PRESETS
    from sglang_legolink_b200.models.qwen import QwenModel
    from sglang_legolink_b200.runtime.engine import Engine
    cfg = PRESETS["qwen2.5-7b"]
    m = QwenModel.random_init(cfg, seed=0, device="cuda", dtype=torch.bfloat16)
    eng = Engine(m, page_size=16, max_context=17000, mem_fraction=0.5, use_cuda_graphs=False)
    seq = eng.prefill(torch.randint(0, cfg.vocab_size, (16384,)).tolist())
    torch.cuda.synchronize()
    eng.decode([seq], int(os.environ.get("DECODE_STEPS", "3")))
torch.cuda.synchronize()
print("ok", case, ops.check_errors("cuda"))
