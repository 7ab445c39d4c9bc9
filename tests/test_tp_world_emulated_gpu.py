"""The fused tensor-parallel kernels at world 4 and 8 on ONE GPU: every
emulated rank's buffers and counters live on this device and each rank's
kernels are launched in turn on one stream.  No launch ever waits on a later
one -- every counter a kernel waits for is already at its target when the
kernel starts -- so the emulation runs no kernels that wait on one another.

Checked against fp32 torch: the scatter GEMM's epilogue (each row into its
owner's slot for this rank, 32-row x 256-column slice counts), the owner's
reduce + residual + RMSNorm + all-gather into every rank's G (and the G
counter increments), the gather-waiting GEMM, and the decode one-shot
all-reduce + RMSNorm (reference: the NCCL all-reduce these replace,
``patched_sglang_files/python/sglang/srt/models/qwen2.py:80-86,162-168``)."""

import pytest
import torch

from sglang_legolink_b200 import ops

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _rel(a, b):
    a, b = a.float().cpu(), b.float().cpu()
    return ((a - b).norm() / (b.norm() + 1e-6)).item()


def _norm(x, w, eps=1e-6):
    x = x.float()
    return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * w.float()


@pytest.mark.parametrize("W", [4, 8])
def test_prefill_boundary_emulated_world(W):
    torch.manual_seed(W)
    ext, err = ops._cuda(), ops.workspace(DEV).err
    R, H, K, N2 = 128, 1024, 512, 768  # T = W x R >= 512, the fused path's minimum
    T = W * R
    a = [(torch.randn(T, K, device=DEV) * 0.5).to(torch.bfloat16) for _ in range(W)]   # rank r's activations
    wo = [(torch.randn(H, K, device=DEV) / 16).to(torch.bfloat16) for _ in range(W)]   # rank r's K-slice of o_proj
    slots = [torch.zeros(W, R, H, device=DEV, dtype=torch.bfloat16) for _ in range(W)]  # owner d: [src rank][R][H]
    G = [torch.zeros(T, H, device=DEV, dtype=torch.bfloat16) for _ in range(W)]
    cnt = [torch.zeros(2, device=DEV, dtype=torch.int64) for _ in range(W)]           # [slot counter, G counter]
    sp, cp = [s.data_ptr() for s in slots], [c.data_ptr() for c in cnt]
    gp, gcp = [g.data_ptr() for g in G], [c.data_ptr() + 8 for c in cnt]
    # 1. every rank's scatter GEMM
    for r in range(W):
        ext.gemm_tp(a[r], wo[r], None, None, 2, H, sp, cp, 0, 0, r, W, R, err)
    torch.cuda.synchronize()
    assert ops.check_errors(DEV) == 0
    per_rank_slices = (R // 32) * ((H + 255) // 256)

    def untile(x):  # a source rank's slot region: [R/32][H/32][32][32] -> [R, H]
        return x.reshape(R // 32, H // 32, 32, 32).permute(0, 2, 1, 3).reshape(R, H)

    for d in range(W):
        assert int(cnt[d][0]) == W * per_rank_slices
        for r in range(W):
            exp = a[r][d * R:(d + 1) * R].float() @ wo[r].float().t()
            assert _rel(untile(slots[d][r]), exp) < 1e-2
    # 2. every owner's reduce + residual + RMSNorm + all-gather
    res0 = [torch.randn(R, H, device=DEV).to(torch.bfloat16) for _ in range(W)]
    res = [x.clone() for x in res0]
    nw = (torch.rand(H, device=DEV) + 0.5).to(torch.bfloat16)
    grids = []
    for d in range(W):
        grids.append(ext.tp_reduce_norm_gather(slots[d], res[d], nw, 1e-6, R, gp, gcp, cp[d],
                                               W * per_rank_slices, d, W, R, err))
    torch.cuda.synchronize()
    assert ops.check_errors(DEV) == 0
    assert len(set(grids)) == 1
    for d in range(W):
        s = res0[d].float() + sum(untile(slots[d][r]).float() for r in range(W))
        assert _rel(res[d], s) < 1e-2
        for e in range(W):
            assert _rel(G[e][d * R:(d + 1) * R], _norm(s, nw)) < 1e-2
    for e in range(W):
        assert int(cnt[e][1]) == W * grids[0]
    # 3. the gather-waiting GEMM of each rank (its counter is already complete)
    w2 = (torch.randn(N2, H, device=DEV) / 32).to(torch.bfloat16)
    for e in (0, W - 1):
        out = torch.empty(T, N2, device=DEV, dtype=torch.bfloat16)
        ext.gemm_tp(G[e], w2, None, out, 0, 0, [], [], gcp[e], W * grids[0], e, W, R, err)
        torch.cuda.synchronize()
        assert ops.check_errors(DEV) == 0
        assert _rel(out, G[e].float() @ w2.float().t()) < 1e-2


@pytest.mark.parametrize("W", [4, 8])
@pytest.mark.parametrize("rows,H", [(1, 5120), (16, 5120)])
def test_decode_boundary_emulated_world(W, rows, H):
    """One decode boundary per emulated rank.  Each rank's kernel adds 1 to
    every rank's arrival counter and waits for its own to reach W; the host
    pre-adds W - 1 to every counter, so each launch finds its wait satisfied."""
    torch.manual_seed(rows + W)
    ext, err = ops._cuda(), ops.workspace(DEV).err
    parts = [torch.randn(rows, H, device=DEV).to(torch.bfloat16) for _ in range(W)]
    w = (torch.rand(H, device=DEV) + 0.5).to(torch.bfloat16)
    cnt = [torch.full((2,), W - 1, device=DEV, dtype=torch.int64) for _ in range(W)]
    pp, cp = [p.data_ptr() for p in parts], [c.data_ptr() for c in cnt]
    base = torch.randn(rows, H, device=DEV).to(torch.bfloat16)
    s = base.float() + torch.stack([p.float() for p in parts]).sum(0)
    for r in range(W):
        res = base.clone()
        out = torch.empty(rows, H, device=DEV, dtype=torch.bfloat16)
        epoch = torch.zeros(2, device=DEV, dtype=torch.int64)
        ext.tp_decode_allreduce_norm(res, w, out, 1e-6, rows, pp, cp, epoch, r, W, err)
        torch.cuda.synchronize()
        assert ops.check_errors(DEV) == 0
        assert int(epoch[0]) == 1
        assert _rel(res, s) < 1e-2
        assert _rel(out, _norm(s, w)) < 1e-2
    for c in cnt:  # W - 1 pre-added + one arrival from each rank
        assert int(c[0]) == 2 * W - 1
