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


def _pair_word(val: float, gidx: int) -> int:
    import struct

    bits = struct.unpack("<I", struct.pack("<f", val))[0]
    x = (bits << 32) | (gidx & 0xFFFFFFFF)
    return x - (1 << 64) if x >= (1 << 63) else x


@pytest.mark.parametrize("W", [2, 4, 8])
def test_vocab_sharded_argmax_emulated_world(W):
    """Greedy over vocab shards in one kernel, rank 0 of an emulated world:
    the host writes the other ranks' (max, index) records for each call's
    epoch into rank 0's slot array before the launch, so the kernel's wait is
    already satisfied; the winner is the largest max, ties to the lowest rank
    (the smallest token id), over three calls (both record parities)."""
    torch.manual_seed(W)
    ext, err = ops._cuda(), ops.workspace(DEV).err
    R, V, RMAX = 16, 1000, 64
    recs = [torch.zeros(2 * RMAX * 8 * 2, device=DEV, dtype=torch.int64) for _ in range(W)]
    ptrs = [r.data_ptr() for r in recs]
    epoch = torch.zeros(2, device=DEV, dtype=torch.int64)
    for call in (1, 2, 3):
        logits = torch.randn(R, V, device=DEV).to(torch.bfloat16)
        lf = logits.float()
        mine_v, mine_i = lf.max(-1)
        par = call & 1
        cands = [[(float(mine_v[i]), int(mine_i[i]))] for i in range(R)]
        for r in range(1, W):
            for i in range(R):
                if i == 0:
                    val = float(mine_v[i])  # a tie with rank 0: rank 0 (the smaller id) wins
                elif i == 1 and r >= 2:
                    val = 50.0  # a tie between the other ranks: the lowest of them wins
                else:
                    val = float(torch.randn(()).item() * 2)
                gidx = r * V + int(torch.randint(0, V, ()).item())
                cands[i].append((val, gidx))
                base = ((par * RMAX + i) * 8 + r) * 2
                recs[0][base] = _pair_word(val, gidx)
                recs[0][base + 1] = call
        out = torch.empty(R, device=DEV, dtype=torch.int32)
        ext.tp_argmax(logits, 0, out, ptrs, epoch, 0, W, RMAX, err)
        torch.cuda.synchronize()
        assert ops.check_errors(DEV) == 0
        exp = [max(c, key=lambda t: (t[0], -t[1]))[1] for c in cands]
        assert out.tolist() == exp
        assert int(epoch[0]) == call
        # rank 0 pushed its own record, tagged with this call's epoch, to every rank
        for d in range(W):
            base = ((par * RMAX + 3) * 8 + 0) * 2
            assert int(recs[d][base + 1]) == call
