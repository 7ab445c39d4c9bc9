"""sm_100a kernels vs plain PyTorch fp32 statements of the same ops."""

import math

import pytest
import torch

from sglang_legolink_b200 import ops
from sglang_legolink_b200.ops import reference as ref

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _rel(a, b):
    a, b = a.float().cpu(), b.float().cpu()
    return ((a - b).norm() / (b.norm() + 1e-6)).item()


@pytest.mark.parametrize("M,N,K", [(128, 256, 128), (256, 512, 1024), (1000, 4608, 3584), (77, 640, 512),
                                   (600, 2200, 768), (1300, 2560, 1024), (257, 2048, 64),
                                   (384, 3584, 18944), (4096, 1024, 512)])
def test_gemm_tcgen05(M, N, K):
    torch.manual_seed(0)
    a = torch.randn(M, K, device=DEV, dtype=torch.bfloat16)
    w = torch.randn(N, K, device=DEV, dtype=torch.bfloat16) / math.sqrt(K)
    bias = torch.randn(N, device=DEV, dtype=torch.bfloat16)
    out = torch.empty(M, N, device=DEV, dtype=torch.bfloat16)
    ops._cuda().gemm(a, w, bias, out, 0, 256 if N >= 2048 else 128, ops.workspace(DEV).err)
    torch.cuda.synchronize()
    assert ops.check_errors(DEV) == 0
    exp = a.float() @ w.float().t() + bias.float()
    assert _rel(out, exp) < 1e-2


@pytest.mark.parametrize("bn", [128, 256])
def test_gemm_tcgen05_both_tiles(bn):
    torch.manual_seed(1)
    M, N, K = 300, 768, 640
    a = torch.randn(M, K, device=DEV, dtype=torch.bfloat16)
    w = torch.randn(N, K, device=DEV, dtype=torch.bfloat16) / math.sqrt(K)
    out = torch.empty(M, N, device=DEV, dtype=torch.bfloat16)
    ops._cuda().gemm(a, w, None, out, 0, bn, ops.workspace(DEV).err)
    assert _rel(out, a.float() @ w.float().t()) < 1e-2


def test_gemm_swiglu_epilogue():
    torch.manual_seed(2)
    M, I, K = 333, 1024, 512
    a = torch.randn(M, K, device=DEV, dtype=torch.bfloat16)
    gate = torch.randn(I, K, device=DEV, dtype=torch.bfloat16) / math.sqrt(K)
    up = torch.randn(I, K, device=DEV, dtype=torch.bfloat16) / math.sqrt(K)
    gu = ops.interleave_gate_up(gate, up)
    out = ops.linear(a, gu, swiglu_epilogue=True)
    exp = torch.nn.functional.silu(a.float() @ gate.float().t()) * (a.float() @ up.float().t())
    assert _rel(out, exp) < 1e-2


@pytest.mark.parametrize("M", [1, 7, 64])
@pytest.mark.parametrize("splits", [1, 0])
def test_gemm_small_m_swiglu_epilogue(M, splits):
    """SwiGLU applied in the small-M GEMM's own epilogue (one split) and in
    its split-K fix-up (auto splits) against fp32 silu(a.gate^T) * a.up^T."""
    torch.manual_seed(4)
    I, K = 1024, 1536
    a = torch.randn(M, K, device=DEV, dtype=torch.bfloat16)
    gate = torch.randn(I, K, device=DEV, dtype=torch.bfloat16) / math.sqrt(K)
    up = torch.randn(I, K, device=DEV, dtype=torch.bfloat16) / math.sqrt(K)
    gu = ops.interleave_gate_up(gate, up)
    ws = ops.workspace(DEV)
    ws.reserve_gemm(32 * M * 2 * I, 2 * I // 128)
    out = torch.empty(M, I, device=DEV, dtype=torch.bfloat16)
    ops._cuda().gemm_small_m(a, gu, None, out, splits, ws.gemm_ws, ws.tickets, ws.err, True)
    torch.cuda.synchronize()
    assert ops.check_errors(DEV) == 0
    exp = torch.nn.functional.silu(a.float() @ gate.float().t()) * (a.float() @ up.float().t())
    assert _rel(out, exp) < 1e-2
    assert torch.equal(ops.linear(a, gu, swiglu_epilogue=True), out) or splits == 1


@pytest.mark.parametrize("M", [1, 5, 40])
def test_gemv_rownorm_and_residual_epilogues(M):
    """Row-scaled GEMV (plain and SwiGLU) and the residual epilogue against
    fp32: y * rsqrt(sumsq / K + eps) + bias; r = bf16(y) + res, res = bf16(r),
    h = bf16(r * w), sumsq += sum(r^2)."""
    torch.manual_seed(6)
    K, N, eps = 1536, 1024, 1e-6
    x = torch.randn(M, K, device=DEV, dtype=torch.bfloat16)
    w = torch.randn(N, K, device=DEV, dtype=torch.bfloat16) / math.sqrt(K)
    bias = torch.randn(N, device=DEV, dtype=torch.bfloat16)
    sumsq = ops.sumsq_from_values(torch.rand(M, device=DEV) * K * 3 + 1.0)  # int64 fixed point on CUDA
    rstd = torch.rsqrt(ops.sumsq_values(sumsq) / K + eps)[:, None]
    out = ops.gemv_rownorm(x, w, bias, sumsq, eps)
    assert _rel(out, (x.float() @ w.float().t()) * rstd + bias.float()) < 1e-2
    gate, up = w[: N // 2], torch.randn(N // 2, K, device=DEV, dtype=torch.bfloat16) / math.sqrt(K)
    sw = ops.gemv_rownorm(x, ops.interleave_gate_up(gate, up), None, sumsq, eps, swiglu=True)
    exp = torch.nn.functional.silu((x.float() @ gate.float().t()) * rstd) * ((x.float() @ up.float().t()) * rstd)
    assert _rel(sw, exp) < 1e-2
    res = torch.randn(M, N, device=DEV, dtype=torch.bfloat16)
    res0 = res.clone()
    nw = torch.rand(N, device=DEV, dtype=torch.bfloat16) + 0.5
    h = torch.empty(M, N, device=DEV, dtype=torch.bfloat16)
    sq = ops.sumsq_buffer(M, DEV)
    ops.gemv_residual(x, w, res, nw, h, sq)
    torch.cuda.synchronize()
    assert ops.check_errors(DEV) == 0
    r = (x.float() @ w.float().t()).to(torch.bfloat16).float() + res0.float()
    assert _rel(res, r) < 1e-2 and _rel(h, r * nw.float()) < 1e-2
    assert _rel(ops.sumsq_values(sq), (r * r).sum(-1)) < 1e-3
    # the fixed-point sums are bit-identical however the tiles finish
    for _ in range(3):
        res.copy_(res0)
        sq2 = ops.sumsq_buffer(M, DEV)
        ops.gemv_residual(x, w, res, nw, h, sq2)
        assert torch.equal(sq2, sq)


@pytest.mark.parametrize("qk_norm,M", [(False, 3), (True, 3), (True, 37)])
def test_gemv_qkv_rope_matches_unfused(qk_norm, M):
    """qkv GEMV with per-head norm, RoPE and the KV write in its stores ==
    GEMV then rope_qkv_write, and == the fp32 CPU definition.  M = 37 puts
    rows past 32, whose positions and slots the epilogue reads from memory."""
    torch.manual_seed(7)
    Hq, Hkv, D, K, ps, pages = 8, 2, 128, 1024, 16, 8
    N = (Hq + 2 * Hkv) * D
    x = torch.randn(M, K, device=DEV, dtype=torch.bfloat16)
    w = torch.randn(N, K, device=DEV, dtype=torch.bfloat16) / math.sqrt(K)
    bias = torch.randn(N, device=DEV, dtype=torch.bfloat16)
    if M == 3:
        pos = torch.tensor([5, 17, 100], device=DEV, dtype=torch.int32)
        slots = torch.tensor([3, 40, 77], device=DEV, dtype=torch.int64)
    else:
        pos = torch.randperm(4096, generator=torch.Generator().manual_seed(M))[:M].to(DEV, torch.int32)
        slots = torch.randperm(pages * ps, generator=torch.Generator().manual_seed(M + 1))[:M].to(DEV)
    cs = ref.rope_cos_sin_table(4096, 128, 1e6).to(DEV)
    qn = (torch.rand(D, device=DEV, dtype=torch.bfloat16) + 0.5) if qk_norm else None
    kn = (torch.rand(D, device=DEV, dtype=torch.bfloat16) + 0.5) if qk_norm else None
    pools = [torch.zeros(pages, Hkv, ps, D, device=DEV, dtype=torch.bfloat16) for _ in range(4)]
    q1 = torch.empty(M, Hq, D, device=DEV, dtype=torch.bfloat16)
    q2 = torch.empty_like(q1)
    ops.gemv_qkv_rope(x, w, bias, pos, slots, cs, q1, pools[0], pools[1], Hq, Hkv, qn, kn, 1e-6)
    torch.cuda.synchronize()
    assert ops.check_errors(DEV) == 0
    ops.rope_qkv_write(ops.linear(x, w, bias), pos, slots, cs, q2, pools[2], pools[3], Hq, Hkv, D, qn, kn, 1e-6)
    assert _rel(q1, q2) < 1e-2 and _rel(pools[0], pools[2]) < 1e-2 and _rel(pools[1], pools[3]) < 1e-2
    kc = torch.zeros(pages, Hkv, ps, D)
    vc = torch.zeros_like(kc)
    qc = torch.empty(M, Hq, D)
    c = lambda t: None if t is None else t.cpu().float()
    ops.gemv_qkv_rope(c(x), c(w), c(bias), pos.cpu(), slots.cpu(), cs.cpu(), qc, kc, vc, Hq, Hkv, c(qn), c(kn), 1e-6)
    assert _rel(q1, qc) < 1e-2 and _rel(pools[0], kc) < 1e-2 and _rel(pools[1], vc) < 1e-2


@pytest.mark.parametrize("max_splits", [8, 1])
@pytest.mark.parametrize("M", [2, 5, 16])
def test_gemv_tile_epilogue_rows_equal_one_row_launches(M, max_splits, monkeypatch):
    """2..16-row GEMVs run the tile epilogue (a row per warp, four features
    per lane); 1-row GEMVs run the one-row epilogue.  Row for row the two
    give the same bits in all four epilogue modes, with the split-K fix-up
    and without it (one split).  Both launches get the same split count
    (8, the cap of the 2..16-row launches), so they sum in the same order."""
    monkeypatch.setattr(ops, "_SMALL_M_MAX_SPLITS", max_splits)
    torch.manual_seed(11)
    K, N, eps = 1536, 1024, 1e-6
    x = torch.randn(M, K, device=DEV, dtype=torch.bfloat16)
    w = torch.randn(N, K, device=DEV, dtype=torch.bfloat16) / math.sqrt(K)
    bias = torch.randn(N, device=DEV, dtype=torch.bfloat16)
    ws = ops.workspace(DEV)
    # plain store with bias
    out = torch.empty(M, N, device=DEV, dtype=torch.bfloat16)
    ops._small_m(ops._cuda(), ws, x, w, bias, out)
    for r in range(M):
        o1 = torch.empty(1, N, device=DEV, dtype=torch.bfloat16)
        ops._small_m(ops._cuda(), ws, x[r:r + 1], w, bias, o1)
        assert torch.equal(out[r], o1[0]), r
    # row-scaled SwiGLU
    sumsq = ops.sumsq_from_values(torch.rand(M, device=DEV) * K * 3 + 1.0)
    sw = ops.gemv_rownorm(x, w, None, sumsq, eps, swiglu=True)
    for r in range(M):
        assert torch.equal(sw[r], ops.gemv_rownorm(x[r:r + 1], w, None, sumsq[r:r + 1], eps, swiglu=True)[0]), r
    # residual add + next-norm data + fixed-point sums of squares
    res0 = torch.randn(M, N, device=DEV, dtype=torch.bfloat16)
    nw = torch.rand(N, device=DEV, dtype=torch.bfloat16) + 0.5
    res, h, sq = res0.clone(), torch.empty(M, N, device=DEV, dtype=torch.bfloat16), ops.sumsq_buffer(M, DEV)
    ops.gemv_residual(x, w, res, nw, h, sq)
    for r in range(M):
        res1, h1, sq1 = res0[r:r + 1].clone(), torch.empty(1, N, device=DEV, dtype=torch.bfloat16), ops.sumsq_buffer(1, DEV)
        ops.gemv_residual(x[r:r + 1], w, res1, nw, h1, sq1)
        assert torch.equal(res[r], res1[0]) and torch.equal(h[r], h1[0]) and torch.equal(sq[r], sq1[0]), r
    # qkv with QK-norm, RoPE and the KV write
    Hq, Hkv, D, ps, pages = 8, 2, 128, 16, 4
    Nq = (Hq + 2 * Hkv) * D
    wq = torch.randn(Nq, K, device=DEV, dtype=torch.bfloat16) / math.sqrt(K)
    bq = torch.randn(Nq, device=DEV, dtype=torch.bfloat16)
    pos = torch.randperm(4096, generator=torch.Generator().manual_seed(M))[:M].to(DEV, torch.int32)
    slots = torch.randperm(pages * ps, generator=torch.Generator().manual_seed(M + 1))[:M].to(DEV)
    cs = ref.rope_cos_sin_table(4096, 128, 1e6).to(DEV)
    qn = torch.rand(D, device=DEV, dtype=torch.bfloat16) + 0.5
    kn = torch.rand(D, device=DEV, dtype=torch.bfloat16) + 0.5
    pools = [torch.zeros(pages, Hkv, ps, D, device=DEV, dtype=torch.bfloat16) for _ in range(4)]
    q = torch.empty(M, Hq, D, device=DEV, dtype=torch.bfloat16)
    ops.gemv_qkv_rope(x, wq, bq, pos, slots, cs, q, pools[0], pools[1], Hq, Hkv, qn, kn, eps)
    for r in range(M):
        q1 = torch.empty(1, Hq, D, device=DEV, dtype=torch.bfloat16)
        ops.gemv_qkv_rope(x[r:r + 1], wq, bq, pos[r:r + 1], slots[r:r + 1], cs, q1, pools[2], pools[3], Hq, Hkv,
                          qn, kn, eps)
        assert torch.equal(q[r], q1[0]), r
    assert torch.equal(pools[0], pools[2]) and torch.equal(pools[1], pools[3])
    torch.cuda.synchronize()
    assert ops.check_errors(DEV) == 0


@pytest.mark.parametrize("M", [1, 3, 16, 17, 64, 100, 128])
@pytest.mark.parametrize("N,K", [(4608, 3584), (3584, 18944), (1000, 512)])
def test_gemm_small_m(M, N, K):
    torch.manual_seed(3)
    a = torch.randn(M, K, device=DEV, dtype=torch.bfloat16)
    w = torch.randn(N, K, device=DEV, dtype=torch.bfloat16) / math.sqrt(K)
    bias = torch.randn(N, device=DEV, dtype=torch.bfloat16)
    out = torch.empty(M, N, device=DEV, dtype=torch.bfloat16)
    ops._small_m(ops._cuda(), ops.workspace(DEV), a, w, bias, out)
    torch.cuda.synchronize()
    assert ops.check_errors(DEV) == 0
    exp = a.float() @ w.float().t() + bias.float()
    assert _rel(out, exp) < 1e-2
    # second call reuses the tickets (must have been reset to zero)
    out2 = torch.empty_like(out)
    ops._small_m(ops._cuda(), ops.workspace(DEV), a, w, bias, out2)
    assert torch.equal(out, out2)


@pytest.mark.parametrize("hidden", [256, 3584, 5120])
def test_rmsnorm_and_fused_add(hidden):
    torch.manual_seed(4)
    x = torch.randn(37, hidden, device=DEV, dtype=torch.bfloat16)
    r = torch.randn(37, hidden, device=DEV, dtype=torch.bfloat16)
    w = torch.randn(hidden, device=DEV, dtype=torch.bfloat16)
    y = ops.rmsnorm(x, w, 1e-6)
    assert _rel(y, ref.rmsnorm(x.cpu().float(), w.cpu().float(), 1e-6)) < 1e-2
    xc, rc = x.clone(), r.clone()
    ops.fused_add_rmsnorm(xc, rc, w, 1e-6)
    xr, rr = x.float().cpu(), r.float().cpu()
    ref.fused_add_rmsnorm(xr, rr, w.float().cpu(), 1e-6)
    assert _rel(rc, rr) < 1e-2 and _rel(xc, xr) < 1e-2


@pytest.mark.parametrize("qk_norm", [False, True])
def test_rope_qkv_write(qk_norm):
    torch.manual_seed(5)
    Hq, Hkv, D, ps, T = 8, 2, 128, 16, 50
    qkv = torch.randn(T, (Hq + 2 * Hkv) * D, device=DEV, dtype=torch.bfloat16)
    pos = torch.randint(0, 4000, (T,), dtype=torch.int32)
    pages = torch.randperm(64)[:8]
    slots = (pages[torch.arange(T) // ps] * ps + torch.arange(T) % ps).to(torch.int64)
    cs = ref.rope_cos_sin_table(4096, D, 1e6)
    qn = torch.randn(D, dtype=torch.bfloat16) if qk_norm else None
    kn = torch.randn(D, dtype=torch.bfloat16) if qk_norm else None
    kp = torch.zeros(64, Hkv, ps, D, device=DEV, dtype=torch.bfloat16)
    vp = torch.zeros_like(kp)
    q = torch.empty(T, Hq, D, device=DEV, dtype=torch.bfloat16)
    ops.rope_qkv_write(qkv, pos.to(DEV), slots.to(DEV), cs.to(DEV), q, kp, vp, Hq, Hkv, D,
                       qn.to(DEV) if qk_norm else None, kn.to(DEV) if qk_norm else None)
    kr, vr = kp.cpu().float().zero_(), vp.cpu().float().zero_()
    qr = ref.rope_qkv_write(qkv.cpu().float(), pos, slots, cs, kr, vr, Hq, Hkv, D,
                            qn.float() if qk_norm else None, kn.float() if qk_norm else None)
    assert _rel(q, qr) < 1e-2
    assert _rel(kp, kr) < 1e-2
    assert torch.equal(vp.cpu().float(), vr)


@pytest.mark.parametrize("ps", [16, 64])
def test_kv_link_rope_matches_fp32_within_one_ulp(ps):
    torch.manual_seed(6)
    L, P, H, D = 3, 96, 4, 128
    k = torch.randn(L, P, H, ps, D, dtype=torch.bfloat16)
    v = torch.randn(L, P, H, ps, D, dtype=torch.bfloat16)
    n = 300
    src = torch.randperm(P * ps // 2)[:n].to(torch.int64)
    dst = (torch.randperm(P * ps // 2)[:n] + P * ps // 2).to(torch.int64)
    lp = torch.randint(0, 8192, (n,), dtype=torch.int32)
    gp = torch.randint(0, 32768, (n,), dtype=torch.int32)
    gp[:10] = lp[:10]  # identity rows
    cs = ref.rope_cos_sin_table(32768, D, 1e6)
    kd, vd = k.to(DEV), v.to(DEV)
    ops.kv_link_rope(kd, vd, src.to(DEV), dst.to(DEV), lp.to(DEV), gp.to(DEV), cs.to(DEV))
    kr, vr = k.float(), v.float()
    ref.kv_link_rope(kr, vr, src, dst, lp, gp, cs)
    got = kd.cpu().float()
    # compare rounded-to-bf16 oracle: within 1 bf16 ulp
    exp = kr.to(torch.bfloat16).float()
    ulp = torch.maximum(exp.abs(), torch.full_like(exp, 1e-30)) * 2.0**-7
    assert bool(((got - exp).abs() <= ulp + 1e-6).all())
    assert torch.equal(vd.cpu(), vr.to(torch.bfloat16))


def _paged_setup(B, lens, Hkv, D, ps, seed=0, contiguous=False):
    g = torch.Generator().manual_seed(seed)
    npages = sum((n + ps - 1) // ps for n in lens) + 4
    perm = torch.arange(npages) if contiguous else torch.randperm(npages, generator=g)
    if contiguous:  # ascending runs with one break, so both load paths of the kernels run
        perm[npages // 3:] = torch.flip(perm[npages // 3:], [0])
    kp = torch.randn(npages, Hkv, ps, D, generator=g).to(torch.bfloat16)
    vp = torch.randn(npages, Hkv, ps, D, generator=g).to(torch.bfloat16)
    maxp = max((n + ps - 1) // ps for n in lens)
    pt = torch.zeros(B, maxp, dtype=torch.int32)
    c = 0
    for b, n in enumerate(lens):
        k = (n + ps - 1) // ps
        pt[b, :k] = perm[c : c + k].to(torch.int32)
        c += k
    return kp, vp, pt


@pytest.mark.parametrize("Hq,Hkv,ps", [(28, 4, 16), (8, 8, 16), (64, 8, 16), (4, 2, 16), (28, 4, 64), (7, 1, 32)])
def test_attention_prefill_sparse_rows(Hq, Hkv, ps):
    D = 128
    lens = [700, 130, 1500]
    kp, vp, pt = _paged_setup(3, lens, Hkv, D, ps)
    g = torch.Generator().manual_seed(1)
    rows, qptr = [], [0]
    for n in lens:
        # sparse repair rows: a prefix, windows, and the tail
        p = sorted(set(list(range(0, 5)) + list(range(100, 140)) + list(range(n - 20, n))))
        p = [x for x in p if x < n]
        rows.extend(p)
        qptr.append(qptr[-1] + len(p))
    T = len(rows)
    q = torch.randn(T, Hq, D, generator=g).to(torch.bfloat16)
    qpos = torch.tensor(rows, dtype=torch.int32)
    qi = torch.tensor(qptr, dtype=torch.int32)
    kvl = torch.tensor(lens, dtype=torch.int32)
    scale = 1 / math.sqrt(D)
    kd, vd = kp[None].to(DEV), vp[None].to(DEV)
    out = ops.attention_prefill(q.to(DEV), kd, vd, 0, qi.to(DEV), qpos.to(DEV), pt.to(DEV), kvl.to(DEV), scale)
    torch.cuda.synchronize()
    assert ops.check_errors(DEV) == 0
    exp = ref.paged_attention(q.float(), kp.float(), vp.float(), qi, qpos, pt, kvl, scale)
    assert _rel(out.cpu(), exp) < 1.5e-2
    legacy = ops.attention_prefill_mma(q.to(DEV), kp.to(DEV), vp.to(DEV), qi.to(DEV), qpos.to(DEV), pt.to(DEV),
                                       scale)
    assert _rel(legacy.cpu(), exp) < 1.5e-2


@pytest.mark.parametrize("variant", [0, 2, 3, 4, 7, 8])
def test_attention_prefill_builds_match_fp32(variant):
    """Builds of the tcgen05 kernel (0: one softmax warpgroup per tile, 2:
    with 2 of 8 exp2 on the FMA pipe, 3 and 4: two warpgroups per tile, 64
    key columns each, 7 and 8: 8-chain max and P stored after the whole row)
    on sparse and full causal rows; the second request's
    queries are scaled up so that running maxima grow mid-row and O is
    rescaled in TMEM."""
    ext = ops._cuda()
    D, Hq, Hkv, ps = 128, 28, 4, 16
    lens = [3000, 900]
    kp, vp, pt = _paged_setup(2, lens, Hkv, D, ps, seed=11)
    g = torch.Generator().manual_seed(12)
    rows = sorted(set(range(0, 40)) | set(range(1000, 1100)) | set(range(2950, 3000)))
    qptr = [0, len(rows), len(rows) + lens[1]]
    rows = rows + list(range(lens[1]))
    q = torch.randn(len(rows), Hq, D, generator=g)
    q[qptr[1]:] *= 4.0
    q = q.to(torch.bfloat16)
    qpos = torch.tensor(rows, dtype=torch.int32)
    qi = torch.tensor(qptr, dtype=torch.int32)
    kvl = torch.tensor(lens, dtype=torch.int32)
    scale = 1 / math.sqrt(D)
    exp = ref.paged_attention(q.float(), kp.float(), vp.float(), qi, qpos, pt, kvl, scale)
    try:
        ext.attn_prefill_tc_set_variant(variant)
        out = ops.attention_prefill(q.to(DEV), kp[None].to(DEV), vp[None].to(DEV), 0, qi.to(DEV), qpos.to(DEV),
                                    pt.to(DEV), kvl.to(DEV), scale)
        torch.cuda.synchronize()
    finally:
        ext.attn_prefill_tc_set_variant(-2)
    assert ops.check_errors(DEV) == 0
    assert _rel(out.cpu(), exp) < 1.5e-2


@pytest.mark.parametrize("variant", [7, 0, 3])
@pytest.mark.parametrize("S", [2, 3, 5])
def test_attention_prefill_key_range_splits_match_fp32(variant, S):
    """Each tile as S work items over equal key ranges, partials merged by
    the combine kernel: one KV head with 8 query heads per kv head (a tensor
    parallel rank's share of Qwen3-32B), rows near the start (their tiles
    have fewer key blocks than S: empty items) and rows deep in a 6K context
    (ranges that mask every key of some rows), queries scaled up so running
    maxima grow mid-range; against the fp32 statement."""
    ext = ops._cuda()
    D, Hq, Hkv, ps = 128, 8, 1, 16
    lens = [6000, 700]
    kp, vp, pt = _paged_setup(2, lens, Hkv, D, ps, seed=21)
    g = torch.Generator().manual_seed(22)
    rows0 = sorted(set(range(0, 48)) | set(range(2000, 2060)) | set(range(5900, 6000)))
    rows1 = list(range(0, 30)) + list(range(650, 700))
    qptr = [0, len(rows0), len(rows0) + len(rows1)]
    rows = rows0 + rows1
    q = torch.randn(len(rows), Hq, D, generator=g)
    q[: len(rows0) // 2] *= 4.0
    q = q.to(torch.bfloat16)
    qpos = torch.tensor(rows, dtype=torch.int32)
    qi = torch.tensor(qptr, dtype=torch.int32)
    kvl = torch.tensor(lens, dtype=torch.int32)
    scale = 1 / math.sqrt(D)
    exp = ref.paged_attention(q.float(), kp.float(), vp.float(), qi, qpos, pt, kvl, scale)
    host = ops.prefill_tiles(qi, qpos, Hq, Hkv, split=S)
    assert ops.tiles_split_count(host) == S and len(host) % S == 0
    try:
        ext.attn_prefill_tc_set_variant(variant)
        out = ops.attention_prefill(q.to(DEV), kp[None].to(DEV), vp[None].to(DEV), 0, qi.to(DEV), qpos.to(DEV),
                                    pt.to(DEV), kvl.to(DEV), scale, tiles=host.to(DEV), nsplit=S)
        torch.cuda.synchronize()
    finally:
        ext.attn_prefill_tc_set_variant(-2)
    assert ops.check_errors(DEV) == 0
    assert _rel(out.cpu(), exp) < 1.5e-2


def test_attention_prefill_split_work_list_mismatch_is_refused():
    """A work list whose encoded split count differs from the launch's is
    recorded as an error and writes nothing (no partial goes to a missing
    workspace)."""
    D, Hq, Hkv, ps = 128, 8, 1, 16
    lens = [600]
    kp, vp, pt = _paged_setup(1, lens, Hkv, D, ps, seed=23)
    rows = list(range(500, 600))
    q = torch.randn(len(rows), Hq, D).to(torch.bfloat16).to(DEV)
    qi = torch.tensor([0, len(rows)], dtype=torch.int32)
    qpos = torch.tensor(rows, dtype=torch.int32)
    host = ops.prefill_tiles(qi, qpos, Hq, Hkv, split=3)
    out = torch.full((len(rows), Hq * D), 7.0, device=DEV).to(torch.bfloat16)
    ops.attention_prefill(q, kp[None].to(DEV), vp[None].to(DEV), 0, qi.to(DEV), qpos.to(DEV), pt.to(DEV),
                          torch.tensor(lens, dtype=torch.int32, device=DEV), 0.1, tiles=host.to(DEV), out=out,
                          nsplit=1)
    torch.cuda.synchronize()
    assert ops.check_errors(DEV) != 0
    assert bool((out.float() == 7.0).all())


@pytest.mark.parametrize("B,Hq,Hkv,n,contiguous", [(1, 28, 4, 16000, False), (1, 28, 4, 16000, True),
                                                   (3, 28, 4, 1000, True), (16, 8, 1, 3000, False),
                                                   (2, 64, 8, 77, False)])
def test_attention_decode(B, Hq, Hkv, n, contiguous):
    D, ps = 128, 16
    lens = [n - 3 * b for b in range(B)]
    kp, vp, pt = _paged_setup(B, lens, Hkv, D, ps, seed=3, contiguous=contiguous)
    g = torch.Generator().manual_seed(2)
    q = torch.randn(B, Hq, D, generator=g).to(torch.bfloat16)
    kvl = torch.tensor(lens, dtype=torch.int32)
    scale = 1 / math.sqrt(D)
    out = ops.attention_decode(q.to(DEV), kp.to(DEV), vp.to(DEV), pt.to(DEV), kvl.to(DEV), scale)
    exp = ref.paged_attention(q.float(), kp.float(), vp.float(), torch.arange(B + 1, dtype=torch.int32),
                              kvl - 1, pt, kvl, scale)
    assert _rel(out.cpu(), exp) < 1.5e-2


@pytest.mark.parametrize("contiguous", [False, True])
def test_attention_prefill_multi_layer_pool_full_causal(contiguous):
    """Full causal prefill of two requests reading layer 1 of a 3-layer pool
    (random page tables, and ascending page runs that use the whole-block
    TMA boxes)."""
    D, ps, Hq, Hkv = 128, 16, 28, 4
    lens = [300, 1000]
    kp, vp, pt = _paged_setup(2, lens, Hkv, D, ps, seed=5, contiguous=contiguous)
    g = torch.Generator().manual_seed(9)
    K3 = torch.randn(3, *kp.shape, generator=g).to(torch.bfloat16)
    V3 = torch.randn(3, *vp.shape, generator=g).to(torch.bfloat16)
    rows = list(range(lens[0])) + list(range(lens[1]))
    qptr = torch.tensor([0, lens[0], lens[0] + lens[1]], dtype=torch.int32)
    q = torch.randn(len(rows), Hq, D, generator=g).to(torch.bfloat16)
    qpos = torch.tensor(rows, dtype=torch.int32)
    kvl = torch.tensor(lens, dtype=torch.int32)
    scale = 1 / math.sqrt(D)
    out = ops.attention_prefill(q.to(DEV), K3.to(DEV), V3.to(DEV), 1, qptr.to(DEV), qpos.to(DEV), pt.to(DEV),
                                kvl.to(DEV), scale)
    exp = ref.paged_attention(q.float(), K3[1].float(), V3[1].float(), qptr, qpos, pt, kvl, scale)
    assert _rel(out.cpu(), exp) < 1.5e-2


def test_swiglu_embedding_argmax():
    torch.manual_seed(7)
    gu = torch.randn(19, 2 * 256, device=DEV, dtype=torch.bfloat16)
    assert _rel(ops.swiglu(gu), ops.ref_swiglu_interleaved(gu.cpu().float())) < 1e-2
    table = torch.randn(1000, 256, device=DEV, dtype=torch.bfloat16)
    ids = torch.randint(0, 1000, (33,), device=DEV, dtype=torch.int32)
    assert torch.equal(ops.embedding(ids, table), table[ids.long()])
    logits = torch.randn(5, 152064, device=DEV, dtype=torch.bfloat16)
    assert torch.equal(ops.argmax(logits).cpu(), torch.argmax(logits.float(), -1).int().cpu())


@pytest.mark.parametrize("M,N,K", [(1, 4608, 3584), (16, 3584, 18944), (64, 1024, 512)])
def test_gemm_small_m_tile_major_weights(M, N, K):
    torch.manual_seed(8)
    a = torch.randn(M, K, device=DEV, dtype=torch.bfloat16)
    w = torch.randn(N, K, device=DEV, dtype=torch.bfloat16) / math.sqrt(K)
    wt = ops.tile_weight(w)
    assert torch.equal(ops.untile_weight(wt), w)
    out = torch.empty(M, N, device=DEV, dtype=torch.bfloat16)
    ops._small_m(ops._cuda(), ops.workspace(DEV), a, wt, None, out)
    assert _rel(out, a.float() @ w.float().t()) < 1e-2


@pytest.mark.gpu
@pytest.mark.parametrize("rows,H", [(1, 5120), (16, 5120), (64, 3584), (7, 1024)])
def test_tp_decode_allreduce_norm_single_rank(rows, H):
    """The decode TP boundary with one rank: residual += partial; out =
    RMSNorm(residual) * w, against fp32 torch; consecutive calls alternate
    buffers and advance the device epoch, also when replayed from a CUDA
    graph."""
    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(rows * 7 + H)
    w = (torch.rand(H, device=dev, generator=g) + 0.5).to(torch.bfloat16)
    res = torch.randn(rows, H, device=dev, generator=g).to(torch.bfloat16)
    parts = [torch.randn(rows, H, device=dev, generator=g).to(torch.bfloat16) for _ in range(2)]
    out = torch.empty(rows, H, device=dev, dtype=torch.bfloat16)
    cnt = torch.zeros(2, dtype=torch.int64, device=dev)
    epoch = torch.zeros(2, dtype=torch.int64, device=dev)
    err = ops.workspace(dev).err
    k = ops._cuda()

    def call(i):
        k.tp_decode_allreduce_norm(res, w, out, 1e-6, rows, [parts[i % 2].data_ptr()], [cnt.data_ptr()], epoch, 0, 1,
                                   err)

    def expect(r, p):
        s = r.float() + p.float()
        return s.to(torch.bfloat16), (s * torch.rsqrt(s.pow(2).mean(-1, keepdim=True) + 1e-6) * w.float())

    for i in range(3):
        r_exp, o_exp = expect(res, parts[i % 2])
        call(i)
        torch.cuda.synchronize()
        assert torch.equal(res, r_exp)
        assert _rel(out.float(), o_exp) < 1e-2
    assert int(epoch[0]) == 3 and int(cnt[0]) == 3 and ops.check_errors(dev) == 0
    graph = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s), torch.cuda.graph(graph, stream=s):
        call(0)
        call(1)
    torch.cuda.current_stream().wait_stream(s)
    for rep in range(3):
        r_exp, _ = expect(res, parts[0])
        r_exp, o_exp = expect(r_exp, parts[1])
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(res, r_exp)
        assert _rel(out.float(), o_exp) < 1e-2
    assert int(epoch[0]) == 9 and int(epoch[1]) == 0 and ops.check_errors(dev) == 0
