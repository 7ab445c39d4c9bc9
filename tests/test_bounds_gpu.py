"""Index checks in the kernels that take slot maps, positions and page
tables: an index past its bound is recorded in the device error word
(kErrBadIndex = 6) and its access skipped; the in-range rows still run.

Every out-of-range index here is the first one past the bound, and every
pool, rope table and page table is a view into a larger allocation, so even
an unchecked access would land in memory the test owns (and the test checks
that memory is untouched)."""

import math

import pytest
import torch

from sglang_legolink_b200 import ops
from sglang_legolink_b200.ops import reference as ref

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")
BAD_INDEX = 6


def _clear():
    torch.cuda.synchronize()
    ops.check_errors(DEV)


def test_kv_link_rope_refuses_out_of_range_rows():
    L, pages, H, ps, D = 2, 4, 2, 16, 128
    big_k = torch.zeros(L + 1, pages, H, ps, D, device=DEV, dtype=torch.bfloat16)
    big_v = torch.zeros_like(big_k)
    kp, vp = big_k[:L], big_v[:L]
    kp.normal_()
    vp.normal_()
    cs_big = ref.rope_cos_sin_table(80, D, 1e6).to(DEV)
    cs = cs_big[:64]
    lim = pages * ps
    src = torch.tensor([0, 1, 2, 3], device=DEV, dtype=torch.int64)
    dst = torch.tensor([40, lim, 42, 43], device=DEV, dtype=torch.int64)  # row 1: first slot past the pool
    lp = torch.tensor([0, 1, 2, 3], device=DEV, dtype=torch.int32)
    gp = torch.tensor([5, 6, 64, 8], device=DEV, dtype=torch.int32)  # row 2: first position past the table
    _clear()
    want_k, want_v = kp.clone(), vp.clone()
    ops.kv_link_rope(kp, vp, src, dst, lp, gp, cs)
    torch.cuda.synchronize()
    assert ops.check_errors(DEV) == BAD_INDEX
    assert big_k[L].abs().sum().item() == 0 and big_v[L].abs().sum().item() == 0
    # rows 0 and 3 were linked, rows 1 and 2 not
    keep = torch.tensor([True, False, False, True], device=DEV)
    ref.kv_link_rope(want_k, want_v, src[keep], dst[keep], lp[keep], gp[keep], cs)
    assert torch.equal(kp[:, 2:], want_k[:, 2:]) and torch.equal(vp[:, 2:], want_v[:, 2:])
    assert ops.check_errors(DEV) == 0


def test_rope_qkv_write_and_fused_qkv_gemv_refuse_out_of_range_rows():
    Hq, Hkv, D, pages, ps, K = 4, 2, 128, 4, 16, 512
    T = 3
    N = (Hq + 2 * Hkv) * D
    big_k = torch.zeros(pages + 1, Hkv, ps, D, device=DEV, dtype=torch.bfloat16)
    big_v = torch.zeros_like(big_k)
    kp, vp = big_k[:pages], big_v[:pages]
    cs = ref.rope_cos_sin_table(96, D, 1e6).to(DEV)[:64]
    pos = torch.tensor([3, 64, 9], device=DEV, dtype=torch.int32)  # row 1: position past the table
    slots = torch.tensor([5, 7, pages * ps], device=DEV, dtype=torch.int64)  # row 2: slot past the pool
    qkv = torch.randn(T, N, device=DEV, dtype=torch.bfloat16)
    q = torch.zeros(T, Hq, D, device=DEV, dtype=torch.bfloat16)
    _clear()
    ops.rope_qkv_write(qkv, pos, slots, cs, q, kp, vp, Hq, Hkv, D)
    torch.cuda.synchronize()
    assert ops.check_errors(DEV) == BAD_INDEX
    assert big_k[pages].abs().sum().item() == 0 and big_v[pages].abs().sum().item() == 0
    assert q[0].abs().sum().item() > 0 and q[1].abs().sum().item() == 0
    x = torch.randn(T, K, device=DEV, dtype=torch.bfloat16)
    w = torch.randn(N, K, device=DEV, dtype=torch.bfloat16) / math.sqrt(K)
    kp.zero_()
    vp.zero_()
    q.zero_()
    ops.gemv_qkv_rope(x, w, None, pos, slots, cs, q, kp, vp, Hq, Hkv)
    torch.cuda.synchronize()
    assert ops.check_errors(DEV) == BAD_INDEX
    assert big_k[pages].abs().sum().item() == 0 and big_v[pages].abs().sum().item() == 0
    assert q[0].abs().sum().item() > 0 and q[1].abs().sum().item() == 0
    assert kp[0, :, 5].abs().sum().item() > 0  # row 0's slot 5 (page 0, offset 5) was written


def test_attention_refuses_keys_past_the_page_table_row():
    Hq, Hkv, D, ps, pages = 8, 2, 128, 16, 8
    kp = torch.randn(1, pages, Hkv, ps, D, device=DEV, dtype=torch.bfloat16)
    vp = torch.randn_like(kp)
    big_pt = torch.zeros(16, device=DEV, dtype=torch.int32)
    big_pt[:4] = torch.arange(4, device=DEV, dtype=torch.int32)
    pt = big_pt[:4].view(1, 4)  # a row of 4 pages = 64 keys (stride 4); entries 4.. belong to the test
    scale = 1.0 / math.sqrt(D)
    q = torch.randn(1, Hq, D, device=DEV, dtype=torch.bfloat16)
    kvl = torch.tensor([70], device=DEV, dtype=torch.int32)  # 6 keys past the row's capacity
    out = torch.empty(1, Hq * D, device=DEV, dtype=torch.bfloat16)
    _clear()
    ops.attention_decode(q, kp[0], vp[0], pt, kvl, scale, nsplit=1, out=out)
    torch.cuda.synchronize()
    assert ops.check_errors(DEV) == BAD_INDEX
    assert torch.isfinite(out.float()).all()
    qp = torch.randn(4, Hq, D, device=DEV, dtype=torch.bfloat16)
    qpos = torch.tensor([60, 61, 62, 66], device=DEV, dtype=torch.int32)  # the last row is past the row
    qi = torch.tensor([0, 4], device=DEV, dtype=torch.int32)
    outp = torch.empty(4, Hq * D, device=DEV, dtype=torch.bfloat16)
    ops.attention_prefill(qp, kp, vp, 0, qi, qpos, pt, torch.tensor([67], device=DEV, dtype=torch.int32), scale,
                          out=outp)
    torch.cuda.synchronize()
    assert ops.check_errors(DEV) == BAD_INDEX
    assert torch.isfinite(outp.float()).all()
    assert torch.equal(big_pt[4:], torch.zeros_like(big_pt[4:]))
