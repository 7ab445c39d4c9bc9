"""Plain PyTorch (fp32) statements of every op the runtime executes.

These are the numerical oracle for the sm_100a kernels in ``csrc/`` and the
execution path of the CPU runtime (the BASELINE "CPU fake-runtime" config).
Each function states the math the corresponding kernel must reproduce.

KV pool layout shared by the oracle and the kernels::

    k_pool, v_pool: [num_layers, num_pages, num_kv_heads, page_size, head_dim]

A *slot* is ``page * page_size + offset``; token ``t`` of a request lives at
slot ``page_table[t // page_size] * page_size + t % page_size``.

RoPE cos/sin table: ``cos_sin[pos] = [cos(pos*f_0..f_{D/2-1}), sin(...)]``
(neox / rotate-half style, as Qwen uses; reference
``patched_sglang_files/python/sglang/srt/pic_runtime.py:1868-1885``).
"""

from __future__ import annotations

import math
from typing import Optional

import torch


def rope_cos_sin_table(max_pos: int, rotary_dim: int, theta: float, device=None) -> torch.Tensor:
    """fp32 table [max_pos, rotary_dim] = [cos | sin], computed in float64."""
    half = rotary_dim // 2
    inv_freq = 1.0 / (theta ** (torch.arange(0, half, dtype=torch.float64) * 2.0 / rotary_dim))
    pos = torch.arange(max_pos, dtype=torch.float64)
    ang = pos[:, None] * inv_freq[None, :]
    table = torch.cat([torch.cos(ang), torch.sin(ang)], dim=-1).to(torch.float32)
    return table.to(device) if device is not None else table


def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    xf = x.float()
    var = xf.pow(2).mean(-1, keepdim=True)
    return (xf * torch.rsqrt(var + eps) * w.float()).to(x.dtype)


def fused_add_rmsnorm(x: torch.Tensor, residual: torch.Tensor, w: torch.Tensor, eps: float):
    """residual <- residual + x ; x <- rmsnorm(residual) * w   (both in place)."""
    r = residual.float() + x.float()
    residual.copy_(r.to(residual.dtype))
    rf = residual.float()
    var = rf.pow(2).mean(-1, keepdim=True)
    x.copy_((rf * torch.rsqrt(var + eps) * w.float()).to(x.dtype))


def apply_rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """x [..., D] fp32, cos/sin [..., D/2] fp32 broadcastable (rotate-half)."""
    half = x.shape[-1] // 2
    x1, x2 = x[..., :half], x[..., half:]
    return torch.cat([x1 * cos - x2 * sin, x2 * cos + x1 * sin], dim=-1)


def rope_qkv_write(
    qkv: torch.Tensor,
    positions: torch.Tensor,
    slots: torch.Tensor,
    cos_sin: torch.Tensor,
    k_pool_l: torch.Tensor,
    v_pool_l: torch.Tensor,
    num_heads: int,
    num_kv_heads: int,
    head_dim: int,
    q_norm_w: Optional[torch.Tensor] = None,
    k_norm_w: Optional[torch.Tensor] = None,
    eps: float = 1e-6,
) -> torch.Tensor:
    """Split fused QKV rows, optional per-head RMSNorm (Qwen3), RoPE q and k at
    ``positions``, write k/v to the pool at ``slots``; return q [T, Hq, D]."""
    T = qkv.shape[0]
    qs, ks = num_heads * head_dim, num_kv_heads * head_dim
    q = qkv[:, :qs].float().view(T, num_heads, head_dim)
    k = qkv[:, qs : qs + ks].float().view(T, num_kv_heads, head_dim)
    v = qkv[:, qs + ks : qs + 2 * ks].view(T, num_kv_heads, head_dim)
    if q_norm_w is not None:
        q = rmsnorm(q, q_norm_w, eps).float()
        k = rmsnorm(k, k_norm_w, eps).float()
    half = head_dim // 2
    cs = cos_sin[positions.long()]
    cos, sin = cs[:, None, :half], cs[:, None, half:]
    q = apply_rope(q, cos, sin)
    k = apply_rope(k, cos, sin)
    ps = k_pool_l.shape[2]
    page = slots.long() // ps
    off = slots.long() % ps
    k_pool_l[page, :, off, :] = k.to(k_pool_l.dtype)
    v_pool_l[page, :, off, :] = v.to(v_pool_l.dtype)
    return q.to(qkv.dtype)


def gather_kv(pool_l: torch.Tensor, page_table_row: torch.Tensor, n: int) -> torch.Tensor:
    """Token-ordered [n, H, D] view of one request's KV from a paged layer pool."""
    ps = pool_l.shape[2]
    t = torch.arange(n, device=pool_l.device)
    page = page_table_row.long()[t // ps]
    return pool_l[page, :, t % ps, :]


def paged_attention(
    q: torch.Tensor,
    k_pool_l: torch.Tensor,
    v_pool_l: torch.Tensor,
    q_indptr: torch.Tensor,
    q_pos: torch.Tensor,
    page_table: torch.Tensor,
    kv_lens: torch.Tensor,
    scale: float,
) -> torch.Tensor:
    """Causal-by-position GQA attention over paged KV.

    Row r of sequence b attends to key positions ``[0, q_pos[r]]`` of b (all
    keys already written).  This one statement covers full prefill, sparse
    boundary repair (rows at arbitrary positions; reference
    ``flashinfer_sparse_repair.py:1241-1263`` explains why the mask must be
    by *global position*, not physical slot) and decode (one row at the end).
    Returns [T, Hq*D].
    """
    T, Hq, D = q.shape
    Hkv = k_pool_l.shape[1]
    g = Hq // Hkv
    out = torch.empty(T, Hq, D, dtype=torch.float32, device=q.device)
    B = q_indptr.numel() - 1
    for b in range(B):
        s, e = int(q_indptr[b]), int(q_indptr[b + 1])
        if e == s:
            continue
        n = int(kv_lens[b])
        K = gather_kv(k_pool_l, page_table[b], n).float()  # [n, Hkv, D]
        V = gather_kv(v_pool_l, page_table[b], n).float()
        qb = q[s:e].float()  # [R, Hq, D]
        K = K.repeat_interleave(g, dim=1)
        V = V.repeat_interleave(g, dim=1)
        scores = torch.einsum("rhd,nhd->hrn", qb, K) * scale
        kpos = torch.arange(n, device=q.device)
        mask = kpos[None, :] <= q_pos[s:e].long()[:, None]
        scores = scores.masked_fill(~mask[None], float("-inf"))
        p = torch.softmax(scores, dim=-1)
        out[s:e] = torch.einsum("hrn,nhd->rhd", p, V)
    return out.reshape(T, Hq * D).to(q.dtype)


def swiglu(gu: torch.Tensor) -> torch.Tensor:
    """gu [T, 2I] = [gate | up] -> silu(gate) * up, [T, I]."""
    inter = gu.shape[-1] // 2
    g, u = gu[:, :inter].float(), gu[:, inter:].float()
    return (torch.nn.functional.silu(g) * u).to(gu.dtype)


def linear(x: torch.Tensor, w: torch.Tensor, bias: Optional[torch.Tensor] = None) -> torch.Tensor:
    y = x.float() @ w.float().t()
    if bias is not None:
        y = y + bias.float()
    return y.to(x.dtype)


def remap_delta(cos_sin: torch.Tensor, local_pos: torch.Tensor, global_pos: torch.Tensor):
    """Rotation that maps RoPE(local) to RoPE(global): R(global) R(local)^-1.

    ``delta_cos = gc*lc + gs*ls``, ``delta_sin = gs*lc - gc*ls`` evaluated in
    fp32 with one rounding per product/sum (reference
    ``pic_runtime.py:6025-6057``)."""
    half = cos_sin.shape[1] // 2
    lc, ls = cos_sin[local_pos.long(), :half], cos_sin[local_pos.long(), half:]
    gc, gs = cos_sin[global_pos.long(), :half], cos_sin[global_pos.long(), half:]
    return gc * lc + gs * ls, gs * lc - gc * ls


def kv_link_rope(
    k_pool: torch.Tensor,
    v_pool: torch.Tensor,
    src_slots: torch.Tensor,
    dst_slots: torch.Tensor,
    local_pos: torch.Tensor,
    global_pos: torch.Tensor,
    cos_sin: torch.Tensor,
    skip: Optional[torch.Tensor] = None,
    src_k_pool: Optional[torch.Tensor] = None,
    src_v_pool: Optional[torch.Tensor] = None,
) -> None:
    """Gather K/V rows at ``src_slots`` (all layers), re-rotate K from
    ``local_pos`` to ``global_pos`` and scatter to ``dst_slots``.

    Rows with ``skip[i]`` true are not written (their K/V will be recomputed
    by repair).  Rows whose local and global position are equal are copied
    unchanged (the identity prefix block, reference ``pic_runtime.py:4771``).
    ``src_*_pool`` default to the destination pools (local link); a peer
    replica's pools make this the cross-replica link.
    """
    src_k_pool = k_pool if src_k_pool is None else src_k_pool
    src_v_pool = v_pool if src_v_pool is None else src_v_pool
    if skip is not None:
        keep = ~skip.bool()
        src_slots, dst_slots = src_slots[keep], dst_slots[keep]
        local_pos, global_pos = local_pos[keep], global_pos[keep]
    if src_slots.numel() == 0:
        return
    ps = k_pool.shape[3]
    sp, so = src_slots.long() // ps, src_slots.long() % ps
    dp, do = dst_slots.long() // ps, dst_slots.long() % ps
    dc, ds = remap_delta(cos_sin, local_pos, global_pos)  # [n, D/2]
    same = (local_pos == global_pos)
    for layer in range(k_pool.shape[0]):
        k = src_k_pool[layer][sp, :, so, :].float()  # [n, H, D]
        v = src_v_pool[layer][sp, :, so, :]
        half = k.shape[-1] // 2
        k1, k2 = k[..., :half], k[..., half:]
        c, s = dc[:, None, :], ds[:, None, :]
        rot = torch.cat([k1 * c - k2 * s, k2 * c + k1 * s], dim=-1)
        rot = torch.where(same[:, None, None], k, rot)
        k_pool[layer][dp, :, do, :] = rot.to(k_pool.dtype)
        v_pool[layer][dp, :, do, :] = v


def argmax(logits: torch.Tensor) -> torch.Tensor:
    return torch.argmax(logits.float(), dim=-1).to(torch.int32)
