"""Runtime ops.  CUDA tensors run the sm_100a kernels of ``legolink_cuda``
(missing build -> :class:`ExtensionMissing`); CPU tensors run the fp32
statements in :mod:`.reference`, which are also the test oracle.

Conventions
-----------
* Linear weights are ``[out_features, in_features]`` (nn.Linear layout).
* The fused gate/up weight is stored *interleaved in groups of 16 rows*:
  rows ``[32j, 32j+16)`` are gate rows ``[16j, 16j+16)`` and rows
  ``[32j+16, 32j+32)`` the matching up rows.  ``swiglu`` and the GEMM's
  SwiGLU epilogue both read that layout (:func:`interleave_gate_up`).
* KV pools are ``[layers, pages, kv_heads, page_size, head_dim]``.
"""

from __future__ import annotations

import math
import os
from typing import Optional

import torch

from . import reference as ref
from ._ext import ExtensionMissing, cuda as _cuda  # noqa: F401

__all__ = [
    "ExtensionMissing", "linear", "rmsnorm", "fused_add_rmsnorm", "rope_qkv_write", "attention_prefill",
    "attention_decode", "swiglu", "embedding", "argmax", "kv_link_rope", "interleave_gate_up",
    "deinterleave_gate_up", "prefill_tiles", "workspace", "check_errors", "gemv_rownorm", "gemv_residual",
    "gemv_qkv_rope",
]

SMALL_M_MAX = 128


# ----------------------------------------------------------------- workspace
class _Workspace:
    """Per-device scratch: error word, split-K partials + tickets, decode
    partials.  Sized up front by the engine; a buffer that has to grow later
    is replaced, and the old one is kept alive, because a captured CUDA graph
    may still point at it."""

    def __init__(self, device: torch.device):
        self.device = device
        self._retired: list = []
        self.err = torch.zeros(1, dtype=torch.int32, device=device)
        self.gemm_ws = torch.empty(0, dtype=torch.float32, device=device)
        self.tickets = torch.zeros(4096, dtype=torch.int32, device=device)
        self.dec_o = torch.empty(0, dtype=torch.float32, device=device)
        self.dec_ml = torch.empty(0, dtype=torch.float32, device=device)
        self.pre_o = torch.empty(0, dtype=torch.float32, device=device)
        self.pre_ml = torch.empty(0, dtype=torch.float32, device=device)

    def reserve_gemm(self, floats: int, tiles: int = 0) -> None:
        if self.gemm_ws.numel() < floats:
            self._retired.append(self.gemm_ws)
            self.gemm_ws = torch.empty(floats, dtype=torch.float32, device=self.device)
        if self.tickets.numel() < tiles:
            self._retired.append(self.tickets)
            self.tickets = torch.zeros(tiles, dtype=torch.int32, device=self.device)

    def reserve_prefill_split(self, rows: int, nsplit: int, head_dim: int = 128) -> None:
        """Partials of split prefill attention ([rows][nsplit][head_dim] fp32
        + [rows][nsplit][2]); grown, never shrunk."""
        need = rows * nsplit
        if self.pre_o.numel() < need * head_dim:
            self._retired += [self.pre_o, self.pre_ml]
            self.pre_o = torch.empty(need * head_dim, dtype=torch.float32, device=self.device)
            self.pre_ml = torch.empty(need * 2, dtype=torch.float32, device=self.device)

    def reserve_decode(self, rows: int, nsplit: int, head_dim: int = 128) -> None:
        need = rows * nsplit
        if self.dec_o.numel() < need * head_dim:
            self._retired += [self.dec_o, self.dec_ml]
            self.dec_o = torch.empty(need * head_dim, dtype=torch.float32, device=self.device)
            self.dec_ml = torch.empty(need * 2, dtype=torch.float32, device=self.device)


_WS: dict[int, _Workspace] = {}


def workspace(device) -> _Workspace:
    device = torch.device(device)
    idx = device.index if device.index is not None else torch.cuda.current_device()
    ws = _WS.get(idx)
    if ws is None:
        ws = _WS[idx] = _Workspace(torch.device("cuda", idx))
    return ws


ERROR_NAMES = {1: "TMA full-barrier wait timed out", 2: "shared-memory empty-barrier wait timed out",
               3: "TMEM full wait timed out", 4: "TMEM empty wait timed out", 5: "peer flag wait timed out",
               6: "index past its bound (slot, position or page-table entry) refused"}


def check_errors(device) -> int:
    """Read (and clear) the device error word set by bounded waits."""
    ws = workspace(device)
    code = int(ws.err.item())
    if code:
        ws.err.zero_()
    return code


# ------------------------------------------------------------------ weights
def interleave_gate_up(gate: torch.Tensor, up: torch.Tensor, group: int = 16) -> torch.Tensor:
    """[I, H] gate + [I, H] up -> [2I, H] interleaved in groups of ``group``."""
    inter, hid = gate.shape
    assert inter % group == 0, "intermediate size must be a multiple of 16"
    g = gate.reshape(inter // group, group, hid)
    u = up.reshape(inter // group, group, hid)
    return torch.stack([g, u], dim=1).reshape(2 * inter, hid).contiguous()


def deinterleave_gate_up(gu: torch.Tensor, group: int = 16):
    two_i, hid = gu.shape
    x = gu.reshape(two_i // (2 * group), 2, group, hid)
    return x[:, 0].reshape(-1, hid), x[:, 1].reshape(-1, hid)


# ---------------------------------------------------------------------- ops
def linear(x: torch.Tensor, w: torch.Tensor, bias: Optional[torch.Tensor] = None,
           out: Optional[torch.Tensor] = None, swiglu_epilogue: bool = False) -> torch.Tensor:
    """``x @ w.T (+ bias)``; with ``swiglu_epilogue`` the result is
    ``silu(gate) * up`` of the interleaved gate/up product (half width)."""
    M, N = x.shape[0], w.shape[0]
    if not x.is_cuda:
        y = ref.linear(x, w, bias)
        if swiglu_epilogue:
            y = ref_swiglu_interleaved(y)
        if out is not None:
            out.copy_(y)
            return out
        return y
    ext = _cuda()
    ws = workspace(x.device)
    if out is None:
        out = torch.empty(M, N // 2 if swiglu_epilogue else N, dtype=x.dtype, device=x.device)
    if M <= SMALL_M_MAX and not (M > 64 and N >= 148 * 256):
        _small_m(ext, ws, x, w, bias, out, swiglu_epilogue)
        return out
    bn = 256 if N >= 2048 else 128
    ext.gemm(x, w, bias, out, 1 if swiglu_epilogue else 0, bn, ws.err)
    return out


def tile_weight(w: torch.Tensor) -> torch.Tensor:
    """[N, K] -> tile-major [N/128, K/64, 128, 64]: each 128-row x 64-column
    TMA box of the small-M GEMM becomes one contiguous 16 KB block."""
    N, K = w.shape
    assert N % 128 == 0 and K % 64 == 0, "tile-major weights need N % 128 == 0 and K % 64 == 0"
    return w.reshape(N // 128, 128, K // 64, 64).permute(0, 2, 1, 3).contiguous()


def untile_weight(wt: torch.Tensor) -> torch.Tensor:
    a, b, c, d = wt.shape
    return wt.permute(0, 2, 1, 3).reshape(a * c, b * d)


def _small_m(ext, ws, x, w, bias, out, swiglu: bool = False):
    M, K = x.shape
    N = w.shape[0] * 128 if w.dim() == 4 else w.shape[0]
    ext.gemm_small_m(x, w, bias, out, _small_m_splits(ws, M, N, K), ws.gemm_ws, ws.tickets, ws.err, swiglu)


EPI_STORE, EPI_SWIGLU, EPI_RESIDUAL, EPI_QKV_ROPE = 0, 1, 2, 3


# LL_SMALL_M_MAX_SPLITS=<n> caps the split-K count of the small-M GEMM
# (a measurement knob for benchmarks/decode_breakdown.py; unset: no cap
# beyond the kernel's own).
_SMALL_M_MAX_SPLITS = int(os.environ.get("LL_SMALL_M_MAX_SPLITS", "0") or 0)


# 2..16-row GEMVs (the tile epilogue) take at most 8 splits: the fix-up loads
# four splits' partials per round.  Measured at 16 rows (2/4/8/automatic
# splits): the cap takes the qkv GEMV of a Qwen3-32B TP=8 rank from 16 splits
# and 12.7 us to 10.8 us, and Qwen2.5-7B's o_proj / down from 10 splits and
# 11.5 / 28.2 us to 10.5 / 27.4 us; 4 splits was up to 8 % faster on some
# shapes and slower on others.  LL_GEMV_TILE_MAX_SPLITS=<n> overrides the cap
# (a measurement knob).
_TILE_MAX_SPLITS = int(os.environ.get("LL_GEMV_TILE_MAX_SPLITS", "8") or 8)


def _small_m_splits(ws, M: int, N: int, K: int) -> int:
    splits = _cuda().gemm_small_m_splits(N, K)
    if 1 < M <= 16 and splits > _TILE_MAX_SPLITS:
        splits = _TILE_MAX_SPLITS
    if _SMALL_M_MAX_SPLITS > 0 and splits > _SMALL_M_MAX_SPLITS:
        splits = _SMALL_M_MAX_SPLITS
    if splits > 1:
        need = splits * M * N
        if ws.gemm_ws.numel() < need or ws.tickets.numel() < (N + 127) // 128:
            if torch.cuda.is_current_stream_capturing():
                raise RuntimeError("GEMM workspace too small during CUDA graph capture; reserve it first")
            ws.reserve_gemm(need, (N + 127) // 128)
    return splits


SUMSQ_ONE = float(1 << 24)


def sumsq_buffer(shape, device) -> torch.Tensor:
    """Zeroed row sums of squares for the decode GEMV epilogues: int64 fixed
    point (units of 2^-24) on CUDA, whose atomic accumulation does not depend
    on tile completion order; fp32 on CPU."""
    dtype = torch.int64 if torch.device(device).type == "cuda" else torch.float32
    return torch.zeros(shape, dtype=dtype, device=device)


def sumsq_values(sumsq: torch.Tensor) -> torch.Tensor:
    """fp32 values of a sums-of-squares buffer (either representation)."""
    return sumsq.double().div(SUMSQ_ONE).float() if sumsq.dtype == torch.int64 else sumsq.float()


def sumsq_from_values(vals: torch.Tensor) -> torch.Tensor:
    """The CUDA (fixed-point) representation of fp32 sums of squares."""
    return torch.round(vals.double() * SUMSQ_ONE).to(torch.int64)


def _row_rstd(sumsq: torch.Tensor, K: int, eps: float) -> torch.Tensor:
    return torch.rsqrt(sumsq_values(sumsq) / K + eps)


def gemv_rownorm(x, w, bias, sumsq, eps: float, out=None, swiglu: bool = False):
    """``(x @ w.T) * rsqrt(sumsq / K + eps)[:, None] + bias`` (SwiGLU of the
    interleaved gate/up product with ``swiglu``): the GEMV of an input whose
    RMSNorm scale is applied after the product (the producer wrote
    ``residual * norm_weight`` and the rows' sums of squares).  Decode sizes
    (M <= 128) only."""
    M, K = x.shape
    N = w.shape[0] * 128 if w.dim() == 4 else w.shape[0]
    if out is None:
        out = torch.empty(M, N // 2 if swiglu else N, dtype=x.dtype, device=x.device)
    if not x.is_cuda:
        y = x.float() @ w.float().t() * _row_rstd(sumsq[:M], K, eps)[:, None]
        if bias is not None:
            y = y + bias.float()
        out.copy_(ref_swiglu_interleaved(y) if swiglu else y)
        return out
    ws = workspace(x.device)
    _cuda().gemm_small_m_epi(x, w, bias, out, _small_m_splits(ws, M, N, K), ws.gemm_ws, ws.tickets, ws.err,
                             EPI_SWIGLU if swiglu else EPI_STORE, sumsq, eps, None, None, None, None, None, None,
                             None, None, None, None, None, None, 0, 0, 0, eps)
    return out


def gemv_residual(x, w, residual, norm_w, h_out, sumsq_out, scale_sumsq=None, eps: float = 1e-6):
    """``y = x @ w.T``; ``r = bf16(y) + residual``; ``residual = bf16(r)``;
    ``h_out = bf16(r * norm_w)``; ``sumsq_out[m] += sum(r[m]^2)`` (fp32
    ``r``) -- the residual add and the data half of the next RMSNorm, done in
    the GEMV's stores.  ``sumsq_out`` must be zero beforehand; on CUDA it is
    int64 fixed point (:func:`sumsq_buffer`)."""
    M, K = x.shape
    N = w.shape[0] * 128 if w.dim() == 4 else w.shape[0]
    if not x.is_cuda:
        y = x.float() @ w.float().t()
        if scale_sumsq is not None:
            y = y * _row_rstd(scale_sumsq[:M], K, eps)[:, None]
        r = y.to(x.dtype).float() + residual.float()
        residual.copy_(r)
        h_out.copy_(r * norm_w.float())
        sumsq_out[:M] += (r * r).sum(-1)
        return h_out
    ws = workspace(x.device)
    _cuda().gemm_small_m_epi(x, w, None, None, _small_m_splits(ws, M, N, K), ws.gemm_ws, ws.tickets, ws.err,
                             EPI_RESIDUAL, scale_sumsq, eps, residual, norm_w, h_out, sumsq_out, None, None, None,
                             None, None, None, None, None, 0, 0, 0, eps)
    return h_out


def gemv_qkv_rope(x, w, bias, positions, slots, cos_sin, q_out, k_pool_l, v_pool_l, num_heads: int,
                  num_kv_heads: int, q_norm_w=None, k_norm_w=None, eps: float = 1e-6, scale_sumsq=None):
    """The qkv GEMV with :func:`rope_qkv_write` in its stores: one 128-wide
    output tile is one head, so the tile's last CTA applies the head's
    RMSNorm (Qwen3), RoPE, and writes Q to ``q_out`` and K/V to the pool
    slot.  The qkv product is rounded to bf16 first, as when it is stored."""
    M, K = x.shape
    N = w.shape[0] * 128 if w.dim() == 4 else w.shape[0]
    if not x.is_cuda:
        y = x.float() @ w.float().t()
        if scale_sumsq is not None:
            y = y * _row_rstd(scale_sumsq[:M], K, eps)[:, None]
        if bias is not None:
            y = y + bias.float()
        return rope_qkv_write(y.to(x.dtype), positions, slots, cos_sin, q_out, k_pool_l, v_pool_l, num_heads,
                              num_kv_heads, 128, q_norm_w, k_norm_w, eps)
    ws = workspace(x.device)
    _cuda().gemm_small_m_epi(x, w, bias, None, _small_m_splits(ws, M, N, K), ws.gemm_ws, ws.tickets, ws.err,
                             EPI_QKV_ROPE, scale_sumsq, eps, None, None, None, None, positions, slots, cos_sin,
                             q_out, k_pool_l, v_pool_l, q_norm_w, k_norm_w, num_heads, num_kv_heads,
                             k_pool_l.shape[-2], eps)
    return q_out


def ref_swiglu_interleaved(gu: torch.Tensor) -> torch.Tensor:
    T, two_i = gu.shape
    x = gu.float().reshape(T, two_i // 32, 2, 16)
    y = torch.nn.functional.silu(x[:, :, 0]) * x[:, :, 1]
    return y.reshape(T, two_i // 2).to(gu.dtype)


def swiglu(gu: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    if not gu.is_cuda:
        y = ref_swiglu_interleaved(gu)
        if out is not None:
            out.copy_(y)
            return out
        return y
    if out is None:
        out = torch.empty(gu.shape[0], gu.shape[1] // 2, dtype=gu.dtype, device=gu.device)
    _cuda().swiglu(out, gu)
    return out


def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    if not x.is_cuda:
        y = ref.rmsnorm(x, w, eps)
        if out is not None:
            out.copy_(y)
            return out
        return y
    if out is None:
        out = torch.empty_like(x)
    _cuda().rmsnorm(out, x, None, w, eps)
    return out


def fused_add_rmsnorm(x: torch.Tensor, residual: torch.Tensor, w: torch.Tensor, eps: float) -> None:
    """residual += x ; x = rmsnorm(residual) * w  (in place, fp32 math)."""
    if not x.is_cuda:
        ref.fused_add_rmsnorm(x, residual, w, eps)
        return
    _cuda().rmsnorm(x, x, residual, w, eps)


def rope_qkv_write(qkv, positions, slots, cos_sin, q_out, k_pool_l, v_pool_l, num_heads, num_kv_heads,
                   head_dim, q_norm_w=None, k_norm_w=None, eps=1e-6):
    if not qkv.is_cuda:
        q = ref.rope_qkv_write(qkv, positions, slots, cos_sin, k_pool_l, v_pool_l, num_heads, num_kv_heads,
                               head_dim, q_norm_w, k_norm_w, eps)
        q_out.copy_(q)
        return q_out
    _cuda().rope_qkv_write(qkv, positions, slots, cos_sin, q_out, k_pool_l, v_pool_l, q_norm_w, k_norm_w,
                           num_heads, num_kv_heads, head_dim, eps, workspace(qkv.device).err)
    return q_out


PREFILL_ROWS_PER_TILE = 256  # packed (token, head) rows per CTA of the tcgen05 kernel (2 tiles of 128)
PREFILL_BLOCK_KEYS = 128     # keys per block step of that kernel
# Timing model of the tcgen05 prefill kernel on B200 (one CTA per SM, CTAs
# placed in list order onto the SM that frees first), fitted to the split
# sweep of benchmarks/attn_split.py (TP = 1/2/4/8 shares of the Qwen3-32B
# Link, S = 1..16): a block step of a CTA (2 x 128 rows x 128 keys) ~2.1 us,
# a CTA's start-up and epilogue ~1 block step, and a split's partials (the
# fp32 write, the combine's read: 520 B per row and split each way) at an
# effective ~2 TB/s plus one ~3 us combine launch.
_PF_BLOCK_US, _PF_ITEM_BLOCKS, _PF_COMBINE_US, _PF_BYTES_PER_US = 2.1, 1.0, 3.0, 2.0e6
PREFILL_SPLIT_CHOICES = (1, 2, 3, 4, 6, 8, 12, 16)
PREFILL_SPLIT_MAX_WS_BYTES = 256 << 20


def prefill_split_time_us(blocks, packed_rows: int, S: int, num_sms: int = 148) -> float:
    """Modelled duration (us) of one prefill attention launch whose tiles
    have ``blocks`` key blocks each, every tile split into S equal key
    ranges (S = 1: no split), including the partials' traffic and the
    combine."""
    import numpy as np

    from . import _ext

    nb = np.asarray(blocks, dtype=np.int64)
    ch = -(-nb // S)
    sizes = np.clip(nb[:, None] - ch[:, None] * np.arange(S)[None, :], 0, ch[:, None]).ravel()
    sizes = np.sort(sizes)[::-1]
    work = np.where(sizes > 0, sizes + _PF_ITEM_BLOCKS, 0.5)
    t = _ext.host().list_schedule_makespan(work, num_sms) * _PF_BLOCK_US
    if S > 1:
        t += _PF_COMBINE_US + packed_rows * (S * 520 * 2 + 256) / _PF_BYTES_PER_US
    return t


def prefill_split_count(blocks, packed_rows: int, num_sms: int = 148) -> int:
    """Key-range split count for a prefill launch whose tiles have ``blocks``
    key blocks each: the one with the smallest modelled time
    (:func:`prefill_split_time_us`), kept only when it is at least 15 %
    faster than no split (the model's error on the sweep it was fitted to is
    up to ~8 %).  Splitting pays when there are too few tiles to
    fill the SMs (few KV heads per rank under tensor parallelism, short
    repair sets over long contexts)."""
    if len(blocks) == 0 or len(blocks) >= 3 * num_sms:  # three or more waves of tiles: no split
        return 1
    base, best, best_t = prefill_split_time_us(blocks, packed_rows, 1, num_sms), 1, None
    for S in PREFILL_SPLIT_CHOICES[1:]:
        if packed_rows * S * 520 > PREFILL_SPLIT_MAX_WS_BYTES:
            break
        t = prefill_split_time_us(blocks, packed_rows, S, num_sms)
        if best_t is None or t < best_t:
            best, best_t = S, t
    return best if best_t is not None and best_t < 0.85 * base else 1


def _split_items(t, S: int):
    """Expands tiles [n, 4] (int64 numpy) into S key-range items each (kv
    head | split << 8 | S << 16 in column 1), longest item first."""
    import numpy as np

    nb = t[:, 3] // PREFILL_BLOCK_KEYS + 1
    ch = (nb + S - 1) // S
    rep = np.repeat(t, S, axis=0)
    sp = np.tile(np.arange(S, dtype=np.int64), len(t))
    size = np.clip(np.repeat(nb, S) - np.repeat(ch, S) * sp, 0, np.repeat(ch, S))
    rep[:, 1] = rep[:, 1] | (sp << 8) | (S << 16)
    order = np.argsort(-size, kind="stable")
    return rep[order]


def tiles_split_count(tiles) -> int:
    """Split count encoded in a work list built by :func:`prefill_tiles`
    (host tensor or array)."""
    if len(tiles) == 0:
        return 1
    return max(1, int(tiles[0][1]) >> 16)


def prefill_tiles(q_indptr_host: torch.Tensor, q_pos_host: torch.Tensor, num_heads: int, num_kv_heads: int,
                  rows_per_tile: int = PREFILL_ROWS_PER_TILE, split: bool | int = False) -> torch.Tensor:
    """Work list for the prefill/repair attention kernels: one int4
    ``(request, kv_head, first_packed_row, max_position_in_tile)`` per CTA,
    longest (largest max position) first.  Packed row ``r`` of a request is
    (token ``r // g``, q-head ``kv_head*g + r % g``), ``g = Hq / Hkv``.
    ``split`` (tcgen05 kernel only): each tile may become S items over equal
    key ranges, S from :func:`prefill_split_count` when ``split`` is True, or
    S = ``split`` when it is an int >= 2 (read it back with
    :func:`tiles_split_count`)."""
    import numpy as np

    return torch.from_numpy(prefill_tiles_np(q_indptr_host.cpu().numpy(), q_pos_host.cpu().numpy(), num_heads,
                                             num_kv_heads, rows_per_tile, split))


def prefill_tiles_np(q_indptr, q_pos, num_heads: int, num_kv_heads: int,
                     rows_per_tile: int = PREFILL_ROWS_PER_TILE, split: bool | int = False):
    """numpy form of :func:`prefill_tiles` (int32 [n, 4]) for the host-side
    batch build."""
    import numpy as np

    g = num_heads // num_kv_heads
    qi = np.asarray(q_indptr, dtype=np.int64)
    qp = np.asarray(q_pos, dtype=np.int64)
    out = []
    for b in range(len(qi) - 1):
        s, e = int(qi[b]), int(qi[b + 1])
        nrows = (e - s) * g
        if nrows <= 0:
            continue
        r0 = np.arange(0, nrows, rows_per_tile, dtype=np.int64)
        mp = qp[s + (np.minimum(r0 + rows_per_tile, nrows) - 1) // g]
        n = len(r0)
        t = np.empty((n * num_kv_heads, 4), dtype=np.int64)
        t[:, 0] = b
        t[:, 1] = np.tile(np.arange(num_kv_heads), n)
        t[:, 2] = np.repeat(r0, num_kv_heads)
        t[:, 3] = np.repeat(mp, num_kv_heads)
        out.append(t)
    if not out:
        return np.zeros((0, 4), dtype=np.int32)
    t = np.concatenate(out)
    order = np.argsort(-t[:, 3], kind="stable")
    t = t[order]
    if split:
        if split is True:
            S = prefill_split_count(t[:, 3] // PREFILL_BLOCK_KEYS + 1, int(qi[-1] - qi[0]) * num_heads)
        else:
            S = int(split)
            if not 1 <= S <= 255:
                raise ValueError(f"split count {S} outside [1, 255]")
        if S > 1:
            t = _split_items(t, S)
    return np.ascontiguousarray(t.astype(np.int32))


def attention_prefill(q, k_pool, v_pool, layer, q_indptr, q_pos, page_table, kv_lens, scale, tiles=None,
                      out=None, nsplit: int = 1) -> torch.Tensor:
    """q [T, Hq, D] -> [T, Hq*D]; rows attend to positions [0, q_pos] of their
    request (positions ascending within a request).  ``k_pool``/``v_pool`` are
    the whole pools; ``layer`` selects one.  CUDA: tcgen05 kernel.  With
    ``tiles`` given, ``nsplit`` is its split count (:func:`tiles_split_count`
    of the host copy); without, the work list is built here with the split
    model."""
    if not q.is_cuda:
        y = ref.paged_attention(q, k_pool[layer], v_pool[layer], q_indptr, q_pos, page_table, kv_lens, scale)
        if out is not None:
            out.copy_(y)
            return out
        return y
    T, Hq, D = q.shape
    if out is None:
        out = torch.empty(T, Hq * D, dtype=q.dtype, device=q.device)
    if tiles is None:
        host = prefill_tiles(q_indptr.cpu(), q_pos.cpu(), Hq, k_pool.shape[2], split=True)
        nsplit = tiles_split_count(host)
        tiles = host.to(q.device)
    ws = workspace(q.device)
    if nsplit > 1:
        ws.reserve_prefill_split(T * Hq, nsplit, D)
        _cuda().attn_prefill_tc(q, k_pool, v_pool, layer, q_indptr, q_pos, page_table, tiles, out, scale, ws.err,
                                nsplit, ws.pre_o, ws.pre_ml)
    else:
        _cuda().attn_prefill_tc(q, k_pool, v_pool, layer, q_indptr, q_pos, page_table, tiles, out, scale, ws.err,
                                1, None, None)
    return out


def attention_prefill_mma(q, k_pool_l, v_pool_l, q_indptr, q_pos, page_table, scale, tiles=None, out=None):
    """Same op on the legacy mma.sync tensor-core path (64-row tiles): the
    baseline the tcgen05 kernel is measured against."""
    T, Hq, D = q.shape
    if out is None:
        out = torch.empty(T, Hq * D, dtype=q.dtype, device=q.device)
    if tiles is None:
        tiles = prefill_tiles(q_indptr.cpu(), q_pos.cpu(), Hq, k_pool_l.shape[1], rows_per_tile=64).to(q.device)
    _cuda().attn_prefill(q, k_pool_l, v_pool_l, q_indptr, q_pos, page_table, tiles, out, scale)
    return out


def decode_splits(batch: int, num_kv_heads: int, max_kv_len: int, num_sms: int = 148) -> int:
    """Split count for decode attention, from a timing model of the kernel
    fitted on B200: two 4-warp CTAs fit on an SM (``2 * num_sms`` per wave);
    a CTA costs ~3 us of start-up + merge and streams at most ~80 keys/us
    (its 3-stage TMA ring), and a wave cannot beat HBM (512 B of K+V per key
    and KV head at ~6.5 TB/s); each split adds a little combine work.  The
    fastest split count under that model is taken (at least 128 keys per
    split, at most 1024 splits).  Split counts just past a wave boundary are
    what the model avoids: at batch 16 / 4 KV heads / 32K keys, 5 splits
    (320 CTAs: a second, nearly empty wave) ran 1.3x slower than 4."""
    slots = 2 * num_sms
    units = max(1, batch * num_kv_heads)
    top = int(max(1, min(math.ceil(max_kv_len / 128), 1024)))
    c0_us, keys_per_us, hbm_bytes_per_us = 3.0, 80.0, 6.5e6

    def wave(active: int, keys: int) -> float:
        return max(c0_us + keys / keys_per_us, active * keys * 512 / hbm_bytes_per_us)

    best, best_t = 1, None
    for s in range(1, top + 1):
        keys = math.ceil(math.ceil(max_kv_len / s) / 64) * 64
        full, rem = divmod(units * s, slots)
        t = full * wave(slots, keys) + (wave(rem, keys) if rem else 0.0) + 0.02 * s
        if best_t is None or t < best_t - 1e-9:
            best, best_t = s, t
    return best


def attention_decode(q, k_pool_l, v_pool_l, page_table, kv_lens, scale, nsplit=None, out=None) -> torch.Tensor:
    """One query token per request: q [B, Hq, D] -> [B, Hq*D]."""
    B, Hq, D = q.shape
    if not q.is_cuda:
        q_indptr = torch.arange(B + 1, dtype=torch.int32)
        q_pos = (kv_lens - 1).to(torch.int32)
        y = ref.paged_attention(q, k_pool_l, v_pool_l, q_indptr, q_pos, page_table, kv_lens, scale)
        if out is not None:
            out.copy_(y)
            return out
        return y
    if out is None:
        out = torch.empty(B, Hq * D, dtype=q.dtype, device=q.device)
    if nsplit is None:
        nsplit = decode_splits(B, k_pool_l.shape[1], int(kv_lens.max()))
    ws = workspace(q.device)
    if nsplit > 1:
        need = B * Hq * nsplit
        if ws.dec_o.numel() < need * D:
            if torch.cuda.is_current_stream_capturing():
                raise RuntimeError("decode workspace too small during CUDA graph capture; reserve it first")
            ws.reserve_decode(B * Hq, nsplit, D)
    _cuda().attn_decode(q, k_pool_l, v_pool_l, page_table, kv_lens, out.view(B, Hq, D), ws.dec_o, ws.dec_ml,
                        nsplit, scale, ws.err)
    return out


def embedding(ids: torch.Tensor, table: torch.Tensor, out: Optional[torch.Tensor] = None,
              vocab_start: int = 0) -> torch.Tensor:
    if not ids.is_cuda:
        local = ids.long() - vocab_start
        mine = (local >= 0) & (local < table.shape[0])
        y = table[local.clamp(0, table.shape[0] - 1)] * mine[:, None].to(table.dtype)
        if out is not None:
            out.copy_(y)
            return out
        return y
    if out is None:
        out = torch.empty(ids.numel(), table.shape[1], dtype=table.dtype, device=ids.device)
    _cuda().embedding(out, ids, table, vocab_start)
    return out


def argmax(logits: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    if not logits.is_cuda:
        y = ref.argmax(logits)
        if out is not None:
            out.copy_(y)
            return out
        return y
    if out is None:
        out = torch.empty(logits.shape[0], dtype=torch.int32, device=logits.device)
    _cuda().argmax(out, logits)
    return out


def kv_link_rope(k_pool, v_pool, src_slots, dst_slots, local_pos, global_pos, cos_sin,
                 src_k_ptr: int = 0, src_v_ptr: int = 0, src_page_size: int = 0, src_layer_stride: int = 0,
                 src_pools=None) -> None:
    """Gather + RoPE delta + scatter over all layers in one launch.
    ``src_*_ptr`` name a peer replica's pools (cross-replica link)."""
    if not k_pool.is_cuda:
        sk, sv = (src_pools if src_pools is not None else (None, None))
        ref.kv_link_rope(k_pool, v_pool, src_slots, dst_slots, local_pos, global_pos, cos_sin,
                         src_k_pool=sk, src_v_pool=sv)
        return
    _cuda().kv_link_rope(k_pool, v_pool, int(src_k_ptr), int(src_v_ptr), int(src_page_size),
                         int(src_layer_stride), src_slots, dst_slots, local_pos, global_pos, cos_sin,
                         workspace(k_pool.device).err)
