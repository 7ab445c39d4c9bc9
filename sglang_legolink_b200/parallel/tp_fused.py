"""Tensor parallelism with the reduction fused into the kernels (no collective
library call on the prefill / Link path).

The reference reduces the row-parallel o_proj / down_proj outputs with an
NCCL all-reduce after each GEMM (reference
``patched_sglang_files/python/sglang/srt/models/qwen2.py:80-86,162-168``).
:class:`FusedTPComm` instead splits the T rows of a forward into ``world``
ranges of ``R`` rows (R a multiple of 32) and drives three kernels per layer
boundary (``csrc/tp_fused.cu``, ``csrc/gemm_tcgen05.cu``):

* :meth:`gemm_scatter` -- the row-parallel GEMM whose epilogue stores every
  output row over NVLink into its owner rank's slot buffer (one slot per
  source rank) and bumps the owner's arrival counter (reduce-scatter fused
  into the GEMM, overlapping the next tiles' MMAs);
* :meth:`reduce_norm_gather` -- on each owner: wait for the slices, sum the
  slots + residual, RMSNorm, and write the normalised rows into every rank's
  gather buffer ``G`` over NVLink (the all-gather fused into the norm);
* :meth:`gemm_from_gather` -- the next column-parallel GEMM, whose TMA
  producer waits for the gather counter and reads ``G`` from local memory.

The buffers live in symmetric memory (``torch.distributed._symmetric_memory``)
so every rank holds the others' base addresses.  The counters only grow;
this object keeps each counter's cumulative target, so every rank must run
the same sequence of fused calls (as it does the same forward).

Decode steps (up to ``MAX_DECODE_ROWS`` rows) use a fourth kernel after
each row-parallel GEMV, :meth:`decode_allreduce_norm`: the GEMV writes its
partial rows into this rank's symmetric buffer (two buffers, alternating
call by call), and the kernel sums every rank's rows over NVLink (one-shot
all-reduce), adds the residual and applies the next RMSNorm.  Its epoch lives
in device memory, so the decode CUDA graphs replay it unchanged.  Greedy
sampling over the vocab-sharded LM head is one kernel as well
(:meth:`argmax_vocab`).  Short prefills keep the NCCL path inherited from
:class:`~.tp.NcclTPComm`.
"""

from __future__ import annotations

import math

import torch
import torch.distributed as dist

from .. import ops
from .tp import NcclTPComm

# below this many (padded) rows a forward takes the NCCL path
MIN_FUSED_ROWS = 512
# decode steps with at most this many rows use the fused decode boundary
MAX_DECODE_ROWS = 64


def _round_up(x: int, m: int) -> int:
    return (x + m - 1) // m * m


class FusedTPComm(NcclTPComm):
    name = "fused"

    def __init__(self, hidden: int, max_rows: int, device, group=None):
        import torch.distributed._symmetric_memory as symm_mem

        super().__init__(group)
        W = self.size
        self.hidden = hidden
        self.r_max = _round_up(math.ceil(max_rows / W), 32)
        n = W * self.r_max * hidden
        group = group or dist.group.WORLD
        gname = group.group_name
        self.slots = symm_mem.empty((n,), dtype=torch.bfloat16, device=device)
        self.gbuf = symm_mem.empty((n,), dtype=torch.bfloat16, device=device)
        self.cnt = symm_mem.empty((2,), dtype=torch.int64, device=device)
        self.gbuf.zero_()
        self.cnt.zero_()
        self._hs = symm_mem.rendezvous(self.slots, gname)
        self._hg = symm_mem.rendezvous(self.gbuf, gname)
        self._hc = symm_mem.rendezvous(self.cnt, gname)
        self.slot_ptrs = [int(p) for p in self._hs.buffer_ptrs]
        self.g_ptrs = [int(p) for p in self._hg.buffer_ptrs]
        self.slot_cnt_ptrs = [int(p) for p in self._hc.buffer_ptrs]
        self.g_cnt_ptrs = [p + 8 for p in self.slot_cnt_ptrs]
        self.slot_target = 0
        self.g_target = 0
        # decode boundary: two partial buffers, one arrival counter per rank,
        # this rank's [epoch, ticket]
        self.dpart = symm_mem.empty((2 * MAX_DECODE_ROWS * hidden,), dtype=torch.bfloat16, device=device)
        self.dcnt = symm_mem.empty((2,), dtype=torch.int64, device=device)
        self.dcnt.zero_()
        self.depoch = torch.zeros(2, dtype=torch.int64, device=device)
        self._hdp = symm_mem.rendezvous(self.dpart, gname)
        self._hdc = symm_mem.rendezvous(self.dcnt, gname)
        self.dpart_ptrs = [int(p) for p in self._hdp.buffer_ptrs]
        self.dcnt_ptrs = [int(p) for p in self._hdc.buffer_ptrs]
        # NVLS (wherever the buffers have a multicast address, unless
        # SGLANG_PIC_TP_NVLS=0): the decode boundary sums the ranks' partial
        # rows with one multimem load through the multicast address instead
        # of one peer load per rank (TP=4, batch 16: 14.99 vs 28.96 ms/step;
        # NCCL 21.59 ms on the same box)
        import os

        mc = int(getattr(self._hdp, "multicast_ptr", 0) or 0)
        self.dpart_mc = mc if (os.getenv("SGLANG_PIC_TP_NVLS", "1") != "0" and mc) else 0
        self._dparity = 0
        # greedy over the vocab shards: per-row (max, index) records pushed
        # to every rank ([2 parities][MAX_DECODE_ROWS][8 ranks][pair, tag])
        self.arec = symm_mem.empty((2 * MAX_DECODE_ROWS * 8 * 2,), dtype=torch.int64, device=device)
        self.arec.zero_()
        self.aepoch = torch.zeros(2, dtype=torch.int64, device=device)
        self._hak = symm_mem.rendezvous(self.arec, gname)
        self.arec_ptrs = [int(p) for p in self._hak.buffer_ptrs]
        torch.cuda.synchronize(device)
        dist.barrier(group=self.group)  # every counter is zero before any peer adds to it
        self.stats = {"fused_gemms": 0, "fused_reduces": 0, "fused_decode_reduces": 0, "fused_argmax": 0,
                      "nvls_decode": bool(self.dpart_mc)}

    # ------------------------------------------------------------ geometry
    def rows_per_rank(self, T: int) -> int:
        return _round_up(math.ceil(T / self.size), 32)

    def use_fused(self, T: int) -> bool:
        R = self.rows_per_rank(T)
        return R <= self.r_max and self.size * R >= MIN_FUSED_ROWS

    def gather_view(self, T: int) -> torch.Tensor:
        R = self.rows_per_rank(T)
        return self.gbuf[: self.size * R * self.hidden].view(self.size * R, self.hidden)

    def slot_view(self, T: int) -> torch.Tensor:
        R = self.rows_per_rank(T)
        return self.slots[: self.size * R * self.hidden].view(self.size, R, self.hidden)

    def decode_fusable(self, T: int) -> bool:
        return T <= MAX_DECODE_ROWS

    def decode_part(self, T: int) -> torch.Tensor:
        """This rank's buffer for the next row-parallel GEMV's partial rows."""
        n = MAX_DECODE_ROWS * self.hidden
        return self.dpart[self._dparity * n: self._dparity * n + T * self.hidden].view(T, self.hidden)

    def decode_allreduce_norm(self, T: int, residual: torch.Tensor, w: torch.Tensor, eps: float,
                              out: torch.Tensor) -> None:
        """residual[:T] += the sum over ranks of their :meth:`decode_part`
        rows; out[:T] = RMSNorm(residual) * w.  Flips the partial buffer."""
        off = self._dparity * MAX_DECODE_ROWS * self.hidden * 2
        ops._cuda().tp_decode_allreduce_norm_nvls(residual, w, out, float(eps), T,
                                                  [p + off for p in self.dpart_ptrs], self.dcnt_ptrs, self.depoch,
                                                  self.rank, self.size, ops.workspace(residual.device).err,
                                                  self.dpart_mc + off if self.dpart_mc else 0)
        self._dparity ^= 1
        self.stats["fused_decode_reduces"] += 1

    def argmax_vocab(self, local: torch.Tensor, vocab_start: int) -> torch.Tensor:
        """Greedy token ids over vocab-sharded logits in one kernel: every
        rank pushes its rows' (max, index) to every rank over NVLink and
        picks the winner (ties: the smallest token id).  Replaces the pair
        all-gather of :class:`~.tp.NcclTPComm` for up to MAX_DECODE_ROWS rows."""
        R = local.shape[0]
        if not local.is_cuda or R > MAX_DECODE_ROWS or local.stride(-1) != 1:
            return super().argmax_vocab(local, vocab_start)
        out = torch.empty(R, dtype=torch.int32, device=local.device)
        ops._cuda().tp_argmax(local, int(vocab_start), out, self.arec_ptrs, self.aepoch, self.rank, self.size,
                              MAX_DECODE_ROWS, ops.workspace(local.device).err)
        self.stats["fused_argmax"] += 1
        return out

    # ------------------------------------------------------------- kernels
    def reduce_norm_gather(self, residual: torch.Tensor, w: torch.Tensor, eps: float, T: int,
                           with_slots: bool = True) -> None:
        """residual [R, H] (this rank's rows) += sum of slots (when
        ``with_slots``); G[rank*R:(rank+1)*R] on every rank = RMSNorm(residual)."""
        R = self.rows_per_rank(T)
        err = ops.workspace(residual.device).err
        grid = ops._cuda().tp_reduce_norm_gather(
            self.slot_view(T) if with_slots else None, residual, w, float(eps), R, self.g_ptrs, self.g_cnt_ptrs,
            self.slot_cnt_ptrs[self.rank] if with_slots else 0, self.slot_target, self.rank, self.size, R, err)
        self.g_target += self.size * int(grid)
        self.stats["fused_reduces"] += 1

    def gemm_from_gather(self, w: torch.Tensor, bias, out: torch.Tensor, T: int, swiglu: bool = False) -> None:
        """out[Tp, N] = G @ w^T (+ bias), after this rank's G is complete."""
        R = self.rows_per_rank(T)
        g = self.gather_view(T)
        ops._cuda().gemm_tp(g, w, bias, out, 1 if swiglu else 0, 0, [], [], self.g_cnt_ptrs[self.rank],
                            self.g_target, self.rank, self.size, R, ops.workspace(g.device).err)
        self.stats["fused_gemms"] += 1

    def gemm_scatter(self, a: torch.Tensor, w: torch.Tensor, T: int) -> None:
        """Partial a @ w^T of all Tp rows, each row stored into its owner's
        slot for this rank (reduce-scatter inside the GEMM epilogue)."""
        R = self.rows_per_rank(T)
        N = w.shape[0]
        ops._cuda().gemm_tp(a, w, None, None, 2, N, self.slot_ptrs, self.slot_cnt_ptrs, 0, 0, self.rank,
                            self.size, R, ops.workspace(a.device).err)
        self.slot_target += self.size * (R // 32) * ((N + 255) // 256)
        self.stats["fused_gemms"] += 1

    def wait_gather(self, device) -> None:
        """Makes the current stream wait until this rank's G is complete
        (before torch ops read it)."""
        ops._cuda().tp_wait(self.g_cnt_ptrs[self.rank], self.g_target, ops.workspace(device).err)
