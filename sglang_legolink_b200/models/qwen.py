"""Qwen2 / Qwen2.5 / Qwen3 dense decoder on the runtime's ops.

Layer structure (reference ``patched_sglang_files/python/sglang/srt/models/
qwen2.py:63-311``): fused-add RMSNorm -> QKV GEMM (+bias on Qwen2) -> [Qwen3:
per-head q/k RMSNorm] -> RoPE + paged KV write -> attention -> o_proj ->
fused-add RMSNorm -> gate_up GEMM with SwiGLU epilogue -> down_proj.

One forward serves every batch kind through :class:`ForwardBatch`:

* ``extend``  -- query rows at arbitrary positions of each request (a Compile
  prefill from position 0, the sparse repair rows of a Link, a plain prefill);
  every row's K/V is written before attention, and attention is causal by
  position over the request's paged KV.
* ``decode``  -- one row per request at position ``kv_len - 1``.

Tensor parallelism (``tp_size > 1``) shards heads / intermediate features
column-wise and reduces after o_proj / down_proj through ``self.comm`` (see
:mod:`sglang_legolink_b200.parallel`).
"""

from __future__ import annotations

import json
import math
import os
from dataclasses import dataclass, field
from typing import Optional

import torch

from .. import ops
from ..ops import reference as ref
from .config import ModelConfig


@dataclass
class ForwardBatch:
    mode: str  # "extend" | "decode"
    input_ids: torch.Tensor  # [T] int32
    positions: torch.Tensor  # [T] int32
    slots: torch.Tensor  # [T] int64   KV write slot of each row
    q_indptr: torch.Tensor  # [B+1] int32  rows of request b: [q_indptr[b], q_indptr[b+1])
    page_table: torch.Tensor  # [B, max_pages] int32
    kv_lens: torch.Tensor  # [B] int32   keys visible to request b after this step's writes
    logit_rows: Optional[torch.Tensor] = None  # [R] int64 rows whose logits are returned
    tiles: Optional[torch.Tensor] = None  # prefill attention work list
    tiles_nsplit: int = 1  # its key-range split count (ops.tiles_split_count)
    decode_nsplit: Optional[int] = None
    # grouped execution rows of one extend forward (row-wise repair compute):
    # {"batch_execution_unit_size": n, "repair_ranges": [{"start", "end"}], ...}
    repair_meta: Optional[dict] = None

    @property
    def num_rows(self) -> int:
        return int(self.input_ids.shape[0])


class LayerWeights:
    __slots__ = ("in_norm", "qkv_w", "qkv_b", "q_norm", "k_norm", "o_w", "post_norm", "gu_w", "down_w")


class QwenModel:
    def __init__(self, cfg: ModelConfig, device="cpu", dtype=torch.float32, tp_rank: int = 0, tp_size: int = 1,
                 comm=None):
        self.cfg = cfg
        self.device = torch.device(device)
        self.dtype = dtype
        self.tp_rank, self.tp_size = tp_rank, tp_size
        self.comm = comm
        self.capture = None  # optional RepairStateCapture (diagnostics; extend forwards only)
        from ..utils.layer_markers import LayerMarkers

        self.markers = LayerMarkers.from_env()  # profiler regions (off unless enabled)
        assert cfg.num_heads % tp_size == 0, "num_heads must divide by tp_size"
        self.hq = cfg.num_heads // tp_size
        # KV heads are split when possible, else replicated (each rank keeps one).
        self.hkv = max(1, cfg.num_kv_heads // tp_size)
        assert cfg.intermediate_size % (16 * tp_size) == 0
        self.inter = cfg.intermediate_size // tp_size
        self.layers: list[LayerWeights] = []
        self.embed: Optional[torch.Tensor] = None
        self.final_norm: Optional[torch.Tensor] = None
        self.lm_head: Optional[torch.Tensor] = None
        self.cos_sin: Optional[torch.Tensor] = None
        self.scale = 1.0 / math.sqrt(cfg.head_dim)
        self._bufs: dict = {}
        self.buf_generation = 0  # bumped whenever a scratch buffer is replaced by a larger one

    # ------------------------------------------------------------ weights
    def _kv_head_range(self) -> tuple[int, int]:
        c = self.cfg
        if c.num_kv_heads >= self.tp_size:
            return self.tp_rank * self.hkv, (self.tp_rank + 1) * self.hkv
        rep = self.tp_size // c.num_kv_heads
        h = self.tp_rank // rep
        return h, h + 1

    def shard_qkv(self, wq, wk, wv, bq=None, bk=None, bv=None):
        c, r, D = self.cfg, self.tp_rank, self.cfg.head_dim
        q0 = r * self.hq * D
        k0, k1 = self._kv_head_range()
        w = torch.cat([wq[q0 : q0 + self.hq * D], wk[k0 * D : k1 * D], wv[k0 * D : k1 * D]], 0)
        b = None
        if bq is not None:
            b = torch.cat([bq[q0 : q0 + self.hq * D], bk[k0 * D : k1 * D], bv[k0 * D : k1 * D]], 0)
        return w, b

    def _place(self, t: torch.Tensor) -> torch.Tensor:
        return t.to(device=self.device, dtype=self.dtype).contiguous()

    def set_weights(self, get) -> None:
        """``get(name)`` returns the full (unsharded) HF tensor for ``name``."""
        c, D, r = self.cfg, self.cfg.head_dim, self.tp_rank
        self.layers = []
        for i in range(c.num_layers):
            p = f"model.layers.{i}."
            lw = LayerWeights()
            lw.in_norm = self._place(get(p + "input_layernorm.weight"))
            lw.post_norm = self._place(get(p + "post_attention_layernorm.weight"))
            bq = bk = bv = None
            if c.qkv_bias:
                bq, bk, bv = (get(p + f"self_attn.{n}_proj.bias") for n in "qkv")
            w, b = self.shard_qkv(get(p + "self_attn.q_proj.weight"), get(p + "self_attn.k_proj.weight"),
                                  get(p + "self_attn.v_proj.weight"), bq, bk, bv)
            lw.qkv_w = self._place(w)
            lw.qkv_b = self._place(b) if b is not None else None
            if c.qk_norm:
                lw.q_norm = self._place(get(p + "self_attn.q_norm.weight"))
                lw.k_norm = self._place(get(p + "self_attn.k_norm.weight"))
            else:
                lw.q_norm = lw.k_norm = None
            o = get(p + "self_attn.o_proj.weight")
            lw.o_w = self._place(o[:, r * self.hq * D : (r + 1) * self.hq * D])
            gate = get(p + "mlp.gate_proj.weight")[r * self.inter : (r + 1) * self.inter]
            up = get(p + "mlp.up_proj.weight")[r * self.inter : (r + 1) * self.inter]
            lw.gu_w = self._place(ops.interleave_gate_up(gate, up))
            lw.down_w = self._place(get(p + "mlp.down_proj.weight")[:, r * self.inter : (r + 1) * self.inter])
            self.layers.append(lw)
        emb = get("model.embed_tokens.weight")
        self.embed = self._place(emb)
        self.final_norm = self._place(get("model.norm.weight"))
        head = emb if c.tie_word_embeddings else get("lm_head.weight")
        v0, v1 = self.vocab_range()
        self.lm_head = self._place(head[v0:v1])
        self.cos_sin = ref.rope_cos_sin_table(c.max_position_embeddings, c.rotary_dim, c.rope_theta).to(self.device)

    def ensure_rope_positions(self, n: int) -> None:
        """Makes the RoPE table cover positions [0, n) (it starts at
        ``max_position_embeddings`` rows).  Called by the engine at
        construction, before any CUDA graph captures the table's address.
        Reference: the cos/sin cache extended on demand, ``pic_runtime.py:5051-5053``."""
        if self.cos_sin is not None and self.cos_sin.shape[0] >= n:
            return
        c = self.cfg
        rows = max(n, c.max_position_embeddings)
        rows = (rows + 4095) // 4096 * 4096
        self.cos_sin = ref.rope_cos_sin_table(rows, c.rotary_dim, c.rope_theta).to(self.device)

    def vocab_range(self) -> tuple[int, int]:
        v = self.cfg.vocab_size
        per = (v + self.tp_size - 1) // self.tp_size
        return self.tp_rank * per, min(v, (self.tp_rank + 1) * per)

    @staticmethod
    def random_hf_state(cfg: ModelConfig, seed: int = 0, dtype=torch.float32, device="cpu", std: float = 0.02):
        """Random-init weights under HF Qwen names (generated on ``device``)."""
        g = torch.Generator(device=device)
        g.manual_seed(seed)
        D, H = cfg.head_dim, cfg.hidden_size

        def rnd(*shape, s=std):
            return (torch.randn(*shape, generator=g, device=device, dtype=torch.float32) * s).to(dtype)

        def ones(n):
            return (1.0 + 0.1 * torch.randn(n, generator=g, device=device, dtype=torch.float32)).to(dtype)

        st = {}
        for i in range(cfg.num_layers):
            p = f"model.layers.{i}."
            st[p + "input_layernorm.weight"] = ones(H)
            st[p + "post_attention_layernorm.weight"] = ones(H)
            st[p + "self_attn.q_proj.weight"] = rnd(cfg.num_heads * D, H)
            st[p + "self_attn.k_proj.weight"] = rnd(cfg.num_kv_heads * D, H)
            st[p + "self_attn.v_proj.weight"] = rnd(cfg.num_kv_heads * D, H)
            if cfg.qkv_bias:
                st[p + "self_attn.q_proj.bias"] = rnd(cfg.num_heads * D, s=0.1)
                st[p + "self_attn.k_proj.bias"] = rnd(cfg.num_kv_heads * D, s=0.1)
                st[p + "self_attn.v_proj.bias"] = rnd(cfg.num_kv_heads * D, s=0.1)
            if cfg.qk_norm:
                st[p + "self_attn.q_norm.weight"] = ones(D)
                st[p + "self_attn.k_norm.weight"] = ones(D)
            st[p + "self_attn.o_proj.weight"] = rnd(H, cfg.num_heads * D)
            st[p + "mlp.gate_proj.weight"] = rnd(cfg.intermediate_size, H)
            st[p + "mlp.up_proj.weight"] = rnd(cfg.intermediate_size, H)
            st[p + "mlp.down_proj.weight"] = rnd(H, cfg.intermediate_size)
        st["model.embed_tokens.weight"] = rnd(cfg.vocab_size, H, s=1.0)
        st["model.norm.weight"] = ones(H)
        if not cfg.tie_word_embeddings:
            st["lm_head.weight"] = rnd(cfg.vocab_size, H)
        return st

    @classmethod
    def random_init(cls, cfg: ModelConfig, seed=0, device="cpu", dtype=torch.float32, tp_rank=0, tp_size=1,
                    comm=None) -> "QwenModel":
        m = cls(cfg, device, dtype, tp_rank, tp_size, comm)
        # Generate per tensor on the target device to keep host memory small.
        gen_dev = device if torch.device(device).type == "cuda" else "cpu"
        state = cls.random_hf_state(cfg, seed, dtype=dtype, device=gen_dev)
        m.set_weights(lambda n: state[n])
        del state
        return m

    @classmethod
    def from_pretrained(cls, path: str, device="cpu", dtype=torch.bfloat16, tp_rank=0, tp_size=1,
                        comm=None) -> "QwenModel":
        cfg = ModelConfig.from_pretrained(path)
        m = cls(cfg, device, dtype, tp_rank, tp_size, comm)
        m.set_weights(SafetensorsReader(path))
        return m

    def save_pretrained(self, path: str, state: dict) -> None:
        save_safetensors_checkpoint(path, self.cfg, state)

    # -------------------------------------------------------------- buffers
    def _buf(self, name, shape, dtype=None):
        dtype = dtype or self.dtype
        b = self._bufs.get(name)
        n = 1
        for s in shape:
            n *= s
        if b is None or b.numel() < n or b.dtype != dtype:
            if b is not None:
                # the old memory is freed: captured decode graphs that point
                # into it must be dropped before they replay (Engine._graph)
                self.buf_generation += 1
            b = torch.empty(max(n, 1), dtype=dtype, device=self.device)
            self._bufs[name] = b
        return b[:n].view(*shape)

    # -------------------------------------------------------------- forward
    def forward(self, fb: ForwardBatch, kv, return_hidden: bool = False) -> torch.Tensor:
        """Runs all layers over ``fb``; returns logits [R, vocab(shard)] for
        ``fb.logit_rows`` (all rows when None)."""
        c = self.cfg
        T = fb.num_rows
        if (fb.mode == "extend" and getattr(self.comm, "name", "") == "fused" and fb.input_ids.is_cuda
                and self.comm.use_fused(T)):
            return self._forward_fused_tp(fb, kv, return_hidden)
        if fb.mode == "decode" and not return_hidden and self._decode_fusable(T):
            return self._forward_decode_fused(fb, kv)
        if (fb.mode == "decode" and not return_hidden and getattr(self.comm, "name", "") == "fused"
                and fb.input_ids.is_cuda and self.comm.decode_fusable(T)):
            return self._forward_decode_tp(fb, kv)
        H, D = c.hidden_size, c.head_dim
        qkv_n = (self.hq + 2 * self.hkv) * D
        x = ops.embedding(fb.input_ids, self.embed, out=self._buf("x", (T, H)))
        residual = self._buf("res", (T, H))
        residual.copy_(x)
        h = self._buf("h", (T, H))
        ops.rmsnorm(residual, self.layers[0].in_norm, c.rms_norm_eps, out=h)
        q = self._buf("q", (T, self.hq, D))
        attn = self._buf("attn", (T, self.hq * D))
        qkv = self._buf("qkv", (T, qkv_n))
        mlp = self._buf("mlp", (T, self.inter))
        o = self._buf("o", (T, H))
        tiles, tiles_nsplit = fb.tiles, fb.tiles_nsplit
        if fb.mode == "extend" and tiles is None and fb.input_ids.is_cuda:
            tiles, tiles_nsplit = self._attn_tiles(fb)
        rw_o = rw_ffn = ()
        if fb.mode == "extend" and fb.repair_meta is not None:
            from ..runtime.repair_diagnostics import rowwise_slices

            rw_o = rowwise_slices(fb.repair_meta, T, "output_projection")
            rw_ffn = rowwise_slices(fb.repair_meta, T, "ffn")
        cap = self.capture if fb.mode == "extend" else None
        mk = self.markers
        cmp_attn = False
        if fb.mode == "extend":
            from ..runtime.repair_diagnostics import compare_enabled

            cmp_attn = compare_enabled("attention")
        for li, lw in enumerate(self.layers):
            if li > 0:
                ops.fused_add_rmsnorm(h, residual, lw.in_norm, c.rms_norm_eps)
            if cap is not None and cap.wants(li):
                cap.on_component(li, "pre_attention_norm", hidden=h, residual=residual)
            ops.linear(h, lw.qkv_w, lw.qkv_b, out=qkv)
            ops.rope_qkv_write(qkv, fb.positions, fb.slots, self.cos_sin, q, kv.k[li], kv.v[li], self.hq, self.hkv,
                               D, lw.q_norm, lw.k_norm, c.rms_norm_eps)
            if cap is not None and cap.wants(li):
                cap.on_component(li, "qkv_projection", qkv=qkv)
                cap.on_component(li, "rope", q=q)
            with mk.region("Attention", li, q=q):
                if fb.mode == "decode":
                    ops.attention_decode(q, kv.k[li], kv.v[li], fb.page_table, fb.kv_lens, self.scale,
                                         nsplit=fb.decode_nsplit, out=attn)
                else:
                    ops.attention_prefill(q, kv.k, kv.v, li, fb.q_indptr, fb.positions, fb.page_table, fb.kv_lens,
                                          self.scale, tiles=tiles, out=attn, nsplit=tiles_nsplit)
                    if cmp_attn:  # diagnostic: native kernel vs the fp32 torch statement, sampled rows
                        from ..runtime.repair_diagnostics import compare_attention
                        from ..utils.trace import emit_trace

                        row = compare_attention(li, q, attn, kv.k[li], kv.v[li], fb.q_indptr, fb.positions,
                                                fb.page_table, fb.kv_lens, self.scale)
                        if fb.repair_meta is not None:
                            fb.repair_meta.setdefault("native_operator_comparisons", []).append(row)
                        emit_trace("repair_attention_compare", **row)
            # row-wise: each grouped row with the shapes it has alone
            for sl in rw_o or (slice(None),):
                self._row_parallel(attn[sl], lw.o_w, o[sl])
            if cap is not None and cap.wants(li):
                cap.on_component(li, "attention", attention_output=attn)
                cap.on_component(li, "output_projection", projected_output=o)
            ops.fused_add_rmsnorm(o, residual, lw.post_norm, c.rms_norm_eps)
            if cap is not None and cap.wants(li):
                cap.on_component(li, "post_attention_norm", hidden=o, residual=residual)
            with mk.region("FFN", li, hidden=o):
                for sl in rw_ffn or (slice(None),):
                    ops.linear(o[sl], lw.gu_w, out=mlp[sl], swiglu_epilogue=True)
                    self._row_parallel(mlp[sl], lw.down_w, h[sl])
            if cap is not None:
                if cap.wants(li):
                    cap.on_component(li, "mlp", mlp_output=h)
                cap.on_layer(li, hidden=h, residual=residual)
        # final: residual += h ; h = norm(residual)
        ops.fused_add_rmsnorm(h, residual, self.final_norm, c.rms_norm_eps)
        rows = h if fb.logit_rows is None else h.index_select(0, fb.logit_rows)
        if return_hidden:
            return rows
        return self.logits(rows)

    def _forward_decode_tp(self, fb: ForwardBatch, kv) -> torch.Tensor:
        """TP decode step whose row-parallel reductions are fused kernels:
        each o_proj / down GEMV writes its partial rows into this rank's
        symmetric buffer, and one kernel per boundary sums every rank's rows
        over NVLink, adds the residual and applies the next RMSNorm (the
        reference's NCCL all-reduce + fused add-norm, ``models/qwen2.py:80-86,
        162-168``)."""
        c, comm, mk = self.cfg, self.comm, self.markers
        T = fb.num_rows
        H, D, eps = c.hidden_size, c.head_dim, c.rms_norm_eps
        x = ops.embedding(fb.input_ids, self.embed, out=self._buf("x", (T, H)))
        residual = self._buf("res", (T, H))
        residual.copy_(x)
        h = self._buf("h", (T, H))
        ops.rmsnorm(residual, self.layers[0].in_norm, eps, out=h)
        q = self._buf("q", (T, self.hq, D))
        attn = self._buf("attn", (T, self.hq * D))
        qkv = self._buf("qkv", (T, (self.hq + 2 * self.hkv) * D))
        mlp = self._buf("mlp", (T, self.inter))
        o = self._buf("o", (T, H))
        n = len(self.layers)
        # the qkv GEMV writes Q and this step's K/V with QK-norm and RoPE in
        # its stores (one launch instead of GEMV + rope_qkv_write)
        qkv_fused = T <= ops.SMALL_M_MAX and D == 128 and c.rotary_dim == 128
        for li, lw in enumerate(self.layers):
            if qkv_fused:
                ops.gemv_qkv_rope(h, lw.qkv_w, lw.qkv_b, fb.positions, fb.slots, self.cos_sin, q, kv.k[li],
                                  kv.v[li], self.hq, self.hkv, lw.q_norm, lw.k_norm, eps)
            else:
                ops.linear(h, lw.qkv_w, lw.qkv_b, out=qkv)
                ops.rope_qkv_write(qkv, fb.positions, fb.slots, self.cos_sin, q, kv.k[li], kv.v[li], self.hq,
                                   self.hkv, D, lw.q_norm, lw.k_norm, eps)
            with mk.region("Attention", li, q=q):
                ops.attention_decode(q, kv.k[li], kv.v[li], fb.page_table, fb.kv_lens, self.scale,
                                     nsplit=fb.decode_nsplit, out=attn)
            ops.linear(attn, lw.o_w, out=comm.decode_part(T))
            comm.decode_allreduce_norm(T, residual, lw.post_norm, eps, o)
            with mk.region("FFN", li, hidden=o):
                ops.linear(o, lw.gu_w, out=mlp, swiglu_epilogue=True)
                ops.linear(mlp, lw.down_w, out=comm.decode_part(T))
                nxt = self.layers[li + 1].in_norm if li + 1 < n else self.final_norm
                comm.decode_allreduce_norm(T, residual, nxt, eps, h)
        rows = h if fb.logit_rows is None else h.index_select(0, fb.logit_rows)
        return self.logits(rows)

    def _decode_fusable(self, T: int) -> bool:
        return (self.embed.is_cuda and (self.tp_size == 1 or self.comm is None) and T <= ops.SMALL_M_MAX
                and self.cfg.head_dim == 128 and self.cfg.rotary_dim == 128 and self.cfg.hidden_size % 32 == 0)

    def _attn_tiles(self, fb: ForwardBatch):
        """Prefill attention work list (with its key-range split count) for a
        batch built without one."""
        host = ops.prefill_tiles(fb.q_indptr.cpu(), fb.positions.cpu(), self.hq, self.hkv, split=True)
        return host.to(self.device), ops.tiles_split_count(host)

    def _forward_decode_fused(self, fb: ForwardBatch, kv) -> torch.Tensor:
        """Decode step as five kernels per layer: the qkv GEMV writes Q and
        the new K/V (per-head norm and RoPE in its stores), attention, and
        three GEMVs whose stores add the residual and produce the next
        RMSNorm's input ``residual * norm_weight`` with the rows' sums of
        squares; the GEMV that reads it applies the ``rsqrt`` row scale.
        Same math as :meth:`forward` with the norm's scale moved after the
        product (reference layer order:
        patched_sglang_files/python/sglang/srt/models/qwen2.py:170-200)."""
        c = self.cfg
        T = fb.num_rows
        H, D, L = c.hidden_size, c.head_dim, len(self.layers)
        eps = c.rms_norm_eps
        x = ops.embedding(fb.input_ids, self.embed, out=self._buf("x", (T, H)))
        residual = self._buf("res", (T, H))
        residual.copy_(x)
        h = self._buf("h", (T, H))
        ops.rmsnorm(residual, self.layers[0].in_norm, eps, out=h)
        hp = self._buf("hp", (T, H))
        q = self._buf("q", (T, self.hq, D))
        attn = self._buf("attn", (T, self.hq * D))
        mlp = self._buf("mlp", (T, self.inter))
        ss = self._buf("rowsq", (2 * L, T), torch.int64)  # fixed-point sums of squares
        ss.zero_()
        for li, lw in enumerate(self.layers):
            ops.gemv_qkv_rope(h, lw.qkv_w, lw.qkv_b, fb.positions, fb.slots, self.cos_sin, q, kv.k[li], kv.v[li],
                              self.hq, self.hkv, lw.q_norm, lw.k_norm, eps,
                              scale_sumsq=ss[2 * li - 1] if li > 0 else None)
            ops.attention_decode(q, kv.k[li], kv.v[li], fb.page_table, fb.kv_lens, self.scale,
                                 nsplit=fb.decode_nsplit, out=attn)
            ops.gemv_residual(attn, lw.o_w, residual, lw.post_norm, hp, ss[2 * li], eps=eps)
            ops.gemv_rownorm(hp, lw.gu_w, None, ss[2 * li], eps, out=mlp, swiglu=True)
            nxt = self.layers[li + 1].in_norm if li + 1 < L else self.final_norm
            ops.gemv_residual(mlp, lw.down_w, residual, nxt, h, ss[2 * li + 1], eps=eps)
        rows, sq = h, ss[2 * L - 1]
        if fb.logit_rows is not None:
            rows, sq = h.index_select(0, fb.logit_rows), sq.index_select(0, fb.logit_rows)
        with self.markers.region("LMHead", hidden=rows):
            return ops.gemv_rownorm(rows, self.lm_head, None, sq, eps)

    def _forward_fused_tp(self, fb: ForwardBatch, kv, return_hidden: bool = False) -> torch.Tensor:
        """Extend forward with the TP reductions fused into the kernels
        (:class:`~sglang_legolink_b200.parallel.tp_fused.FusedTPComm`): this
        rank keeps the residual of its R rows only; every layer boundary is
        GEMM-with-scatter -> reduce+norm+all-gather -> GEMM-from-gather."""
        c, comm = self.cfg, self.comm
        T = fb.num_rows
        H, D = c.hidden_size, c.head_dim
        W, rank = comm.size, comm.rank
        R = comm.rows_per_rank(T)
        Tp = W * R
        qkv_n = (self.hq + 2 * self.hkv) * D
        r0 = rank * R
        nv = max(0, min(R, T - r0))
        ids = self._buf("tp_ids", (R,), torch.int32)
        ids.zero_()
        if nv:
            ids[:nv].copy_(fb.input_ids[r0 : r0 + nv])
        res = ops.embedding(ids, self.embed, out=self._buf("tp_res", (R, H)))
        comm.reduce_norm_gather(res, self.layers[0].in_norm, c.rms_norm_eps, T, with_slots=False)
        q = self._buf("q", (T, self.hq, D))
        attn = self._buf("tp_attn", (Tp, self.hq * D))
        if Tp > T:
            attn[T:].zero_()
        qkv = self._buf("tp_qkv", (Tp, qkv_n))
        mlp = self._buf("tp_mlp", (Tp, self.inter))
        tiles, tiles_nsplit = fb.tiles, fb.tiles_nsplit
        if tiles is None:
            tiles, tiles_nsplit = self._attn_tiles(fb)
        nl = len(self.layers)
        for li, lw in enumerate(self.layers):
            comm.gemm_from_gather(lw.qkv_w, lw.qkv_b, qkv, T)
            ops.rope_qkv_write(qkv[:T], fb.positions, fb.slots, self.cos_sin, q, kv.k[li], kv.v[li], self.hq,
                               self.hkv, D, lw.q_norm, lw.k_norm, c.rms_norm_eps)
            ops.attention_prefill(q, kv.k, kv.v, li, fb.q_indptr, fb.positions, fb.page_table, fb.kv_lens,
                                  self.scale, tiles=tiles, out=attn[:T], nsplit=tiles_nsplit)
            comm.gemm_scatter(attn, lw.o_w, T)
            comm.reduce_norm_gather(res, lw.post_norm, c.rms_norm_eps, T)
            comm.gemm_from_gather(lw.gu_w, None, mlp, T, swiglu=True)
            comm.gemm_scatter(mlp, lw.down_w, T)
            nxt = self.layers[li + 1].in_norm if li + 1 < nl else self.final_norm
            comm.reduce_norm_gather(res, nxt, c.rms_norm_eps, T)
        comm.wait_gather(self.device)
        g = comm.gather_view(T)[:T]
        rows = g if fb.logit_rows is None else g.index_select(0, fb.logit_rows)
        if return_hidden:
            return rows
        return self.logits(rows)

    def _row_parallel(self, x: torch.Tensor, w: torch.Tensor, out: torch.Tensor) -> None:
        if self.tp_size == 1 or self.comm is None:
            ops.linear(x, w, out=out)
        else:
            self.comm.gemm_allreduce(x, w, out)

    def logits(self, hidden: torch.Tensor) -> torch.Tensor:
        """Logits of this rank's vocab shard (the full vocab when tp_size == 1)."""
        with self.markers.region("LMHead", hidden=hidden):
            return ops.linear(hidden, self.lm_head)

    def full_logits(self, local: torch.Tensor) -> torch.Tensor:
        if self.tp_size > 1 and self.comm is not None:
            return self.comm.all_gather_vocab(local, self.cfg.vocab_size)
        return local

    def greedy(self, local_logits: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Greedy token ids [R] int32 from (vocab-sharded) logits."""
        if self.tp_size > 1 and self.comm is not None:
            ids = self.comm.argmax_vocab(local_logits, self.vocab_range()[0])
            if out is not None:
                out.copy_(ids)
                return out
            return ids
        return ops.argmax(local_logits, out=out)


# ------------------------------------------------------------ safetensors IO
class SafetensorsReader:
    """Lazy name -> tensor reader over an HF checkpoint directory."""

    def __init__(self, path: str):
        from safetensors import safe_open

        self.path = path
        idx = os.path.join(path, "model.safetensors.index.json")
        if os.path.exists(idx):
            with open(idx, encoding="utf-8") as f:
                wm = json.load(f)["weight_map"]
            files = sorted(set(wm.values()))
        else:
            files = [f for f in os.listdir(path) if f.endswith(".safetensors")]
            wm = None
        self._handles = {f: safe_open(os.path.join(path, f), framework="pt") for f in files}
        self._where = {}
        for f, h in self._handles.items():
            for k in h.keys():
                self._where[k] = f

    def __call__(self, name: str) -> torch.Tensor:
        if name not in self._where:
            raise KeyError(f"checkpoint has no tensor '{name}'")
        return self._handles[self._where[name]].get_tensor(name)

    def keys(self):
        return list(self._where)


def save_safetensors_checkpoint(path: str, cfg: ModelConfig, state: dict, shard_bytes: int = 4 << 30) -> None:
    """Writes an HF-layout checkpoint (config.json + sharded safetensors + index)."""
    from safetensors.torch import save_file

    os.makedirs(path, exist_ok=True)
    with open(os.path.join(path, "config.json"), "w", encoding="utf-8") as f:
        json.dump(cfg.to_hf_dict(), f, indent=1)
    shards, cur, size = [], {}, 0
    for k in sorted(state):
        t = state[k].contiguous().cpu()
        if cur and size + t.numel() * t.element_size() > shard_bytes:
            shards.append(cur)
            cur, size = {}, 0
        cur[k] = t
        size += t.numel() * t.element_size()
    if cur:
        shards.append(cur)
    wm = {}
    for i, sh in enumerate(shards):
        name = f"model-{i + 1:05d}-of-{len(shards):05d}.safetensors"
        save_file(sh, os.path.join(path, name), metadata={"format": "pt"})
        for k in sh:
            wm[k] = name
    with open(os.path.join(path, "model.safetensors.index.json"), "w", encoding="utf-8") as f:
        json.dump({"metadata": {}, "weight_map": wm}, f, indent=1)
