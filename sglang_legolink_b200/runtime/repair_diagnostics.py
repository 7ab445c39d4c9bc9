"""Row-wise repair compute and opt-in repair diagnostics.

* :func:`rowwise_slices` -- when one extend forward carries several grouped
  execution rows (the Compiles of one scheduler batch; ``repair_ranges`` give
  each row's flattened token range), the output projection and/or the FFN
  can be applied row by row, each call with the shapes the row would have
  alone, so a row's numerics do not depend on what it was batched with.
  Enabled per forward (``rowwise_ffn_enabled`` /
  ``rowwise_output_projection_enabled``) or by
  ``SGLANG_PIC_SPARSE_REPAIR_ROWWISE_FFN`` /
  ``SGLANG_PIC_SPARSE_REPAIR_ROWWISE_OUTPUT_PROJECTION``; the observed row
  count and lengths are written back into the metadata.
* :class:`RepairStateCapture` -- diagnostic capture for equivalence gates:
  every layer's output, the components of selected layers
  (``SGLANG_PIC_SPARSE_REPAIR_CAPTURE_COMPONENT_LAYERS``), the repaired K/V
  of the repair rows and the logits, saved once to
  ``<dir>/sparse_repair_state.pt``.  It copies to the host on every call, so
  it is never on a measured path.
* :class:`RepairRowView` -- immutable identity of one contiguous repair row
  (request, destination slots, positions, a digest of the slots).

Reference: ``patched_sglang_files/python/sglang/srt/sparse_repair_compute.py``
(row slices ``:25-114``, ``SparseRepairStateCapture`` ``:125-332``,
``UnifiedSparseRepairMetadataView`` ``:336-383``).
"""

from __future__ import annotations

import hashlib
import os
from dataclasses import dataclass
from pathlib import Path
from typing import Optional, Sequence

import torch


class SparseRepairComputeError(RuntimeError):
    pass


_ROWWISE = {
    "ffn": ("rowwise_ffn_enabled", "SGLANG_PIC_SPARSE_REPAIR_ROWWISE_FFN", "FFN"),
    "output_projection": ("rowwise_output_projection_enabled", "SGLANG_PIC_SPARSE_REPAIR_ROWWISE_OUTPUT_PROJECTION",
                          "output projection"),
}


def _flag(name: str) -> bool:
    return os.getenv(name, "0").strip().lower() in {"1", "true", "yes", "on"}


def rowwise_slices(meta: Optional[dict], token_count: int, which: str) -> tuple[slice, ...]:
    """Flattened token slices, one per grouped execution row, for a
    row-by-row ``which`` ("ffn" or "output_projection"); () when disabled or
    when the forward holds a single row."""
    if not isinstance(meta, dict):
        return ()
    override_key, env, label = _ROWWISE[which]
    override = meta.get(override_key)
    if override is not None and not isinstance(override, bool):
        raise SparseRepairComputeError(f"row-wise {label} override must be boolean")
    if not (override if override is not None else _flag(env)):
        return ()
    units = int(meta.get("batch_execution_unit_size", 1))
    if units <= 1:
        return ()
    ranges = meta.get("repair_ranges")
    if not isinstance(ranges, list) or len(ranges) != units:
        raise SparseRepairComputeError(f"row-wise {label} requires one repair range per grouped execution row")
    lengths = []
    for r in ranges:
        if not isinstance(r, dict):
            raise SparseRepairComputeError(f"row-wise {label} repair ranges must use start/end mappings")
        a, b = int(r.get("start", -1)), int(r.get("end", -1))
        if a < 0 or b <= a:
            raise SparseRepairComputeError(f"row-wise {label} received an invalid range")
        lengths.append(b - a)
    if sum(lengths) != int(token_count):
        raise SparseRepairComputeError(f"row-wise {label} ranges do not match the flattened token count")
    prefix = "rowwise_" + which
    meta[prefix + "_observed"] = True
    meta[prefix + "_row_count"] = len(lengths)
    meta[prefix + "_lengths"] = list(lengths)
    out, o = [], 0
    for n in lengths:
        out.append(slice(o, o + n))
        o += n
    return tuple(out)


@dataclass(frozen=True)
class RepairRowView:
    request_id: str
    destination_slots: tuple
    positions: tuple
    slot_digest: str

    @classmethod
    def of(cls, request_id: str, slots: Sequence[int], positions: Sequence[int]) -> "RepairRowView":
        s = tuple(int(x) for x in slots)
        p = tuple(int(x) for x in positions)
        if len(s) != len(p) or not s:
            raise SparseRepairComputeError("a repair row needs one slot per position")
        return cls(str(request_id), s, p, hashlib.sha256(repr(s).encode()).hexdigest())

    @property
    def token_count(self) -> int:
        return len(self.destination_slots)


COMPONENTS = ("pre_attention_norm", "qkv_projection", "rope", "attention", "output_projection",
              "post_attention_norm", "mlp")


class RepairStateCapture:
    """Attach as ``model.capture``; the extend forward reports each layer's
    output (``on_layer``) and, for the layers named in
    ``component_layers``, each component (``on_component``)."""

    def __init__(self, output_path: Path, component_layers: Sequence[int] = ()):
        self.output_path = Path(output_path)
        self.component_layers = set(int(x) for x in component_layers)
        self.layer_outputs: dict[int, list[dict]] = {}
        self.component_outputs: dict[int, dict[str, list[dict]]] = {}

    @classmethod
    def create_if_enabled(cls, output_dir: Optional[str], num_layers: int) -> Optional["RepairStateCapture"]:
        if not output_dir:
            return None
        path = Path(output_dir) / "sparse_repair_state.pt"
        if path.exists():  # one capture per directory
            return None
        raw = os.getenv("SGLANG_PIC_SPARSE_REPAIR_CAPTURE_COMPONENT_LAYERS", "").strip()
        layers: set = set()
        if raw:
            try:
                layers = {int(v.strip()) for v in raw.split(",")}
            except ValueError as e:
                raise SparseRepairComputeError("component capture layers must be comma-separated integers") from e
            if any(not 0 <= li < num_layers for li in layers):
                raise SparseRepairComputeError("component capture layer is outside the model")
        return cls(path, sorted(layers))

    @staticmethod
    def _host(tensors: dict) -> dict:
        return {k: v.detach().float().cpu().clone() for k, v in tensors.items() if isinstance(v, torch.Tensor)}

    def wants(self, layer: int) -> bool:
        return layer in self.component_layers

    def on_layer(self, layer: int, **tensors) -> None:
        if not tensors:
            raise SparseRepairComputeError(f"layer {layer} produced no tensor output")
        self.layer_outputs.setdefault(layer, []).append(self._host(tensors))

    def on_component(self, layer: int, name: str, **tensors) -> None:
        if name not in COMPONENTS:
            raise SparseRepairComputeError(f"unknown component {name}")
        if layer in self.component_layers:
            self.component_outputs.setdefault(layer, {}).setdefault(name, []).append(self._host(tensors))

    def save(self, kv, repair_slots: torch.Tensor, repair_positions: Sequence[int],
             execution_units: Sequence[Sequence[int]], logits: Optional[torch.Tensor]) -> Path:
        """K/V of the repair rows (per layer, logical repair order) and the
        logits, with everything captured during the forward."""
        slots = repair_slots.long().to(kv.k.device)
        ps = kv.k.shape[3]
        page, off = slots // ps, slots % ps
        repaired = {}
        for li in range(kv.k.shape[0]):
            repaired[li] = {"key": kv.k[li][page, :, off].detach().float().cpu().clone(),
                            "value": kv.v[li][page, :, off].detach().float().cpu().clone()}
        payload = {
            "schema_version": 2,
            "diagnostic_only": True,
            "repair_positions": torch.tensor(list(repair_positions), dtype=torch.long),
            "execution_units": [list(u) for u in execution_units],
            "layer_outputs": self.layer_outputs,
            "component_outputs": self.component_outputs,
            "repaired_kv": repaired,
            "logits": logits.detach().float().cpu().clone() if logits is not None else None,
        }
        self.output_path.parent.mkdir(parents=True, exist_ok=True)
        torch.save(payload, self.output_path)
        return self.output_path


# ----------------------------------------------------------- debug compares
def compare_enabled(kind: str) -> bool:
    """``kv_link``: ``SGLANG_PIC_COMPARE_FUSED_TORCH_KV_LINK``;
    ``attention``: ``SGLANG_PIC_COMPARE_NATIVE_REFERENCE_ATTENTION``."""
    return _flag({"kv_link": "SGLANG_PIC_COMPARE_FUSED_TORCH_KV_LINK",
                  "attention": "SGLANG_PIC_COMPARE_NATIVE_REFERENCE_ATTENTION"}[kind])


def _stats(got: torch.Tensor, want: torch.Tensor) -> dict:
    d = got.float() - want.float()
    return {"max_abs_error": float(d.abs().max().item()) if d.numel() else 0.0,
            "mean_abs_error": float(d.abs().mean().item()) if d.numel() else 0.0,
            "exact": bool(torch.equal(got.to(want.dtype), want)),
            "allclose_bf16": bool(torch.allclose(got.float(), want.float(), atol=2e-2, rtol=2e-2))}


def compare_kv_link(k_pool, v_pool, src_slots, dst_slots, local_pos, global_pos, cos_sin) -> dict:
    """Destination rows the fused link kernel wrote, against the torch fp32
    statement recomputed from the (untouched) source rows, all layers."""
    from ..ops import reference as ref

    ps = k_pool.shape[3]
    dev = k_pool.device
    src, dst = src_slots.long().to(dev), dst_slots.long().to(dev)
    lp, gp = local_pos.long().to(dev), global_pos.long().to(dev)
    # the reference writes into scratch pools holding only these rows
    n = src.numel()
    npg = (n + ps - 1) // ps
    sk = torch.zeros(k_pool.shape[0], npg, *k_pool.shape[2:], dtype=k_pool.dtype, device=dev)
    sv = torch.zeros_like(sk)
    scratch = torch.arange(n, device=dev)
    ref.kv_link_rope(sk, sv, src, scratch, lp, gp, cos_sin.to(dev), src_k_pool=k_pool, src_v_pool=v_pool)
    kf = k_pool[:, dst // ps, :, dst % ps]
    vf = v_pool[:, dst // ps, :, dst % ps]
    kr = sk[:, scratch // ps, :, scratch % ps]
    vr = sv[:, scratch // ps, :, scratch % ps]
    return {"rows": int(n), "layers": int(k_pool.shape[0]), "key": _stats(kf, kr), "value": _stats(vf, vr)}


def compare_attention(layer: int, q: torch.Tensor, out: torch.Tensor, k_pool_l, v_pool_l, q_indptr, q_pos,
                      page_table, kv_lens, scale: float, max_rows: int = 128) -> dict:
    """The repair attention's output rows against the fp32 torch statement
    on a sample of at most ``max_rows`` rows (evenly spaced; every row is
    independent given its position)."""
    from ..ops import reference as ref

    T = q.shape[0]
    take = torch.linspace(0, T - 1, steps=min(T, max_rows)).round().long().unique().to(q.device)
    qi = q_indptr.long().cpu()
    req = torch.bucketize(take.cpu(), qi[1:], right=True)  # request of each sampled row
    rows, got = [], []
    for b in req.unique().tolist():
        sel = take[(req == b).to(take.device)]
        ptr = torch.tensor([0, sel.numel()], dtype=torch.int32, device=q.device)
        y = ref.paged_attention(q[sel], k_pool_l, v_pool_l, ptr, q_pos[sel], page_table[b:b + 1], kv_lens[b:b + 1],
                                scale)
        rows.append(y)
        got.append(out[sel])
    want, have = torch.cat(rows), torch.cat(got)
    return {"layer_id": int(layer), "rows_compared": int(want.shape[0]), "shape": list(out.shape),
            **_stats(have, want), "native_norm": float(have.float().norm().item()),
            "reference_norm": float(want.float().norm().item())}
