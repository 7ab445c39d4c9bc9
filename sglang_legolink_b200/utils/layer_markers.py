"""Layer-wise profiler markers: ``LegoLink::Attention``, ``LegoLink::FFN``,
``LegoLink::LMHead`` and ``LegoLink::Sampling`` regions around the model's
parts, as ``torch.profiler.record_function`` regions (they show up in the
``/start_profile`` trace) and NVTX ranges whose payload names the part, the
layer and the input shapes.

The model is not a tree of ``nn.Module`` objects, so the markers are placed
explicitly around each part of the forward instead of by module hooks.  Off
by default (``SGLANG_ENABLE_LAYERWISE_NVTX_MARKER=1``, the server's
``--enable-layerwise-nvtx-marker``, or ``LayerMarkers(True)``); when off,
``region`` returns one shared null context.  Nothing is marked while a CUDA
graph is being captured (the decode step), since host ranges there would only
mark the capture.

Reference: ``patched_sglang_files/python/sglang/srt/utils/nvtx_pytorch_hooks.py``
(region names ``:44-60``), ``model_executor/model_runner.py:1320``.
"""

from __future__ import annotations

import contextlib
import os
from typing import Optional

import torch

_NULL = contextlib.nullcontext()
KINDS = ("Attention", "FFN", "LMHead", "Sampling")


class LayerMarkers:
    def __init__(self, enabled: bool = False):
        self.enabled = bool(enabled)
        self.pushed = 0  # NVTX ranges opened (tests and diagnostics)

    @classmethod
    def from_env(cls) -> "LayerMarkers":
        return cls(os.getenv("SGLANG_ENABLE_LAYERWISE_NVTX_MARKER", "0").strip().lower() in {"1", "true", "yes"})

    def region(self, kind: str, layer: Optional[int] = None, **inputs):
        if not self.enabled:
            return _NULL
        if torch.cuda.is_available() and torch.cuda.is_current_stream_capturing():
            return _NULL
        return self._region(kind, layer, inputs)

    @contextlib.contextmanager
    def _region(self, kind: str, layer: Optional[int], inputs: dict):
        if kind not in KINDS:
            raise ValueError(f"unknown marker region {kind}")
        name = f"LegoLink::{kind}"
        payload = {"Module": name if layer is None else f"{name}[{layer}]",
                   "Inputs": {k: list(v.shape) for k, v in inputs.items() if isinstance(v, torch.Tensor)}}
        nvtx = torch.cuda.is_available()
        with torch.profiler.record_function(name):
            if nvtx:
                torch.cuda.nvtx.range_push(str(payload))
            self.pushed += 1
            try:
                yield payload
            finally:
                if nvtx:
                    torch.cuda.nvtx.range_pop()
