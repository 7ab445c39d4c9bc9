"""Token sampling: greedy (the default, and what exact-repair equivalence is
measured with), temperature, top-k and top-p with per-request seeds
(reference: the PyTorch sampling backend, ``layers/sampler.py``; the host
harness sends temperature 0 / top_k 1, ``sglang_adapter.py:324-333``).

Greedy rows use the fused argmax kernel; sampled rows use torch ops on the
logits the decode graph already produced (a [B, vocab] softmax is tiny next to
the GEMMs).
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Optional, Sequence

import torch


@dataclass(frozen=True)
class SamplingParams:
    temperature: float = 0.0
    top_p: float = 1.0
    top_k: int = 0
    seed: Optional[int] = None

    @property
    def greedy(self) -> bool:
        return self.temperature <= 0.0 or self.top_k == 1

    @classmethod
    def from_request(cls, payload: dict) -> "SamplingParams":
        return cls(float(payload.get("temperature", 0.0) or 0.0), float(payload.get("top_p", 1.0) or 1.0),
                   int(payload.get("top_k", 0) or 0), payload.get("seed"))


GREEDY = SamplingParams()


def sample_rows(logits: torch.Tensor, params: Sequence[SamplingParams],
                generators: Optional[Sequence[Optional[torch.Generator]]] = None) -> torch.Tensor:
    """One token per row of ``logits`` [B, vocab] (full vocab)."""
    B = logits.shape[0]
    out = torch.argmax(logits.float(), dim=-1).to(torch.int32)
    for i, p in enumerate(params[:B]):
        if p.greedy:
            continue
        x = logits[i].float() / max(p.temperature, 1e-5)
        if p.top_k and p.top_k > 0:
            kth = torch.topk(x, min(p.top_k, x.numel())).values[-1]
            x = torch.where(x < kth, torch.full_like(x, float("-inf")), x)
        probs = torch.softmax(x, dim=-1)
        if p.top_p < 1.0:
            sp, si = torch.sort(probs, descending=True)
            cum = torch.cumsum(sp, dim=-1)
            keep = cum - sp < p.top_p
            sp = torch.where(keep, sp, torch.zeros_like(sp))
            probs = torch.zeros_like(probs).scatter_(0, si, sp)
            probs = probs / probs.sum()
        g = generators[i] if generators is not None else None
        out[i] = torch.multinomial(probs, 1, generator=g).to(torch.int32)[0]
    return out


def make_generator(params: SamplingParams, device) -> Optional[torch.Generator]:
    if params.greedy or params.seed is None:
        return None
    g = torch.Generator(device=device)
    g.manual_seed(int(params.seed))
    return g
