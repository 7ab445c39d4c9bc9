"""Compile economics: whether compiling a block pays for itself, from measured
latencies rather than a constant token floor.

The trade is a break-even, per block:

    compile once + N x (link + repair)    versus    N x native prefill

so the decision needs four measured latencies (prefill, compile, link,
optionally repair) of *this* deployment, an expectation of N, and what
keeping the KV resident costs.  This module holds those terms and the
arithmetic; the policy that uses them is ``CostBenefitCompilePolicy`` in
``host/planner.py``.

Honesty rules:

* a :class:`LatencyCurve` answers only inside its measured range (piecewise
  linear between measured points); asked elsewhere it raises
  :class:`CompileCostUnavailable` rather than extrapolating or clamping;
* a :class:`CompileCostProfile` carries the provenance of its numbers
  (hardware, model, dtype, TP size, attention backend, when, from what) and
  is refused for a deployment it was not measured on (strict by default);
* expected reuse always names its source; residency cost is explicitly
  disabled until measured, and every decision records which model it used.

:func:`measure_engine_profile` builds a profile by timing this runtime's own
engine (full prefill, Compile, Link with a stated repair window) at several
lengths -- the curves the B200 deployment actually has.

Reference behaviour: ``noc_context_manager/compile_cost.py:81-875``
(curves, provenance, profile, expectations, residency, breakdown, the
arithmetic).
"""

from __future__ import annotations

import hashlib
import json
from abc import ABC, abstractmethod
from dataclasses import dataclass
from pathlib import Path
from typing import Any, Mapping, Optional, Sequence

COMPILE_COST_SCHEMA_VERSION = 1
COMPILE_COST_POLICY_VERSION = "compile-cost-benefit-v1"


class CompileCostError(RuntimeError):
    pass


class CompileCostProfileError(CompileCostError):
    """A profile is malformed or inconsistent."""


class CompileCostUnavailable(CompileCostError):
    """No honest estimate exists (no profile, length outside the measured
    range, a profile of another deployment, an unstated repair window)."""


# ------------------------------------------------------------------ curves
@dataclass(frozen=True)
class LatencyCurve:
    """Milliseconds as a function of model tokens over measured points."""

    name: str
    points: tuple
    statistic: str = "median"
    samples_per_point: int = 0

    def __post_init__(self):
        if not self.points:
            raise CompileCostProfileError(f"{self.name}: no measured points")
        xs = [int(x) for x, _ in self.points]
        if min(xs) < 0 or any(float(y) < 0 for _, y in self.points):
            raise CompileCostProfileError(f"{self.name}: negative length or latency")
        if any(b <= a for a, b in zip(xs, xs[1:])):
            raise CompileCostProfileError(f"{self.name}: token counts must strictly increase")

    @property
    def measured_range(self) -> tuple:
        return int(self.points[0][0]), int(self.points[-1][0])

    def covers(self, tokens: int) -> bool:
        lo, hi = self.measured_range
        return lo <= int(tokens) <= hi

    def estimate_ms(self, tokens: int) -> float:
        n = int(tokens)
        if not self.covers(n):
            lo, hi = self.measured_range
            raise CompileCostUnavailable(f"{self.name} was measured over {lo}..{hi} tokens, not {n}; extend the "
                                         "profile instead of extrapolating")
        pts = [(int(x), float(y)) for x, y in self.points]
        for (x0, y0), (x1, y1) in zip(pts, pts[1:]):
            if x0 <= n <= x1:
                return y0 + (y1 - y0) * (n - x0) / (x1 - x0)
        return pts[0][1]  # a single measured point

    def to_dict(self) -> dict:
        return {"name": self.name, "points": [[int(x), float(y)] for x, y in self.points],
                "statistic": self.statistic, "samples_per_point": int(self.samples_per_point)}

    @classmethod
    def from_payload(cls, name: str, d: Mapping) -> "LatencyCurve":
        return cls(str(d.get("name") or name), tuple((int(x), float(y)) for x, y in d.get("points", ())),
                   str(d.get("statistic") or "median"), int(d.get("samples_per_point") or 0))


def build_curve(points: Sequence[Sequence[float]], *, name: str, **kw) -> LatencyCurve:
    return LatencyCurve(name, tuple((int(x), float(y)) for x, y in points), **kw)


# --------------------------------------------------------------- provenance
@dataclass(frozen=True)
class DeploymentIdentity:
    """What is being served, to check a profile against."""
    hardware_id: str
    model_id: str
    dtype: str = ""
    tensor_parallel_size: Optional[int] = None
    attention_backend: str = ""

    def to_dict(self) -> dict:
        return dict(self.__dict__)


@dataclass(frozen=True)
class ProfileProvenance:
    profile_version: str
    hardware_id: str
    model_id: str
    dtype: str = ""
    tensor_parallel_size: int = 1
    runtime_version: str = ""
    attention_backend: str = ""
    measured_at: str = ""
    source_artifact: str = ""
    notes: str = ""

    def __post_init__(self):
        for f in ("profile_version", "hardware_id", "model_id"):
            if not str(getattr(self, f) or "").strip():
                raise CompileCostProfileError(f"a compile cost profile must state its {f}")

    def to_dict(self) -> dict:
        return dict(self.__dict__)

    @classmethod
    def from_payload(cls, d: Mapping) -> "ProfileProvenance":
        kw = {k: d.get(k) for k in cls.__dataclass_fields__ if d.get(k) is not None}
        if "sglang_version" in d and "runtime_version" not in kw:  # profiles written by the reference tooling
            kw["runtime_version"] = d["sglang_version"]
        kw["tensor_parallel_size"] = int(kw.get("tensor_parallel_size") or 1)
        return cls(**{k: (v if k == "tensor_parallel_size" else str(v)) for k, v in kw.items()})


PROFILE_MATCHED, PROFILE_MISMATCHED, PROFILE_UNCHECKED = "matched", "mismatched", "unchecked"


@dataclass(frozen=True)
class CompileCostProfile:
    """Measured latencies of one model on one hardware configuration.  No
    ``repair_ms`` curve means the link curve already contains the repair the
    measured runs did (recorded on every decision)."""

    provenance: ProfileProvenance
    prefill_ms: LatencyCurve
    compile_ms: LatencyCurve
    link_ms: LatencyCurve
    repair_ms: Optional[LatencyCurve] = None

    @property
    def repair_folded_into_link(self) -> bool:
        return self.repair_ms is None

    @property
    def profile_id(self) -> str:
        body = json.dumps(self.to_dict(), sort_keys=True, separators=(",", ":")).encode()
        return "sha256:" + hashlib.sha256(body).hexdigest()[:16]

    def check_compatibility(self, deployment: Optional[DeploymentIdentity], *, strict: bool = True) -> str:
        """Hardware and model are always compared; dtype, TP size and backend
        when both sides state them."""
        if deployment is None:
            return PROFILE_UNCHECKED
        p, d = self.provenance, deployment
        diffs = []
        if d.hardware_id != p.hardware_id:
            diffs.append(f"hardware {p.hardware_id!r} != {d.hardware_id!r}")
        if d.model_id != p.model_id:
            diffs.append(f"model {p.model_id!r} != {d.model_id!r}")
        if d.dtype and p.dtype and d.dtype != p.dtype:
            diffs.append(f"dtype {p.dtype!r} != {d.dtype!r}")
        if d.tensor_parallel_size is not None and int(d.tensor_parallel_size) != int(p.tensor_parallel_size):
            diffs.append(f"TP {p.tensor_parallel_size} != {d.tensor_parallel_size}")
        if d.attention_backend and p.attention_backend and d.attention_backend != p.attention_backend:
            diffs.append(f"attention backend {p.attention_backend!r} != {d.attention_backend!r}")
        if not diffs:
            return PROFILE_MATCHED
        if strict:
            raise CompileCostUnavailable(f"profile {self.profile_id} does not match the deployment: "
                                         + "; ".join(diffs))
        return PROFILE_MISMATCHED

    def to_dict(self) -> dict:
        return {"schema_version": COMPILE_COST_SCHEMA_VERSION, "provenance": self.provenance.to_dict(),
                "prefill_ms": self.prefill_ms.to_dict(), "compile_ms": self.compile_ms.to_dict(),
                "link_ms": self.link_ms.to_dict(),
                "repair_ms": self.repair_ms.to_dict() if self.repair_ms is not None else None}

    @classmethod
    def from_payload(cls, d: Mapping) -> "CompileCostProfile":
        missing = [n for n in ("prefill_ms", "compile_ms", "link_ms") if not d.get(n)]
        if missing:
            raise CompileCostProfileError(f"profile is missing curves: {missing}")
        return cls(ProfileProvenance.from_payload(d.get("provenance") or {}),
                   *(LatencyCurve.from_payload(n, d[n]) for n in ("prefill_ms", "compile_ms", "link_ms")),
                   LatencyCurve.from_payload("repair_ms", d["repair_ms"]) if d.get("repair_ms") else None)

    @classmethod
    def from_json(cls, path) -> "CompileCostProfile":
        return cls.from_payload(json.loads(Path(path).read_text(encoding="utf-8")))

    def write_json(self, path) -> Path:
        p = Path(path)
        p.parent.mkdir(parents=True, exist_ok=True)
        p.write_text(json.dumps({**self.to_dict(), "profile_id": self.profile_id}, indent=2, sort_keys=True) + "\n",
                     encoding="utf-8")
        return p


# ----------------------------------------------------------- expected reuse
@dataclass(frozen=True)
class ReuseEstimate:
    """How often a block comes back, and on whose word."""
    expected_future_reuses: float
    reuse_probability: float
    source: str
    evidence_id: Optional[str] = None

    def __post_init__(self):
        if self.expected_future_reuses < 0:
            raise CompileCostError("expected_future_reuses must be non-negative")
        if not 0.0 <= self.reuse_probability <= 1.0:
            raise CompileCostError("reuse_probability must be in [0, 1]")
        if not str(self.source or "").strip():
            raise CompileCostError("a reuse estimate must name its source")

    @property
    def effective_reuses(self) -> float:
        return float(self.expected_future_reuses) * float(self.reuse_probability)

    def to_dict(self) -> dict:
        return {"expected_future_reuses": float(self.expected_future_reuses),
                "reuse_probability": float(self.reuse_probability), "effective_reuses": self.effective_reuses,
                "source": self.source, "evidence_id": self.evidence_id}


class ReuseExpectation(ABC):
    name = "abstract"

    @abstractmethod
    def estimate(self, *, cache_key: str, context_field: str, planned_future_reuse: int) -> ReuseEstimate:
        ...


class FixedReuseExpectation(ReuseExpectation):
    name = "fixed"

    def __init__(self, expected_future_reuses: float, *, probability: float = 1.0):
        self.n, self.p = float(expected_future_reuses), float(probability)

    def estimate(self, *, cache_key, context_field, planned_future_reuse):
        return ReuseEstimate(self.n, self.p, f"fixed:{self.n:g}")


class PlannedTurnsReuseExpectation(ReuseExpectation):
    """The caller's declared future turns, discounted (a plan is not an
    observation)."""
    name = "planned_turns"

    def __init__(self, *, probability: float = 0.5):
        if not 0.0 <= probability <= 1.0:
            raise CompileCostError("probability must be in [0, 1]")
        self.p = float(probability)

    def estimate(self, *, cache_key, context_field, planned_future_reuse):
        return ReuseEstimate(float(max(int(planned_future_reuse), 0)), self.p,
                             f"planned_turns:{planned_future_reuse}")


class ObservedReuseExpectation(ReuseExpectation):
    """Reuse counts recorded for a key in earlier turns; ``default`` for a
    key never seen."""
    name = "observed"

    def __init__(self, observations: Optional[Mapping[str, int]] = None, *, default: float = 0.0,
                 probability: float = 1.0, evidence_id: Optional[str] = None):
        self.obs = dict(observations or {})
        self.default, self.p, self.evidence_id = float(default), float(probability), evidence_id

    def record_reuse(self, cache_key: str, count: int = 1) -> None:
        self.obs[cache_key] = self.obs.get(cache_key, 0) + int(count)

    def estimate(self, *, cache_key, context_field, planned_future_reuse):
        seen = self.obs.get(cache_key)
        if seen is None:
            return ReuseEstimate(self.default, self.p, "observed:unseen", self.evidence_id)
        return ReuseEstimate(float(seen), self.p, f"observed:{seen}", self.evidence_id)


class NoReuseExpectation(ReuseExpectation):
    """Expect nothing: compiles nothing, visibly."""
    name = "none"

    def estimate(self, *, cache_key, context_field, planned_future_reuse):
        return ReuseEstimate(0.0, 0.0, "none:no_reuse_evidence")


# ----------------------------------------------------------------- residency
class ResidencyCostModel(ABC):
    name = "abstract"

    @abstractmethod
    def estimate_ms(self, *, model_tokens: int, expected_hold_reuses: float, memory_pressure: float) -> float:
        ...


class DisabledResidencyCost(ResidencyCostModel):
    """Zero, recorded as ``disabled`` (the cost is unmeasured, not zero)."""
    name = "disabled"

    def estimate_ms(self, *, model_tokens, expected_hold_reuses, memory_pressure):
        return 0.0


class LinearPressureResidencyCost(ResidencyCostModel):
    """coefficient x tokens x expected holds x memory pressure; the caller
    asserts the coefficient and the decision names this model."""
    name = "linear_pressure"

    def __init__(self, *, ms_per_model_token_hold: float):
        if ms_per_model_token_hold < 0:
            raise CompileCostError("ms_per_model_token_hold must be non-negative")
        self.k = float(ms_per_model_token_hold)

    def estimate_ms(self, *, model_tokens, expected_hold_reuses, memory_pressure):
        return self.k * max(int(model_tokens), 0) * max(float(expected_hold_reuses), 0.0) * max(memory_pressure, 0.0)


# ------------------------------------------------------------- the decision
REPAIR_FROM_PLAN = "planned_repair_tokens"
REPAIR_FOLDED_INTO_LINK = "folded_into_link_curve"
REPAIR_WINDOW_UNSPECIFIED = "unspecified"
REPAIR_WINDOW_CALLER_SUPPLIED = "caller_supplied_unvalidated"
REPAIR_WINDOW_EVIDENCE_GATED = "repair_window_policy_evidence_gated"


@dataclass(frozen=True)
class CompileCandidate:
    """One block as the economics see it.  ``preceding_model_tokens`` is
    provenance only (no term reads it): a window sized from position arrives
    as ``planned_repair_model_tokens`` with its ``repair_window_source``."""
    sub_context_id: str
    cache_key: str
    context_field: str
    model_tokens: int
    immutable: bool = True
    reuse_candidate: bool = True
    invalidated: bool = False
    preceding_model_tokens: int = 0
    planned_repair_model_tokens: Optional[int] = None
    repair_window_source: str = REPAIR_WINDOW_UNSPECIFIED
    cache_present: bool = False


@dataclass(frozen=True)
class CompileCostBreakdown:
    model_tokens: int
    expected_future_reuses: float
    expected_reuse_probability: float
    effective_reuses: float
    reuse_source: str
    estimated_prefill_ms: float
    estimated_compile_ms: float
    estimated_link_ms: float
    estimated_repair_ms: float
    estimated_residency_cost_ms: float
    per_reuse_saved_ms: float
    expected_saved_ms: float
    total_cost_ms: float
    net_benefit_ms: float
    repair_model_tokens: int
    repair_source: str
    residency_cost_model: str
    repair_window_source: str = REPAIR_WINDOW_UNSPECIFIED
    compile_cost_sunk: bool = False

    @property
    def is_profitable(self) -> bool:
        """Strictly positive: breaking even does not pay for a plan change."""
        return self.net_benefit_ms > 0.0

    def to_dict(self) -> dict:
        d = dict(self.__dict__)
        d["model_token_count"] = d.pop("model_tokens")
        d["repair_model_token_count"] = d.pop("repair_model_tokens")
        return d


def evaluate_compile_economics(c: CompileCandidate, *, profile: CompileCostProfile, reuse: ReuseExpectation,
                               residency: ResidencyCostModel, planned_future_reuse: int,
                               memory_pressure: float = 0.0) -> CompileCostBreakdown:
    """per_reuse_saved = max(prefill - link - repair, 0);
    saved = effective_reuses x per_reuse_saved; cost = compile + residency
    (compile is sunk, charged 0, when the block is already compiled);
    net = saved - cost.  Compile iff net > 0."""
    n = int(c.model_tokens)
    est = reuse.estimate(cache_key=c.cache_key, context_field=c.context_field,
                         planned_future_reuse=planned_future_reuse)
    prefill = profile.prefill_ms.estimate_ms(n)
    link = profile.link_ms.estimate_ms(n)
    compile_ms = 0.0 if c.cache_present else profile.compile_ms.estimate_ms(n)
    if profile.repair_folded_into_link:
        repair, rtok, rsrc, wsrc = 0.0, 0, REPAIR_FOLDED_INTO_LINK, REPAIR_FOLDED_INTO_LINK
    else:
        if c.planned_repair_model_tokens is None:
            raise CompileCostUnavailable(f"profile {profile.profile_id} prices repair separately but block "
                                         f"{c.sub_context_id} states no repair window")
        rtok = int(c.planned_repair_model_tokens)
        repair, rsrc, wsrc = profile.repair_ms.estimate_ms(rtok), REPAIR_FROM_PLAN, c.repair_window_source
    hold = residency.estimate_ms(model_tokens=n, expected_hold_reuses=est.effective_reuses,
                                 memory_pressure=memory_pressure)
    per = max(prefill - link - repair, 0.0)
    saved = est.effective_reuses * per
    cost = compile_ms + hold
    return CompileCostBreakdown(n, est.expected_future_reuses, est.reuse_probability, est.effective_reuses, est.source,
                                prefill, compile_ms, link, repair, hold, per, saved, cost, saved - cost, rtok, rsrc,
                                residency.name, wsrc, c.cache_present)


# ------------------------------------------------------- measuring a profile
def measure_engine_profile(engine, lengths: Sequence[int], *, hardware_id: str, model_id: str, repeats: int = 3,
                           repair_window: int = 32, seed: int = 0, notes: str = "") -> CompileCostProfile:
    """Times this runtime's engine on the current device: a full prefill of
    n tokens (+ a 32-token turn), a Compile of n tokens, and a Link of that
    block followed by the same turn with ``repair_window`` rows repaired at
    the boundary.  Device time (CUDA events; wall clock on CPU), median of
    ``repeats`` after one warm-up.  The link curve therefore contains the
    repair the runs did (no separate repair curve)."""
    import random
    import statistics
    import time as _time

    import torch

    rng = random.Random(seed)
    V = engine.cfg.vocab_size
    cuda = engine.is_cuda

    def timed(fn):
        if cuda:
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            torch.cuda.synchronize(engine.device)
            a.record()
            out = fn()
            b.record()
            b.synchronize()
            return a.elapsed_time(b), out
        t0 = _time.perf_counter()
        out = fn()
        return (_time.perf_counter() - t0) * 1e3, out

    curves = {"prefill_ms": [], "compile_ms": [], "link_ms": []}
    for n in sorted(set(int(x) for x in lengths)):
        samples = {k: [] for k in curves}
        for r in range(repeats + 1):
            toks = [rng.randrange(V) for _ in range(n)]
            turn = [rng.randrange(V) for _ in range(32)]
            key = f"compile-cost-profile-{n}-{r}-{seed}"
            t_pre, seq = timed(lambda: engine.prefill(toks + turn))
            engine.free(seq)
            t_cmp, _ = timed(lambda: engine.compile(toks, key))
            plan = {"cache_keys": [key], "recompute_initial_tokens": int(repair_window),
                    "recompute_first_block": False}
            t_lnk, seq = timed(lambda: engine.link(plan, turn))
            engine.free(seq)
            engine.unregister_block(key)
            if r:  # the first round is the warm-up
                for k, v in (("prefill_ms", t_pre), ("compile_ms", t_cmp), ("link_ms", t_lnk)):
                    samples[k].append(v)
        for k in curves:
            curves[k].append((n, statistics.median(samples[k])))
    dev = engine.device
    prov = ProfileProvenance(
        profile_version="measured-engine-v1", hardware_id=hardware_id, model_id=model_id,
        dtype=str(engine.model.dtype).replace("torch.", ""), tensor_parallel_size=int(engine.model.tp_size),
        runtime_version="sglang_legolink_b200", attention_backend="sglang_legolink_b200.paged_sm100a" if cuda else "cpu",
        measured_at=_time.strftime("%Y-%m-%dT%H:%M:%SZ", _time.gmtime()),
        source_artifact=f"measure_engine_profile on {dev}",
        notes=notes or f"median of {repeats}; link includes a {repair_window}-row boundary repair and a 32-token turn")
    return CompileCostProfile(prov, *(build_curve(curves[k], name=k, samples_per_point=repeats)
                                      for k in ("prefill_ms", "compile_ms", "link_ms")))
