"""The stage registry matches the source: files exist, symbols resolve, and
every recorded call edge appears in its caller (CPU)."""

import importlib
import inspect
import os

import pytest

from sglang_legolink_b200 import stages

PKG = os.path.dirname(os.path.abspath(stages.__file__))


def _module_name(rel: str) -> str:
    mod = rel[:-3].replace("/", ".")
    if mod.endswith(".__init__"):
        mod = mod[: -len(".__init__")]
    return "sglang_legolink_b200." + mod


def _resolve(rel: str, symbol: str):
    path = os.path.join(PKG, rel)
    assert os.path.exists(path), f"{rel} is missing"
    if rel.endswith(".cu"):
        with open(path, encoding="utf-8") as f:
            assert symbol in f.read(), f"{symbol} not found in {rel}"
        return None
    obj = importlib.import_module(_module_name(rel))
    for part in symbol.split("."):
        obj = getattr(obj, part)
    return obj


@pytest.mark.parametrize("stage", stages.STAGES, ids=lambda s: f"{s.step}-{s.name}")
def test_stage_symbols_resolve(stage):
    _resolve(stage.file, stage.symbol)
    for h in stage.helpers:
        rel, sym = h.split(":")
        _resolve(rel, sym)


@pytest.mark.parametrize("edge", stages.CALL_EDGES, ids=lambda e: f"{e.src}->{e.dst}:{e.caller}")
def test_call_edges_exist(edge):
    fn = _resolve(edge.file, edge.caller)
    assert edge.callee in inspect.getsource(fn), f"{edge.caller} does not call {edge.callee}"


def test_steps_are_unique_and_ordered():
    steps = [s.step for s in stages.STAGES]
    assert steps == sorted(set(steps))
    known = set(steps)
    assert all(e.src in known and e.dst in known for e in stages.CALL_EDGES)
