"""JSON Schemas (draft 2020-12) of the wire objects the host and the runtime
exchange or persist, and a validator for them.

Schemas (``<name>.schema.json`` beside this file):

* ``session_event`` -- one structured ingress event (``host.events.SessionEvent``);
* ``sub_context`` -- a stored sub-context with its identity and cache key
  (``host.store.SubContext``);
* ``agent_context_manifest`` -- one turn's selection (``host.manager.AgentContextManifest``);
* ``execution_plan`` -- the planner's decision (``host.planner.ExecutionPlan``);
* ``pic_link`` -- the Link contract object; unknown and runtime-owned fields
  are refused, as ``contract.validate_pic_link_request`` refuses them;
* ``legolink_request`` -- the ``/v1/chat/completions`` body of a Compile
  (``sub_context``) or a Link (``pic_link``);
* ``metric_row`` -- one per-turn ``metrics.jsonl`` row (``host.metrics.AgentMetric``).

The reference keeps its wire schemas as JSON files too
(``schemas/noc_*.schema.json``); these describe this implementation's own
objects, and ``tests/test_schemas.py`` checks them against the objects the host
pipeline and the contract actually produce.  Schemas refer to one another by
file name (``{"$ref": "pic_link.schema.json"}``); :func:`validate` resolves
those references locally, never over a network.
"""

from __future__ import annotations

import functools
import json
import os
from typing import Any

HERE = os.path.dirname(os.path.abspath(__file__))
BASE_URI = "https://legolink-b200.invalid/schemas/"
SCHEMA_NAMES = ("session_event", "sub_context", "agent_context_manifest", "execution_plan", "pic_link",
                "legolink_request", "metric_row")


class SchemaValidationError(ValueError):
    """An object does not match its schema; ``path`` locates the offending
    value (a list of keys / indices from the root)."""

    def __init__(self, schema: str, message: str, path: list):
        super().__init__(f"{schema}: {message} (at {'/'.join(map(str, path)) or '<root>'})")
        self.schema, self.path = schema, path


def path_of(name: str) -> str:
    if name not in SCHEMA_NAMES:
        raise KeyError(f"unknown schema {name!r}; known: {', '.join(SCHEMA_NAMES)}")
    return os.path.join(HERE, f"{name}.schema.json")


@functools.lru_cache(maxsize=None)
def load(name: str) -> dict:
    with open(path_of(name), encoding="utf-8") as f:
        return json.load(f)


@functools.lru_cache(maxsize=None)
def _registry():
    from referencing import Registry, Resource

    return Registry().with_resources(
        (BASE_URI + f"{n}.schema.json", Resource.from_contents(load(n))) for n in SCHEMA_NAMES)


@functools.lru_cache(maxsize=None)
def _validator(name: str):
    from jsonschema import Draft202012Validator

    return Draft202012Validator(load(name), registry=_registry())


def errors(name: str, obj: Any) -> list:
    """Every violation of schema ``name`` by ``obj`` (empty when it matches)."""
    return sorted(_validator(name).iter_errors(obj), key=lambda e: list(e.absolute_path))


def validate(name: str, obj: Any) -> None:
    """Raise :class:`SchemaValidationError` for the first violation."""
    errs = errors(name, obj)
    if errs:
        e = errs[0]
        raise SchemaValidationError(name, e.message, list(e.absolute_path))


def check_schemas() -> None:
    """Each schema file is itself a valid draft 2020-12 schema."""
    from jsonschema import Draft202012Validator

    for n in SCHEMA_NAMES:
        Draft202012Validator.check_schema(load(n))
