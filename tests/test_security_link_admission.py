"""Link admission hardening on CPU.

L1 -- a Link may not ask for input-token log-probabilities (its input rows
are linked, not computed): every form of the request (OpenAI ``echo`` +
``logprobs``, ``input_logprobs``, native ``return_logprob`` with a
``logprob_start_len`` >= 0) is refused as a bad request, while a normal Link
and a non-Link request asking for them pass.

L2 -- every value of a ``pic_link`` field that breaks its declared shape is
a contract error (a ``ValueError`` the scheduler turns into a request
refusal), never another exception type; recompute modes are accepted in any
case; the accepted modes are the ones the link planner implements; the
scheduler refuses the request and keeps serving.

Reference: ``tests/test_security_l1_link_input_logprobs.py``,
``tests/test_security_l2_pic_link_validation.py``."""

import copy

import pytest
import torch

from sglang_legolink_b200 import contract as C
from sglang_legolink_b200.host.tokenizer import HashTokenizer
from sglang_legolink_b200.models.config import PRESETS
from sglang_legolink_b200.models.qwen import QwenModel
from sglang_legolink_b200.runtime.engine import Engine
from sglang_legolink_b200.runtime.scheduler import Request, RequestRejected, Scheduler
from sglang_legolink_b200.server.http_server import RuntimeService, asks_input_logprobs


@pytest.fixture(scope="module")
def svc():
    eng = Engine(QwenModel.random_init(PRESETS["tiny-qwen2"], seed=0), num_pages=256, page_size=16)
    g = torch.Generator().manual_seed(3)
    eng.compile(torch.randint(0, 1024, (40,), generator=g).tolist(), "sec-a")
    sch = Scheduler(eng, legolink_only=True)
    return RuntimeService(sch, HashTokenizer(1024))


def _link(**extra):
    return {"messages": [{"role": "user", "content": "go"}], "max_tokens": 2,
            "pic_link": {"cache_keys": ["sec-a"], "recompute_initial_tokens": 2}, **extra}


# ------------------------------------------------------------------------ L1
@pytest.mark.parametrize("extra", [
    {"return_logprob": True, "logprob_start_len": 0},
    {"return_logprob": True, "logprob_start_len": 7},
    {"return_logprob": True, "logprob_start_len": "3"},
    {"input_logprobs": True},
    {"echo": True, "logprobs": 1},
])
def test_a_link_asking_for_input_logprobs_is_refused(svc, extra):
    with pytest.raises(RequestRejected, match="input logprobs"):
        svc.build_request(_link(**extra))


@pytest.mark.parametrize("extra", [
    {}, {"return_logprob": True}, {"return_logprob": True, "logprob_start_len": -1},
    {"logprobs": True}, {"echo": True}, {"return_logprob": False, "logprob_start_len": 0},
])
def test_a_link_without_input_logprobs_is_admitted(svc, extra):
    req = svc.build_request(_link(**extra))
    assert req.kind == "link"


def test_a_non_link_request_with_input_logprobs_is_untouched():
    body = {"prompt": [1, 2, 3], "return_logprob": True, "logprob_start_len": 0}
    assert asks_input_logprobs(body)
    eng = Engine(QwenModel.random_init(PRESETS["tiny-qwen2"], seed=0), num_pages=64, page_size=16)
    s = RuntimeService(Scheduler(eng, legolink_only=False), HashTokenizer(1024))
    assert s.build_request(body).kind == "plain"


@pytest.mark.parametrize("link", ["sec-a", ["sec-a"], 5])
def test_a_malformed_pic_link_is_a_contract_refusal_not_a_logprob_one(svc, link):
    body = {"messages": [{"role": "user", "content": "x"}], "pic_link": link, "return_logprob": True,
            "logprob_start_len": 0}
    with pytest.raises((RequestRejected, C.ContractError)):
        svc.build_request(body)


def test_the_refusal_is_request_scoped(svc):
    """The refused Link leaves nothing behind: the next Link is served."""
    with pytest.raises(RequestRejected):
        svc.build_request(_link(input_logprobs=True))
    out = svc.scheduler.run_sync(svc.build_request(_link()))
    assert out["tokens"]


# ------------------------------------------------------------------------ L2
ODD = [None, True, False, -1, 2 ** 40, 1.5, float("nan"), "", "x", [], [1], [None], ["a", 1], {}, {"a": 1}, [[1]]]
FIELDS = sorted(C.PIC_LINK_REQUEST_FIELDS | C.PIC_LINK_RUNTIME_OWNED_FIELDS)


def _plan():
    return {"cache_keys": ["a", "b"], "recompute_initial_tokens": 4}


@pytest.mark.parametrize("field", FIELDS)
def test_no_mutation_of_a_field_escapes_as_another_exception_type(field):
    for v in ODD:
        plan = _plan()
        plan[field] = copy.deepcopy(v)
        try:
            C.validate_pic_link_request(plan, allow_legacy_fields=False, require_formal=False, profile=None)
        except C.ContractError:
            pass


@pytest.mark.parametrize("field,value", [
    ("cache_keys", "a"), ("cache_keys", []), ("cache_keys", [1]), ("cache_keys", None),
    ("recompute_initial_tokens", -1), ("recompute_initial_tokens", "4"), ("recompute_initial_tokens", True),
    ("recompute_initial_tokens", None), ("recompute_tokens_per_block", [1]), ("recompute_tokens_per_block", [1, -2]),
    ("recompute_first_block", "yes"), ("recompute_mode", "sideways"), ("recompute_mode", 3),
    ("block_ids", ["x", "y", "z"]), ("concurrency", -3), ("profiling_warmup", 1), ("variant", 7),
    ("adapter_id", ["x"]), ("execution_group_key", 9), ("promote_reconstructed_group", "1"),
])
def test_each_shape_violation_is_a_contract_error(field, value):
    plan = _plan()
    plan[field] = value
    with pytest.raises(C.ContractError):
        C.validate_pic_link_request(plan, allow_legacy_fields=False, require_formal=False, profile=None)


def test_a_missing_required_field_and_a_non_object_are_contract_errors():
    with pytest.raises(C.ContractError, match="cache_keys"):
        C.validate_pic_link_request({"recompute_initial_tokens": 4}, require_formal=False, profile=None)
    for bad in (None, "x", ["a"], 3):
        with pytest.raises(C.ContractError, match="object"):
            C.validate_pic_link_request(bad, require_formal=False, profile=None)


def test_a_valid_link_with_every_optional_field_is_admitted():
    plan = {"cache_keys": ["a", "b"], "block_ids": ["ba", "bb"], "request_id": "r1", "task_id": 3,
            "variant": "legolink", "profiling_warmup": False, "concurrency": 8, "adapter_id": "base",
            "segmentation_policy_version": "s1", "legolink_policy_version": C.LEGOLINK_POLICY_VERSION,
            "recompute_mode": "batched", "recompute_initial_tokens": 4, "recompute_first_block": True,
            "recompute_first_block_tokens": 4, "recompute_tokens_per_block": [4, 2]}
    C.validate_pic_link_request(plan, require_formal=False, profile=None)


@pytest.mark.parametrize("mode", ["batched", "BATCHED", "Tokenwise", "full_causal", "FULL_CAUSAL"])
def test_recompute_modes_are_accepted_in_any_case(mode):
    C.validate_pic_link_request({"cache_keys": ["a"], "recompute_mode": mode}, require_formal=False, profile=None)


def test_the_mode_enum_matches_what_the_link_planner_implements(monkeypatch):
    from sglang_legolink_b200.runtime.link_plan import resolve_link_plan

    toks = {"a": list(range(40)), "b": list(range(100, 130))}
    rows = {}
    for mode in sorted(C.PIC_LINK_RECOMPUTE_MODES):
        plan = {"cache_keys": ["a", "b"], "recompute_initial_tokens": 4, "recompute_mode": mode}
        r = resolve_link_plan(plan, [7, 8], toks.get)
        assert r.recompute_mode == mode
        rows[mode] = len(r.recompute_positions)
    assert rows["batched"] == rows["tokenwise"] < rows["full_causal"]
    with pytest.raises(C.ContractError):
        resolve_link_plan({"cache_keys": ["a"], "recompute_mode": "sideways"}, [7], toks.get)


def test_the_scheduler_refuses_a_malformed_link_and_keeps_serving(svc):
    sch = svc.scheduler
    bad = Request("link", "bad", [1, 2], 2, pic_link={"cache_keys": ["sec-a"], "recompute_initial_tokens": -5})
    with pytest.raises(RequestRejected, match="recompute_initial_tokens"):
        sch.run_sync(bad)
    good = sch.run_sync(Request("link", "good", [1, 2], 2,
                                pic_link={"cache_keys": ["sec-a"], "recompute_initial_tokens": 2}))
    assert good["tokens"]
