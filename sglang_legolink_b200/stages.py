"""The pipeline's stages pinned to the code that implements them.

Data only: nothing on a serving path imports this module.
``tests/test_stage_registry.py`` checks every entry against the source -- the
file exists, the symbol resolves (a Python attribute path, or a kernel name
present in a ``.cu`` file), and every recorded call edge really appears in
the caller's source -- so a refactor that moves a stage fails a test instead
of silently outdating the map.  The reference keeps the same kind of
registry for its own files (``noc_context_manager/architecture_stages.py:41,196``).

Paths are relative to the package directory.
"""

from __future__ import annotations

from dataclasses import dataclass

HOST, RUNTIME, KERNEL = "host", "runtime", "kernel"


@dataclass(frozen=True)
class Stage:
    step: int
    name: str
    side: str
    file: str
    symbol: str
    helpers: tuple = ()


@dataclass(frozen=True)
class CallEdge:
    src: int
    dst: int
    file: str
    caller: str
    callee: str  # a name that must appear in the caller's source


STAGES: tuple[Stage, ...] = (
    Stage(1, "Agent / ingress", HOST, "host/agent.py", "AgentLLM.call",
          ("server/proxy.py:LegoLinkProxy.chat_completion", "host/events.py:openai_request_events")),
    Stage(2, "Session events + field extraction", HOST, "host/events.py", "FieldExtractor.extract",
          ("host/events.py:EventCollector.add_events",)),
    Stage(3, "Semantic segmentation", HOST, "host/manager.py", "DeterministicSegmenter.segment",
          ("host/manager.py:validate_segments",)),
    Stage(4, "Sub-context identity + store", HOST, "host/store.py", "semantic_cache_key",
          ("host/store.py:SubContextStore.replace_source_revisions",)),
    Stage(5, "Context selection", HOST, "host/manager.py", "ContextManager.select"),
    Stage(6, "Compile policy + planner", HOST, "host/planner.py", "Planner.plan"),
    Stage(7, "Stitch + physical framing", HOST, "host/framing.py", "build_layout",
          ("host/framing.py:Stitcher.stitch",)),
    Stage(8, "Repair windows", HOST, "host/framing.py", "RepairWindowPlanner.plan"),
    Stage(9, "Link contract", HOST, "contract.py", "validate_pic_link_request", ("host/framing.py:frame_link",)),
    Stage(10, "Adapter + residency recovery", HOST, "host/adapter.py", "RuntimeAdapter.link",
          ("host/adapter.py:ResidencyRecoveryCoordinator",)),
    Stage(11, "Runtime admission", RUNTIME, "runtime/scheduler.py", "Scheduler._admit_batch",
          ("server/http_server.py:RuntimeService.build_request",)),
    Stage(12, "Link plan resolution", RUNTIME, "runtime/link_plan.py", "resolve_link_plan"),
    Stage(13, "KV link + RoPE delta remap", RUNTIME, "runtime/engine.py", "Engine._run_kv_links",
          ("ops/__init__.py:kv_link_rope",)),
    Stage(14, "Sparse boundary repair forward", RUNTIME, "models/qwen.py", "QwenModel.forward",
          ("ops/__init__.py:attention_prefill",)),
    Stage(15, "Native decode", RUNTIME, "runtime/engine.py", "Engine.decode_step",
          ("ops/__init__.py:attention_decode",)),
    Stage(16, "Fused KV link kernel", KERNEL, "csrc/elementwise.cu", "kv_link_rope_kernel"),
    Stage(17, "Repair attention kernel", KERNEL, "csrc/attention_tc.cu", "attn_prefill_tc_kernel"),
    Stage(18, "Decode attention kernel", KERNEL, "csrc/attention_tc.cu", "attn_decode_tma_kernel"),
    Stage(19, "GEMM kernels", KERNEL, "csrc/gemm_tcgen05.cu", "gemm_tcgen05_2sm_kernel",
          ("csrc/gemm_tcgen05.cu:gemm_swapab_kernel",)),
    Stage(20, "TP reduction kernels", KERNEL, "csrc/tp_fused.cu", "tp_reduce_norm_gather_kernel"),
)

CALL_EDGES: tuple[CallEdge, ...] = (
    CallEdge(1, 2, "host/agent.py", "AgentLLM.call", "execute"),
    CallEdge(1, 2, "host/adapter.py", "RequestPipeline.execute", "ingest"),
    CallEdge(2, 3, "host/manager.py", "ContextManager._store_changed", "segment"),
    CallEdge(3, 4, "host/manager.py", "ContextManager._store_changed", "replace_source_revisions"),
    CallEdge(4, 5, "host/adapter.py", "RequestPipeline.execute", "select"),
    CallEdge(5, 6, "host/adapter.py", "RequestPipeline.execute", "plan"),
    CallEdge(6, 7, "host/adapter.py", "RequestPipeline.execute", "build_layout"),
    CallEdge(7, 10, "host/adapter.py", "RequestPipeline.execute", "link"),
    CallEdge(10, 11, "server/http_server.py", "RuntimeService.complete", "build_request"),
    CallEdge(11, 12, "runtime/engine.py", "Engine._link_prepare", "resolve_link_plan"),
    CallEdge(12, 13, "runtime/engine.py", "Engine.extend_step", "_run_kv_links"),
    CallEdge(13, 14, "runtime/engine.py", "Engine.extend_step", "forward"),
    CallEdge(13, 16, "ops/__init__.py", "kv_link_rope", "kv_link_rope"),
    CallEdge(14, 17, "ops/__init__.py", "attention_prefill", "attn_prefill_tc"),
    CallEdge(15, 18, "ops/__init__.py", "attention_decode", "attn_decode"),
)
