"""LegoLink on B200: position-independent KV reuse (Compile / Link) for
Qwen2 / Qwen3 serving, with sm_100a kernels.

Subpackages: ``host`` (context manager, planner, contract framing, adapter),
``runtime`` (registry, link plans, engine, scheduler), ``server`` (HTTP API,
OpenAI proxy), ``models``, ``ops`` (kernels), ``parallel`` (TP / DP over
NVLink), ``utils``.
"""

__version__ = "0.1.0"
