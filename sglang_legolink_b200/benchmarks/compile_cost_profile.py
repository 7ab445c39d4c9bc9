"""Measures this deployment's compile cost profile (prefill / Compile / Link
latency curves over block length) on the engine itself and writes it as
JSON for ``CostBenefitCompilePolicy``.

    python -m sglang_legolink_b200.benchmarks.compile_cost_profile --model qwen2.5-7b \\
        --lengths 64,256,1024,4096,8192 --out profile.json

Device time (CUDA events), median of ``--repeats`` after one warm-up; the
Link includes a ``--repair``-row boundary repair and a 32-token turn.
"""

from __future__ import annotations

import argparse
import json


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="qwen2.5-7b")
    ap.add_argument("--lengths", default="64,256,1024,4096,8192")
    ap.add_argument("--repeats", type=int, default=3)
    ap.add_argument("--repair", type=int, default=32)
    ap.add_argument("--hardware-id", default=None, help="defaults to the CUDA device name")
    ap.add_argument("--out", default="compile_cost_profile.json")
    a = ap.parse_args()

    import torch

    from ..host.compile_cost import measure_engine_profile
    from ..models.config import PRESETS
    from ..models.qwen import QwenModel
    from ..runtime.engine import Engine

    dev = torch.device("cuda", 0) if torch.cuda.is_available() else torch.device("cpu")
    dtype = torch.bfloat16 if dev.type == "cuda" else torch.float32
    cfg = PRESETS[a.model]
    lengths = [int(x) for x in a.lengths.split(",")]
    eng = Engine(QwenModel.random_init(cfg, seed=0, device=dev, dtype=dtype), page_size=16,
                 max_context=max(lengths) + 1024, num_pages=4 * (max(lengths) + 1024) // 16 + 256)
    hw = a.hardware_id or (torch.cuda.get_device_name(dev) if dev.type == "cuda" else "cpu")
    prof = measure_engine_profile(eng, lengths, hardware_id=hw, model_id=cfg.name, repeats=a.repeats,
                                  repair_window=a.repair)
    prof.write_json(a.out)
    print(json.dumps({"profile_id": prof.profile_id, "out": a.out,
                      **{k: prof.to_dict()[k]["points"] for k in ("prefill_ms", "compile_ms", "link_ms")}}))


if __name__ == "__main__":
    main()
