"""Two-rank TP worker (launched by tests/test_tp_gpu.py): TP=2 prefill logits
of a small Qwen3 match the unsharded model's within bf16 tolerance, and a TP
Link + graph decode runs on both ranks with identical tokens."""

import os
import sys

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from datetime import timedelta  # noqa: E402

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402


def main():
    rank, local = int(os.environ["RANK"]), int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=60), device_id=dev)
    from sglang_legolink_b200.models.config import PRESETS
    from sglang_legolink_b200.models.qwen import QwenModel
    from sglang_legolink_b200.parallel.tp import NcclTPComm
    from sglang_legolink_b200.runtime.engine import Engine

    cfg = PRESETS["small-qwen3"]
    g = torch.Generator().manual_seed(1)
    prompt = torch.randint(0, cfg.vocab_size, (300,), generator=g).tolist()
    tp = QwenModel.random_init(cfg, seed=0, device=dev, dtype=torch.bfloat16, tp_rank=rank, tp_size=2,
                               comm=NcclTPComm())
    eng = Engine(tp, num_pages=1024, max_context=4096)
    seq = eng.prefill(prompt)
    fb = eng._extend_batch([(prompt[-8:], list(range(292, 300)), seq.pages, 300)])
    local_logits = tp.forward(fb, eng.kv)
    full = tp.full_logits(local_logits).float()
    ok = True
    if rank == 0:
        single = QwenModel.random_init(cfg, seed=0, device=dev, dtype=torch.bfloat16)
        e1 = Engine(single, num_pages=1024, max_context=4096)
        s1 = e1.prefill(prompt)
        fb1 = e1._extend_batch([(prompt[-8:], list(range(292, 300)), s1.pages, 300)])
        ref = single.forward(fb1, e1.kv).float()
        rel = ((full - ref).norm() / ref.norm()).item()
        print("tp2 vs single rel", rel, flush=True)
        ok = rel < 3e-2
    for i, n in enumerate((100, 150)):
        eng.compile(torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist(), f"b{i}")
    s = eng.link({"cache_keys": ["b1", "b0"], "recompute_initial_tokens": 16, "recompute_first_block": True},
                 [5, 6, 7, 8])
    eng.decode([s], 6)
    outs = [None, None]
    dist.all_gather_object(outs, s.output_ids)
    ok = ok and outs[0] == outs[1]
    if rank == 0 and ok:
        print("TP_OK", outs[0], flush=True)
    eng._graphs.clear()
    dist.barrier()
    dist.destroy_process_group()
    sys.exit(0 if ok else 1)


if __name__ == "__main__":
    main()
