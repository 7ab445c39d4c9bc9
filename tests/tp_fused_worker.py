"""Two-rank worker (launched by tests/test_tp_gpu.py): the fused TP forward
(GEMM with reduce-scatter epilogue -> reduce + RMSNorm + all-gather over
NVLink -> GEMM waiting on the gather) gives the same logits as the NCCL
all-reduce path on the same weights, and a Link + decode through the fused
path yields identical tokens on both ranks."""

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
    from sglang_legolink_b200 import ops
    from sglang_legolink_b200.models.config import PRESETS
    from sglang_legolink_b200.models.qwen import QwenModel
    from sglang_legolink_b200.parallel.tp import NcclTPComm
    from sglang_legolink_b200.parallel.tp_fused import FusedTPComm
    from sglang_legolink_b200.runtime.engine import Engine

    ok = True
    for name in ("small-qwen3", "small-qwen2"):
        cfg = PRESETS[name]
        fused = FusedTPComm(cfg.hidden_size, 4096, dev)
        nccl = NcclTPComm()
        m = QwenModel.random_init(cfg, seed=0, device=dev, dtype=torch.bfloat16, tp_rank=rank, tp_size=2,
                                  comm=fused)
        eng = Engine(m, num_pages=1024, max_context=4096)
        g = torch.Generator().manual_seed(3)
        for T in (1000, 777):
            prompt = torch.randint(0, cfg.vocab_size, (T,), generator=g).tolist()
            pages = eng._alloc_pages((T + 15) // 16)
            fb = eng._extend_batch([(prompt, list(range(T)), pages, T)])
            fb.logit_rows = None
            m.comm = fused
            a = m.forward(fb, eng.kv).float()
            m.comm = nccl
            b = m.forward(fb, eng.kv).float()
            m.comm = fused
            torch.cuda.synchronize()
            e = ops.check_errors(dev)
            rel = ((a - b).norm() / b.norm()).item()
            if rank == 0:
                print(name, "T", T, "fused vs nccl rel", rel, "err", e, flush=True)
            ok = ok and rel < 2e-2 and e == 0
            eng.alloc.release(pages)
        # Link + decode through the fused path (repair rows >= 512)
        for i, n in enumerate((400, 500)):
            eng.compile(torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist(), f"b{i}")
        s = eng.link({"cache_keys": ["b1", "b0"], "recompute_initial_tokens": 400, "recompute_first_block": True},
                     list(range(5, 200)))
        eng.decode([s], 6)
        outs = [None, None]
        dist.all_gather_object(outs, s.output_ids)
        ok = ok and outs[0] == outs[1] and fused.stats["fused_gemms"] > 0
        ok = ok and fused.stats["fused_decode_reduces"] > 0
        if rank == 0:
            print(name, "link tokens", outs[0], "fused stats", fused.stats, flush=True)
        # one eager decode step: the fused decode boundary (one-shot all-reduce
        # + add + RMSNorm over NVLink) against NCCL all-reduce + add-norm
        from sglang_legolink_b200.runtime.engine import ForwardBatch

        for B in (1, 4):
            seqs = [s] * B
            ids, pos, slots, pt, kvl = eng._decode_inputs(seqs, B, len(s.pages))
            fb = ForwardBatch(mode="decode", input_ids=ids.to(dev), positions=pos.to(dev), slots=slots.to(dev),
                              q_indptr=torch.arange(B + 1, dtype=torch.int32).to(dev), page_table=pt.to(dev),
                              kv_lens=kvl.to(dev), logit_rows=None)
            m.comm = fused
            a = m.forward(fb, eng.kv).float()
            m.comm = nccl
            b = m.forward(fb, eng.kv).float()
            m.comm = fused
            torch.cuda.synchronize()
            e = ops.check_errors(dev)
            rel = ((a - b).norm() / b.norm()).item()
            if rank == 0:
                print(name, "decode B", B, "fused vs nccl rel", rel, "err", e, flush=True)
            ok = ok and rel < 2e-2 and e == 0
        eng._graphs.clear()
    if rank == 0 and ok:
        print("TP_FUSED_OK", flush=True)
    dist.barrier()
    dist.destroy_process_group()
    sys.exit(0 if ok else 1)


if __name__ == "__main__":
    main()
