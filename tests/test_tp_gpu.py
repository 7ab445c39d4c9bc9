"""TP=2 on two GPUs (collective-library baseline): logits match the
unsharded model and both ranks decode the same tokens after a Link."""

import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.gpu
@pytest.mark.multigpu
def test_tp2_gpu():
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr=127.0.0.1", "--master-port=29534",
           os.path.join(ROOT, "tests", "tp_worker.py")]
    r = subprocess.run(cmd, capture_output=True, text=True, env={**os.environ, "NCCL_NVLS_ENABLE": "0"})
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert "TP_OK" in r.stdout


@pytest.mark.gpu
@pytest.mark.multigpu
def test_tp2_fused_gpu():
    """Fused TP path (reduce-scatter in the GEMM epilogue, all-gather in the
    norm kernel, over NVLink peer stores) matches the NCCL path."""
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr=127.0.0.1", "--master-port=29538",
           os.path.join(ROOT, "tests", "tp_fused_worker.py")]
    env = {**os.environ, "NCCL_NVLS_ENABLE": "0", "TORCH_SYMM_MEM_DISABLE_MULTICAST": "1"}
    r = subprocess.run(cmd, capture_output=True, text=True, env=env)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert "TP_FUSED_OK" in r.stdout


@pytest.mark.gpu
@pytest.mark.multigpu
def test_tp2_fused_nvls_gpu():
    """The same checks with multicast available: the decode boundary reads
    the ranks' partial rows through NVLS multimem loads (no rank is lost in
    this test)."""
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr=127.0.0.1", "--master-port=29542",
           os.path.join(ROOT, "tests", "tp_fused_worker.py")]
    env = {k: v for k, v in os.environ.items() if k != "TORCH_SYMM_MEM_DISABLE_MULTICAST"}
    env["SGLANG_PIC_TP_NVLS"] = "1"
    r = subprocess.run(cmd, capture_output=True, text=True, env=env)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert "TP_FUSED_OK" in r.stdout

