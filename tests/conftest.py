import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 GPU (sm_100a)")
    config.addinivalue_line("markers", "multigpu: needs two or more CUDA GPUs")
    config.addinivalue_line("markers", "slow: long-running test")
    _ensure_host_extension()


def _ensure_host_extension():
    """The C++ runtime core (page allocator, block registry) is CPU-only and
    every engine test needs it; build it in-tree when a fresh checkout has
    none yet.  The CUDA extension is never built here: GPU tests expect it
    prebuilt and fail loudly without it."""
    from sglang_legolink_b200.ops import _ext

    if not _ext.so_path("legolink_host"):
        from sglang_legolink_b200 import build_ext

        build_ext.build_host()


def pytest_collection_modifyitems(config, items):
    import torch

    have_gpu = torch.cuda.is_available()
    ngpu = torch.cuda.device_count() if have_gpu else 0
    for item in items:
        if "gpu" in item.keywords and not have_gpu:
            item.add_marker(pytest.mark.skip(reason="no CUDA device"))
        if "multigpu" in item.keywords and ngpu < 2:
            item.add_marker(pytest.mark.skip(reason="needs >= 2 CUDA devices"))
