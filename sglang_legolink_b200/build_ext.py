"""Build the in-tree native extensions.

* ``legolink_cuda`` -- every sm_100a kernel (``csrc/*.cu``) plus the torch
  bindings, compiled with ``-gencode arch=compute_100a,code=sm_100a``.
* ``legolink_host`` -- the C++ runtime core (page allocator, block registry,
  radix prefix index, scheduler admission), CPU only.

Both land in ``sglang_legolink_b200/_ext/<name>/<name>.so`` and are imported
from there by path (``sglang_legolink_b200.ops._ext``), so a prebuilt tree
travels to another machine and is never rebuilt at import time.

Usage: ``python -m sglang_legolink_b200.build_ext [cuda|host|all]``.
"""

from __future__ import annotations

import os
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(PKG, "csrc")
EXT_DIR = os.path.join(PKG, "_ext")

CUDA_SOURCES = [
    "bindings.cpp",
    "gemm_tcgen05.cu",
    "elementwise.cu",
    "attention.cu",
    "attention_tc.cu",
    "gemm_small_m_noalloc.cu",
    "tp_fused.cu",
]
HOST_SOURCES = ["host_runtime.cpp"]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "--expt-relaxed-constexpr",
    "-U__CUDA_NO_HALF_OPERATORS__", "-U__CUDA_NO_HALF_CONVERSIONS__",
    "-U__CUDA_NO_BFLOAT16_CONVERSIONS__", "-U__CUDA_NO_BFLOAT162_OPERATORS__",
]


def _load(name: str, sources: list[str], cuda: bool, verbose: bool = False):
    from torch.utils.cpp_extension import load

    build_dir = os.path.join(EXT_DIR, name)
    os.makedirs(build_dir, exist_ok=True)
    kw = dict(
        name=name,
        sources=[os.path.join(CSRC, s) for s in sources],
        build_directory=build_dir,
        extra_cflags=["-O3", "-std=c++17"],
        verbose=verbose,
    )
    if cuda:
        # Only sm_100a: keep torch from adding its own arch list.
        os.environ["TORCH_CUDA_ARCH_LIST"] = "10.0a"
        kw["extra_cuda_cflags"] = NVCC_FLAGS
        kw["extra_include_paths"] = [CSRC]
    else:
        kw["with_cuda"] = False
    return load(**kw)


def build_cuda(verbose: bool = False):
    os.environ.setdefault("MAX_JOBS", str(max(1, (os.cpu_count() or 4))))
    return _load("legolink_cuda", CUDA_SOURCES, cuda=True, verbose=verbose)


def build_host(verbose: bool = False):
    return _load("legolink_host", HOST_SOURCES, cuda=False, verbose=verbose)


def build_all(verbose: bool = False) -> None:
    build_host(verbose)
    build_cuda(verbose)


if __name__ == "__main__":
    what = sys.argv[1] if len(sys.argv) > 1 else "all"
    v = "-v" in sys.argv
    if what in ("host", "all"):
        build_host(v)
    if what in ("cuda", "all"):
        build_cuda(v)
    print("built", what)
