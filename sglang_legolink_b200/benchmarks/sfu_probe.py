"""Throughput of the softmax building blocks (exp2 on MUFU, the polynomial
exp2 on the FMA/ALU pipes, the bf16x2 pack, and their mixes), element-ops
per clock per SM, one JSON line per (mode, threads per block).

    python -m sglang_legolink_b200.benchmarks.sfu_probe

Compiles ``sfu_probe.cu`` (next to this file) with nvcc for sm_100a into a
temporary directory and runs it on GPU 0.
"""

from __future__ import annotations

import os
import subprocess
import sys
import tempfile

HERE = os.path.dirname(os.path.abspath(__file__))


def main() -> int:
    with tempfile.TemporaryDirectory() as d:
        exe = os.path.join(d, "sfu_probe")
        subprocess.run(["nvcc", "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-std=c++17",
                        os.path.join(HERE, "sfu_probe.cu"), "-o", exe], check=True)
        return subprocess.run([exe]).returncode


if __name__ == "__main__":
    sys.exit(main())
