"""Source rules of this repository, checked on every run (CPU):

* nothing committed imports, reads or runs the scratch directory;
* none of the batched-copy runtime/driver calls that are closed on this GPU
  pool appears anywhere (their names are assembled here, not spelled);
* comments and docstrings name no build notes file and no machine path.
"""

import re
import subprocess
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent
SELF = Path(__file__).resolve()


def _sources(*suffixes):
    out = subprocess.run(["git", "ls-files"], cwd=ROOT, capture_output=True, text=True).stdout.split()
    files = [ROOT / f for f in out if f.endswith(suffixes)]
    if not files:  # not a git checkout (an exported snapshot): walk the package and tests
        files = [p for d in ("sglang_legolink_b200", "tests") for p in (ROOT / d).rglob("*") if p.suffix in suffixes]
        files += [ROOT / "bench.py", ROOT / "__graft_entry__.py"]
    return [f for f in files if f.exists() and f.resolve() != SELF]


def test_no_committed_code_uses_the_scratch_directory():
    pat = re.compile(r"""(['"/]_work[/'"]|import\s+_work|from\s+_work)""")
    bad = [str(f.relative_to(ROOT)) for f in _sources(".py", ".sh", ".cu", ".cpp") if pat.search(f.read_text())]
    assert not bad, bad


def test_closed_batched_copy_calls_are_absent():
    names = [p + "Memcpy" + d + "Batch" + "Async" for p in ("cuda", "cu") for d in ("", "3D")]
    bad = [f"{f.relative_to(ROOT)}: {n}" for f in _sources(".py", ".cu", ".cuh", ".h", ".cpp", ".sh")
           for n in names if n in f.read_text()]
    assert not bad, bad


def test_sources_name_no_notes_file_or_machine_path():
    notes = ["SUR" + "VEY", "DES" + "IGN.md", "VER" + "DICT", "ADV" + "ICE.md", "BASE" + "LINE.md"]
    bad = []
    for f in _sources(".py", ".cu", ".cuh", ".h", ".cpp"):
        text = f.read_text()
        for n in notes + ["/ro" + "ot/"]:
            if n in text:
                bad.append(f"{f.relative_to(ROOT)}: {n}")
    assert not bad, bad


def test_benchmark_modules_import_and_share_the_headline_workload():
    """Every benchmark module with a ``main`` imports on CPU (``ncu_cases``
    is a script that runs its case on import), and the library-baseline
    bench builds the same Link layout as the headline bench (5087 repair rows
    of a 16416-token request)."""
    import importlib
    import sys

    sys.path.insert(0, str(ROOT))
    pkg = ROOT / "sglang_legolink_b200" / "benchmarks"
    for f in sorted(pkg.glob("*.py")):
        if f.stem != "__init__" and "def main(" in f.read_text():
            importlib.import_module(f"sglang_legolink_b200.benchmarks.{f.stem}")
    from sglang_legolink_b200.benchmarks.baselines import link_workload

    plan = link_workload()
    assert len(plan.recompute_positions) == 5087 and plan.total_token_count == 16416
