"""Validate JSON files against one of the wire schemas.

    python -m sglang_legolink_b200.schemas <schema> FILE [FILE ...]

A ``.jsonl`` file is checked line by line (blank lines skipped); any other
file holds one JSON document.  Prints one line per violation and exits 1 if
there was any, else prints ``ok <count>`` and exits 0.
"""

from __future__ import annotations

import json
import sys

from . import SCHEMA_NAMES, errors


def main(argv=None) -> int:
    argv = list(sys.argv[1:] if argv is None else argv)
    if len(argv) < 2 or argv[0] not in SCHEMA_NAMES:
        print(f"usage: python -m sglang_legolink_b200.schemas {{{','.join(SCHEMA_NAMES)}}} FILE [FILE ...]",
              file=sys.stderr)
        return 2
    name, bad, count = argv[0], 0, 0
    for path in argv[1:]:
        with open(path, encoding="utf-8") as f:
            docs = ([(i + 1, line) for i, line in enumerate(f) if line.strip()] if path.endswith(".jsonl")
                    else [(0, f.read())])
        for lineno, text in docs:
            count += 1
            where = f"{path}:{lineno}" if lineno else path
            try:
                obj = json.loads(text)
            except json.JSONDecodeError as e:
                print(f"{where}: not JSON ({e.msg})")
                bad += 1
                continue
            for e in errors(name, obj):
                print(f"{where}: {'/'.join(map(str, e.absolute_path)) or '<root>'}: {e.message}")
                bad += 1
    if bad:
        return 1
    print(f"ok {count}")
    return 0


if __name__ == "__main__":
    sys.exit(main())
