"""Writes ``core_golden.json``: the reference core's traces (``tests/core_traces.py``), from the unmodified reference
installed under ``baseline/_ref``.

    python tests/golden/make_core_golden.py
"""

import json
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.dirname(HERE))
sys.path.insert(0, ROOT)

import core_traces  # noqa: E402


def main() -> None:
    import logging

    logging.disable(logging.WARNING)  # the cost model warns about clamped contexts on these synthetic tables
    ref = core_traces.reference(os.path.join(ROOT, "baseline", "_ref"))
    if ref is None:
        raise SystemExit("the reference is not installed under baseline/_ref")
    traces = core_traces.all_traces(ref)
    with open(os.path.join(HERE, "core_golden.json"), "w", encoding="utf-8") as f:
        json.dump(traces, f, sort_keys=True, separators=(",", ":"))
        f.write("\n")
    print("wrote", len(traces), "traces")


if __name__ == "__main__":
    main()
