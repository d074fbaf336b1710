"""Command line: ``python -m braidinfer_b200.utils.check_compatibility_cli MODEL [-v] [--threshold S] [--export F]``.

Exit codes as in ``braidinfer/utils/check_compatibility_cli.py:24-162``:
0 compatible, 1 warning, 2 incompatible, 3 error.  ``--threshold`` overrides
the score below which the model is reported incompatible.
"""
from __future__ import annotations

import argparse
import sys

from .kernel_compatibility import (FusedKernelCompatibilityChecker, export_json,
                                   generate_compatibility_report)


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description="Check q/k-norm weight ranges of a checkpoint")
    ap.add_argument("model", help="checkpoint directory (HF layout)")
    ap.add_argument("-v", "--verbose", action="store_true")
    ap.add_argument("--threshold", type=float, default=None, help="incompatible below this score (default 0.5)")
    ap.add_argument("--export", default=None, help="write the result as JSON")
    a = ap.parse_args(argv)
    try:
        res = FusedKernelCompatibilityChecker().check_model(a.model, a.model)
    except Exception as e:  # noqa: BLE001 - reported as exit code 3
        print(f"error: {e}", file=sys.stderr)
        return 3
    if a.threshold is not None:
        res.status = "INCOMPATIBLE" if res.score < a.threshold else res.status
    print(generate_compatibility_report(res, a.model, a.verbose))
    if a.export:
        export_json(res, a.export)
    return {"COMPATIBLE": 0, "WARNING": 1, "INCOMPATIBLE": 2}[res.status]


if __name__ == "__main__":
    sys.exit(main())
