"""Validate the READY manifests in a serve log: ``python -m oscar_b200.serve.check_ready LOG``.

Same checks as the reference's ``delivery/check_ready.py:8-29``: every tensor-parallel
rank reported, all ranks carry the same FULL-layer set, and all run the same source
(optionally a given sha256, or ``--sha256 auto`` for this checkout's fingerprint).
"""
from __future__ import annotations

import argparse
import sys

from ..engine.budget import BudgetError, parse_ready_lines, source_fingerprint, validate


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("log")
    ap.add_argument("--world", type=int, default=None)
    ap.add_argument("--sha256", default=None)
    args = ap.parse_args(argv)
    with open(args.log, errors="replace") as f:
        mans = parse_ready_lines(f.read())
    sha = source_fingerprint() if args.sha256 == "auto" else args.sha256
    try:
        validate(mans, world_size=args.world, sha256=sha)
    except BudgetError as e:
        print(f"NOT READY: {e}")
        return 1
    print(f"READY: {len(mans)} rank(s), layers {mans[0]['layer_ids']}, source {mans[0]['sha256'][:12]}")
    return 0


if __name__ == "__main__":
    sys.exit(main())
