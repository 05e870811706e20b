"""Per-kernel device-time breakdown of a few engine steps, one file per rank.

Runs a callable under ``torch.profiler`` (CUPTI kernel activity, which also sees the
kernels of replayed CUDA graphs and NCCL's kernels) and sums device time per kernel
name.  Numbers taken under the profiler are for shares only, never a benchmark value:
CUPTI adds a little time per launch.  Every rank writes ``{prefix}.rank{r}.json``::

    {"rank": r, "steps": n, "total_us": ..., "kernels": [[name, count, us], ...]}

so that the collective kernels of a tensor-parallel step can be compared with the
compute kernels of the same rank, and the max over ranks taken by the reader.
"""
from __future__ import annotations

import json
from collections import defaultdict


def _short(name: str) -> str:
    """Kernel name without ``void`` and the argument list (template arguments kept)."""
    if name.startswith("void "):
        name = name[5:]
    name = name.replace("(anonymous namespace)::", "")
    i = name.find("(")
    if i > 0:
        name = name[:i]
    return name[:120]


def profile_steps(fn, steps: int, prefix: str, rank: int) -> dict:
    """Run ``fn()`` ``steps`` times under the profiler; write and return the summary.

    The caller runs the steps eagerly (CUDA graphs off): replays of graphs that were
    captured before the profiler started are not traced reliably; the eager steps launch
    the same kernels."""
    import torch
    from torch.profiler import ProfilerActivity, profile

    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA], record_shapes=False) as prof:
        for _ in range(steps):
            fn()
        torch.cuda.synchronize()
    agg: dict = defaultdict(lambda: [0, 0.0])
    for ev in prof.key_averages():
        us = float(getattr(ev, "self_device_time_total", 0.0) or 0.0)
        if us > 0:
            a = agg[_short(ev.key)]
            a[0] += int(ev.count)
            a[1] += us
    rows = sorted(([k, v[0], round(v[1], 1)] for k, v in agg.items()), key=lambda r: -r[2])
    out = {"rank": rank, "steps": steps, "total_us": round(sum(r[2] for r in rows), 1), "kernels": rows}
    with open(f"{prefix}.rank{rank}.json", "w") as f:
        json.dump(out, f, indent=0)
    return out
