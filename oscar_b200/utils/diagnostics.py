"""Opt-in per-stage PERF capture of the serving engine.

Behaviour follows the reference's diagnostics (``oscar_ascend/diagnostics.py:36-267``):

* enabled by ``OSCAR_ASCEND_PROFILE_STEPS=N`` (> 0), on rank 0 only; nothing is
  wrapped otherwise;
* only the first ``N`` steps whose schedule matches the filters are captured:
  ``OSCAR_ASCEND_PROFILE_MIN_REQUESTS`` (at least that many requests in the step) and
  ``OSCAR_ASCEND_PROFILE_MAX_TOKENS_PER_REQUEST`` (no request with more tokens), 0
  meaning "no filter";
* every hooked stage records inclusive, device-synchronised wall time: the time spent
  draining earlier GPU work before the stage (``wait_before_ms``), the first and the
  largest duration and the sum; ``OSCAR_PROFILE_TIMER=events`` instead brackets each
  stage with CUDA events and an NVTX range (no synchronisation inside the step);
* a ``TorchDispatchMode`` counts ``aten::sort``/``argsort`` calls inside the step and
  keeps the Python stacks of integer-dtype sorts (the reference hunted host-visible
  integer sorts on the serving path);
* the code identity of the engine step is the sha256 of its marshalled code object;
* each captured step prints one ``[oscar-b200] PERF {json}`` line.

Capturing synchronises the device around every stage, so CUDA-graph replay is
turned off for the engine while diagnostics are installed.
"""
from __future__ import annotations

import hashlib
import json
import marshal
import os
import time
import traceback
from contextlib import contextmanager
from dataclasses import dataclass, field

import torch
from torch.utils._python_dispatch import TorchDispatchMode

PREFIX = "[oscar-b200] PERF "


def _env_int(name: str) -> int:
    try:
        return int(os.environ.get(name, "0") or 0)
    except ValueError:
        return 0


@dataclass
class Record:
    """Inclusive timings of one stage within a captured step."""

    count: int = 0
    total_ms: float = 0.0
    first_ms: float = -1.0
    max_ms: float = 0.0
    wait_before_ms: float = 0.0

    def add(self, ms: float, wait_ms: float) -> None:
        self.count += 1
        self.total_ms += ms
        if self.first_ms < 0:
            self.first_ms = ms
        self.max_ms = max(self.max_ms, ms)
        self.wait_before_ms += wait_ms

    def as_dict(self) -> dict:
        return {"count": self.count, "ms": round(self.total_ms, 4), "first_ms": round(self.first_ms, 4),
                "max_ms": round(self.max_ms, 4), "wait_before_ms": round(self.wait_before_ms, 4)}


class SortTrace(TorchDispatchMode):
    """Counts sort/argsort ops; keeps the stacks of integer-dtype sorts."""

    _SORTS = ("sort", "argsort")

    def __init__(self, max_stacks: int = 8):
        super().__init__()
        self.count = 0
        self.int_count = 0
        self.stacks: list[str] = []
        self.max_stacks = max_stacks

    def __torch_dispatch__(self, func, types, args=(), kwargs=None):
        name = func.overloadpacket.__name__ if hasattr(func, "overloadpacket") else str(func)
        if name in self._SORTS or name.startswith("sort"):
            self.count += 1
            x = args[0] if args else None
            if isinstance(x, torch.Tensor) and not x.is_floating_point():
                self.int_count += 1
                if len(self.stacks) < self.max_stacks:
                    self.stacks.append("".join(traceback.format_stack(limit=8)[:-1]))
        return func(*args, **(kwargs or {}))


@dataclass
class Diagnostics:
    steps: int = 0
    min_requests: int = 0
    max_tokens_per_request: int = 0
    rank: int = 0
    sink: object = None  # callable(str) for the PERF lines (default: print)
    captured: int = 0
    seen: int = 0
    lines: list = field(default_factory=list)
    _stages: dict | None = None
    _last_end: float = 0.0
    code_sha256: str | None = None
    mode: str = "sync"  # "sync" | "events" (CUDA events + NVTX, no syncs in the step)
    _pending: list = field(default_factory=list)

    @classmethod
    def from_env(cls, rank: int = 0, sink=None) -> "Diagnostics":
        return cls(steps=_env_int("OSCAR_ASCEND_PROFILE_STEPS"),
                   min_requests=_env_int("OSCAR_ASCEND_PROFILE_MIN_REQUESTS"),
                   max_tokens_per_request=_env_int("OSCAR_ASCEND_PROFILE_MAX_TOKENS_PER_REQUEST"),
                   rank=rank, sink=sink, mode=os.environ.get("OSCAR_PROFILE_TIMER", "sync"))

    @property
    def enabled(self) -> bool:
        return self.steps > 0 and self.rank == 0

    # ------------------------------------------------------------ filters
    def matches(self, shape: dict) -> bool:
        if self.captured >= self.steps:
            return False
        if self.min_requests and shape["requests"] < self.min_requests:
            return False
        if self.max_tokens_per_request and shape["max_tokens_per_request"] > self.max_tokens_per_request:
            return False
        return True

    # ------------------------------------------------------------ stage timing
    @staticmethod
    def _sync():
        if torch.cuda.is_available() and torch.cuda.is_initialized():
            torch.cuda.synchronize()

    @contextmanager
    def timed(self, name: str):
        """Inclusive timing of a stage (no-op outside a captured step).

        ``mode == "sync"`` (default, and always on the CPU): device-synchronised wall
        time, with the time spent draining earlier work as ``wait_before_ms``.
        ``mode == "events"`` on CUDA: CUDA events around the stage on the current stream
        and an NVTX range, no synchronisation inside the step; resolved after the step.
        """
        if self._stages is None:
            yield
            return
        if self.mode == "events" and torch.cuda.is_available() and torch.cuda.is_initialized():
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            torch.cuda.nvtx.range_push(name)
            s.record()
            try:
                yield
            finally:
                e.record()
                torch.cuda.nvtx.range_pop()
                self._pending.append((name, s, e))
            return
        t0 = time.perf_counter()
        self._sync()
        t1 = time.perf_counter()
        try:
            yield
        finally:
            self._sync()
            t2 = time.perf_counter()
            self._stages.setdefault(name, Record()).add((t2 - t1) * 1e3, (t1 - t0) * 1e3)

    def wrap(self, obj, attr: str, stage: str) -> None:
        """Replace ``obj.attr`` by a timed wrapper (instance attribute)."""
        fn = getattr(obj, attr)
        diag = self

        def wrapped(*a, **k):
            with diag.timed(stage):
                return fn(*a, **k)

        wrapped.__wrapped__ = fn
        setattr(obj, attr, wrapped)

    # ------------------------------------------------------------ step capture
    def capture_step(self, step_fn, shape: dict):
        """Run ``step_fn()``; when the step matches, time it and emit a PERF line."""
        self.seen += 1
        if not self.matches(shape):
            return step_fn()
        if self.code_sha256 is None:
            code = getattr(step_fn, "__code__", None) or getattr(getattr(step_fn, "__func__", None), "__code__", None)
            if code is not None:
                self.code_sha256 = hashlib.sha256(marshal.dumps(code)).hexdigest()
        self._stages = {}
        trace = SortTrace()
        t0 = time.perf_counter()
        try:
            with trace, self.timed("step"):
                out = step_fn()
        finally:
            stages, self._stages = self._stages, None  # context always reset, also on exceptions
            if self._pending:
                torch.cuda.synchronize()
                for name, s, e in self._pending:
                    stages.setdefault(name, Record()).add(s.elapsed_time(e), 0.0)
                self._pending = []
        self.captured += 1
        rec = {"step": self.seen, "shape": shape, "wall_ms": round((time.perf_counter() - t0) * 1e3, 4),
               "stages": {k: v.as_dict() for k, v in stages.items()},
               "sorts": trace.count, "int_sorts": trace.int_count, "int_sort_stacks": trace.stacks,
               "code_sha256": self.code_sha256}
        line = PREFIX + json.dumps(rec, sort_keys=True)
        self.lines.append(line)
        (self.sink or print)(line)
        return out


def scheduled_shape(sched) -> dict:
    """Shape of a step's schedule ``[(rid, kind, n_tokens), ...]``."""
    toks = [n for _, _, n in sched]
    return {"requests": len(sched), "tokens": int(sum(toks)), "max_tokens_per_request": int(max(toks, default=0)),
            "prefill": sum(1 for _, k, _ in sched if k == "prefill")}


def install(engine, diag: Diagnostics | None = None) -> Diagnostics | None:
    """Hook an :class:`~oscar_b200.engine.engine.LLMEngine` (no-op when disabled)."""
    diag = diag or Diagnostics.from_env(rank=getattr(engine.model.tp, "rank", 0) if hasattr(engine.model, "tp") else 0)
    if not diag.enabled:
        return None
    engine.use_graphs = False
    model = engine.model
    diag.wrap(model, "forward", "forward")
    for mixer, mlp in model.layers:
        if hasattr(mixer, "attention"):
            diag.wrap(mixer, "attention", "full_attention")
        else:
            diag.wrap(mixer, "mixer", "gdn")
    if getattr(model, "mtp", None) is not None:
        diag.wrap(model.mtp, "forward", "mtp_draft")
    diag.wrap(model, "sample", "sample")
    step = engine.step
    sched_fn = engine._schedule

    def hooked_step():
        sched = sched_fn()
        shape = scheduled_shape(sched)
        engine._schedule = lambda: sched  # the step runs exactly this schedule
        try:
            return diag.capture_step(step, shape)
        finally:
            engine._schedule = sched_fn

    engine.step = hooked_step
    engine.diagnostics = diag
    return diag
