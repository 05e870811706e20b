"""Engine worker: runs the serving engine in lockstep on every tensor-parallel rank.

Rank 0 owns the request queue.  Every iteration it drains newly submitted requests,
broadcasts them (with a stop flag) to the other ranks over a CPU (gloo) control
group, adds them to its engine and runs one engine step; the other ranks receive the
same message, add the same requests (with their sampling parameters) in the same order
and run the same step.  The scheduler is deterministic and the sampled tokens are
identical on every rank (the vocab-parallel argmax, or the sampler's per-rank
statistics, are all-gathered and every rank draws the same seeded noise), so the
engines stay in lockstep without any other coordination.  While idle, rank 0 sends an empty message every
``heartbeat_s`` so that the followers' blocking receive never hits the process-group
timeout.
"""
from __future__ import annotations

import itertools
import queue
import threading
import time
from concurrent.futures import Future
from dataclasses import dataclass, field

import torch.distributed as dist

from ..ops.sampling import SamplingParams


class Histogram:
    """Fixed-bucket histogram in the Prometheus form (cumulative bucket counts, sum, count):
    constant memory however long the server runs."""

    def __init__(self, bounds):
        self.bounds = list(bounds)
        self.counts = [0] * (len(self.bounds) + 1)  # last: +Inf
        self.sum = 0.0
        self.count = 0

    def observe(self, v: float) -> None:
        i = next((j for j, b in enumerate(self.bounds) if v <= b), len(self.bounds))
        self.counts[i] += 1
        self.sum += v
        self.count += 1

    @property
    def mean(self) -> float:
        return self.sum / max(1, self.count)

    def lines(self, name: str) -> list[str]:
        out, acc = [f"# TYPE {name} histogram"], 0
        for b, c in zip(self.bounds + ["+Inf"], self.counts):
            acc += c
            out.append(f'{name}_bucket{{le="{b}"}} {acc}')
        return out + [f"{name}_sum {self.sum}", f"{name}_count {self.count}"]


TTFT_BUCKETS = (0.01, 0.025, 0.05, 0.1, 0.25, 0.5, 1, 2.5, 5, 10, 25, 50, 100)
TPOT_BUCKETS = (0.001, 0.0025, 0.005, 0.0075, 0.01, 0.015, 0.02, 0.03, 0.05, 0.1, 0.25, 0.5)


@dataclass
class Metrics:
    requests: int = 0
    finished: int = 0
    tokens_out: int = 0
    ttft: Histogram = field(default_factory=lambda: Histogram(TTFT_BUCKETS))
    tpot: Histogram = field(default_factory=lambda: Histogram(TPOT_BUCKETS))
    finish_reasons: dict = field(default_factory=dict)
    accepted: dict = field(default_factory=dict)  # drafts accepted in a verify step -> count
    steps: int = 0
    started: float = field(default_factory=time.perf_counter)

    def snapshot(self, engine) -> dict:
        el = max(1e-9, time.perf_counter() - self.started)
        st = engine.stats
        acc = st.get("drafts_accepted", 0) / max(1, st.get("drafts_proposed", 0))
        return {"requests": self.requests, "finished": self.finished, "tokens_out": self.tokens_out,
                "tok_per_s": self.tokens_out / el, "steps": self.steps, "draft_acceptance": acc,
                "ttft_ms_mean": 1e3 * self.ttft.mean, "tpot_ms_mean": 1e3 * self.tpot.mean,
                "kv_blocks_free": engine.bm.free_blocks, "running": len(engine.running),
                "waiting": len(engine.waiting), "preempted": st.get("preempted", 0)}

    def exposition(self, engine) -> str:
        """Prometheus text: the snapshot as gauges, the latency histograms, finish reasons."""
        lines = [f"oscar_{k} {float(v)}" for k, v in self.snapshot(engine).items() if v is not None]
        lines += self.ttft.lines("oscar_ttft_seconds") + self.tpot.lines("oscar_tpot_seconds")
        lines.append("# TYPE oscar_finish_reason_total counter")
        lines += [f'oscar_finish_reason_total{{reason="{r}"}} {n}' for r, n in sorted(self.finish_reasons.items())]
        lines.append("# TYPE oscar_verify_steps_total counter")
        lines += [f'oscar_verify_steps_total{{accepted="{k}"}} {n}' for k, n in sorted(self.accepted.items())]
        return "\n".join(lines) + "\n"


class ControlChannel:
    """Broadcast of (new requests, aborted request ids, stop) from rank 0 over a gloo group."""

    def __init__(self, group=None, src: int = 0):
        self.group = group
        self.src = src

    @classmethod
    def create(cls, ranks=None):
        g = dist.new_group(ranks=ranks, backend="gloo")
        return cls(g, src=min(ranks) if ranks else 0)

    def exchange(self, msg=None):
        obj = [msg]
        dist.broadcast_object_list(obj, src=self.src, group=self.group)
        return obj[0]


def _settle(fut: Future, result=None, error: BaseException | None = None) -> None:
    """Resolves ``fut`` unless its consumer already cancelled it."""
    if fut.done():
        return
    try:
        if error is not None:
            fut.set_exception(error)
        else:
            fut.set_result(result)
    except Exception:  # noqa: BLE001 - cancelled concurrently
        pass


class EngineWorker:
    """Rank-0 side: thread-safe submission, background stepping, futures per request.

    A request's future resolves to its generated token ids (``fut.finish_reason`` is set
    first: ``"stop"``, ``"length"`` or ``"abort"``).  ``on_tokens(new_ids, finish_reason)``
    is called from the engine thread after every step that produced tokens for the
    request (``finish_reason`` None until the last call); :meth:`abort` ends a request
    between steps, on every rank."""

    def __init__(self, engine, control: ControlChannel | None = None, heartbeat_s: float = 1.0):
        self.engine = engine
        self.control = control
        self.heartbeat_s = heartbeat_s
        self.q: queue.Queue = queue.Queue()
        self.aborts: queue.Queue = queue.Queue()
        self.futures: dict[int, Future] = {}
        self.metrics = Metrics()
        self._stop = threading.Event()
        self._thread: threading.Thread | None = None
        self._last_msg = 0.0
        self._handles = itertools.count()
        self._rid_of: dict[int, int] = {}   # handle -> request id
        self._sent: dict[int, int] = {}     # request id -> tokens passed to on_tokens
        self.error: BaseException | None = None

    def submit(self, prompt: list[int], max_tokens: int, sampling=None, stop_ids=None, on_tokens=None,
               logprobs: int | None = None) -> Future:
        """Queues a request; ``sampling`` is a :class:`SamplingParams` (None: greedy),
        ``stop_ids`` token ids that end it.  The future has a ``handle`` for :meth:`abort`."""
        if self.error is not None:
            raise RuntimeError(f"engine worker failed: {self.error!r}")
        if sampling is not None:
            sampling.validate()
        self.engine.validate_request(prompt, max_tokens)  # raises here, not in the engine thread
        fut: Future = Future()
        fut.handle = next(self._handles)
        fut.finish_reason = None
        fut.on_tokens = on_tokens
        fut.logprobs = None
        self.q.put((list(map(int, prompt)), int(max_tokens), sampling,
                    tuple(int(t) for t in (stop_ids or ())), logprobs, fut))
        if self.error is not None:  # the loop died while this was being queued
            self._fail_queued(self.error)
        return fut

    def abort(self, fut: Future) -> None:
        """Ends the request of ``fut`` at the next step boundary (no effect once finished)."""
        self.aborts.put(fut.handle)

    def _fail_queued(self, err: BaseException) -> None:
        while True:
            try:
                *_, fut = self.q.get_nowait()
            except queue.Empty:
                return
            _settle(fut, error=err)

    def start(self) -> "EngineWorker":
        self._thread = threading.Thread(target=self._run, name="oscar-engine", daemon=True)
        self._thread.start()
        return self

    def stop(self, timeout: float = 30.0) -> None:
        self._stop.set()
        if self._thread is not None:
            self._thread.join(timeout)

    # -------------------------------------------------------------- loop
    def _drain(self, block: bool) -> list:
        items = []
        try:
            items.append(self.q.get(timeout=min(0.05, self.heartbeat_s)) if block else self.q.get_nowait())
            while True:
                items.append(self.q.get_nowait())
        except queue.Empty:
            pass
        return items

    def _take_aborts(self, new: list) -> tuple[list, list]:
        """Aborted handles -> (requests of this iteration still to add, request ids to abort)."""
        handles = set()
        while True:
            try:
                handles.add(self.aborts.get_nowait())
            except queue.Empty:
                break
        if not handles:
            return new, []
        keep = []
        for item in new:  # aborted before it was ever added: resolve it empty
            fut = item[-1]
            if fut.handle in handles:
                fut.finish_reason = "abort"
                if fut.on_tokens is not None:
                    try:
                        fut.on_tokens([], "abort")
                    except Exception:  # noqa: BLE001
                        pass
                _settle(fut, [])
            else:
                keep.append(item)
        rids = [self._rid_of[h] for h in handles if h in self._rid_of]
        return keep, rids

    def _run(self) -> None:
        eng = self.engine
        new: list = []
        try:
            while True:
                stop = self._stop.is_set()
                new = self._drain(block=not eng.has_work() and not stop and self.aborts.empty())
                new, aborts = self._take_aborts(new)
                now = time.perf_counter()
                if self.control is not None and (new or aborts or eng.has_work() or stop
                                                 or now - self._last_msg > self.heartbeat_s):
                    self.control.exchange(([(p, m, None if sp is None else sp.to_dict(), st, lp)
                                            for p, m, sp, st, lp, _ in new], aborts, stop))
                    self._last_msg = now
                if stop:
                    break
                for p, m, sp, st, lp, fut in new:
                    rid = eng.add_request(p, m, sp, st, lp)
                    self.futures[rid] = fut
                    self._rid_of[fut.handle] = rid
                    self.metrics.requests += 1
                new = []
                for rid in aborts:
                    eng.abort(rid)
                if eng.has_work():
                    eng.step()
                    self.metrics.steps += 1
                self._resolve()
        except BaseException as e:  # noqa: BLE001 - surfaced to every pending request
            self.error = e
            for fut in list(self.futures.values()) + [item[-1] for item in new]:
                _settle(fut, error=e)
            self._fail_queued(e)

    def _resolve(self) -> None:
        eng = self.engine
        for rid, fut in list(self.futures.items()):
            r = eng.requests[rid]
            cb = fut.on_tokens
            if cb is not None:
                sent = self._sent.get(rid, 0)
                if len(r.output) > sent or r.finished:
                    self._sent[rid] = len(r.output)
                    if r.logprobs is not None:  # what a streaming consumer reads for these tokens
                        fut.lp_live = list(r.lp)
                    try:
                        cb(list(r.output[sent:]), r.finish_reason if r.finished else None)
                    except Exception:  # noqa: BLE001 - a consumer that went away must not stop the engine
                        fut.on_tokens = None
            if not r.finished:
                continue
            out = r.output[:r.max_new_tokens]
            self.metrics.finished += 1
            self.metrics.tokens_out += len(out)
            if r.first_token_time is not None:
                self.metrics.ttft.observe(r.first_token_time - r.arrival)
                if len(out) > 1 and r.finish_time is not None:
                    self.metrics.tpot.observe((r.finish_time - r.first_token_time) / (len(out) - 1))
            fr = r.finish_reason or "unknown"
            self.metrics.finish_reasons[fr] = self.metrics.finish_reasons.get(fr, 0) + 1
            for k in r.accepted:  # the accepted-length histogram of MTP verification
                self.metrics.accepted[k] = self.metrics.accepted.get(k, 0) + 1
            self.futures.pop(rid)
            self._sent.pop(rid, None)
            self._rid_of.pop(fut.handle, None)
            fut.finish_reason = r.finish_reason
            fut.logprobs = list(r.lp) if r.logprobs is not None else None
            _settle(fut, out)
            eng.release(rid)


def follower_loop(engine, control: ControlChannel) -> None:
    """Ranks != 0: mirror rank 0's requests and steps until it says stop."""
    while True:
        new, aborts, stop = control.exchange(None)
        if stop:
            return
        for p, m, sp, st, lp in new:
            engine.add_request(p, m, None if sp is None else SamplingParams(**sp), st, lp)
        for rid in aborts:
            engine.abort(rid)
        if engine.has_work():
            engine.step()
            for rid in [rid for rid, r in engine.requests.items() if r.finished]:
                engine.release(rid)
