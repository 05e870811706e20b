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

import queue
import threading
import time
from concurrent.futures import Future
from dataclasses import dataclass, field

import torch.distributed as dist

from ..ops.sampling import SamplingParams


@dataclass
class Metrics:
    requests: int = 0
    finished: int = 0
    tokens_out: int = 0
    ttft_s: list = field(default_factory=list)
    tpot_s: list = field(default_factory=list)
    steps: int = 0
    started: float = field(default_factory=time.perf_counter)

    def snapshot(self, engine) -> dict:
        el = max(1e-9, time.perf_counter() - self.started)
        st = engine.stats
        acc = st.get("drafts_accepted", 0) / max(1, st.get("drafts_proposed", 0))
        return {"requests": self.requests, "finished": self.finished, "tokens_out": self.tokens_out,
                "tok_per_s": self.tokens_out / el, "steps": self.steps, "draft_acceptance": acc,
                "ttft_ms_mean": 1e3 * sum(self.ttft_s) / max(1, len(self.ttft_s)),
                "tpot_ms_mean": 1e3 * sum(self.tpot_s) / max(1, len(self.tpot_s)),
                "kv_blocks_free": engine.bm.free_blocks}


class ControlChannel:
    """Broadcast of (new requests, stop) from rank 0 over a gloo group."""

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


class EngineWorker:
    """Rank-0 side: thread-safe submission, background stepping, futures per request."""

    def __init__(self, engine, control: ControlChannel | None = None, heartbeat_s: float = 1.0):
        self.engine = engine
        self.control = control
        self.heartbeat_s = heartbeat_s
        self.q: queue.Queue = queue.Queue()
        self.futures: dict[int, Future] = {}
        self.metrics = Metrics()
        self._stop = threading.Event()
        self._thread: threading.Thread | None = None
        self._last_msg = 0.0
        self.error: BaseException | None = None

    def submit(self, prompt: list[int], max_tokens: int, sampling=None) -> Future:
        """Queues a request; ``sampling`` is a :class:`SamplingParams` (None: greedy)."""
        if self.error is not None:
            raise RuntimeError(f"engine worker failed: {self.error!r}")
        if sampling is not None:
            sampling.validate()
        fut: Future = Future()
        self.q.put((list(map(int, prompt)), int(max_tokens), sampling, fut))
        if self.error is not None:  # the loop died while this was being queued
            self._fail_queued(self.error)
        return fut

    def _fail_queued(self, err: BaseException) -> None:
        while True:
            try:
                *_, fut = self.q.get_nowait()
            except queue.Empty:
                return
            if not fut.done():
                fut.set_exception(err)

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

    def _run(self) -> None:
        eng = self.engine
        new: list = []
        try:
            while True:
                stop = self._stop.is_set()
                new = self._drain(block=not eng.has_work() and not stop)
                now = time.perf_counter()
                if self.control is not None and (new or eng.has_work() or stop or now - self._last_msg > self.heartbeat_s):
                    self.control.exchange(([(p, m, None if sp is None else sp.to_dict()) for p, m, sp, _ in new],
                                           stop))
                    self._last_msg = now
                if stop:
                    break
                for p, m, sp, fut in new:
                    rid = eng.add_request(p, m, sp)
                    self.futures[rid] = fut
                    self.metrics.requests += 1
                new = []
                if eng.has_work():
                    eng.step()
                    self.metrics.steps += 1
                    self._resolve()
        except BaseException as e:  # noqa: BLE001 - surfaced to every pending request
            self.error = e
            for fut in list(self.futures.values()) + [item[-1] for item in new]:
                if not fut.done():
                    fut.set_exception(e)
            self._fail_queued(e)

    def _resolve(self) -> None:
        eng = self.engine
        done = [rid for rid, f in self.futures.items() if eng.requests[rid].finished]
        for rid in done:
            r = eng.requests[rid]
            out = r.output[:r.max_new_tokens]
            self.metrics.finished += 1
            self.metrics.tokens_out += len(out)
            if r.first_token_time is not None:
                self.metrics.ttft_s.append(r.first_token_time - r.arrival)
                if len(out) > 1 and r.finish_time is not None:
                    self.metrics.tpot_s.append((r.finish_time - r.first_token_time) / (len(out) - 1))
            self.futures.pop(rid).set_result(out)
            eng.release(rid)


def follower_loop(engine, control: ControlChannel) -> None:
    """Ranks != 0: mirror rank 0's requests and steps until it says stop."""
    while True:
        new, stop = control.exchange(None)
        if stop:
            return
        for p, m, sp in new:
            engine.add_request(p, m, None if sp is None else SamplingParams(**sp))
        if engine.has_work():
            engine.step()
            for rid in [rid for rid, r in engine.requests.items() if r.finished]:
                engine.release(rid)
