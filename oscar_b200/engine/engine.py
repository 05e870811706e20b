"""Serving engine: continuous batching, chunked prefill, MTP speculative decoding.

One ``LLMEngine`` drives one tensor-parallel model replica (every rank of the TP
group runs the same engine loop on identical host state; only rank 0 reports).
A step:

1. schedules verify groups (``1 + num_spec`` tokens) for decoding requests and
   prefill chunks (FCFS) within ``max_batched_tokens`` (15,360 by default, the
   reference's packed serve setting ``delivery/serve_oscar.sh:64-74``);
2. builds all step metadata on the host (block tables, slots, staging seat plan,
   attention work list, GDN commit counts) and uploads it once;
3. runs the main model, verifies drafts (greedy, a seeded acceptance pattern, or, for
   requests with sampling parameters, exact speculative sampling: see
   :mod:`oscar_b200.ops.sampling`), then runs the MTP head over the step's rows and
   chains ``num_spec - 1`` more single-token draft passes.

The GDN layers use deferred commit (see :mod:`oscar_b200.ops.gdn`), so a rejected
draft costs no state rollback; FULL-layer KV of rejected positions is simply
overwritten by the next step.
"""
from __future__ import annotations

import itertools
import os
import time
from dataclasses import dataclass, field

import numpy as np
import torch

from ..kv.offload import HostKVStore
from ..models.qwen35 import P_MAX, HybridModel, StepBatch
from ..ops import attention as A
from ..ops.functional import num_sms, reserve_split_workspace
from ..ops import sampling as samp
from . import checks
from .block_manager import BlockManager, SlotManager
from .staging import seat_plan
from ..kv.oracle import window_row
from ..utils import launches as _launches


@dataclass
class Request:
    rid: int
    prompt: list
    max_new_tokens: int
    output: list = field(default_factory=list)
    num_computed: int = 0          # positions whose KV / state are final
    last_token: int | None = None  # token at position num_computed (next to feed)
    drafts: list = field(default_factory=list)
    pending_commit: int = 0
    slot: int = -1
    arrival: float = 0.0
    first_token_time: float | None = None
    finish_time: float | None = None
    accepted: list = field(default_factory=list)
    sampling: samp.SamplingParams | None = None  # None or temperature 0: greedy
    seed: int = 0
    stop_ids: frozenset = frozenset()  # generating one of these ends the request (it is kept)
    stopped: bool = False
    aborted: bool = False
    logprobs: int | None = None  # report the k most likely tokens per output token (0: the token's only)
    lp: list = field(default_factory=list)  # per output token: (logprob, [(id, logprob), ...])

    @property
    def prefill_done(self) -> bool:
        return self.num_computed >= len(self.prompt)

    @property
    def finished(self) -> bool:
        return self.stopped or self.aborted or len(self.output) >= self.max_new_tokens

    @property
    def finish_reason(self) -> str | None:
        """``"stop"`` (a stop token), ``"length"`` (max_new_tokens), ``"abort"``, or None."""
        if self.aborted:
            return "abort"
        if self.stopped:
            return "stop"
        return "length" if len(self.output) >= self.max_new_tokens else None

    def emit(self, tokens: list) -> int:
        """Appends generated tokens up to the first stop token or max_new_tokens; returns
        how many were kept."""
        n = 0
        for t in tokens:
            if len(self.output) >= self.max_new_tokens or self.stopped:
                break
            self.output.append(t)
            n += 1
            if t in self.stop_ids:
                self.stopped = True
        return n


class SeededAcceptance:
    """Deterministic acceptance pattern: accepted drafts per (request, step) ~ target mean."""

    def __init__(self, num_spec: int, mean_accepted: float, seed: int = 0):
        self.k = num_spec
        p = min(max(mean_accepted / num_spec, 0.0), 1.0)
        self.rng = np.random.default_rng(seed)
        self.p = p

    def __call__(self, rid: int) -> int:
        return int(self.rng.binomial(self.k, self.p))


class LLMEngine:
    def __init__(self, model: HybridModel, num_blocks: int, max_slots: int, max_batched_tokens: int = 15360,
                 num_spec: int = 3, acceptance: SeededAcceptance | None = None, prefill_policy: str = "fcfs",
                 timer=time.perf_counter, offload: bool = False, seed: int = 0):
        self.model = model
        self.seed = int(seed)  # seeds the sampled requests that bring no seed of their own
        self.dev = model.device
        self.num_spec = num_spec if model.mtp is not None else 0
        self.bm = BlockManager(num_blocks)
        self.slots = SlotManager(max_slots)
        self.max_batched_tokens = max_batched_tokens
        self.acceptance = acceptance
        self.prefill_policy = prefill_policy
        self.requests: dict[int, Request] = {}
        self.waiting: list[int] = []
        self.running: list[int] = []
        self.finished: list[int] = []
        self._ids = itertools.count()
        self.timer = timer
        self.stats = {"steps": 0, "tokens_out": 0, "drafts_proposed": 0, "drafts_accepted": 0}
        # device-busy time of the model work (CUDA events around every GPU segment)
        self.record_device_time = False
        # Next-step metadata built while the drafting phase runs on the device (see
        # _prepare_next); OSCAR_LOOKAHEAD=0 turns it off.
        self.lookahead = os.environ.get("OSCAR_LOOKAHEAD", "1") != "0"
        self._pre = None
        # OSCAR_HOST_PROFILE=1: seconds of host time per step phase (see _mark)
        self.host_profile = {} if os.environ.get("OSCAR_HOST_PROFILE") == "1" else None
        self._mark_t = 0.0
        self._events: list = []
        # CUDA graphs of the pure-decode (verify + drafting) steps
        self.use_graphs = model.device.type == "cuda"
        self._graphs: dict = {}
        self._seen: dict = {}
        self._graph_pool = torch.cuda.graph_pool_handle() if self.use_graphs else None
        self._hid_static = None
        model.allocate_cache(num_blocks, max_slots)
        model.setup_row_reduce(max_batched_tokens + max_slots * (1 + self.num_spec))
        if self.dev.type == "cuda":
            reserve_split_workspace(self.dev)
        cfg = model.oscar
        self.stage_rows = model.stage_rows
        self._owner_host = np.full(max(1, self.stage_rows) * 128, -1, dtype=np.int32)
        self.sink, self.recent = cfg.sink_tokens, cfg.recent_tokens
        self.g = model.full_layers[0].Hq // model.full_layers[0].Hk if model.full_layers else 1
        self.Hk = model.full_layers[0].Hk if model.full_layers else 1
        self.sms = num_sms(self.dev) if self.dev.type == "cuda" else 148
        # preemption by swapping to pinned host memory (off: requests wait for blocks)
        self.offload = HostKVStore(model) if offload else None
        self.swapped_q: list[int] = []

    # ------------------------------------------------------------------ API
    def close(self) -> None:
        """Release the captured CUDA graphs (they may hold NCCL work: drop them before
        the process group is destroyed)."""
        if self.use_graphs:
            torch.cuda.synchronize(self.dev)
        self._graphs.clear()
        self._seen.clear()

    def release(self, rid: int) -> None:
        """Forget a finished request (its cache blocks and slot were freed when it finished)."""
        r = self.requests.get(rid)
        if r is None or not r.finished:
            return
        del self.requests[rid]
        if rid in self.finished:
            self.finished.remove(rid)

    def max_request_tokens(self) -> int:
        """Longest prompt + output a request may have: the RoPE tables end at the model's
        ``max_position`` (a position past it would index outside them on the device), and a
        request must fit in the KV pool with room for its speculative positions."""
        spare = 2 * self.num_spec + 2
        return min(self.model.cfg.max_position, self.bm.num_blocks * self.bm.page) - spare

    def validate_request(self, prompt, max_new_tokens: int) -> None:
        """Raises ValueError for a request the engine could never run (safe to call from
        any thread: it reads only constants)."""
        if len(prompt) == 0:
            raise ValueError("empty prompt")
        if int(max_new_tokens) < 1:
            raise ValueError("max_new_tokens must be >= 1")
        V = self.model.cfg.vocab_size
        lo, hi = min(prompt), max(prompt)
        if lo < 0 or hi >= V:
            raise ValueError(f"prompt token ids must be in [0, {V})")
        n, cap = len(prompt) + int(max_new_tokens), self.max_request_tokens()
        if n > cap:
            raise ValueError(f"prompt ({len(prompt)}) + max_new_tokens ({max_new_tokens}) = {n} tokens exceeds "
                             f"the {cap} this engine serves")

    def add_request(self, prompt, max_new_tokens: int, sampling: samp.SamplingParams | None = None,
                    stop_ids=None, logprobs: int | None = None) -> int:
        """Queues a request; ``stop_ids``: token ids that end it (an EOS id, say);
        ``logprobs``: record every output token's log-probability and the ``logprobs`` most
        likely tokens (steps with such requests run without CUDA graphs)."""
        self.validate_request(prompt, max_new_tokens)
        if logprobs is not None and not 0 <= int(logprobs) <= 20:
            raise ValueError(f"logprobs {logprobs} must be in [0, 20]")
        rid = next(self._ids)
        r = Request(rid, list(map(int, prompt)), int(max_new_tokens), arrival=self.timer(),
                    stop_ids=frozenset(int(t) for t in (stop_ids or ())),
                    logprobs=None if logprobs is None else int(logprobs))
        if sampling is not None and not sampling.validate().greedy:
            r.sampling = sampling
            r.seed = int(sampling.seed) if sampling.seed is not None else int(
                samp.hash32(torch.tensor([(self.seed * 0x9E3779B1 + rid) & 0xFFFFFFFF])).item())
        self.requests[rid] = r
        self.waiting.append(rid)
        return rid

    def has_work(self) -> bool:
        return bool(self.waiting or self.running or self.swapped_q)

    def abort(self, rid: int) -> None:
        """Ends a request between steps (a client went away, a stop string was seen): its
        blocks and state slot are freed; the tokens generated so far stay in ``output``."""
        r = self.requests.get(rid)
        if r is None or r.finished:
            return
        r.aborted = True
        r.finish_time = self.timer()
        if rid in self.waiting:
            self.waiting.remove(rid)
        if rid in self.running:
            self.running.remove(rid)
        if rid in self.swapped_q:
            self.swapped_q.remove(rid)
            self.offload.discard(rid)
        else:
            self.bm.free(rid)
            self.slots.release(rid)
        r.slot = -1
        self.finished.append(rid)
        self.stats["aborted"] = self.stats.get("aborted", 0) + 1

    # ------------------------------------------------------------------ preemption
    def _swap_out(self, rid: int) -> None:
        r = self.requests[rid]
        off = self.offload
        sw = off.swap_out(rid, list(self.bm.table(rid)), r.slot, self.slots.parity[r.slot],
                          on_freed=lambda: (self.bm.free(rid), self.slots.release(rid)))
        if sw.owner_cleared is not None and len(sw.owner_cleared):
            self._owner_host[sw.owner_cleared] = -1
        off.drain()  # blocks and slot are reusable in this very step
        r.slot = -1
        self.running.remove(rid)
        self.swapped_q.append(rid)
        self.stats["preempted"] = self.stats.get("preempted", 0) + 1

    def _swap_in_ready(self) -> None:
        while self.swapped_q:
            rid = self.swapped_q[0]
            n = self.offload.swapped[rid].n_blocks
            if n > self.bm.free_blocks or not self.slots.free_slots:
                return
            self.swapped_q.pop(0)
            blocks = self.bm.ensure(rid, n * self.bm.page)
            r = self.requests[rid]
            r.slot = self.slots.acquire(rid)
            parity, seats, tags = self.offload.swap_in(rid, list(blocks), r.slot)
            self.slots.parity[r.slot] = parity
            if seats is not None:
                self._owner_host[seats] = tags
            self.running.append(rid)

    def _preempt_for(self, rid: int, tokens: int, scheduled: set) -> bool:
        """Swap out the newest running requests not in this step until ``rid`` fits."""
        if self.offload is None:
            return False
        while not self.bm.can_allocate(rid, tokens):
            victims = [v for v in reversed(self.running) if v != rid and v not in scheduled]
            if not victims:
                return False
            self._swap_out(victims[0])
        return True

    def generate(self, prompts, max_new_tokens: int, sampling=None, stop_ids=None) -> list[list[int]]:
        """Runs ``prompts`` to completion; ``sampling`` is one :class:`SamplingParams` for
        all of them, a list with one per prompt, or None (greedy)."""
        sps = sampling if isinstance(sampling, (list, tuple)) else [sampling] * len(prompts)
        ids = [self.add_request(p, max_new_tokens, sp, stop_ids) for p, sp in zip(prompts, sps)]
        while self.has_work():
            self.step()
        return [self.requests[i].output[:max_new_tokens] for i in ids]

    # ------------------------------------------------------------------ scheduling
    def _schedule(self):
        """Returns a list of (rid, kind, n_tokens) with kind in {"verify", "prefill"}."""
        sched = []
        budget = self.max_batched_tokens
        if self.offload is not None:
            self.offload.poll()
            self._swap_in_ready()
        scheduled: set = set()
        for rid in list(self.running):
            if rid not in self.running:  # swapped out for an earlier request of this step
                continue
            r = self.requests[rid]
            if not r.prefill_done:
                continue
            n = 1 + len(r.drafts)
            extra = 2 * self.num_spec + 2
            if not self.bm.can_allocate(rid, r.num_computed + n + extra) and not self._preempt_for(
                    rid, r.num_computed + n + extra, scheduled):
                continue  # no space this step and nothing to preempt
            self.bm.ensure(rid, r.num_computed + n + extra)
            sched.append((rid, "verify", n))
            scheduled.add(rid)
            budget -= n
        fresh: list = []  # state slots of requests starting this step
        candidates = [rid for rid in self.running if not self.requests[rid].prefill_done] + list(self.waiting)
        if self.prefill_policy == "wide" and candidates:
            share = max(1, budget // len(candidates))
        for rid in candidates:
            if budget <= 0:
                break
            r = self.requests[rid]
            remaining = len(r.prompt) - r.num_computed
            n = min(remaining, budget if self.prefill_policy == "fcfs" else min(share, budget))
            if n <= 0:
                continue
            extra = 2 * self.num_spec + 2 if n == remaining else 0
            if not self.bm.can_allocate(rid, r.num_computed + n + extra) or (r.slot < 0 and not self.slots.free_slots):
                break
            self.bm.ensure(rid, r.num_computed + n + extra)
            if r.slot < 0:
                r.slot = self.slots.acquire(rid)
                fresh.append(r.slot)
            if rid in self.waiting:
                self.waiting.remove(rid)
                self.running.append(rid)
            sched.append((rid, "prefill", n))
            budget -= n
        self.model.reset_state_slots(fresh)
        return sched

    # ------------------------------------------------------------------ metadata
    def _tensor(self, x, dtype=torch.int32):
        a = np.ascontiguousarray(np.asarray(x))
        self.stats["h2d_bytes"] = self.stats.get("h2d_bytes", 0) + a.nbytes
        return torch.as_tensor(a, dtype=dtype).to(self.dev, non_blocking=True)

    def _upload(self, arrays: dict) -> dict:
        """Pack int32 host arrays into one pinned buffer and upload them with one copy."""
        flat = [np.ascontiguousarray(np.asarray(v, dtype=np.int32)).reshape(-1) for v in arrays.values()]
        n = sum((f.size + 3) // 4 * 4 for f in flat)
        if self.dev.type != "cuda":
            out, off = {}, 0
            for (k, v), f in zip(arrays.items(), flat):
                out[k] = torch.from_numpy(f.copy()).view(np.asarray(v).shape) if f.size else torch.zeros(np.asarray(v).shape, dtype=torch.int32)
            return out
        if getattr(self, "_pin", None) is None or self._pin.numel() < n:
            self._pin = torch.empty(max(n, 1 << 16), dtype=torch.int32, pin_memory=True)
            self._dbuf = torch.empty(max(n, 1 << 16), dtype=torch.int32, device=self.dev)
        # the previous step's copy must be finished before the pinned buffer is reused
        if getattr(self, "_pin_event", None) is not None:
            self._pin_event.synchronize()
        host = self._pin.numpy()
        off = 0
        spans = []
        for f in flat:
            host[off:off + f.size] = f
            spans.append((off, f.size))
            off += (f.size + 3) // 4 * 4  # keep every array 16-byte aligned (int4 loads)
        dbuf = torch.empty(n, dtype=torch.int32, device=self.dev)
        dbuf.copy_(self._pin[:n], non_blocking=True)
        self._pin_event = torch.cuda.Event()
        self._pin_event.record()
        self.stats["h2d_bytes"] = self.stats.get("h2d_bytes", 0) + 4 * n
        out = {}
        for (k, v), (o, sz) in zip(arrays.items(), spans):
            out[k] = dbuf[o:o + sz].view(np.asarray(v).shape)
        return out

    def _arrays(self, rows, logit_rows, commit_info, keep, static: bool = False, extra: dict | None = None):
        """Host metadata of one batch: ``(arrays, meta)``.

        ``static=True`` makes every array shape depend only on the batch shape (bucketed
        block-table width, fixed attention splits, owner updates padded to one per token),
        the form a captured CUDA graph can replay.
        """
        toks, poss, slots, tok_req, q_start, seq_lens, bts = [], [], [], [], [0], [], []
        req_slot, n_commit, keep_p, parity = [], [], [], []
        order = []
        for rid, tok, pos in rows:
            if not order or order[-1] != rid:
                order.append(rid)
                q_start.append(q_start[-1])
            q_start[-1] += 1
            toks.append(tok)
            poss.append(pos)
            slots.append(self.bm.slot(rid, pos))
            tok_req.append(len(order) - 1)
        maxp = 1
        for i, rid in enumerate(order):
            b = q_start[i + 1]
            seq_lens.append(poss[b - 1] + 1)
            t = self.bm.table(rid)
            bts.append(t)
            maxp = max(maxp, len(t))
            r = self.requests[rid]
            req_slot.append(r.slot)
            n_commit.append(commit_info.get(rid, 0))
            keep_p.append(1 if keep.get(rid, False) else 0)
            parity.append(self.slots.parity[r.slot])
        if static:
            maxp = 1 << (maxp - 1).bit_length()
        bt = np.zeros((len(order), maxp), dtype=np.int32)
        for i, t in enumerate(bts):
            bt[i, :len(t)] = t
        slots_np = np.asarray(slots, dtype=np.int64)
        pos_np = np.asarray(poss, dtype=np.int64)
        seq_np = np.asarray(seq_lens, dtype=np.int64)[np.asarray(tok_req, dtype=np.int64)]
        token_rows = None
        lay = getattr(self.model, "stage_layout", None)
        if lay is not None and self.stage_rows:  # per-request window rows (sink rows never shared)
            slot_of_tok = np.asarray(req_slot, dtype=np.int64)[np.asarray(tok_req, dtype=np.int64)]
            token_rows = window_row(slot_of_tok, pos_np // 128, lay[0], lay[1])
        stage_seat, owner_seat, owner_val = seat_plan(slots_np, pos_np, seq_np, self.stage_rows, self.sink,
                                                      self.recent, token_rows=token_rows)
        if self.stage_rows:
            self._owner_host[owner_seat] = owner_val
            if static:  # pad to one update per token with idempotent rewrites
                pad = len(rows) - owner_seat.shape[0]
                if pad > 0:
                    fill = owner_seat[:1] if owner_seat.shape[0] else np.zeros(1, np.int32)
                    owner_seat = np.concatenate([owner_seat, np.repeat(fill, pad)]).astype(np.int32)
                    owner_val = self._owner_host[owner_seat].astype(np.int32)
        arrays = dict(tokens=toks, positions=poss, slots=slots, q_start=q_start, seq_lens=seq_lens, bt=bt,
                      tok_req=tok_req, stage_seat=stage_seat, owner_seat=owner_seat, owner_val=owner_val,
                      req_slot=req_slot, n_commit=n_commit, keep=keep_p, parity=parity, logit_rows=logit_rows)
        if extra:
            arrays.update(extra)
        meta = {"q_start": q_start, "seq_lens": seq_lens, "order": order,
                "max_qlen": max((q_start[i + 1] - q_start[i] for i in range(len(order))), default=0)}
        if self.dev.type == "cuda":
            fixed = 0
            decode_only = all((q_start[i + 1] - q_start[i]) * self.g <= A.LONG_ROWS for i in range(len(order)))
            if static or decode_only:
                # decode / verify steps use the fixed split layout whether or not they are
                # replayed from a CUDA graph, so both paths compute the same partials
                fixed = A.decode_splits(q_start, self.g, self.Hk, self.sms)
            plan_np = A.plan_attention_host(q_start, seq_lens, self.g, self.Hk, self.sms, fixed_splits=fixed)
            arrays.update(work=plan_np[0], item_first=plan_np[1], item_count=plan_np[2], tiles=plan_np[5])
            meta["max_rb"], meta["n_work"] = plan_np[3], plan_np[4]
            meta["n_short"], meta["rpi_short"] = plan_np[6], plan_np[7]
            meta["n_tiles"] = int((plan_np[5][:, 2] >= 0).sum()) if plan_np[4] > plan_np[6] else 0
        if checks.enabled():  # OSCAR_CHECK_STEPS=1: validate what the kernels will index with
            checks.check_step(arrays, meta, num_blocks=self.bm.num_blocks, max_slots=self.slots.n, g=self.g,
                              stage_rows=self.stage_rows, max_pending=P_MAX)
        return arrays, meta

    def _batch(self, d: dict, meta: dict) -> StepBatch:
        plan = None
        if "work" in d:
            plan = A.AttnPlan(d["work"], d["item_first"], d["item_count"], meta["max_rb"], meta["n_work"], d["tiles"],
                              meta["n_tiles"], meta["n_short"], meta["rpi_short"])
        b = StepBatch(
            tokens=d["tokens"], positions=d["positions"], slots=d["slots"], q_start=d["q_start"],
            seq_lens=d["seq_lens"], block_tables=d["bt"], tok_req=d["tok_req"], q_start_l=meta["q_start"],
            seq_lens_l=meta["seq_lens"], plan=plan,
            stage_seat=d["stage_seat"] if self.stage_rows else None,
            owner_seat=d["owner_seat"] if self.stage_rows else None,
            owner_val=d["owner_val"] if self.stage_rows else None,
            req_slot=d["req_slot"], n_commit=d["n_commit"], keep_pending=d["keep"], parity=d["parity"],
            logit_rows=d["logit_rows"].long())
        b.extra["order"] = meta["order"]
        b.extra["max_qlen"] = meta["max_qlen"]
        if "samp_t" in d:
            b.extra["sampling"] = samp.rows_from_arrays(d)
        return b

    def _build(self, rows, logit_rows, commit_info, keep, extra: dict | None = None):
        """Eager batch: host metadata uploaded with one copy."""
        arrays, meta = self._arrays(rows, logit_rows, commit_info, keep, extra=extra)
        return self._batch(self._upload(arrays), meta)

    # ------------------------------------------------------------------ CUDA graphs
    def _run_phase(self, name: str, specs: list, fn):
        """Run ``fn(batches)`` for host metadata ``specs = [(arrays, meta), ...]``.

        With graphs enabled, the second occurrence of a metadata shape is captured into
        a CUDA graph whose metadata lives in a static device buffer; later occurrences
        copy the new metadata into that buffer (one pinned host-to-device copy) and replay.
        """
        if not self.use_graphs or self.dev.type != "cuda":
            return fn([self._batch(self._upload(a), m) for a, m in specs])
        sig = (name,) + tuple(tuple((k, np.shape(v)) for k, v in a.items()) + (m.get("max_rb"), m.get("n_work"))
                              for a, m in specs)
        ent = self._graphs.get(sig)
        if ent is not None:
            self._fill_static(ent, specs)
            ent["graph"].replay()
            _launches.add(ent["launches"])
            return ent["out"]
        self._seen[sig] = self._seen.get(sig, 0) + 1
        if self._seen[sig] < 2:
            return fn([self._batch(self._upload(a), m) for a, m in specs])
        # capture (kernel attributes and tensor maps were initialised by the eager run)
        layout, n = [], 0
        for a, _ in specs:
            lay = {}
            for k, v in a.items():
                sz = int(np.prod(np.shape(v))) if np.ndim(v) else 1
                lay[k] = (n, np.shape(v))
                n += (sz + 3) // 4 * 4
            layout.append(lay)
        ent = {"layout": layout, "n": n, "dbuf": torch.zeros(max(n, 4), dtype=torch.int32, device=self.dev),
               "pin": torch.empty(max(n, 4), dtype=torch.int32, pin_memory=True), "event": None}
        self._fill_static(ent, specs)
        batches = []
        for (a, m), lay in zip(specs, layout):
            d = {k: ent["dbuf"][o:o + int(np.prod(shp))].view(shp) for k, (o, shp) in lay.items()}
            batches.append(self._batch(d, m))
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        n0 = _launches.count()
        with torch.cuda.graph(g, pool=self._graph_pool):
            out = fn(batches)
        ent["launches"] = _launches.count() - n0  # kernels of this package inside the graph
        ent["graph"], ent["out"] = g, out
        self._graphs[sig] = ent
        g.replay()
        return out

    def _fill_static(self, ent, specs):
        if ent["event"] is not None:
            ent["event"].synchronize()
        host = ent["pin"].numpy()
        for (a, _), lay in zip(specs, ent["layout"]):
            for k, v in a.items():
                o, shp = lay[k]
                f = np.asarray(v, dtype=np.int32).reshape(-1)
                host[o:o + f.size] = f
        ent["dbuf"].copy_(ent["pin"][:ent["dbuf"].numel()], non_blocking=True)
        ev = torch.cuda.Event()
        ev.record()
        ent["event"] = ev
        self.stats["h2d_bytes"] = self.stats.get("h2d_bytes", 0) + 4 * ent["n"]

    # ------------------------------------------------------------------ step
    def _mark(self, name: str) -> None:
        """Host-time breakdown of steps (OSCAR_HOST_PROFILE=1): seconds since the previous mark."""
        if self.host_profile is not None:
            now = time.perf_counter()
            self.host_profile[name] = self.host_profile.get(name, 0.0) + now - self._mark_t
            self._mark_t = now

    # ------------------------------------------------------------------ lookahead
    def _steady(self, rids) -> bool:
        """Every running request verifies its drafts this step, greedily, nothing waits."""
        if not self.lookahead or self.num_spec <= 0 or self.offload is not None or self.waiting or not rids:
            return False
        for rid in rids:
            r = self.requests[rid]
            if not r.prefill_done or r.finished or r.sampling is not None or r.logprobs is not None:
                return False
        return True

    def _prepare_next(self) -> None:
        """Build the next verify step's metadata while this step's drafting runs.

        In a steady decode step every running request verifies ``1 + num_spec`` rows at
        known positions; only the draft tokens are not known until the drafts are read
        back, so the rows carry placeholders that ``_take_prepared`` fills in.  Block
        allocation is done here (it is idempotent); the host mirror of the staging owner
        tags is snapshotted so that a discarded batch leaves no trace in it.
        """
        self._pre = None
        rids = list(self.running)
        if not self.use_graphs or not self._steady(rids):
            return
        n = 1 + self.num_spec
        extra = 2 * self.num_spec + 2
        reqs = [self.requests[rid] for rid in rids]
        if not all(self.bm.can_allocate(rid, r.num_computed + n + extra) for rid, r in zip(rids, reqs)):
            return
        for rid, r in zip(rids, reqs):
            self.bm.ensure(rid, r.num_computed + n + extra)
        snapshot = self._owner_host.copy() if self.stage_rows else None
        rows, logit_rows, commit, keep, info = [], [], {}, {}, []
        for rid, r in zip(rids, reqs):
            base = len(rows)
            keep[rid] = True
            logit_rows.extend(range(base, base + n))
            commit[rid] = r.pending_commit
            rows.append((rid, r.last_token, r.num_computed))
            rows.extend((rid, 0, r.num_computed + i) for i in range(1, n))
            info.append((rid, "verify", n, base))
        arrays, meta = self._arrays(rows, logit_rows, commit, keep, static=True)
        self._pre = dict(rids=tuple(rids), nc=tuple(r.num_computed for r in reqs), rows=rows, logit_rows=logit_rows,
                         commit=commit, keep=keep, info=info, arrays=arrays, meta=meta, snapshot=snapshot)

    def _take_prepared(self):
        """The prepared batch with its draft tokens filled in, or None (and the staging
        mirror restored) when the running set changed since it was built."""
        pre, self._pre = self._pre, None
        if pre is None:
            return None
        rids = tuple(self.running)
        ok = (rids == pre["rids"] and self._steady(rids)
              and tuple(self.requests[rid].num_computed for rid in rids) == pre["nc"]
              and all(len(self.requests[rid].drafts) == self.num_spec for rid in rids))
        if not ok:
            if pre["snapshot"] is not None:
                self._owner_host[:] = pre["snapshot"]
            return None
        toks, rows = pre["arrays"]["tokens"], pre["rows"]
        for rid, _, n, base in pre["info"]:
            d = self.requests[rid].drafts
            for i in range(1, n):
                toks[base + i] = d[i - 1]
                rows[base + i] = (rid, d[i - 1], rows[base + i][2])
        return pre

    def step(self) -> dict:
        if self.host_profile is not None:
            self._mark_t = time.perf_counter()
        pre = self._take_prepared()
        if pre is not None:
            self.stats["lookahead_steps"] = self.stats.get("lookahead_steps", 0) + 1
            return self._step_body(pre["rows"], pre["logit_rows"], pre["commit"], pre["keep"], pre["info"], None,
                                   None, (pre["arrays"], pre["meta"]))
        sched = self._schedule()
        if not sched:
            return {}
        rows, logit_rows, commit, keep = [], [], {}, {}
        info = []
        sp_rows = []  # per logit row: (request, position sampled, draft verified there or -1)
        for rid, kind, n in sched:
            r = self.requests[rid]
            base = len(rows)
            if kind == "verify":
                toks = [r.last_token] + r.drafts
                keep[rid] = True
                logit_rows.extend(range(base, base + n))
                sp_rows += [(r, r.num_computed + i + 1, r.drafts[i] if i < len(r.drafts) else -1) for i in range(n)]
            else:
                toks = r.prompt[r.num_computed:r.num_computed + n]
                keep[rid] = False
                if r.num_computed + n == len(r.prompt):
                    logit_rows.append(base + n - 1)
                    sp_rows.append((r, len(r.prompt), -1))
            commit[rid] = r.pending_commit
            for i, t in enumerate(toks):
                rows.append((rid, t, r.num_computed + i))
            info.append((rid, kind, n, base))
        sampled = None
        if any(r.sampling is not None for r, _, _ in sp_rows):
            sampled = samp.host_rows([r.sampling for r, _, _ in sp_rows], [r.seed for r, _, _ in sp_rows],
                                     [p for _, p, _ in sp_rows], [d for _, _, d in sp_rows])
        return self._step_body(rows, logit_rows, commit, keep, info, sampled, sched, None)

    def _step_body(self, rows, logit_rows, commit, keep, info, sampled, sched, prepared):
        lp_k = max((self.requests[rid].logprobs for rid, _, _, _ in info
                    if self.requests[rid].logprobs is not None), default=None)
        static = self.use_graphs and lp_k is None and all(kind == "verify" for _, kind, _, _ in info)
        self._mark("schedule")
        if static:
            if prepared is not None:
                arrays, meta = prepared
            else:
                arrays, meta = self._arrays(rows, logit_rows, commit, keep, static=True, extra=sampled)
            b = (arrays, meta)
            self._mark("main_metadata")
            with self._segment():
                hid, tok = self._run_phase("main", [(arrays, meta)], lambda bs: self._main_fn(bs[0]))
        else:
            b = self._build(rows, logit_rows, commit, keep, extra=sampled)
            if lp_k is not None:
                b.extra["logprobs_k"] = lp_k
            with self._segment():
                hid, tok = self._main_fn(b)
        self._mark("main_launch")
        tok_h = tok.tolist()
        self._mark("main_wait")
        lp_h = None
        if lp_k is not None:
            tl, ti, tv = self.model.last_logprobs
            lp_h = (tl.tolist(), ti.tolist(), tv.tolist())
        self.stats["d2h_bytes"] = self.stats.get("d2h_bytes", 0) + 4 * len(tok_h)
        self.last = (hid, tok)
        self._check_status()
        # ---------------- verify / sample -----------------
        now = self.timer()
        li = 0
        next_row_tok = [0] * len(rows)
        draft_rows = []  # (rid, row index in step) rows whose MTP output starts drafting
        for rid, kind, n, base in info:
            r = self.requests[rid]
            for i in range(n):
                p = r.num_computed + i
                next_row_tok[base + i] = r.prompt[p + 1] if p + 1 < len(r.prompt) else 0
            if kind == "verify":
                targets = tok_h[li:li + n]
                li0 = li
                li += n
                d = r.drafts
                if self.acceptance is not None:
                    n_acc = min(self.acceptance(rid), len(d))
                else:
                    n_acc = 0
                    while n_acc < len(d) and d[n_acc] == targets[n_acc]:
                        n_acc += 1
                emitted = d[:n_acc] + [targets[n_acc]]
                for i in range(n):
                    next_row_tok[base + i] = d[i] if i < n_acc else targets[i]
                self.stats["drafts_proposed"] += len(d)
                self.stats["drafts_accepted"] += n_acc
                r.accepted.append(n_acc)
                r.num_computed += n_acc + 1
                r.pending_commit = n_acc + 1
                self.slots.parity[r.slot] ^= 1
                kept = r.emit(emitted)
                self.stats["tokens_out"] += kept
                if r.logprobs is not None:  # an accepted draft is its row's token
                    self._record_lp(r, lp_h, li0, kept)
                r.last_token = emitted[-1]
                draft_rows.append((rid, base + n_acc))
            else:
                r.num_computed += n
                r.pending_commit = 0
                self.slots.parity[r.slot] ^= 1
                if r.prefill_done:
                    y = tok_h[li]
                    kept = r.emit([y])
                    if r.logprobs is not None:
                        self._record_lp(r, lp_h, li, kept)
                    li += 1
                    next_row_tok[base + n - 1] = y
                    self.stats["tokens_out"] += kept
                    r.last_token = y
                    r.first_token_time = now
                    draft_rows.append((rid, base + n - 1))
            if r.first_token_time is None and r.output:
                r.first_token_time = now
        self._mark("accept")
        # ---------------- MTP drafting -----------------
        if self.num_spec > 0 and draft_rows:
            self._draft(b, hid, rows, next_row_tok, draft_rows)
        # ---------------- retire -----------------
        for rid, kind, n, base in info:
            r = self.requests[rid]
            if r.finished:
                r.finish_time = now
                self.running.remove(rid)
                self.finished.append(rid)
                self.bm.free(rid)
                self.slots.release(rid)
        self.stats["steps"] += 1
        self._mark("retire")
        return {"scheduled": sched if sched is not None else [(rid, kind, n) for rid, kind, n, _ in info]}

    @staticmethod
    def _record_lp(r: Request, lp_h, row0: int, n: int) -> None:
        tl, ti, tv = lp_h
        for j in range(row0, row0 + n):
            r.lp.append((tl[j], list(zip(ti[j][:r.logprobs], tv[j][:r.logprobs]))))

    def _main_fn(self, b: StepBatch):
        """Main model; the hidden states land in a persistent buffer so that a captured
        drafting graph always reads them from the same address."""
        hid, tok = self.model.forward(b)
        T, H = hid.shape
        if self._hid_static is None or self._hid_static.shape[0] < T:
            self._graphs = {k: v for k, v in self._graphs.items() if k[0] != "mtp"}  # their input moved
            self._hid_static = torch.empty(max(T, self.max_batched_tokens), H, dtype=hid.dtype, device=hid.device)
        self._hid_static[:T].copy_(hid)
        return self._hid_static[:T], tok

    def _draft(self, b, hid, rows, next_row_tok, draft_rows):
        """MTP pass over the step's rows, then num_spec-1 chained single-token passes.

        All passes run back to back on the device: the draft tokens of pass k are the
        input tokens of pass k+1 without a host round trip; the host reads every draft
        once at the end.
        """
        m = self.model
        rows_sel = [ri for _, ri in draft_rows]

        def chain(batches):
            b1, later = batches[0], batches[1:]
            h1, e = m.mtp.forward(b1, hid)
            outs = [e]
            h = h1[b1.logit_rows]
            for bk in later:
                h, e = m.mtp.forward(bk, h, tokens=e)
                outs.append(e)
            return torch.stack(outs, 1)

        if isinstance(b, tuple):  # static (graph) metadata of a pure decode step
            arrays, meta = b
            a1 = dict(arrays)
            a1["tokens"] = next_row_tok
            a1["logit_rows"] = rows_sel
            specs = [(a1, meta)]
            for k in range(1, self.num_spec):
                # the MTP row after ``ri`` sits one position further; tokens come from the device
                prow = [(rid, 0, rows[ri][2] + k) for rid, ri in draft_rows]
                specs.append(self._arrays(prow, list(range(len(prow))), {}, {}, static=True))
            self._mark("draft_metadata")
            with self._segment():
                drafts_t = self._run_phase("mtp", specs, chain)
            self._mark("draft_launch")
            self._prepare_next()  # overlaps the drafting on the device
        else:
            up = self._upload({"tokens": next_row_tok, "rows": rows_sel})
            b.tokens = up["tokens"]
            b.logit_rows = up["rows"].long()
            later = []
            for k in range(1, self.num_spec):
                prow = [(rid, 0, rows[ri][2] + k) for rid, ri in draft_rows]
                later.append(self._build(prow, list(range(len(prow))), {}, {}))
            with self._segment():
                drafts_t = chain([b] + later)
        self._mark("prepare_next")
        d = drafts_t.tolist()
        self._mark("draft_wait")
        self.stats["d2h_bytes"] = self.stats.get("d2h_bytes", 0) + 4 * drafts_t.numel()
        for (rid, _), row in zip(draft_rows, d):
            self.requests[rid].drafts = [int(x) for x in row]

    class _Seg:
        def __init__(self, eng):
            self.eng = eng

        def __enter__(self):
            if self.eng.record_device_time:
                self.a = torch.cuda.Event(enable_timing=True)
                self.a.record()

        def __exit__(self, *exc):
            if self.eng.record_device_time:
                b = torch.cuda.Event(enable_timing=True)
                b.record()
                self.eng._events.append((self.a, b))

    def _segment(self):
        return LLMEngine._Seg(self)

    def device_ms(self, reset: bool = True) -> float:
        """Sum of recorded GPU segment durations (synchronises)."""
        torch.cuda.synchronize()
        t = sum(a.elapsed_time(b) for a, b in self._events)
        if reset:
            self._events = []
        return t

    def _check_status(self):
        st = self.model.status
        if st is not None:
            v = int(st.item())
            if v != 0:
                raise RuntimeError(f"kernel reported status {v} (bounded wait expired or bad index)")
