"""Host-side checks of one step's kernel metadata (opt-in: ``OSCAR_CHECK_STEPS=1``).

The kernels trust their metadata: a block-table entry past the pool, a slot that does
not match its block table or an attention work item past a request's keys turns into
an out-of-bounds access on the device.  Compute-sanitizer is not available everywhere
this framework runs, so this module is the cheap stand-in: before a step's metadata is
uploaded it checks, in numpy, every invariant the kernels rely on and raises
:class:`StepMetadataError` naming the first violation.  It costs a few milliseconds per
step, so it is meant for debugging and tests, not for serving.

Checked (the array names of :meth:`LLMEngine._arrays`):

* ``q_start`` starts at 0 and is non-decreasing; every request has ``seq_len >= q_len``;
* ``positions`` of request ``r`` are ``seq_len - q_len .. seq_len - 1`` in order;
* every block-table entry a request needs (``ceil(seq_len / page)`` of them) lies in
  ``[0, num_blocks)`` and no block is held by two requests of the step;
* every KV slot equals ``block_table[pos // page] * page + pos % page``;
* ``req_slot`` lies in ``[0, max_slots)`` without duplicates, ``parity`` is 0 or 1,
  ``n_commit`` lies in ``[0, max_pending]``;
* staging seats and owner updates lie inside the staging arena and owner values are
  ``-1`` or a block of the step;
* attention work items (``work``: request, first row, key range) stay inside their
  request's rows and keys, each (request, 64-row block) has items covering its keys
  from 0, and prefill tiles name items of their own request.
"""
from __future__ import annotations

import os

import numpy as np

PAGE = 128
ROWS = 64


class StepMetadataError(RuntimeError):
    """A step's kernel metadata violates an invariant the kernels rely on."""


def enabled() -> bool:
    return os.environ.get("OSCAR_CHECK_STEPS", "0") == "1"


def _fail(msg: str):
    raise StepMetadataError(msg)


def check_step(arrays: dict, meta: dict, *, num_blocks: int, max_slots: int, g: int, stage_rows: int = 0,
               max_pending: int = 16, page: int = PAGE) -> None:
    """Raises :class:`StepMetadataError` on the first violated invariant."""
    q_start = np.asarray(arrays["q_start"], dtype=np.int64)
    seq_lens = np.asarray(arrays["seq_lens"], dtype=np.int64)
    R = len(seq_lens)
    if len(q_start) != R + 1 or q_start[0] != 0 or np.any(np.diff(q_start) < 0):
        _fail(f"q_start {q_start.tolist()} is not a prefix sum over {R} requests")
    qlen = np.diff(q_start)
    if np.any(seq_lens < qlen):
        r = int(np.argmax(seq_lens < qlen))
        _fail(f"request {r}: seq_len {int(seq_lens[r])} < q_len {int(qlen[r])}")
    T = int(q_start[-1])
    pos = np.asarray(arrays["positions"], dtype=np.int64)
    slots = np.asarray(arrays["slots"], dtype=np.int64)
    if len(pos) != T or len(slots) != T:
        _fail(f"{len(pos)} positions / {len(slots)} slots for {T} tokens")
    bt = np.asarray(arrays["bt"], dtype=np.int64).reshape(R, -1) if R else np.zeros((0, 1), np.int64)
    seen_blocks: dict[int, int] = {}
    for r in range(R):
        a, b = int(q_start[r]), int(q_start[r + 1])
        want = np.arange(seq_lens[r] - (b - a), seq_lens[r])
        if not np.array_equal(pos[a:b], want):
            _fail(f"request {r}: positions {pos[a:b].tolist()[:8]}... are not {want.tolist()[:8]}...")
        need = int((seq_lens[r] + page - 1) // page)
        if need > bt.shape[1]:
            _fail(f"request {r}: needs {need} pages, block table holds {bt.shape[1]}")
        blocks = bt[r, :need]
        bad = (blocks < 0) | (blocks >= num_blocks)
        if np.any(bad):
            i = int(np.argmax(bad))
            _fail(f"request {r}: block table entry {i} = {int(blocks[i])} outside [0, {num_blocks})")
        for blk in blocks.tolist():
            if seen_blocks.setdefault(blk, r) != r:
                _fail(f"block {blk} is held by requests {seen_blocks[blk]} and {r}")
        want_slots = blocks[pos[a:b] // page] * page + pos[a:b] % page
        if not np.array_equal(slots[a:b], want_slots):
            i = int(np.argmax(slots[a:b] != want_slots))
            _fail(f"request {r}: token {i} slot {int(slots[a + i])} != block table slot {int(want_slots[i])}")
    if "req_slot" in arrays:
        rs = np.asarray(arrays["req_slot"], dtype=np.int64)
        if len(rs) != R or np.any(rs < 0) or np.any(rs >= max_slots) or len(set(rs.tolist())) != R:
            _fail(f"req_slot {rs.tolist()} invalid for {max_slots} slots")
    if "parity" in arrays and np.any(~np.isin(np.asarray(arrays["parity"]), (0, 1))):
        _fail(f"parity {np.asarray(arrays['parity']).tolist()} is not 0/1")
    if "n_commit" in arrays:
        nc = np.asarray(arrays["n_commit"], dtype=np.int64)
        if np.any(nc < 0) or np.any(nc > max_pending):
            _fail(f"n_commit {nc.tolist()} outside [0, {max_pending}]")
    if stage_rows:
        cap = stage_rows * page
        for key in ("stage_seat", "owner_seat"):
            if key in arrays:
                v = np.asarray(arrays[key], dtype=np.int64)
                keep = v >= 0 if key == "stage_seat" else np.ones_like(v, dtype=bool)
                if np.any(v[keep] >= cap) or (key == "owner_seat" and np.any(v < 0)):
                    _fail(f"{key} outside the staging arena of {cap} seats")
        if "owner_val" in arrays:
            ov = np.asarray(arrays["owner_val"], dtype=np.int64)
            ok = (ov == -1) | np.isin(ov, list(seen_blocks))
            if not np.all(ok):
                _fail(f"owner value {int(ov[~ok][0])} is neither -1 nor a block of the step")
    if "work" in arrays:
        _check_plan(arrays, meta, q_start, seq_lens, g)


def _check_plan(arrays: dict, meta: dict, q_start, seq_lens, g: int) -> None:
    R = len(seq_lens)
    n_work = int(meta["n_work"])
    work = np.asarray(arrays["work"], dtype=np.int64).reshape(-1, 4)[:n_work]
    max_rb = int(meta["max_rb"])
    first = np.asarray(arrays["item_first"], dtype=np.int64)
    count = np.asarray(arrays["item_count"], dtype=np.int64)
    for i, (r, row0, b0, b1) in enumerate(work.tolist()):
        if not 0 <= r < R:
            _fail(f"work item {i}: request {r} outside [0, {R})")
        rows = int(q_start[r + 1] - q_start[r]) * g
        prefix = int(seq_lens[r] - (q_start[r + 1] - q_start[r]))
        if row0 % ROWS or not 0 <= row0 < max(rows, 1):
            _fail(f"work item {i}: first row {row0} invalid for {rows} rows")
        need = prefix + (min(rows, row0 + ROWS) - 1) // g + 1
        if not 0 <= b0 <= b1 <= need:
            _fail(f"work item {i}: keys [{b0}, {b1}) outside [0, {need})")
    for r in range(R):
        rows = int(q_start[r + 1] - q_start[r]) * g
        prefix = int(seq_lens[r] - (q_start[r + 1] - q_start[r]))
        for rb in range((rows + ROWS - 1) // ROWS):
            f, c = int(first[r * max_rb + rb]), int(count[r * max_rb + rb])
            if c < 1 or f < 0 or f + c > n_work:
                _fail(f"request {r} block {rb}: items [{f}, {f + c}) outside the {n_work} work items")
            items = work[f:f + c]
            if np.any(items[:, 0] != r) or np.any(items[:, 1] != rb * ROWS):
                _fail(f"request {r} block {rb}: items name another request or block")
            need = prefix + (min(rows, (rb + 1) * ROWS) - 1) // g + 1
            if int(items[:, 2].min()) != 0 or int(items[:, 3].max()) != need:
                _fail(f"request {r} block {rb}: items cover [{int(items[:, 2].min())}, {int(items[:, 3].max())}), "
                      f"not [0, {need})")
    n_tiles = int(meta.get("n_tiles", 0))
    if n_tiles:
        tiles = np.asarray(arrays["tiles"], dtype=np.int64).reshape(-1, 4)[:n_tiles]
        for i, (r, row0, ia, ib) in enumerate(tiles.tolist()):
            if not 0 <= r < R or row0 % (2 * ROWS):
                _fail(f"tile {i}: request {r} / first row {row0} invalid")
            for it, off in ((ia, 0), (ib, ROWS)):
                if it < 0:
                    continue
                if not 0 <= it < n_work or work[it, 0] != r or work[it, 1] != row0 + off:
                    _fail(f"tile {i}: item {it} is not rows {row0 + off}.. of request {r}")
