"""Host-side staging seat plan (sink/recent fp32 window with owner tags).

Same semantics as the reference staging write (``oscar_ascend/backend.py:439-481``):
a token is *kept* if ``pos >= seq - recent`` or ``pos < sink_eff``; its seat is
``row * 128 + slot % 128`` with ``row = slot // 128 % rows`` in the reference's hashed
arena, or the request's own row for the token's logical page in the window layout
(``kv.oracle.window_row``: sink pages have rows of their own, so they are never
evicted); among tokens of a step that share a seat
the last one (in token order) wins; the owner tag becomes the block id, or -1 when
the winner is not kept (invalidating recycled seats).

The plan depends only on the step's slots and positions, so it is computed once per
step on the host (no device sort) and shared by all FULL layers; only the first
layer's store launch writes the owner tags, every layer writes its own values.
"""
from __future__ import annotations

import numpy as np

PAGE = 128


def seat_plan(slots: np.ndarray, pos: np.ndarray, seq_of_tok: np.ndarray, rows: int, sink_tokens: int,
              recent_tokens: int, page: int = PAGE, token_rows: np.ndarray | None = None):
    """Returns ``(stage_seat [T], owner_seat [n], owner_val [n])`` as int32 arrays.

    ``stage_seat[t]`` is the seat token ``t`` writes its fp32 K/V to (winner and kept),
    else -1.  ``token_rows[t]`` is token ``t``'s staging row in the per-request window
    layout; without it the row is ``block % rows`` (the reference's hashed arena).
    """
    T = slots.shape[0]
    stage_seat = np.full(T, -1, dtype=np.int32)
    if rows <= 0 or T == 0:
        return stage_seat, np.zeros(0, np.int32), np.zeros(0, np.int32)
    sink_eff = (sink_tokens // page) * page
    keep = (pos >= seq_of_tok - recent_tokens) | (pos < sink_eff)
    valid = np.nonzero(slots >= 0)[0]
    s = slots[valid].astype(np.int64)
    row = (s // page % rows) if token_rows is None else token_rows[valid].astype(np.int64)
    seats = row * page + s % page
    # last writer per seat in token order: stable sort, take the final index of each run
    order = np.argsort(seats, kind="stable")
    ss = seats[order]
    last = np.ones(ss.shape[0], dtype=bool)
    if ss.shape[0] > 1:
        last[:-1] = ss[1:] != ss[:-1]
    tok = valid[order[last]]
    seat = ss[last]
    owner = np.where(keep[tok], s[order[last]] // page, -1)
    kept = keep[tok]
    stage_seat[tok[kept]] = seat[kept]
    return stage_seat, seat.astype(np.int32), owner.astype(np.int32)
