"""Attention work planner (host side): short requests' split items first, one item per
64-row block of a prefill request, 128-row prefill tiles pairing those items."""
import math

import numpy as np

from oscar_b200.ops import attention as A


def test_plan_orders_short_items_first_and_tiles_long_requests():
    g = 6
    q_start = [0, 4, 204, 205, 245]       # verify (4), prefill (200), decode (1), prefill (40)
    seq_lens = [9000, 1500, 300, 40]
    work, first, count, max_rb, n_work, tiles, n_short, rpi_short = A.plan_attention_host(
        q_start, seq_lens, g, Hk=2, sms=148)
    work = work[:n_work]
    R = len(seq_lens)
    rows = [(q_start[r + 1] - q_start[r]) * g for r in range(R)]
    long_req = {r for r in range(R) if rows[r] > A.LONG_ROWS}
    assert long_req == {1, 3}
    # short items first, their rows fit the decode/verify kernel
    assert all(int(w[0]) not in long_req for w in work[:n_short])
    assert all(int(w[0]) in long_req for w in work[n_short:])
    assert rpi_short == 24
    # every (request, 64-row block) has its items; long blocks exactly one covering [0, need)
    for r in range(R):
        rb_n = (rows[r] + A.ROWS - 1) // A.ROWS
        prefix = seq_lens[r] - (q_start[r + 1] - q_start[r])
        for rb in range(rb_n):
            f, c = int(first[r * max_rb + rb]), int(count[r * max_rb + rb])
            items = work[f:f + c]
            assert all(int(w[0]) == r and int(w[1]) == rb * A.ROWS for w in items)
            need = prefix + (min(rows[r], (rb + 1) * A.ROWS) - 1) // g + 1
            if r in long_req:
                assert c == 1 and int(items[0][2]) == 0 and int(items[0][3]) == need
            else:
                assert int(items[0][2]) == 0 and int(items[-1][3]) == need
    # tiles: one per 128 rows of each long request, pairing consecutive block items
    n_tiles = int((tiles[:, 2] >= 0).sum())
    assert n_tiles == sum((rows[r] + 127) // 128 for r in long_req)
    for req, row0, ia, ib in tiles[:n_tiles]:
        req, row0, ia, ib = int(req), int(row0), int(ia), int(ib)
        assert row0 % 128 == 0
        assert ia == int(first[req * max_rb + row0 // A.ROWS])
        if row0 + A.ROWS < rows[req]:
            assert ib == int(first[req * max_rb + row0 // A.ROWS + 1])
        else:
            assert ib == -1
    # the tiles with the most keys come first
    keys = [seq_lens[int(t[0])] - (q_start[int(t[0]) + 1] - q_start[int(t[0])]) + int(t[1]) // g
            for t in tiles[:n_tiles]]
    assert keys == sorted(keys, reverse=True)


def test_plan_without_prefill_has_no_tiles():
    work, first, count, max_rb, n_work, tiles, n_short, rpi_short = A.plan_attention_host(
        [0, 1, 2, 6], [100, 5000, 300], 6, Hk=1, sms=148)
    assert n_short == n_work
    assert int((tiles[:, 2] >= 0).sum()) == 0
    assert rpi_short == 24
    assert np.all(count[:3] >= 1)


def _plan_loop(q_start: list[int], seq_lens: list[int], g: int, Hk: int, sms: int,
                        min_chunk: int = 256, waves: int = 3, fixed_splits: int = 0, long_rows: int = A.LONG_ROWS):
    """The planner as a plain loop over blocks and splits (the oracle of the vectorised one)."""
    R = len(seq_lens)
    blocks = []  # (req, row0, kv_need, long)
    max_rb = 1
    for r in range(R):
        n = q_start[r + 1] - q_start[r]
        if n <= 0:
            continue
        prefix = seq_lens[r] - n
        rows = n * g
        rb = (rows + A.ROWS - 1) // A.ROWS
        max_rb = max(max_rb, rb)
        for b in range(rb):
            last_row = min(rows, (b + 1) * A.ROWS) - 1
            blocks.append((r, b * A.ROWS, prefix + last_row // g + 1, rows > long_rows))
    short = [bk for bk in blocks if not bk[3]]
    longb = [bk for bk in blocks if bk[3]]
    total = sum(k for _, _, k, _ in short)
    target_items = max(1, (waves * sms) // max(Hk, 1))
    # page-aligned (128-token) split ranges: every split streams whole pages
    chunk = max(min_chunk, int(math.ceil(total / target_items / 128.0)) * 128) if total else min_chunk
    work = []
    first = np.zeros(R * max_rb, dtype=np.int32)
    count = np.zeros(R * max_rb, dtype=np.int32)
    rpi_short = 0
    for r, row0, need, _ in short:
        rb = row0 // A.ROWS
        rows = (q_start[r + 1] - q_start[r]) * g
        rpi_short = max(rpi_short, min(A.ROWS, rows - row0))
        first[r * max_rb + rb] = len(work)
        if fixed_splits > 0:
            splits = fixed_splits
            per = max(128, int(math.ceil(need / splits / 128.0)) * 128)
            for s in range(splits):
                b0 = min(need, s * per)
                work.append((r, row0, b0, min(need, b0 + per)))
        else:
            splits = max(1, (need + chunk - 1) // chunk)
            for s in range(splits):
                work.append((r, row0, s * chunk, min(need, (s + 1) * chunk)))
        count[r * max_rb + rb] = splits
    n_short = len(work)
    for r, row0, need, _ in longb:
        rb = row0 // A.ROWS
        first[r * max_rb + rb] = len(work)
        count[r * max_rb + rb] = 1
        work.append((r, row0, 0, need))
    tiles = []
    for r, row0, need, _ in longb:
        if row0 % (2 * A.ROWS):
            continue
        rb = row0 // A.ROWS
        rows = (q_start[r + 1] - q_start[r]) * g
        item_b = int(first[r * max_rb + rb + 1]) if row0 + A.ROWS < rows else -1
        tiles.append((r, row0, int(first[r * max_rb + rb]), item_b))
    # longest tiles (most keys) first
    tiles.sort(key=lambda t: -(seq_lens[t[0]] - (q_start[t[0] + 1] - q_start[t[0]]) + t[1] // g))
    n_work = len(work)
    wt = np.asarray(work if work else [(0, 0, 0, 0)], dtype=np.int32).reshape(-1, 4)
    tt = np.asarray(tiles if tiles else [(0, 0, -1, -1)], dtype=np.int32).reshape(-1, 4)
    return wt, first, count, max_rb, n_work, tt, n_short, rpi_short



def test_vectorised_planner_equals_the_loop():
    rng = np.random.default_rng(0)
    for case in range(300):
        R = int(rng.integers(1, 40))
        g = int(rng.choice([1, 3, 6]))
        Hk = int(rng.choice([1, 2, 4]))
        qlen = rng.choice([1, 2, 4, 5, 37, 300, 1000], size=R, p=[.3, .1, .3, .1, .1, .05, .05])
        if case % 7 == 0:
            qlen[rng.integers(0, R)] = 0  # a request with no rows this step
        q_start = [0] + np.cumsum(qlen).tolist()
        seq_lens = (qlen + rng.integers(0, 40000, size=R)).tolist()
        fixed = int(rng.choice([0, 0, 3, 13]))
        got = A.plan_attention_host(q_start, seq_lens, g, Hk, 148, fixed_splits=fixed)
        want = _plan_loop(q_start, seq_lens, g, Hk, 148, fixed_splits=fixed)
        for x, y in zip(got, want):
            if isinstance(y, np.ndarray):
                assert x.dtype == y.dtype and x.shape == y.shape and np.array_equal(x, y), case
            else:
                assert x == y, case
