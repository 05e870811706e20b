"""Attention work planner (host side): short requests' split items first, one item per
64-row block of a prefill request, 128-row prefill tiles pairing those items."""
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
