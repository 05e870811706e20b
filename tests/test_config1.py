"""BASELINE config 1 on the CPU: single-layer OSCAR decode vs the SDPA oracle.

Hq = 6, Hk = 1 (6:1 GQA), head_dim 256, 128-token pages, 24,579-token history plus a
4-token MTP query chunk; Q/K/V ~ N(0, 1) in fp32 cast to bf16 from seed 0; per-layer
random orthogonal K/V rotations from the QR of a seeded Gaussian; clip K 0.96 / V 0.92;
sink 128, recent 256, staging 8192.

The OSCAR read path (rotate -> INT2 store + staging -> paged multi-query attention in
rotated space -> @ R_v^T) must equal SDPA over the dequantised, staging-spliced cache
brought back to the original domain within the reference's decode tolerance (1e-4).
"""
import math

import torch

from oscar_b200.kv import format as fmt
from oscar_b200.kv import oracle as O


def test_config1_decode_vs_sdpa_oracle():
    g = torch.Generator().manual_seed(0)
    hq, hk, D, hist, n = 6, 1, 256, 24579, 4
    q = torch.randn(n, hq, D, generator=g).to(torch.bfloat16).float()
    k = torch.randn(hist + n, hk, D, generator=g).to(torch.bfloat16).float()
    v = torch.randn(hist + n, hk, D, generator=g).to(torch.bfloat16).float()
    Rk = torch.linalg.qr(torch.randn(D, D, generator=g))[0]
    Rv = torch.linalg.qr(torch.randn(D, D, generator=g))[0]
    pages = (hist + n + 127) // 128
    pool = torch.zeros(pages, hk, fmt.page_head_bytes(D), dtype=torch.uint8)
    slots = torch.arange(hist)
    k_rot, v_rot = O.store_ref(k[:hist], v[:hist], pool, slots, Rk, Rv, 0.96, 0.92)
    rows = O.staging_rows(128, 256, 8192)
    stage = O.StagingArena(rows, hk, D)
    stage.write(O.seat_plan(slots, slots, torch.full((hist,), hist + n), rows, 128, 256), k_rot, v_rot)
    bt = torch.arange(pages, dtype=torch.int32).view(1, -1)
    scale = 1 / math.sqrt(D)
    out = O.oscar_attention_ref(q, k[hist:], v[hist:], pool, bt, [0, n], [hist + n], scale, Rk, Rv, stage)

    # oracle: dequantised history, staged tokens spliced, back to the original domain
    kh, vh = O.gather_history(pool, bt[0], hist, D, stage)
    kk = torch.cat([kh @ Rk.t(), k[hist:]])
    vv = torch.cat([vh @ Rv.t(), v[hist:]])
    ref = O.sdpa_causal(q, kk, vv, scale, hist)
    err = float((out - ref).norm() / ref.norm())
    assert err <= fmt.DECODE_TOL, err

    # quality of INT2 + window against exact attention on the unquantised cache
    exact = O.sdpa_causal(q, k, v, scale, hist)
    q_err = float((out - exact).norm() / exact.norm())
    assert q_err < 1.0
    # the staging window holds the recent tokens (history positions >= seq - 256); with
    # 193 pages hashed onto 64 rows the sink page's seats were rewritten by later,
    # unkept tokens (owner -1): the reference's last-writer-wins arena behaves the same
    own = stage.owner.view(-1)
    assert int((own >= 0).sum()) == hist - (hist + n - 256)
    assert int((own == 0).sum()) == 0


def test_config1_window_layout_keeps_the_sink():
    """The per-request window layout (this framework's default) gives the sink page rows of
    its own: at the same 24,579-token shape every one of the first 128 tokens stays staged
    (fp32) next to the recent window, and the read path still equals the SDPA oracle over
    the staging-spliced cache within 1e-4."""
    g = torch.Generator().manual_seed(0)
    hq, hk, D, hist, n = 6, 1, 256, 24579, 4
    q = torch.randn(n, hq, D, generator=g).to(torch.bfloat16).float()
    k = torch.randn(hist + n, hk, D, generator=g).to(torch.bfloat16).float()
    v = torch.randn(hist + n, hk, D, generator=g).to(torch.bfloat16).float()
    Rk = torch.linalg.qr(torch.randn(D, D, generator=g))[0]
    Rv = torch.linalg.qr(torch.randn(D, D, generator=g))[0]
    pages = (hist + n + 127) // 128
    pool = torch.zeros(pages, hk, fmt.page_head_bytes(D), dtype=torch.uint8)
    slots = torch.arange(hist)
    k_rot, v_rot = O.store_ref(k[:hist], v[:hist], pool, slots, Rk, Rv, 0.96, 0.92)
    sink_pages, ring = O.window_layout(128, 256)
    req_slot = 3
    rows = O.arena_rows(128, 256, 8192, "window", max_slots=4)
    token_rows = O.window_row(req_slot, slots // 128, sink_pages, ring)
    stage = O.StagingArena(rows, hk, D)
    stage.write(O.seat_plan(slots, slots, torch.full((hist,), hist + n), rows, 128, 256, token_rows=token_rows),
                k_rot, v_rot)
    page_rows = O.window_row(req_slot, torch.arange(pages), sink_pages, ring)
    bt = torch.arange(pages, dtype=torch.int32).view(1, -1)
    # the sink page keeps its row: all 128 tags equal its block (block 0)
    assert int((stage.owner[int(page_rows[0])] == 0).sum()) == 128
    kh, vh = O.gather_history(pool, bt[0], hist, D, stage, page_rows)
    assert torch.equal(kh[:128], k_rot[:128]) and torch.equal(vh[:128], v_rot[:128])  # unquantised sink
    assert torch.equal(kh[hist + n - 256:], k_rot[hist + n - 256:])  # and the recent window
    scale = 1 / math.sqrt(D)
    kk = torch.cat([kh @ Rk.t(), k[hist:]])
    vv = torch.cat([vh @ Rv.t(), v[hist:]])
    ref = O.sdpa_causal(q, kk, vv, scale, hist)
    exact = O.sdpa_causal(q, k, v, scale, hist)
    assert float((ref - exact).norm() / exact.norm()) < 1.0
