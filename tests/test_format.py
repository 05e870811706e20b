"""INT2 numeric contract (N-01..N-04) and page layout, CPU only.

Golden behaviours mirror the reference's numeric tests (``tests/test_numeric.py``):
quant/dequant round trip <= 1e-5, slot round trip, round-half-up (not banker's),
scale floor, fp16-first scale/zero, little-endian meta, 2-bit packing order.
"""
import math

import torch

from oscar_b200.kv import format as fmt
from oscar_b200.kv import oracle


def test_quant_dequant_roundtrip():
    torch.manual_seed(0)
    x = torch.randn(5, 3, 64) * 1.5
    packed, s, z = fmt.quantize(x)
    rec = fmt.dequant(packed, s, z, 64)
    q = torch.clamp(torch.floor((x - z) / s + 0.5), 0, 3)
    assert (rec - (q * s + z)).abs().max() <= fmt.DEQUANT_TOL


def test_round_half_up_not_bankers():
    # (x - zero) / scale == 0.5 exactly must round up to 1 (torch.round would give 0)
    x = torch.tensor([[0.0, 0.5, 1.5, 3.0]])
    _, s, z = fmt.quantize(x)
    assert s.item() == 1.0 and z.item() == 0.0
    codes = fmt.unpack(fmt.quantize(x)[0], 4)
    assert codes.tolist() == [[0, 1, 2, 3]]


def test_scale_floor_and_constant_vector():
    x = torch.full((1, 16), 3.25)
    p, s, z = fmt.quantize(x)
    assert s.item() == 2.0 ** -14
    assert fmt.unpack(p, 16).eq(0).all()
    assert torch.allclose(fmt.dequant(p, s, z, 16), x)


def test_scale_zero_rounded_to_fp16_first():
    x = torch.tensor([[0.1, 0.7, 0.33, 1.0000001]])
    _, s, z = fmt.quantize(x)
    assert s.item() == torch.tensor((1.0000001 - 0.1) / 3).half().float().item()
    assert z.item() == torch.tensor(0.1).half().float().item()


def test_pack_order():
    q = torch.tensor([[1, 2, 3, 0, 3, 3, 3, 3]])
    b = fmt.pack(q)
    assert b.tolist() == [[1 | (2 << 2) | (3 << 4), 255]]
    assert fmt.unpack(b, 8).tolist() == q.tolist()


def test_slot_bytes_roundtrip_and_le_meta():
    torch.manual_seed(1)
    k, v = torch.randn(4, 2, 256), torch.randn(4, 2, 256)
    slot = fmt.make_slot_bytes(k, v)
    assert slot.shape == (4, 2, 160)
    assert slot[..., 8:32].eq(0).all()
    _, ks, _ = fmt.quantize(k)
    lo = slot[..., 0].to(torch.int32)
    hi = slot[..., 1].to(torch.int32)
    assert torch.equal(((hi << 8) | lo).to(torch.int16).view(torch.float16).float(), ks.squeeze(-1))
    kr, vr = fmt.parse_slot_bytes(slot, 256)
    kp, ks, kz = fmt.quantize(k)
    assert torch.allclose(kr, fmt.dequant(kp, ks, kz, 256))


def test_page_layout_and_store_ref_matches_slot_contract():
    torch.manual_seed(2)
    D, H, N = 256, 2, 9
    pool = torch.zeros(3, H, fmt.page_head_bytes(D), dtype=torch.uint8)
    assert fmt.page_head_bytes(D) == 17408
    k, v = torch.randn(N, H, D), torch.randn(N, H, D)
    slots = torch.tensor([0, 1, 2, 130, 131, -1, 255, 300, 301])
    oracle.store_ref(k, v, pool, slots)
    valid = slots >= 0
    s = slots[valid]
    got = fmt.pool_to_slots(pool, s // 128, s % 128, D)
    want = fmt.make_slot_bytes(k[valid], v[valid])
    assert torch.equal(got, want)


def test_clip_threshold_rule():
    x = torch.arange(1, 257, dtype=torch.float32).view(1, 256)
    c = fmt.clip_sorted(x, 0.96)  # idx = int(245.76) = 245 -> 246th smallest |x| = 246
    assert c.max().item() == 246.0
    assert fmt.clip_sorted(x, 0.0).equal(x)


def test_staging_rows_formula():
    # rows = max(ceil(staging/bs), sink_pages + tail_pages + 2) (backend.py:418-437)
    assert oracle.staging_rows(128, 256, 8192) == 64
    assert oracle.staging_rows(128, 256, 0) == 1 + (2 + 1) + 2
    assert oracle.staging_rows(64, 256, 128) == 0 + 3 + 2


def test_seat_plan_last_writer_and_invalidation():
    from oscar_b200.engine.staging import seat_plan
    import numpy as np

    rows = 2
    # tokens 0 and 2 share seat 0 (blocks 0 and 2 hash to row 0); token 2 is last and not kept
    slots = np.array([0, 128 + 5, 256], dtype=np.int64)
    pos = np.array([10, 20, 5000], dtype=np.int64)
    seq = np.array([6000, 6000, 6000], dtype=np.int64)
    stage_seat, seat, owner = seat_plan(slots, pos, seq, rows, sink_tokens=128, recent_tokens=256)
    d = dict(zip(seat.tolist(), owner.tolist()))
    assert d[0] == -1          # last writer (token 2, pos 5000) is outside the window
    assert d[128 + 5] == 1     # block 1, kept as sink token
    assert stage_seat.tolist() == [-1, 128 + 5, -1]


def test_paged_attention_ref_equals_dense_sdpa():
    """Oracle self-consistency: paged reads == dense SDPA over the dequantized cache."""
    torch.manual_seed(3)
    D, hk, hq = 64, 1, 4
    prefix, n = 300, 4
    pool = torch.zeros(4, hk, fmt.page_head_bytes(D), dtype=torch.uint8)
    k, v = torch.randn(prefix, hk, D), torch.randn(prefix, hk, D)
    bt = torch.tensor([[3, 1, 0, 2]])
    pos = torch.arange(prefix)
    slots = bt[0, pos // 128] * 128 + pos % 128
    oracle.store_ref(k, v, pool, slots)
    q, kn, vn = torch.randn(n, hq, D), torch.randn(n, hk, D), torch.randn(n, hk, D)
    out = oracle.paged_attention_ref(q, kn, vn, pool, bt, [0, n], [prefix + n], 0.125)
    kd, vd = fmt.dequant_tokens(pool, bt[0, pos // 128], pos % 128, D)
    want = oracle.sdpa_causal(q, torch.cat([kd, kn]), torch.cat([vd, vn]), 0.125, prefix)
    assert torch.allclose(out, want, atol=1e-5)
