"""INT2 KV numeric contract and the page-packed physical layout.

Numeric contract (identical semantics to the reference's ``oscar_ascend/format.py``):

* per (token, head) vector ``x`` (fp32, already rotated and clipped):
  ``scale = max((max(x) - min(x)) / 3, 2**-14)`` and ``zero = min(x)``, both rounded
  to fp16 *before* use (``format.py:51-64``);
* ``q = clamp(floor((x - zero) / scale + 0.5), 0, 3)`` with true fp32 division and
  round-half-up, not banker's rounding (``format.py:67-88``);
* four codes per byte, code ``4b+k`` in bits ``2k..2k+1`` (``format.py:84-87``);
* the 160-byte logical slot (N-01): ``[0:2]`` K scale, ``[2:4]`` K zero, ``[4:6]`` V
  scale, ``[6:8]`` V zero (fp16 little-endian), ``[8:32]`` zero pad, ``[32:96]`` K codes,
  ``[96:160]`` V codes (``format.py:25-33``).  It is kept as an exchange format so that
  stored bytes can be compared with the reference oracle exactly.

Physical layout (this framework): the pool is page-major structure-of-arrays.  One
128-token page of one KV head is a contiguous block of ``PAGE*D/2 + 8*PAGE`` bytes
(17,408 B at D=256, i.e. 136 B per token and head)::

    [K codes  PAGE x D/4] [V codes PAGE x D/4]
    [K scale  PAGE fp16 ] [K zero  PAGE fp16 ] [V scale PAGE fp16] [V zero PAGE fp16]

so an attention CTA fetches one page-head with a single 16-byte-aligned bulk copy.

Bit order inside the pool differs from the exchange format: each little-endian
32-bit word of a code row covers 16 consecutive dims, and dim ``16w + 2m + e`` sits at
bit ``16e + 2m``.  Adjacent dims 2m, 2m+1 are then the two halves of
``(word >> 2m) & 0x00030003``, which the attention kernel widens to an fp16 pair
with one logic op.  ``pack_page``/``unpack_page`` convert.
"""
from __future__ import annotations

import torch

BITS = 2
LEVELS = 4
VALUES_PER_BYTE = 4
D_DEFAULT = 256
PAGE = 128  # tokens per kernel page

# Logical slot (exchange format, N-01)
SLOT_SIZE = 160
META_BYTES = 8
K_IDX_OFF = 32
V_IDX_OFF = 96

DEQUANT_TOL = 1e-5
DECODE_TOL = 1e-4
SCALE_FLOOR = 2.0 ** -14


def check_d(D: int) -> None:
    if D % VALUES_PER_BYTE != 0:
        raise ValueError(f"D={D} must be divisible by {VALUES_PER_BYTE} for INT2 packing")
    if D // VALUES_PER_BYTE > V_IDX_OFF - K_IDX_OFF:
        raise ValueError(f"D={D} does not fit the 160-byte logical slot")


# ---------------------------------------------------------------------------
# page geometry
# ---------------------------------------------------------------------------
def code_bytes(D: int) -> int:
    return D // VALUES_PER_BYTE


def page_head_bytes(D: int, page: int = PAGE) -> int:
    """Bytes of one page of one KV head: K codes + V codes + 4 fp16 meta arrays."""
    return page * code_bytes(D) * 2 + 4 * 2 * page


def page_offsets(D: int, page: int = PAGE) -> dict[str, int]:
    cb = code_bytes(D)
    k = 0
    v = page * cb
    ks = 2 * page * cb
    return {"k": k, "v": v, "k_scale": ks, "k_zero": ks + 2 * page,
            "v_scale": ks + 4 * page, "v_zero": ks + 6 * page,
            "total": ks + 8 * page}


# ---------------------------------------------------------------------------
# quantize / dequantize
# ---------------------------------------------------------------------------
def vector_scales(x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Per-vector (scale, zero), rounded to fp16 and returned as fp32 ``[..., 1]``."""
    x = x.float()
    lo = x.amin(dim=-1, keepdim=True)
    hi = x.amax(dim=-1, keepdim=True)
    scale = (hi - lo) / float(LEVELS - 1)
    scale = torch.where(scale > SCALE_FLOOR, scale, torch.full_like(scale, SCALE_FLOOR))
    return scale.half().float(), lo.half().float()


def codes(x: torch.Tensor, scale: torch.Tensor, zero: torch.Tensor) -> torch.Tensor:
    """Integer codes 0..3 (int32) with round-half-up on the true quotient."""
    return torch.clamp(torch.floor((x.float() - zero) / scale + 0.5), 0, LEVELS - 1).to(torch.int32)


def pack(q: torch.Tensor) -> torch.Tensor:
    """Codes ``[..., D]`` (0..3) -> bytes ``[..., D/4]`` with code 4b+k at bits 2k."""
    q4 = q.to(torch.int32).reshape(*q.shape[:-1], q.shape[-1] // 4, 4)
    b = q4[..., 0] | (q4[..., 1] << 2) | (q4[..., 2] << 4) | (q4[..., 3] << 6)
    return b.to(torch.uint8)


def unpack(packed: torch.Tensor, D: int) -> torch.Tensor:
    """Bytes ``[..., D/4]`` -> codes ``[..., D]`` (int32)."""
    p = packed.to(torch.int32)
    parts = [(p >> (2 * k)) & 3 for k in range(4)]
    return torch.stack(parts, dim=-1).reshape(*p.shape[:-1], D)


def _page_bit_positions(D: int) -> torch.Tensor:
    """Bit position (within the code row) of every dim in the pool's bit order."""
    d = torch.arange(D)
    w, j = d // 16, d % 16
    return w * 32 + 16 * (j % 2) + 2 * (j // 2)


def pack_page(q: torch.Tensor) -> torch.Tensor:
    """Codes ``[..., D]`` -> pool-order bytes ``[..., D/4]``."""
    D = q.shape[-1]
    pos = _page_bit_positions(D).to(q.device)
    byte, shift = pos // 8, pos % 8
    out = torch.zeros(*q.shape[:-1], D // 4, dtype=torch.int32, device=q.device)
    vals = (q.to(torch.int32) & 3) << shift.to(torch.int32)
    out.index_add_(-1 if out.dim() == 1 else out.dim() - 1, byte, vals)
    return out.to(torch.uint8)


def unpack_page(b: torch.Tensor, D: int) -> torch.Tensor:
    """Pool-order bytes ``[..., D/4]`` -> codes ``[..., D]`` (int32)."""
    pos = _page_bit_positions(D).to(b.device)
    byte, shift = pos // 8, pos % 8
    return (b.to(torch.int32)[..., byte] >> shift) & 3


def quantize(x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """``x [..., D]`` fp32 -> (packed ``[..., D/4]`` uint8, scale ``[...,1]``, zero ``[...,1]``)."""
    scale, zero = vector_scales(x)
    return pack(codes(x, scale, zero)), scale, zero


def dequant(packed: torch.Tensor, scale: torch.Tensor, zero: torch.Tensor, D: int) -> torch.Tensor:
    return unpack(packed, D).to(torch.float32) * scale + zero


def clip_sorted(x: torch.Tensor, ratio: float) -> torch.Tensor:
    """Per-vector clip at the ``min(int(ratio*D), D-1)``-th smallest ``|x|`` (ascending).

    Same threshold rule as the reference's sort-based clip (``backend.py:129-147``);
    ``ratio == 0`` disables clipping.
    """
    x = x.float()
    if ratio <= 0.0:
        return x
    D = x.shape[-1]
    idx = min(int(ratio * D), D - 1)
    thr = x.abs().sort(dim=-1).values[..., idx: idx + 1]
    return torch.maximum(torch.minimum(x, thr), -thr)


# ---------------------------------------------------------------------------
# fp16 little-endian helpers and the 160-byte logical slot
# ---------------------------------------------------------------------------
def f16_le(x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    bits = x.contiguous().half().view(torch.int16).to(torch.int32) & 0xFFFF
    return (bits & 0xFF).to(torch.uint8), ((bits >> 8) & 0xFF).to(torch.uint8)


def f16_from_le(lo: torch.Tensor, hi: torch.Tensor) -> torch.Tensor:
    bits = (lo.to(torch.int32) | (hi.to(torch.int32) << 8)).to(torch.int16)
    return bits.view(torch.float16).float()


def make_slot_bytes(k_rot: torch.Tensor, v_rot: torch.Tensor) -> torch.Tensor:
    """``[N, H, D]`` rotated K/V -> ``[N, H, 160]`` logical slots (N-01 byte order)."""
    N, H, D = k_rot.shape
    check_d(D)
    cb = code_bytes(D)
    kp, ks, kz = quantize(k_rot)
    vp, vs, vz = quantize(v_rot)
    slot = torch.zeros(N, H, SLOT_SIZE, dtype=torch.uint8, device=k_rot.device)
    for i, t in enumerate((ks, kz, vs, vz)):
        lo, hi = f16_le(t)
        slot[..., 2 * i: 2 * i + 1] = lo
        slot[..., 2 * i + 1: 2 * i + 2] = hi
    slot[..., K_IDX_OFF: K_IDX_OFF + cb] = kp
    slot[..., V_IDX_OFF: V_IDX_OFF + cb] = vp
    return slot


def parse_slot_bytes(slot: torch.Tensor, D: int) -> tuple[torch.Tensor, torch.Tensor]:
    check_d(D)
    cb = code_bytes(D)
    meta = [f16_from_le(slot[..., 2 * i: 2 * i + 1], slot[..., 2 * i + 1: 2 * i + 2]) for i in range(4)]
    k = dequant(slot[..., K_IDX_OFF: K_IDX_OFF + cb], meta[0], meta[1], D)
    v = dequant(slot[..., V_IDX_OFF: V_IDX_OFF + cb], meta[2], meta[3], D)
    return k, v


# ---------------------------------------------------------------------------
# page-packed pool views
# ---------------------------------------------------------------------------
def page_views(pool: torch.Tensor, D: int, page: int = PAGE):
    """Split a ``[blocks, Hk, page_head_bytes]`` uint8 pool into typed views.

    Returns ``(k_codes [B,Hk,page,D/4], v_codes_t [B,Hk,D,page/4], k_scale [B,Hk,page]
    fp16, k_zero, v_scale, v_zero)``.  K codes are token-major (one row of ``D/4`` bytes
    per token, dims in the pool bit order, 16-byte chunks swizzled by the token, see
    :func:`k_chunk_perm`); V codes are dim-major (one row of ``page/4`` bytes per dim,
    tokens in the same bit order), which is the operand layout of the P.V product in
    the attention kernels.
    """
    nb, hk, pb = pool.shape
    off = page_offsets(D, page)
    assert pb == off["total"], f"pool page size {pb} != {off['total']}"
    cb = code_bytes(D)
    kc = pool[:, :, off["k"]: off["v"]].view(nb, hk, page, cb)
    vt = pool[:, :, off["v"]: off["k_scale"]].view(nb, hk, D, page // 4)
    meta = pool.view(torch.float16)[:, :, off["k_scale"] // 2: off["total"] // 2].view(nb, hk, 4, page)
    return kc, vt, meta[:, :, 0], meta[:, :, 1], meta[:, :, 2], meta[:, :, 3]


def k_chunk_perm(offs: torch.Tensor, D: int) -> torch.Tensor:
    """Byte permutation of the K code rows of tokens ``offs``: the row's 16-byte chunk
    ``c`` is stored at chunk ``c ^ ((off >> 1) & (D/64 - 1))`` (bank-conflict-free reads
    of one row per thread in the attention kernels).  Returns ``[T, D/4]`` byte indices:
    ``stored[:, idx[t]] == logical``."""
    cb = code_bytes(D)
    nch = cb // 16
    b = torch.arange(cb, device=offs.device)
    ch, within = b // 16, b % 16
    sw = (ch.unsqueeze(0) ^ ((offs.long().unsqueeze(1) >> 1) & (nch - 1))) * 16 + within.unsqueeze(0)
    return sw


def read_k_codes(kc: torch.Tensor, b: torch.Tensor, o: torch.Tensor, D: int) -> torch.Tensor:
    """Codes ``[T, Hk, D]`` of tokens ``(b, o)`` from the token-major K view."""
    rows = kc[b.long(), :, o.long()]  # [T, Hk, D/4] stored order
    idx = k_chunk_perm(o, D).unsqueeze(1).expand(-1, rows.shape[1], -1)
    return unpack_page(torch.gather(rows, 2, idx), D)


def write_k_codes(kc: torch.Tensor, b: torch.Tensor, o: torch.Tensor, q: torch.Tensor) -> None:
    D = q.shape[-1]
    logical = pack_page(q)  # [T, Hk, D/4]
    idx = k_chunk_perm(o, D).unsqueeze(1).expand(-1, logical.shape[1], -1)
    stored = torch.empty_like(logical)
    stored.scatter_(2, idx, logical)
    kc[b.long(), :, o.long()] = stored


def _token_byte_shift(offs: torch.Tensor, page: int = PAGE):
    pos = _page_bit_positions(page).to(offs.device)[offs.long()]
    return pos // 8, pos % 8


def read_v_codes(vt: torch.Tensor, b: torch.Tensor, o: torch.Tensor) -> torch.Tensor:
    """Codes ``[T, Hk, D]`` of tokens ``(b, o)`` from the dim-major V view."""
    byte, shift = _token_byte_shift(o, vt.shape[-1] * 4)
    raw = vt[b.long(), :, :, byte].to(torch.int32)  # [T, Hk, D]
    return (raw >> shift.view(-1, 1, 1).to(torch.int32)) & 3


def write_v_codes(vt: torch.Tensor, b: torch.Tensor, o: torch.Tensor, q: torch.Tensor) -> None:
    """Store codes ``q [T, Hk, D]`` of tokens ``(b, o)`` into the dim-major V view.  Four
    tokens share a byte, so the writes go in four passes of non-colliding tokens."""
    page = vt.shape[-1] * 4
    byte, shift = _token_byte_shift(o, page)
    lane = ((o.long() % 16) // 2) % 4  # tokens of one byte differ here
    for p in range(4):
        sel = torch.nonzero(lane == p, as_tuple=True)[0]
        if sel.numel() == 0:
            continue
        bb, by, sh = b[sel].long(), byte[sel], shift[sel].view(-1, 1, 1).to(torch.int32)
        cur = vt[bb, :, :, by].to(torch.int32)
        new = (cur & ~(3 << sh)) | ((q[sel].to(torch.int32) & 3) << sh)
        vt[bb, :, :, by] = new.to(torch.uint8)


def pool_to_slots(pool: torch.Tensor, blocks: torch.Tensor, offs: torch.Tensor, D: int) -> torch.Tensor:
    """Read tokens ``(blocks[i], offs[i])`` of a page-packed pool as ``[T, Hk, 160]`` slots."""
    kc, vt, ks, kz, vs, vz = page_views(pool, D)
    b, o = blocks.long(), offs.long()
    T, hk = b.numel(), pool.shape[1]
    cb = code_bytes(D)
    slot = torch.zeros(T, hk, SLOT_SIZE, dtype=torch.uint8, device=pool.device)
    for i, t in enumerate((ks, kz, vs, vz)):
        lo, hi = f16_le(t[b, :, o].float().unsqueeze(-1))
        slot[..., 2 * i: 2 * i + 1] = lo
        slot[..., 2 * i + 1: 2 * i + 2] = hi
    slot[..., K_IDX_OFF: K_IDX_OFF + cb] = pack(read_k_codes(kc, b, o, D))
    slot[..., V_IDX_OFF: V_IDX_OFF + cb] = pack(read_v_codes(vt, b, o))
    return slot


def dequant_tokens(pool: torch.Tensor, blocks: torch.Tensor, offs: torch.Tensor, D: int):
    """Dequantize tokens of a page-packed pool -> ``(k [T,Hk,D], v [T,Hk,D])`` fp32 (rotated space)."""
    kc, vt, ks, kz, vs, vz = page_views(pool, D)
    b, o = blocks.long(), offs.long()
    k = read_k_codes(kc, b, o, D).float() * ks[b, :, o].float().unsqueeze(-1) + kz[b, :, o].float().unsqueeze(-1)
    v = read_v_codes(vt, b, o).float() * vs[b, :, o].float().unsqueeze(-1) + vz[b, :, o].float().unsqueeze(-1)
    return k, v


def write_tokens(pool: torch.Tensor, blocks: torch.Tensor, offs: torch.Tensor, k_c: torch.Tensor,
                 v_c: torch.Tensor) -> None:
    """Quantize clipped rotated ``k_c/v_c [T,Hk,D]`` into the pool at ``(blocks, offs)``."""
    D = k_c.shape[-1]
    kc, vt, ks, kz, vs, vz = page_views(pool, D)
    b, o = blocks.long(), offs.long()
    for is_v, x, sv, zv in ((False, k_c, ks, kz), (True, v_c, vs, vz)):
        scale, zero = vector_scales(x)
        q = codes(x, scale, zero)
        if is_v:
            write_v_codes(vt, b, o, q)
        else:
            write_k_codes(kc, b, o, q)
        sv[b, :, o] = scale.squeeze(-1).half()
        zv[b, :, o] = zero.squeeze(-1).half()


def rotate(x: torch.Tensor, R: torch.Tensor) -> torch.Tensor:
    return torch.matmul(x.float(), R)
