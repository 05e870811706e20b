"""OSCAR FULL-attention ops: fused KV store, paged INT2/BF16 attention, split merge.

GPU path (three launches per layer and step):

1. ``kv_store``  - q/k RMSNorm + partial RoPE + fp32 rotation + clip + INT2 quantise +
   page write + fp32 staging write (or a BF16 page write for the MTP draft layer);
2. ``paged_attention`` - split-KV multi-query GQA attention over pages, staging and
   the current chunk, tensor-core tiles, partial (O, LSE) per work item;
3. ``attn_merge`` - split combine, ``o_rot @ R_vᵀ``, sigmoid output gate, int8 quant.

The CPU path computes the same result with the torch oracle
(:mod:`oscar_b200.kv.oracle`).
"""
from __future__ import annotations

import math
import os
from dataclasses import dataclass

import numpy as np
import torch
import torch.nn.functional as F

from ..kv import format as fmt
from ._ext import ext
from .functional import apply_rope_ref, head_rmsnorm_ref, quantize_rows_ref, _bf16_round

ROWS = 64  # rows (query token x head-in-group) per attention work item
# INT2 work items of <= 32 rows run on the tcgen05/TMEM kernel (OSCAR_ATTN_TC=0 keeps
# every item on the warp-level mma.sync kernel, for A/B comparisons)
USE_TC = os.environ.get("OSCAR_ATTN_TC", "1") != "0"


def _rpi(plan: "AttnPlan", q_start: list[int], g: int) -> int:
    """Rows per item the decode/verify kernel is instantiated for (0: warp-level kernel)."""
    if not USE_TC:
        return 0
    return plan.rpi_short if plan.n_tiles > 0 else rows_per_item(q_start, g)


# INT2 prefill chunks run on the tcgen05 prefill kernel when USE_TC is set (the
# OSCAR_ATTN_PREFILL_TC=0 environment switch of the extension keeps them on the
# warp-level kernel for A/B comparisons).


def rows_per_item(q_start: list[int], g: int) -> int:
    """Largest number of query rows (q_len x g, capped at ROWS) of any work item."""
    n = max((q_start[i + 1] - q_start[i] for i in range(len(q_start) - 1)), default=0)
    return min(ROWS, n * g)


@dataclass
class AttnPlan:
    """Host-built work decomposition of one step (shared by every FULL layer)."""

    work: torch.Tensor        # [n_work, 4] int32: req, row0, kv_begin, kv_end
    item_first: torch.Tensor  # [R * max_rb] int32
    item_count: torch.Tensor  # [R * max_rb] int32
    max_rb: int
    n_work: int
    # prefill tiles of 128 rows for the INT2 tensor-core prefill kernel:
    # [n_tiles, 4] int32 (req, row0, item of rows 0-63, item of rows 64-127 or -1)
    tiles: torch.Tensor | None = None
    n_tiles: int = 0
    n_short: int = -1    # items of the short (decode / verify) requests come first
    rpi_short: int = 0   # largest row count of a short request's item


LONG_ROWS = 32  # requests with more query rows (q_len x g) are prefill ("long") requests


def plan_attention_host(q_start: list[int], seq_lens: list[int], g: int, Hk: int, sms: int,
                        min_chunk: int = 256, waves: int = 3, fixed_splits: int = 0, long_rows: int = LONG_ROWS):
    """Work list as numpy arrays:
    ``(work [n,4], item_first, item_count, max_rb, n_work, tiles [n_tiles,4], n_short, rpi_short)``.

    Items of short requests (<= ``long_rows`` query rows) come first and are split over
    the KV range for parallelism; ``fixed_splits > 0`` gives each of their row blocks
    exactly that many page-aligned splits (some may be empty), so the work-list shape
    depends only on the batch shape - the form a captured CUDA graph replays.  Long
    (prefill) requests get one item per 64-row block covering their whole KV range,
    paired into 128-row ``tiles`` for the tensor-core prefill kernel.
    """
    R = len(seq_lens)
    blocks = []  # (req, row0, kv_need, long)
    max_rb = 1
    for r in range(R):
        n = q_start[r + 1] - q_start[r]
        if n <= 0:
            continue
        prefix = seq_lens[r] - n
        rows = n * g
        rb = (rows + ROWS - 1) // ROWS
        max_rb = max(max_rb, rb)
        for b in range(rb):
            last_row = min(rows, (b + 1) * ROWS) - 1
            blocks.append((r, b * ROWS, prefix + last_row // g + 1, rows > long_rows))
    short = [bk for bk in blocks if not bk[3]]
    longb = [bk for bk in blocks if bk[3]]
    total = sum(k for _, _, k, _ in short)
    target_items = max(1, (waves * sms) // max(Hk, 1))
    # page-aligned (128-token) split ranges: every split streams whole pages
    chunk = max(min_chunk, int(math.ceil(total / target_items / 128.0)) * 128) if total else min_chunk
    first = np.zeros(R * max_rb, dtype=np.int32)
    count = np.zeros(R * max_rb, dtype=np.int32)
    rpi_short = 0
    if short:
        sb = np.asarray([(r, row0, need) for r, row0, need, _ in short], dtype=np.int64)
        r_, row0_, need_ = sb[:, 0], sb[:, 1], sb[:, 2]
        qs = np.asarray(q_start, dtype=np.int64)
        rows_ = (qs[r_ + 1] - qs[r_]) * g
        rpi_short = int(np.minimum(ROWS, rows_ - row0_).max())
        if fixed_splits > 0:
            splits = np.full(len(short), fixed_splits, dtype=np.int64)
            step = np.maximum(128, np.ceil(need_ / splits / 128.0).astype(np.int64) * 128)
        else:
            splits = np.maximum(1, (need_ + chunk - 1) // chunk)
            step = np.full(len(short), chunk, dtype=np.int64)
        off = np.concatenate([[0], np.cumsum(splits)[:-1]])
        slot = r_ * max_rb + row0_ // ROWS
        first[slot] = off
        count[slot] = splits
        blk = np.repeat(np.arange(len(short)), splits)
        sidx = np.arange(int(splits.sum())) - off[blk]
        b0 = np.minimum(need_[blk], sidx * step[blk])
        b1 = np.minimum(need_[blk], b0 + step[blk])
        work_short = np.stack([r_[blk], row0_[blk], b0, b1], axis=1)
    else:
        work_short = np.zeros((0, 4), dtype=np.int64)
    work = []
    n_short = int(work_short.shape[0])
    for r, row0, need, _ in longb:
        rb = row0 // ROWS
        first[r * max_rb + rb] = n_short + len(work)
        count[r * max_rb + rb] = 1
        work.append((r, row0, 0, need))
    tiles = []
    for r, row0, need, _ in longb:
        if row0 % (2 * ROWS):
            continue
        rb = row0 // ROWS
        rows = (q_start[r + 1] - q_start[r]) * g
        item_b = int(first[r * max_rb + rb + 1]) if row0 + ROWS < rows else -1
        tiles.append((r, row0, int(first[r * max_rb + rb]), item_b))
    # longest tiles (most keys) first
    tiles.sort(key=lambda t: -(seq_lens[t[0]] - (q_start[t[0] + 1] - q_start[t[0]]) + t[1] // g))
    n_work = n_short + len(work)
    wt = np.concatenate([work_short, np.asarray(work, dtype=np.int64).reshape(-1, 4)]).astype(np.int32)
    if not n_work:
        wt = np.zeros((1, 4), dtype=np.int32)
    tt = np.asarray(tiles if tiles else [(0, 0, -1, -1)], dtype=np.int32).reshape(-1, 4)
    return wt, first, count, max_rb, n_work, tt, n_short, rpi_short


def decode_splits(q_start: list[int], g: int, Hk: int, sms: int) -> int:
    """Page-aligned splits per row block of a decode / verify step: about three CTAs per
    SM over all (row block, KV head) pairs.  The result depends only on the batch shape,
    which a replayed CUDA graph needs."""
    n_blocks = sum((q_start[i + 1] - q_start[i]) * g // ROWS + 1 for i in range(len(q_start) - 1))
    return max(1, (3 * sms) // max(1, Hk * n_blocks))


def plan_attention(q_start: list[int], seq_lens: list[int], g: int, Hk: int, sms: int,
                   device, min_chunk: int = 256, waves: int = 3) -> AttnPlan:
    wt, first, count, max_rb, n_work, tt, n_short, rpi_short = plan_attention_host(q_start, seq_lens, g, Hk, sms,
                                                                                   min_chunk, waves)
    n_tiles = int((tt[:, 2] >= 0).sum()) if n_work > n_short else 0
    return AttnPlan(torch.from_numpy(wt).to(device), torch.from_numpy(first).to(device),
                    torch.from_numpy(count).to(device), max_rb, n_work, torch.from_numpy(tt).to(device), n_tiles,
                    n_short, rpi_short)


# ---------------------------------------------------------------------------
# KV store
# ---------------------------------------------------------------------------
def clip_by_index(x: torch.Tensor, idx: int) -> torch.Tensor:
    if idx < 0:
        return x
    thr = x.abs().sort(dim=-1).values[..., idx: idx + 1]
    return torch.maximum(torch.minimum(x, thr), -thr)


def split_rotation(R: torch.Tensor | None):
    """``R^T`` as bf16 hi + lo parts (``R^T ~ hi + lo`` to ~2^-16) for the tensor-core rotation."""
    if R is None:
        return None, None
    RT = R.t().contiguous().float()
    hi = RT.to(torch.bfloat16)
    lo = (RT - hi.float()).to(torch.bfloat16)
    return hi.contiguous(), lo.contiguous()


def kv_store(qkv, *, q_off, q_head_stride, k_off, v_off, Hq, Hk, D, q_norm_w, k_norm_w, eps, norm_offset,
             positions, rope_cos, rope_sin, rot_dim, Rk, Rv, k_clip_idx, v_clip_idx, q_out, k_fresh, v_fresh,
             kv_mode, pool, kc, vc, slots, stage_k=None, stage_v=None, stage_seat=None, owner=None,
             owner_seat=None, owner_val=None, status=None, rk_split=None, rv_split=None):
    """Fused write path of one FULL layer; see the module docstring.

    ``rk_split``/``rv_split`` are the precomputed :func:`split_rotation` of ``Rk``/``Rv``.
    """
    if qkv.is_cuda:
        if rk_split is None:
            rk_split = split_rotation(Rk)
        if rv_split is None:
            rv_split = split_rotation(Rv)
        xbuf = torch.empty(qkv.shape[0] * (Hq + 2 * Hk) * D, dtype=torch.bfloat16, device=qkv.device)
        ext().kv_store(qkv, q_off, q_head_stride, k_off, v_off, Hq, Hk, D, q_norm_w, k_norm_w, float(eps),
                       float(norm_offset), positions, rope_cos, rope_sin, rot_dim, Rk, Rv, k_clip_idx, v_clip_idx,
                       q_out, k_fresh, v_fresh, kv_mode, pool, kc, vc, slots, stage_k, stage_v, stage_seat, owner,
                       owner_seat, owner_val, status, rk_split[0], rk_split[1], rv_split[0], rv_split[1], xbuf)
        return
    T = qkv.shape[0]
    x = qkv.float()
    q = torch.stack([x[:, q_off + h * q_head_stride: q_off + h * q_head_stride + D] for h in range(Hq)], 1)
    k = x[:, k_off:k_off + Hk * D].reshape(T, Hk, D)
    v = x[:, v_off:v_off + Hk * D].reshape(T, Hk, D)
    if q_norm_w is not None:
        q = head_rmsnorm_ref(q, q_norm_w, eps, norm_offset)
    if k_norm_w is not None:
        k = head_rmsnorm_ref(k, k_norm_w, eps, norm_offset)
    if rope_cos is not None and rot_dim > 0:
        q = apply_rope_ref(q, positions, rope_cos, rope_sin, rot_dim)
        k = apply_rope_ref(k, positions, rope_cos, rope_sin, rot_dim)
    qr = q @ Rk if Rk is not None else q
    kr = k @ Rk if Rk is not None else k
    vr = v @ Rv if Rv is not None else v
    q_out.copy_(qr.half())
    k_fresh.copy_(kr.half())
    v_fresh.copy_(vr.half())
    if owner_seat is not None and owner_seat.numel():
        owner.view(-1)[owner_seat.long()] = owner_val.to(owner.dtype)
    if stage_seat is not None:
        sel = torch.nonzero(stage_seat >= 0, as_tuple=True)[0]
        if sel.numel():
            seats = stage_seat[sel].long()
            stage_k.view(-1, Hk, D)[seats] = kr[sel]
            stage_v.view(-1, Hk, D, fmt.PAGE)[seats // fmt.PAGE, :, :, seats % fmt.PAGE] = vr[sel]
    valid = torch.nonzero(slots >= 0, as_tuple=True)[0]
    if valid.numel() == 0:
        return
    s = slots[valid].long()
    blk, off = s // fmt.PAGE, s % fmt.PAGE
    if kv_mode == 1:
        kc[blk, off] = kr[valid].to(torch.bfloat16)
        vc[blk, off] = vr[valid].to(torch.bfloat16)
        return
    fmt.write_tokens(pool, blk, off, clip_by_index(kr[valid], k_clip_idx), clip_by_index(vr[valid], v_clip_idx))


# ---------------------------------------------------------------------------
# attention + merge
# ---------------------------------------------------------------------------
def _history_fp16(kv_mode, pool, kc, vc, stage, bt_row, count, hk_idx, D):
    """History K/V ``[count, D]`` of one KV head as the kernel sees it (fp16-rounded)."""
    pos = torch.arange(count, device=bt_row.device)
    blocks = bt_row[pos // fmt.PAGE].long()
    offs = pos % fmt.PAGE
    if kv_mode == 1:
        k = kc[blocks, offs, hk_idx].float()
        v = vc[blocks, offs, hk_idx].float()
    else:
        kk, vv = fmt.dequant_tokens(pool, blocks, offs, D)
        k, v = kk[:, hk_idx], vv[:, hk_idx]
    if stage is not None and count:
        sk, sv, owner, rows = stage[:4]
        lay = stage[4] if len(stage) > 4 else None  # (slot of this request, sink pages, ring)
        if lay is None:
            r = blocks % rows
        else:
            from ..kv.oracle import window_row
            r = window_row(int(lay[0]), pos // fmt.PAGE, lay[1], lay[2])
        hit = (owner.view(rows, fmt.PAGE)[r, offs].long() == blocks).unsqueeze(-1)
        k = torch.where(hit, sk.view(rows, fmt.PAGE, -1, D)[r, offs, hk_idx], k)
        v = torch.where(hit, sv.view(rows, -1, D, fmt.PAGE)[r, hk_idx, :, offs], v)
    return k.half().float(), v.half().float()


def attention_ref(q, k_fresh, v_fresh, *, Hq, Hk, D, scale, kv_mode, pool, kc, vc, stage, block_tables,
                  q_start: list[int], seq_lens: list[int]) -> torch.Tensor:
    """Rotated-space attention output ``[T, Hq, D]`` (fp32) with the kernel's inputs."""
    T = q.shape[0]
    g = Hq // Hk
    out = torch.zeros(T, Hq, D, dtype=torch.float32, device=q.device)
    for r in range(len(seq_lens)):
        a, b = q_start[r], q_start[r + 1]
        if b <= a:
            continue
        n = b - a
        prefix = seq_lens[r] - n
        st = stage
        if stage is not None and len(stage) > 4 and stage[4] is not None:
            lay = stage[4]  # per-request layout: this request's state slot
            st = stage[:4] + ((int(lay[0][r]), lay[1], lay[2]),)
        for h in range(Hk):
            kh, vh = _history_fp16(kv_mode, pool, kc, vc, st, block_tables[r], prefix, h, D)
            kk = torch.cat([kh, k_fresh[a:b, h].float()])
            vv = torch.cat([vh, v_fresh[a:b, h].float()])
            qq = q[a:b, h * g:(h + 1) * g].float()  # [n, g, D]
            s = torch.einsum("ngd,ld->ngl", qq, kk) * scale
            kpos = torch.arange(prefix + n, device=q.device)
            lim = prefix + torch.arange(n, device=q.device)
            mask = kpos.view(1, 1, -1) <= lim.view(-1, 1, 1)
            s = s.masked_fill(~mask, float("-inf"))
            p = torch.softmax(s, dim=-1)
            out[a:b, h * g:(h + 1) * g] = torch.einsum("ngl,ld->ngd", p, vv)
    return out


def merge_ref(o_rot: torch.Tensor, RvT, gate, want_bf16: bool, want_q: bool):
    """``o = bf16(o_rot @ R_vᵀ * sigmoid(gate))`` -> (bf16 ``[T, Hq*D]``, int8, scale)."""
    T, Hq, D = o_rot.shape
    o = o_rot @ RvT if RvT is not None else o_rot
    if gate is not None:
        o = o * torch.sigmoid(gate.float())
    o = _bf16_round(o).reshape(T, Hq * D)
    q, s = quantize_rows_ref(o) if want_q else (None, None)
    return (o.to(torch.bfloat16) if want_bf16 else None), q, s


def attention(q, k_fresh, v_fresh, *, Hq, Hk, D, scale, kv_mode, pool, kc, vc, stage, block_tables,
              q_start_t, seq_lens_t, q_start: list[int], seq_lens: list[int], plan: AttnPlan | None,
              tok_req, RvT, gate, gate_ld, gate_hstride, want_bf16=False, want_q=True,
              part_o=None, part_lse=None, status=None, rv_merge_split=None):
    """Attention + merge.  Returns ``(o_bf16 | None, o_int8 | None, o_scale | None)``.

    ``stage`` is ``(stage_k [rows*128, Hk, D], stage_v [rows, Hk, D, 128], owner, rows, layout)``
    or ``None``; ``layout`` is ``None`` (the hashed arena) or ``(req_slot [R], sink_pages,
    ring)`` of the per-request window layout; ``gate`` is the bf16
    qkv buffer view whose ``[t, h*gate_hstride + d]`` element gates output ``(t, h, d)``.
    """
    T = q.shape[0]
    if not q.is_cuda:
        o_rot = attention_ref(q, k_fresh, v_fresh, Hq=Hq, Hk=Hk, D=D, scale=scale, kv_mode=kv_mode, pool=pool,
                              kc=kc, vc=vc, stage=stage, block_tables=block_tables, q_start=q_start,
                              seq_lens=seq_lens)
        g = None
        if gate is not None:
            g = torch.stack([gate[:, h * gate_hstride: h * gate_hstride + D] for h in range(Hq)], 1)
        return merge_ref(o_rot, RvT, g, want_bf16, want_q)
    e = ext()
    assert plan is not None
    if part_o is None or part_o.numel() < plan.n_work * Hk * ROWS * D:
        part_o = torch.empty(plan.n_work * Hk * ROWS * D, dtype=torch.float32, device=q.device)
        part_lse = torch.empty(plan.n_work * Hk * ROWS, dtype=torch.float32, device=q.device)
    sk = sv = own = None
    rows = 0
    lay = None
    if stage is not None:
        sk, sv, own, rows = stage[:4]
        lay = stage[4] if len(stage) > 4 else None
    e.paged_attention(q, k_fresh, v_fresh, Hq, Hk, D, float(scale), kv_mode, pool, kc, vc, sk, sv, own, rows,
                      block_tables, q_start_t, seq_lens_t, plan.work, part_o, part_lse, status,
                      _rpi(plan, q_start, Hq // Hk), plan.tiles if (USE_TC and plan.n_tiles > 0) else None,
                      plan.n_tiles if USE_TC else 0, plan.n_short if (USE_TC and plan.n_tiles > 0) else 0,
                      None if lay is None else lay[0], 0 if lay is None else lay[1], 0 if lay is None else lay[2])
    if RvT is not None:
        # tensor-core merge + rotation + gate, then the vectorised row quantiser
        if rv_merge_split is None:
            rv_merge_split = split_rotation(RvT)
        o_bf16 = torch.empty(T, Hq * D, dtype=torch.bfloat16, device=q.device)
        e.attn_merge_rot(part_o, part_lse, plan.item_first, plan.item_count, plan.max_rb, tok_req, q_start_t, Hq,
                         Hk, D, gate, gate_ld, gate_hstride, o_bf16, T, rv_merge_split[0], rv_merge_split[1])
        o_q = o_s = None
        if want_q:
            from .functional import act_quant
            o_q, o_s = act_quant(o_bf16)
        return (o_bf16 if want_bf16 else None), o_q, o_s
    o_bf16 = torch.empty(T, Hq * D, dtype=torch.bfloat16, device=q.device) if want_bf16 else None
    o_q = torch.empty(T, Hq * D, dtype=torch.int8, device=q.device) if want_q else None
    o_s = torch.empty(T, dtype=torch.float32, device=q.device) if want_q else None
    e.attn_merge(part_o, part_lse, plan.item_first, plan.item_count, plan.max_rb, tok_req, q_start_t, Hq, Hk, D,
                 RvT, gate, gate_ld, gate_hstride, o_bf16, o_q, o_s, T)
    return o_bf16, o_q, o_s
