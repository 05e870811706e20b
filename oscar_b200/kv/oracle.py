"""CPU (pure torch) oracle of every OSCAR KV operation, over the page-packed pool.

These functions define the semantics that the sm_100a kernels must reproduce and are
what the GPU tests compare against.  They mirror the reference behaviours:

* store: rotate (fp32) -> sort-threshold clip -> per-vector INT2 quantize -> page
  write; negative slots are skipped (``store_kernel.py:54-102``, ``backend.py:129-189``);
* staging: sink/recent tokens kept unclipped in fp32 rotated space in a hashed arena
  with owner tags and deterministic last-writer-wins seats (``backend.py:418-481``);
* paged multi-query attention in rotated space: query ``i`` of a request with ``n``
  query tokens and sequence length ``s`` sees keys ``0..s-n+i``; history comes from INT2
  pages, replaced by staged fp32 values where the owner tag matches the page's block,
  and the current chunk always uses its unquantized K/V (``paged_attention.py:20-64,
  136-260``); output is ``o_rot @ R_vᵀ``.
"""
from __future__ import annotations

import itertools
import math

import torch
import torch.nn.functional as F

from . import format as fmt


# ---------------------------------------------------------------------------
# store
# ---------------------------------------------------------------------------
def rotate_clip(x: torch.Tensor, R: torch.Tensor | None, ratio: float) -> tuple[torch.Tensor, torch.Tensor]:
    """Returns ``(rotated_unclipped, rotated_clipped)`` in fp32."""
    xr = x.float() if R is None else torch.matmul(x.float(), R.float())
    return xr, fmt.clip_sorted(xr, ratio)


def store_ref(k: torch.Tensor, v: torch.Tensor, pool: torch.Tensor, slots: torch.Tensor,
              R_k: torch.Tensor | None = None, R_v: torch.Tensor | None = None,
              k_clip: float = 0.0, v_clip: float = 0.0):
    """Quantize ``k/v [N,Hk,D]`` into ``pool [blocks,Hk,page_bytes]`` at ``slots [N]``.

    Returns the rotated, unclipped ``(k_rot, v_rot)`` (fp32) for the staging window.
    """
    N, hk, D = k.shape
    k_rot, k_c = rotate_clip(k, R_k, k_clip)
    v_rot, v_c = rotate_clip(v, R_v, v_clip)
    valid = slots >= 0
    if valid.any():
        s = slots[valid].long()
        fmt.write_tokens(pool, s // fmt.PAGE, s % fmt.PAGE, k_c[valid], v_c[valid])
    return k_rot, v_rot


# ---------------------------------------------------------------------------
# staging window
# ---------------------------------------------------------------------------
def staging_rows(sink_tokens: int, recent_tokens: int, staging_tokens: int, page: int = fmt.PAGE) -> int:
    sink_pages = (sink_tokens // page)
    tail_pages = (recent_tokens + page - 1) // page + 1
    return max((staging_tokens + page - 1) // page, sink_pages + tail_pages + 2)


def window_layout(sink_tokens: int, recent_tokens: int, page: int = fmt.PAGE) -> tuple[int, int]:
    """``(sink_pages, ring)`` of the per-request staging layout: the sink pages keep rows of
    their own and the recent pages cycle through ``ring`` rows, enough that the pages
    holding the last ``recent_tokens`` tokens (up to ``ceil(recent / page) + 1`` of them)
    never share a row."""
    return sink_tokens // page, (recent_tokens + page - 1) // page + 2


def arena_rows(sink_tokens: int, recent_tokens: int, staging_tokens: int, layout: str, max_slots: int,
               page: int = fmt.PAGE) -> int:
    """Rows (of ``page`` tokens) of a FULL layer's staging arena: ``max_slots`` requests'
    own rows in the window layout, the shared hashed arena otherwise."""
    if layout == "window":
        sp, ring = window_layout(sink_tokens, recent_tokens, page)
        return max_slots * (sp + ring)
    return staging_rows(sink_tokens, recent_tokens, staging_tokens, page)


def window_row(req_slot, lp, sink_pages: int, ring: int):
    """Staging row of logical page ``lp`` of the request in state slot ``req_slot`` (ints,
    numpy arrays or tensors; the attention kernels use the same formula)."""
    per = sink_pages + ring
    if isinstance(lp, int):
        return req_slot * per + (lp if lp < sink_pages else sink_pages + lp % ring)
    mod = lp % ring
    return req_slot * per + ((lp < sink_pages) * lp + (lp >= sink_pages) * (sink_pages + mod))


def token_positions(qsl: list[int], seqs: list[int], n_tokens: int) -> tuple[torch.Tensor, torch.Tensor]:
    """Per token: request index and absolute position (``seq - q_len + i``)."""
    req = torch.full((n_tokens,), -1, dtype=torch.long)
    pos = torch.full((n_tokens,), -1, dtype=torch.long)
    for r, (a, b) in enumerate(itertools.pairwise(qsl)):
        a, b = min(a, n_tokens), min(b, n_tokens)
        if b <= a:
            continue
        req[a:b] = r
        pos[a:b] = seqs[r] - (qsl[r + 1] - qsl[r]) + torch.arange(b - a)
    return req, pos


def seat_plan(slots: torch.Tensor, pos: torch.Tensor, seq_of_token: torch.Tensor,
              rows: int, sink_tokens: int, recent_tokens: int, page: int = fmt.PAGE,
              token_rows: torch.Tensor | None = None):
    """Deterministic staging plan for one step (shared by every FULL layer).

    Returns ``(token_idx, seat, owner)``: for every distinct seat the last writer in
    token order, its seat, and the owner tag to store (the block id, or -1 when the
    token is outside the sink/recent window).  ``token_rows`` gives each token's staging
    row (the window layout); by default the row is ``block % rows`` (the hashed arena).
    """
    sink_eff = (sink_tokens // page) * page
    keep = (pos >= seq_of_token - recent_tokens) | (pos < sink_eff)
    valid = torch.nonzero(slots >= 0, as_tuple=True)[0]
    s = slots[valid].long()
    row = (s // page % rows) if token_rows is None else token_rows[valid].long()
    seats = row * page + s % page
    order = torch.argsort(seats, stable=True)
    ss = seats[order]
    last = torch.ones_like(ss, dtype=torch.bool)
    if ss.numel() > 1:
        last[:-1] = ss[1:] != ss[:-1]
    tok = valid[order[last]]
    seat = ss[last]
    owner = torch.where(keep[tok], slots[tok].long() // page, torch.full_like(seat, -1))
    return tok, seat, owner


class StagingArena:
    """fp32 sink/recent staging of one FULL layer: ``[rows, PAGE, Hk, D]`` K and V.

    The owner table ``[rows, PAGE]`` is identical for every layer of a step, so one
    table is shared by all layers of a model (``owner`` may be passed in).
    """

    def __init__(self, rows: int, hk: int, D: int, device="cpu", owner: torch.Tensor | None = None):
        self.rows, self.hk, self.D = rows, hk, D
        self.k = torch.zeros(rows, fmt.PAGE, hk, D, dtype=torch.float32, device=device)
        self.v = torch.zeros_like(self.k)
        self.owner = owner if owner is not None else torch.full(
            (rows, fmt.PAGE), -1, dtype=torch.int32, device=device)

    def write(self, plan, k_rot: torch.Tensor, v_rot: torch.Tensor, write_owner: bool = True) -> None:
        tok, seat, owner = plan
        r, o = seat // fmt.PAGE, seat % fmt.PAGE
        if write_owner:
            self.owner[r, o] = owner.to(self.owner.dtype)
        kept = owner >= 0
        self.k[r[kept], o[kept]] = k_rot[tok[kept]].float()
        self.v[r[kept], o[kept]] = v_rot[tok[kept]].float()


# ---------------------------------------------------------------------------
# attention
# ---------------------------------------------------------------------------
def sdpa_causal(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: float,
                prefix: int, qblock: int = 512) -> torch.Tensor:
    """Right-aligned causal GQA attention: ``q [n,Hq,D]``, ``k/v [prefix+n,Hk,D]``.

    Query ``i`` attends keys ``0..prefix+i``.  Queries are processed in blocks of
    ``qblock`` rows to bound the mask size (``decode_kernel.py:70-117``).
    """
    n, hq, D = q.shape
    hk = k.shape[1]
    kt = k.transpose(0, 1).unsqueeze(0)
    vt = v.transpose(0, 1).unsqueeze(0)
    out = torch.empty(n, hq, D, dtype=q.dtype, device=q.device)
    kpos = torch.arange(k.shape[0], device=q.device)
    for q0 in range(0, n, qblock):
        q1 = min(n, q0 + qblock)
        qt = q[q0:q1].transpose(0, 1).unsqueeze(0)
        mask = kpos.unsqueeze(0) <= torch.arange(prefix + q0, prefix + q1, device=q.device).unsqueeze(1)
        o = F.scaled_dot_product_attention(qt, kt, vt, attn_mask=mask, scale=scale,
                                           enable_gqa=hq != hk)
        out[q0:q1] = o[0].transpose(0, 1)
    return out


def gather_history(pool: torch.Tensor, block_row: torch.Tensor, count: int, D: int,
                   stage: StagingArena | None = None, page_rows: torch.Tensor | None = None):
    """Dequantized (and staging-spliced) rotated history ``k/v [count,Hk,D]`` (fp32).
    ``page_rows[lp]``: the staging row of logical page ``lp`` (window layout); by default
    ``block % rows`` (hashed arena)."""
    pos = torch.arange(count)
    blocks = block_row[pos // fmt.PAGE].long()
    offs = pos % fmt.PAGE
    k, v = fmt.dequant_tokens(pool, blocks, offs, D)
    if stage is not None and count:
        rows = blocks % stage.rows if page_rows is None else page_rows[pos // fmt.PAGE].long()
        hit = (stage.owner[rows, offs].long() == blocks).view(-1, 1, 1)
        k = torch.where(hit, stage.k[rows, offs], k)
        v = torch.where(hit, stage.v[rows, offs], v)
    return k, v


def paged_attention_ref(q_rot: torch.Tensor, k_new: torch.Tensor, v_new: torch.Tensor,
                        pool: torch.Tensor, block_tables: torch.Tensor, qsl: list[int],
                        seqs: list[int], scale: float, stage: StagingArena | None = None,
                        dtype=torch.float32, qblock: int = 512) -> torch.Tensor:
    """Multi-query OSCAR attention in rotated space (fp32 by default) -> ``[T,Hq,D]``."""
    D = q_rot.shape[-1]
    out = torch.zeros(q_rot.shape, dtype=torch.float32)
    for r, (a, b) in enumerate(itertools.pairwise(qsl)):
        if b <= a:
            continue
        n = b - a
        prefix = seqs[r] - n
        hk_, hv_ = gather_history(pool, block_tables[r], prefix, D, stage)
        k = torch.cat([hk_, k_new[a:b].float()]).to(dtype)
        v = torch.cat([hv_, v_new[a:b].float()]).to(dtype)
        out[a:b] = sdpa_causal(q_rot[a:b].to(dtype), k, v, scale, prefix, qblock).float()
    return out


def oscar_attention_ref(q, k, v, pool, block_tables, qsl, seqs, scale, R_k, R_v,
                        stage=None, dtype=torch.float32):
    """Original-domain output of the full read path: rotate q/k/v, attend, ``@ R_vᵀ``."""
    o = paged_attention_ref(q.float() @ R_k, k.float() @ R_k, v.float() @ R_v, pool,
                            block_tables, qsl, seqs, scale, stage, dtype)
    return o @ R_v.t()


def bf16_paged_attention_ref(q, k_new, v_new, k_cache, v_cache, block_tables, qsl, seqs, scale):
    """Plain BF16 paged attention (MTP draft layer / BF16-KV baseline).

    ``k_cache/v_cache [blocks, PAGE, Hk, D]``; history positions read the cache and the
    current chunk reads ``k_new/v_new``.
    """
    out = torch.zeros(q.shape, dtype=torch.float32)
    for r, (a, b) in enumerate(itertools.pairwise(qsl)):
        if b <= a:
            continue
        n = b - a
        prefix = seqs[r] - n
        pos = torch.arange(prefix)
        blocks = block_tables[r][pos // fmt.PAGE].long()
        kh = k_cache[blocks, pos % fmt.PAGE].float()
        vh = v_cache[blocks, pos % fmt.PAGE].float()
        kk = torch.cat([kh, k_new[a:b].float()])
        vv = torch.cat([vh, v_new[a:b].float()])
        out[a:b] = sdpa_causal(q[a:b].float(), kk, vv, scale, prefix)
    return out


def default_scale(D: int) -> float:
    return 1.0 / math.sqrt(D)
