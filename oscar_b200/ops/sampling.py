"""Token sampling over vocab-parallel logits, and exact verification of greedy MTP drafts.

Sampling is the Gumbel-max trick: ``argmax_v (l_v / T + G_v)`` with ``G_v`` independent
standard Gumbel noise is an exact sample of ``softmax(l / T)``.  The noise is a
counter-based hash of (request seed, position of the sampled token, vocabulary id):

* every tensor-parallel rank draws the noise of its own vocabulary shard with no
  communication, and the global choice is the same max-reduction over ranks as greedy
  decoding (each rank proposes its best score and token id);
* a request's samples depend only on its seed and positions, not on the batch it runs
  in or on the tensor-parallel size.

The hash is ``lowbias32`` (C. Wellons, "Hash function prospector", public domain):
``x ^= x >> 16; x *= 0x7feb352d; x ^= x >> 15; x *= 0x846ca68b; x ^= x >> 16`` on 32-bit
words, evaluated exactly in int64 tensors (products split into 16-bit halves).

Truncation is a per-row threshold ``tau`` on the scaled logits ``z = l / T``: a token is
allowed when ``z >= tau``.  ``top_k`` gives the k-th largest ``z``; ``top_p`` the smallest
``z`` of the nucleus of the (top-k truncated, renormalised) distribution, found among the
``CANDIDATES`` largest logits of every rank.  The nucleus is exact when it has at most
``CANDIDATES`` tokens (it always has, for ``top_k <= CANDIDATES``); a wider nucleus leaves
the row untruncated by ``top_p``.  Tokens tied at ``tau`` are all allowed.

Verification of a draft token ``d`` at a row (speculative sampling with a deterministic
draft, Leviathan et al. 2023 and Chen et al. 2023): accept with probability ``p(d)`` (the
truncated distribution); on rejection the token is a sample of ``p`` restricted to
``v != d``.  The emitted token is then distributed exactly as ``p``.  An accepted draft
is emitted as ``d`` and a rejected one never is, so the engine's acceptance loop ("accept
while the row's token equals the draft") serves greedy and sampled requests alike.

Rows with ``temperature <= 0`` are greedy: the token is the argmax of the logits.

On the GPU the per-element work (scaling, truncation mask, the max and exponential sum,
the draft's mass, the hashed Gumbel noise and the masked arg-max) is one pass of the
``sample_pass`` kernel over the vocabulary shard, in 4,096-column chunks; only steps
with top-k / top-p rows also run :func:`phase1` (the candidate top-k) for the
threshold.  The CPU path computes the same quantities with torch ops (the test oracle).

The reference serves through vLLM's sampler (``delivery/serve_oscar.sh:76-99`` runs
``vllm serve``); its benchmark decodes greedily, like this framework's bench.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

CANDIDATES = 1024        # per-rank candidates for the top-k / top-p thresholds
MAX_TOP_K = CANDIDATES   # top_k is exact up to this
_ACCEPT_SALT = 0xFFFFFFFF  # "vocabulary id" of the acceptance draw (outside any vocabulary)
_M16 = 0xFFFF
_M32 = 0xFFFFFFFF


@dataclass
class SamplingParams:
    """Per-request sampling (the OpenAI completions fields of the same names).  The
    offline API (:class:`oscar_b200.LLM`) also reads ``max_tokens``, ``stop_token_ids``,
    ``ignore_eos`` and ``stop``; the engine takes the token-level ones as arguments of
    ``add_request``."""

    temperature: float = 0.0   # <= 0: greedy
    top_k: int = 0             # 0: off
    top_p: float = 1.0         # 1: off
    seed: int | None = None    # None: derived from the engine seed and the request id
    max_tokens: int = 16
    stop_token_ids: list | None = None
    ignore_eos: bool = False
    stop: list | None = None   # stop strings (the offline API and the server cut the text there)
    logprobs: int | None = None  # the offline API reports the k most likely tokens per output token

    def validate(self) -> "SamplingParams":
        if int(self.max_tokens) < 1:
            raise ValueError(f"max_tokens {self.max_tokens} must be >= 1")
        if not np.isfinite(self.temperature) or self.temperature < 0:
            raise ValueError(f"temperature {self.temperature} must be >= 0")
        if not 0 <= int(self.top_k) <= MAX_TOP_K:
            raise ValueError(f"top_k {self.top_k} must be in [0, {MAX_TOP_K}]")
        if not 0.0 < self.top_p <= 1.0:
            raise ValueError(f"top_p {self.top_p} must be in (0, 1]")
        return self

    @property
    def greedy(self) -> bool:
        return self.temperature <= 0

    def to_dict(self) -> dict:
        return {"temperature": self.temperature, "top_k": self.top_k, "top_p": self.top_p, "seed": self.seed,
                "max_tokens": self.max_tokens, "stop_token_ids": self.stop_token_ids, "ignore_eos": self.ignore_eos,
                "stop": self.stop, "logprobs": self.logprobs}


@dataclass
class SampleRows:
    """Device tensors, one entry per logit row."""

    temperature: torch.Tensor  # f32 [n]
    top_k: torch.Tensor        # i32 [n]
    top_p: torch.Tensor        # f32 [n]
    seed: torch.Tensor         # i32 [n], non-negative
    pos: torch.Tensor          # i32 [n], position of the token this row samples
    draft: torch.Tensor        # i32 [n], global id of the draft verified at this row, -1: none
    truncated: bool = True     # some row has top_k > 0 or top_p < 1 (then phase 1 runs)


def host_rows(params: list, seeds: list, positions: list, drafts: list) -> dict:
    """int32 host arrays of :class:`SampleRows` (floats as their bit patterns), the form
    the engine uploads with the rest of a step's metadata."""
    t = np.asarray([p.temperature if p is not None else 0.0 for p in params], dtype=np.float32)
    tp = np.asarray([p.top_p if p is not None else 1.0 for p in params], dtype=np.float32)
    trunc = any(p is not None and p.temperature > 0 and (p.top_k > 0 or p.top_p < 1.0) for p in params)
    # whether any row is truncated is carried in the shape of "samp_trunc" (length 1 or 0),
    # so that steps with and without the threshold phase are different CUDA graphs
    return {"samp_t": t.view(np.int32), "samp_k": [p.top_k if p is not None else 0 for p in params],
            "samp_p": tp.view(np.int32), "samp_seed": [s & 0x7FFFFFFF for s in seeds], "samp_pos": positions,
            "samp_draft": drafts, "samp_trunc": np.zeros(1 if trunc else 0, dtype=np.int32)}


def rows_from_arrays(d: dict) -> SampleRows:
    trunc = "samp_trunc" not in d or d["samp_trunc"].numel() > 0
    return SampleRows(d["samp_t"].view(torch.float32), d["samp_k"], d["samp_p"].view(torch.float32),
                      d["samp_seed"], d["samp_pos"], d["samp_draft"], trunc)


# ----------------------------------------------------------------------------- hashing
def _mul32(x: torch.Tensor, c: int) -> torch.Tensor:
    """``(x * c) mod 2^32`` for int64 ``x`` in ``[0, 2^32)`` without int64 overflow."""
    lo = (x & _M16) * c
    hi = ((x >> 16) * c) & _M16
    return (lo + (hi << 16)) & _M32


def hash32(x: torch.Tensor) -> torch.Tensor:
    """lowbias32 of int64 ``x`` in ``[0, 2^32)``."""
    x = x ^ (x >> 16)
    x = _mul32(x, 0x7FEB352D)
    x = x ^ (x >> 15)
    x = _mul32(x, 0x846CA68B)
    return x ^ (x >> 16)


def _row_key(seed: torch.Tensor, pos: torch.Tensor) -> torch.Tensor:
    return hash32(hash32(seed.long() & _M32) ^ (pos.long() & _M32))


def uniform(key: torch.Tensor, col: torch.Tensor) -> torch.Tensor:
    """float32 uniform in (0, 1), 24 bits, of the row key and a column id (broadcasting)."""
    h = hash32((key ^ (col.long() & _M32)) & _M32)
    return ((h >> 8).float() + 0.5) * (1.0 / (1 << 24))


def gumbel(key: torch.Tensor, col: torch.Tensor) -> torch.Tensor:
    return -torch.log(-torch.log(uniform(key, col)))


# ----------------------------------------------------------------------------- phases
def _scaled(logits: torch.Tensor, rows: SampleRows) -> torch.Tensor:
    t = rows.temperature.float()
    return logits.float() / torch.where(t > 0, t, torch.ones_like(t)).unsqueeze(1)


def phase1(logits: torch.Tensor, rows: SampleRows) -> torch.Tensor:
    """Per-rank statistics ``[n, 2 + CANDIDATES]``: max of ``z``, ``sum exp(z - max)``,
    the largest ``z`` in descending order (padded with -inf)."""
    z = _scaled(logits, rows)
    n, v = z.shape
    k = min(CANDIDATES, v)
    top = torch.topk(z, k, dim=1).values
    if k < CANDIDATES:
        top = torch.cat([top, top.new_full((n, CANDIDATES - k), float("-inf"))], dim=1)
    mx = top[:, 0]
    s = torch.exp(z - mx.unsqueeze(1)).sum(dim=1)
    return torch.cat([mx.unsqueeze(1), s.unsqueeze(1), top], dim=1)


def combine1(stats: torch.Tensor, rows: SampleRows) -> tuple[torch.Tensor, torch.Tensor]:
    """``stats [world, n, 2 + C]`` of every rank -> (global max ``m``, threshold ``tau``)."""
    mr, sr, cand = stats[:, :, 0], stats[:, :, 1], stats[:, :, 2:]
    m = mr.max(dim=0).values
    Z = (sr * torch.exp(mr - m)).sum(dim=0)
    c = cand.permute(1, 0, 2).reshape(m.shape[0], -1)
    c = torch.sort(c, dim=1, descending=True).values
    n, nc = c.shape
    neg = torch.full_like(m, float("-inf"))
    k = rows.top_k.long().clamp(0, nc)
    tau_k = torch.where(k > 0, c.gather(1, (k - 1).clamp(min=0).unsqueeze(1)).squeeze(1), neg)
    # top-p on the top-k truncated distribution
    w = torch.exp(c - m.unsqueeze(1))
    idx = torch.arange(nc, device=c.device).unsqueeze(0)
    w = torch.where((k.unsqueeze(1) == 0) | (idx < k.unsqueeze(1)), w, torch.zeros_like(w))
    Zk = torch.where(k > 0, w.sum(dim=1), Z)
    cum = torch.cumsum(w, dim=1) / Zk.unsqueeze(1)
    p = rows.top_p.float()
    reach = cum >= p.unsqueeze(1)
    first = torch.where(reach.any(dim=1), reach.float().argmax(dim=1), torch.full_like(k, nc - 1))
    tau_p = torch.where((p < 1.0) & reach.any(dim=1), c.gather(1, first.unsqueeze(1)).squeeze(1), neg)
    return m, torch.maximum(tau_k, tau_p)


def phase2(logits: torch.Tensor, vocab_begin: int, rows: SampleRows, m: torch.Tensor,
           tau: torch.Tensor) -> torch.Tensor:
    """Per-rank ``[n, 4]``: allowed mass, draft mass (relative to ``exp(m)``), best score
    and its global token id."""
    z = _scaled(logits, rows)
    n, v = z.shape
    samp = rows.temperature > 0
    cols = torch.arange(vocab_begin, vocab_begin + v, device=z.device).unsqueeze(0)
    allowed = z >= tau.unsqueeze(1)
    e = torch.where(allowed, torch.exp(z - m.unsqueeze(1)), torch.zeros_like(z))
    zt = e.sum(dim=1)
    d = rows.draft.long()
    local = (d >= vocab_begin) & (d < vocab_begin + v)
    pd = torch.where(local, e.gather(1, (d - vocab_begin).clamp(0, v - 1).unsqueeze(1)).squeeze(1),
                     torch.zeros_like(zt))
    key = _row_key(rows.seed, rows.pos).unsqueeze(1)
    score = z + gumbel(key, cols)
    score = torch.where(allowed & (cols != d.unsqueeze(1)), score, torch.full_like(score, float("-inf")))
    score = torch.where(samp.unsqueeze(1), score, logits.float())
    best, arg = score.max(dim=1)
    return torch.stack([zt, pd, best, (arg + vocab_begin).float()], dim=1)


def combine2(parts: torch.Tensor, rows: SampleRows) -> torch.Tensor:
    """``parts [world, n, 4]`` of every rank -> token ids ``[n]`` (int64)."""
    zt = parts[:, :, 0].sum(dim=0)
    pd = parts[:, :, 1].sum(dim=0) / zt.clamp_min(1e-30)
    r = parts[:, :, 2].argmax(dim=0)  # first rank with the best score
    tok = parts[:, :, 3].gather(0, r.unsqueeze(0)).squeeze(0).long()
    key = _row_key(rows.seed, rows.pos)
    u = uniform(key, torch.full_like(key, _ACCEPT_SALT))
    d = rows.draft.long()
    accept = (rows.temperature > 0) & (d >= 0) & (u < pd)
    return torch.where(accept, d, tok)


def _pass_cuda(logits: torch.Tensor, vocab_begin: int, rows: SampleRows, tau: torch.Tensor) -> torch.Tensor:
    """This rank's ``[n, 5]``: max ``m`` of the allowed scaled logits, ``sum exp(z - m)``,
    the draft's scaled logit (or -inf), the best (Gumbel) score and its global token id
    - one ``sample_pass`` kernel over the shard, then a merge of its chunks."""
    from ._ext import ext

    n, V = logits.shape
    chunk = 4096
    nc = (V + chunk - 1) // chunk
    part = torch.empty(n, nc, 5, dtype=torch.float32, device=logits.device)
    ext().sample_pass(logits, vocab_begin, rows.temperature.float().contiguous(), tau.float().contiguous(),
                      rows.draft.int().contiguous(), rows.seed.int().contiguous(), rows.pos.int().contiguous(), part)
    m_c, s_c, zd_c, b_c, id_c = part.unbind(2)
    m = m_c.max(dim=1).values
    finite = m_c > float("-inf")
    mm = torch.where(m > float("-inf"), m, torch.zeros_like(m))
    s = torch.where(finite, s_c * torch.exp(m_c - mm.unsqueeze(1)), torch.zeros_like(s_c)).sum(dim=1)
    zd = zd_c.max(dim=1).values
    best, at = b_c.max(dim=1)  # first chunk on ties: the lowest token id
    tok = id_c.gather(1, at.unsqueeze(1)).squeeze(1)
    return torch.stack([m, s, zd, best, tok], dim=1)


def _combine_cuda(parts: torch.Tensor, rows: SampleRows) -> torch.Tensor:
    """``parts [world, n, 5]`` of every rank -> token ids ``[n]`` (int64)."""
    mr, sr, zdr, br, idr = parts.unbind(2)
    m = mr.max(dim=0).values
    mm = torch.where(m > float("-inf"), m, torch.zeros_like(m))
    Z = torch.where(mr > float("-inf"), sr * torch.exp(mr - mm), torch.zeros_like(sr)).sum(dim=0)
    pd = torch.exp(zdr.max(dim=0).values - mm) / Z.clamp_min(1e-30)
    r = br.argmax(dim=0)  # first rank with the best score
    tok = idr.gather(0, r.unsqueeze(0)).squeeze(0).long()
    key = _row_key(rows.seed, rows.pos)
    u = uniform(key, torch.full_like(key, _ACCEPT_SALT))
    d = rows.draft.long()
    accept = (rows.temperature > 0) & (d >= 0) & (u < pd)
    return torch.where(accept, d, tok)


def sample(logits: torch.Tensor, vocab_begin: int, rows: SampleRows, tp=None) -> torch.Tensor:
    """Token of every row of this rank's vocabulary shard ``logits [n, V_local]``; every
    rank of ``tp`` returns the same tokens (two all-gathers of ``[n, 2 + C]`` and ``[n, 4]``
    on the CPU path; on the GPU one of ``[n, 5]``, plus the threshold's when some row is
    truncated)."""
    world = 1 if tp is None else tp.world
    if logits.is_cuda:
        n = logits.shape[0]
        if rows.truncated:
            st = phase1(logits, rows).unsqueeze(0)
            if world > 1:
                st = tp.all_gather(st)
            _, tau = combine1(st, rows)
        else:
            tau = torch.full((n,), float("-inf"), dtype=torch.float32, device=logits.device)
        parts = _pass_cuda(logits, vocab_begin, rows, tau).unsqueeze(0)
        if world > 1:
            parts = tp.all_gather(parts)
        return _combine_cuda(parts, rows)
    st = phase1(logits, rows).unsqueeze(0)
    if world > 1:
        st = tp.all_gather(st)
    m, tau = combine1(st, rows)
    parts = phase2(logits, vocab_begin, rows, m, tau).unsqueeze(0)
    if world > 1:
        parts = tp.all_gather(parts)
    return combine2(parts, rows)


def probabilities(logits: torch.Tensor, params: SamplingParams) -> torch.Tensor:
    """The truncated sampling distribution of one full-vocabulary row (a float64 CPU
    reference for tests): softmax of ``l / T`` over top-k, then the top-p nucleus."""
    z = logits.double() / params.temperature
    order = torch.argsort(z, descending=True)
    zs = z[order]
    keep = torch.ones_like(zs, dtype=torch.bool)
    if params.top_k > 0:
        keep[params.top_k:] = False
    w = torch.where(keep, torch.exp(zs - zs[0]), torch.zeros_like(zs))
    if params.top_p < 1.0:
        cum = torch.cumsum(w, 0) / w.sum()
        cut = int(torch.nonzero(cum >= params.top_p)[0])
        keep[cut + 1:] = False
        w = torch.where(keep, w, torch.zeros_like(w))
    p = torch.zeros_like(z)
    p[order] = w / w.sum()
    return p


def logprobs(logits: torch.Tensor, vocab_begin: int, tokens: torch.Tensor, k: int, tp=None):
    """Log-probabilities under the model's distribution (the raw logits, before temperature
    or truncation) of ``tokens [n]`` and the ``k`` most likely tokens of every row, over
    vocab-parallel logits (one all-gather of ``[n, 3 + 2k]``).  Returns ``(token_lp [n],
    top_ids [n, k], top_lp [n, k])``."""
    z = logits.float()
    n, v = z.shape
    kk = max(1, min(int(k), v))
    mx = z.max(dim=1).values
    s = torch.exp(z - mx.unsqueeze(1)).sum(dim=1)
    tv, ti = torch.topk(z, kk, dim=1)
    t = tokens.long()
    local = (t >= vocab_begin) & (t < vocab_begin + v)
    tl = torch.where(local, z.gather(1, (t - vocab_begin).clamp(0, v - 1).unsqueeze(1)).squeeze(1),
                     torch.full_like(mx, float("-inf")))
    pack = torch.cat([mx.unsqueeze(1), s.unsqueeze(1), tl.unsqueeze(1), tv, (ti + vocab_begin).float()], dim=1)
    pack = pack.unsqueeze(0)
    if tp is not None and tp.world > 1:
        pack = tp.all_gather(pack)
    mr, sr, tlr = pack[:, :, 0], pack[:, :, 1], pack[:, :, 2]
    m = mr.max(dim=0).values
    lse = m + torch.log((sr * torch.exp(mr - m)).sum(dim=0))
    tok_lp = tlr.max(dim=0).values - lse
    vals = pack[:, :, 3:3 + kk].permute(1, 0, 2).reshape(n, -1)
    ids = pack[:, :, 3 + kk:].permute(1, 0, 2).reshape(n, -1)
    best, where = torch.topk(vals, kk, dim=1)
    return tok_lp, ids.gather(1, where).long(), best - lse.unsqueeze(1)
