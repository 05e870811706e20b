"""Device-dispatching functional ops.

CUDA tensors always run the hand-written sm_100a kernels of ``oscar_b200._C`` (the
call raises if the extension is missing); CPU tensors run a pure-torch reference of
the same computation with the same rounding points.  The references are the
numerics oracle of the GPU tests.
"""
from __future__ import annotations

import math
import os
from dataclasses import dataclass

import torch

from ..kv import format as fmt
from ._ext import ext

_NUM_SMS: dict[int, int] = {}


def num_sms(device: torch.device) -> int:
    idx = device.index if device.index is not None else torch.cuda.current_device()
    if idx not in _NUM_SMS:
        _NUM_SMS[idx] = torch.cuda.get_device_properties(idx).multi_processor_count
    return _NUM_SMS[idx]


def _bf16_round(x: torch.Tensor) -> torch.Tensor:
    return x.to(torch.bfloat16).float()


# ---------------------------------------------------------------------------
# activation quantisation
# ---------------------------------------------------------------------------
def quantize_rows_ref(v: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Per-row symmetric int8: ``q = rint(v * 127 / absmax)``, ``scale = absmax / 127``."""
    v = v.float()
    amax = v.abs().amax(dim=-1)
    inv = torch.where(amax > 0, 127.0 / amax, torch.zeros_like(amax))
    q = torch.clamp(torch.round(v * inv.unsqueeze(-1)), -127, 127).to(torch.int8)
    scale = torch.where(amax > 0, amax / 127.0, torch.ones_like(amax))
    return q, scale


def act_quant(x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """bf16 ``[T, K]`` -> (int8 ``[T, K]``, fp32 scale ``[T]``)."""
    if x.is_cuda:
        T, K = x.shape
        q = torch.empty(T, K, dtype=torch.int8, device=x.device)
        s = torch.empty(T, dtype=torch.float32, device=x.device)
        ext().act_quant(x, q, s)
        return q, s
    return quantize_rows_ref(x.float())


def rmsnorm_quant(x: torch.Tensor, w: torch.Tensor, eps: float, offset: float = 1.0,
                  delta: torch.Tensor | None = None, want_q: bool = True, want_bf16: bool = False,
                  out_q=None, out_s=None, out_bf16=None, wait=None, zero_delta: bool = False, status=None):
    """RMSNorm of the fp32 residual ``x`` (optionally ``x += delta`` first, in place).

    ``y = bf16(x * rsqrt(mean(x^2) + eps) * (offset + w))``; returns
    ``(q int8, scale, y_bf16)`` with the parts not requested set to ``None``.  ``wait =
    (signal_pad_ptr, epoch_tensor, world[, budget_ms])`` first waits for every rank's
    completion flag of a fused GEMM + all-reduce producing ``delta`` (bounded: after
    ``budget_ms``, default 5000, the kernel records a timeout in ``status`` and goes on);
    ``zero_delta`` clears ``delta`` after reading it.
    """
    T, H = x.shape
    if x.is_cuda:
        q = out_q if out_q is not None else (torch.empty(T, H, dtype=torch.int8, device=x.device) if want_q else None)
        s = out_s if out_s is not None else (torch.empty(T, dtype=torch.float32, device=x.device) if want_q else None)
        y = out_bf16 if out_bf16 is not None else (torch.empty(T, H, dtype=torch.bfloat16, device=x.device) if want_bf16 else None)
        sig, ep, world, budget_ms = (tuple(wait) + (5000,))[:4] if wait is not None else (0, None, 0, 5000)
        ext().rmsnorm_quant(x, delta, w, float(offset), float(eps), q, s, y, int(sig), ep, int(world),
                            int(zero_delta), status, int(budget_ms * 1e6))
        return q, s, y
    if delta is not None:
        x += delta.float()
        if zero_delta:
            delta.zero_()
    xf = x.float()
    inv = torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    y = _bf16_round(xf * inv * (offset + w.float()))
    q, s = quantize_rows_ref(y) if want_q else (None, None)
    return q, s, (y.to(torch.bfloat16) if want_bf16 else None)


def swiglu_quant(gu: torch.Tensor, I: int) -> tuple[torch.Tensor, torch.Tensor]:
    """bf16 ``[T, 2I]`` laid out ``[gate | up]`` -> int8 ``silu(gate) * up`` + scale."""
    T = gu.shape[0]
    if gu.is_cuda:
        q = torch.empty(T, I, dtype=torch.int8, device=gu.device)
        s = torch.empty(T, dtype=torch.float32, device=gu.device)
        ext().swiglu_quant(gu, I, q, s)
        return q, s
    g = gu[:, :I].float()
    u = gu[:, I:2 * I].float()
    return quantize_rows_ref(_bf16_round(torch.nn.functional.silu(g) * u))


# ---------------------------------------------------------------------------
# W8A8 GEMM
# ---------------------------------------------------------------------------
@dataclass
class GemmPlan:
    swap: bool
    bn: int
    splits: int


# split-K work units per SM for accumulate GEMMs with fewer output tiles than SMs
SPLIT_WAVES = int(os.environ.get("OSCAR_GEMM_SPLIT_WAVES", "1"))


def plan_gemm(M: int, N: int, K: int, sms: int, allow_split: bool) -> GemmPlan:
    """Tile plan for ``y[M,N] = x[M,K] W[N,K]^T`` on ``sms`` SMs."""
    kblocks = max(1, (K + 127) // 128)
    if M <= 256:
        bn = 32 if M <= 32 else 64 if M <= 64 else 128 if M <= 128 else 256
        tiles = (N + 127) // 128
        swap = True
    else:
        bn = 256 if N >= 2048 else 128
        tiles = ((M + 127) // 128) * ((N + bn - 1) // bn)
        swap = False
    splits = 1
    if allow_split and tiles < sms:
        splits = max(1, min((SPLIT_WAVES * sms) // max(tiles, 1), kblocks // 4, 16))
    return GemmPlan(swap, bn, splits)


# Split-K GEMMs with a bf16 result sum their fp32 partials in a per-device workspace
# that is all zero between calls (the kernel's last split of a tile re-zeroes its
# rows).  Buffers only grow, outside CUDA-graph capture, and replaced ones are kept
# alive: a captured graph may still address them.
_SPLIT_WS: dict[int, tuple[torch.Tensor, torch.Tensor]] = {}
_SPLIT_WS_OLD: list = []
SPLIT_BF16 = os.environ.get("OSCAR_GEMM_SPLIT_BF16", "1") != "0"


def _split_ws(device: torch.device, elems: int, counters: int):
    idx = device.index if device.index is not None else torch.cuda.current_device()
    cur = _SPLIT_WS.get(idx)
    if cur is not None and cur[0].numel() >= elems and cur[1].numel() >= counters:
        return cur
    if torch.cuda.is_current_stream_capturing():
        return None
    n_ws = max(elems, cur[0].numel() if cur else 0, 1 << 20)
    n_cnt = max(counters, cur[1].numel() if cur else 0, 1 << 12)
    if cur is not None:
        _SPLIT_WS_OLD.append(cur)
    cur = (torch.zeros(n_ws, dtype=torch.float32, device=device), torch.zeros(n_cnt, dtype=torch.int32, device=device))
    _SPLIT_WS[idx] = cur
    return cur


def reserve_split_workspace(device: torch.device, sms: int | None = None) -> None:
    """Size the split-K workspace up front (before any CUDA-graph capture).  A GEMM is
    split only when it has fewer output tiles than SMs, so its result has at most
    ``sms x 128 x 256`` elements (the largest tile) and ``sms x 8`` tiles of the swapped
    layout's 32-token minimum, four counters each."""
    sms = sms or num_sms(device)
    _split_ws(device, sms * 128 * 256, sms * 8 * 4)


def linear_i8(xq: torch.Tensor, xs: torch.Tensor, wq: torch.Tensor, ws: torch.Tensor,
              out: torch.Tensor | None = None, accumulate: bool = False,
              status: torch.Tensor | None = None) -> torch.Tensor:
    """``out = (xq @ wq^T) * xs[:, None] * ws[None, :]``.

    bf16 output by default.  With ``accumulate=True`` the result is *added* in fp32 to
    ``out`` (the fp32 residual-delta buffer).  Either way a GEMM with fewer output tiles
    than SMs is split along K (bf16 results through the zeroed fp32 workspace).
    """
    M, K = xq.shape
    N = wq.shape[0]
    if not xq.is_cuda:
        y = (xq.double() @ wq.double().t()) * xs.double().unsqueeze(1) * ws.double().unsqueeze(0)
        if accumulate:
            assert out is not None
            out += y.float()
            return out
        y = y.float().to(torch.bfloat16)
        if out is not None:
            out.copy_(y)
            return out
        return y
    e = ext()
    plan = plan_gemm(M, N, K, num_sms(xq.device), allow_split=accumulate or SPLIT_BF16)
    if accumulate:
        assert out is not None and out.dtype == torch.float32
        mode = 1
    else:
        if out is None:
            out = torch.empty(M, N, dtype=torch.bfloat16, device=xq.device)
        mode = 0
        if plan.splits > 1:
            ld = out.stride(0)
            elems = (N - 1) * ld + M if plan.swap else (M - 1) * ld + N
            rows, cols = (N, M) if plan.swap else (M, N)
            tiles = ((rows + 127) // 128) * ((cols + plan.bn - 1) // plan.bn)
            wsb = _split_ws(xq.device, elems, tiles * 4) if ld % 4 == 0 else None
            if wsb is not None:
                if plan.swap:
                    e.gemm_i8_split(wq, xq, ws, xs, out, 1, plan.bn, plan.splits, wsb[0], wsb[1], status)
                else:
                    e.gemm_i8_split(xq, wq, xs, ws, out, 0, plan.bn, plan.splits, wsb[0], wsb[1], status)
                return out
            plan = GemmPlan(plan.swap, plan.bn, 1)
    if plan.swap:
        e.gemm_i8(wq, xq, ws, xs, out, mode, 1, plan.bn, plan.splits if accumulate else 1, status)
    else:
        e.gemm_i8(xq, wq, xs, ws, out, mode, 0, plan.bn, plan.splits if accumulate else 1, status)
    return out


def quantize_weight(w: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Per-output-channel symmetric int8 weight quantisation: ``w ~ q * s[:, None]``."""
    amax = w.float().abs().amax(dim=1).clamp(min=1e-8)
    s = amax / 127.0
    q = torch.clamp(torch.round(w.float() / s.unsqueeze(1)), -127, 127).to(torch.int8)
    return q, s.float()


# ---------------------------------------------------------------------------
# embedding / sampling
# ---------------------------------------------------------------------------
def embed(tokens: torch.Tensor, table: torch.Tensor, vocab_begin: int, out: torch.Tensor) -> torch.Tensor:
    """fp32 rows of a (vocab-parallel) bf16 table; ids outside this shard give zeros."""
    V = table.shape[0]
    if tokens.is_cuda:
        ext().embed(tokens, table, vocab_begin, vocab_begin + V, out)
        return out
    ids = tokens.long() - vocab_begin
    mine = (ids >= 0) & (ids < V)
    rows = table[ids.clamp(0, V - 1)].float()
    out.copy_(torch.where(mine.unsqueeze(1), rows, torch.zeros_like(rows)))
    return out


def argmax(logits: torch.Tensor, index_offset: int = 0) -> tuple[torch.Tensor, torch.Tensor]:
    """Row-wise (max value, global index) of bf16 logits; ties -> lowest index."""
    T = logits.shape[0]
    if logits.is_cuda:
        v = torch.empty(T, dtype=torch.float32, device=logits.device)
        i = torch.empty(T, dtype=torch.int32, device=logits.device)
        ext().argmax(logits, index_offset, v, i)
        return v, i
    v, i = logits.float().max(dim=-1)
    return v, (i + index_offset).to(torch.int32)


# ---------------------------------------------------------------------------
# RoPE tables
# ---------------------------------------------------------------------------
def rope_inv_freq(rot_dim: int, theta: float, scaling: dict | None = None,
                  max_position: int | None = None) -> tuple[torch.Tensor, float]:
    """float64 inverse frequencies ``[rot_dim / 2]`` and the cos/sin scale of RoPE.

    ``scaling`` None (or ``rope_type`` "default"): ``theta^(-2j / rot_dim)``, scale 1.
    ``rope_type`` "yarn" (Peng et al. 2023, "YaRN: Efficient Context Window Extension of
    Large Language Models"), with ``factor`` s (default ``max_position /
    original_max_position_embeddings``), ``original_max_position_embeddings`` L,
    ``beta_fast`` (32) and ``beta_slow`` (1): the dimension whose wavelength completes r
    rotations over L is ``d(r) = rot_dim ln(L / (2 pi r)) / (2 ln theta)``; frequencies of
    index ``j <= d(beta_fast)`` are kept, those of index ``j >= d(beta_slow)`` divided by s
    (bounds floored / ceiled unless ``truncate`` is false, clamped to the dimensions), with
    a linear ramp in ``j`` between.  The scale is ``0.1 ln s + 1`` (s > 1), or the ratio of
    that form with ``mscale`` / ``mscale_all_dim`` when both are given, or an explicit
    ``attention_factor``."""
    j = torch.arange(0, rot_dim // 2, dtype=torch.float64)
    base = 1.0 / (theta ** (2.0 * j / rot_dim))
    kind = (scaling or {}).get("rope_type", (scaling or {}).get("type", "default"))
    if kind in ("default", None, "mrope"):
        return base, 1.0
    if kind != "yarn":
        raise ValueError(f"unsupported rope scaling {kind!r} (supported: default, yarn)")
    L = float(scaling["original_max_position_embeddings"])
    s = scaling.get("factor")
    s = float(s) if s is not None else float(max_position) / L

    def ms(x: float, m: float = 1.0) -> float:
        return 1.0 if x <= 1 else 0.1 * m * math.log(x) + 1.0

    scale = scaling.get("attention_factor")
    if scale is None:
        m1, m2 = scaling.get("mscale"), scaling.get("mscale_all_dim")
        scale = ms(s, m1) / ms(s, m2) if (m1 and m2) else ms(s)

    def dim_of(rot: float) -> float:
        return rot_dim * math.log(L / (2 * math.pi * rot)) / (2 * math.log(theta))

    lo, hi = dim_of(float(scaling.get("beta_fast") or 32)), dim_of(float(scaling.get("beta_slow") or 1))
    if scaling.get("truncate", True):
        lo, hi = math.floor(lo), math.ceil(hi)
    lo, hi = max(lo, 0), min(hi, rot_dim - 1)
    if hi == lo:
        hi += 0.001
    ramp = ((j - lo) / (hi - lo)).clamp(0.0, 1.0)  # 0: keep the frequency, 1: divide it by s
    return base * (1.0 - ramp) + (base / s) * ramp, float(scale)


def rope_tables(max_pos: int, rot_dim: int, theta: float, device,
                scaling: dict | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """fp32 ``cos/sin [max_pos, rot_dim/2]`` for rotate-half RoPE (scaled by the RoPE
    scaling's cos/sin factor; see :func:`rope_inv_freq`)."""
    inv, scale = rope_inv_freq(rot_dim, theta, scaling, max_pos)
    ang = torch.arange(max_pos, dtype=torch.float64).unsqueeze(1) * inv.unsqueeze(0)
    return (ang.cos() * scale).float().to(device), (ang.sin() * scale).float().to(device)


def apply_rope_ref(x: torch.Tensor, pos: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, rot_dim: int):
    """``x [T, H, D]`` fp32; rotate-half RoPE on the first ``rot_dim`` dims, bf16-rounded."""
    half = rot_dim // 2
    c = cos[pos.long()].unsqueeze(1)
    s = sin[pos.long()].unsqueeze(1)
    a = x[..., :half].clone()
    b = x[..., half:rot_dim].clone()
    out = x.clone()
    out[..., :half] = _bf16_round(a * c - b * s)
    out[..., half:rot_dim] = _bf16_round(b * c + a * s)
    return out


def head_rmsnorm_ref(x: torch.Tensor, w: torch.Tensor, eps: float, offset: float) -> torch.Tensor:
    inv = torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps)
    return _bf16_round(x * inv * (offset + w.float()))


def default_softmax_scale(D: int) -> float:
    return 1.0 / math.sqrt(D)


__all__ = [
    "act_quant", "rmsnorm_quant", "swiglu_quant", "linear_i8", "plan_gemm", "quantize_weight",
    "quantize_rows_ref", "embed", "argmax", "rope_tables", "apply_rope_ref", "head_rmsnorm_ref",
    "num_sms", "fmt",
]
