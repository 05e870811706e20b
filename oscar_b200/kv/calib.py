"""Rotation calibration: capture Q/K/V, build the K/V objectives, compose ``R = U·H·P_br``.

Capture (reference ``oscar_ascend/calib.py:33-83``): each FULL-attention layer of the
model records up to ``OSCAR_ASCEND_CALIB_TOKEN_CAP`` (default 512) tokens of
unquantized ``q [n,Hq,D]``, ``k [n,Hk,D]``, ``v [n,Hk,D]``; MTP and linear-attention
layers are never captured.

Objectives (``calib.py:93-149``), averaged over KV heads with GQA group ``g``:

* ``Σ_Q = mean_h  sym(Q_hᵀ Q_h / (n g))``  — the K rotation ("qqt");
* ``Σ_S = mean_h  sym((V_h √w)ᵀ (V_h √w) / n)`` with ``w_i = k_iᵀ Σ_Qh k_i`` normalised
  to mean 1 — the score-weighted V rotation ("sst").

Composition (``tools/gen_rotations.py:93-146``): eigen-decompose in fp64 on the CPU
(``eigh(cov + 1e-6 I)``), then ``R = U · H · P_br`` with ``H`` the normalised Sylvester
Hadamard matrix and ``P_br`` placing the eigenvalue-sorted directions at bit-reversed
positions.  Cross-rank statistics merge count-weighted (``gen_rotations.py:73-87``).
"""
from __future__ import annotations

import math
import os

import torch

from .rotation import save_rotations


class CalibrationCapture:
    """Collects per-layer Q/K/V samples during ordinary forwards."""

    def __init__(self, token_cap: int | None = None):
        self.token_cap = token_cap if token_cap is not None else int(
            os.environ.get("OSCAR_ASCEND_CALIB_TOKEN_CAP", "512"))
        self.samples: dict[str, dict[str, list[torch.Tensor]]] = {}

    def reset(self) -> None:
        self.samples = {}

    def wants(self, layer_name: str) -> bool:
        if ".mtp." in layer_name or layer_name.startswith("mtp."):
            return False
        if ".linear_attn" in layer_name:
            return False
        return ".self_attn" in layer_name

    def record(self, layer_name: str, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
               num_heads: int, num_kv_heads: int, head_dim: int) -> None:
        """Append samples; accepts 2-D ``[n, H*D]`` or 3-D ``[n, H, D]`` inputs."""
        if not self.wants(layer_name):
            return
        d = self.samples.setdefault(layer_name, {"q": [], "k": [], "v": []})
        have = sum(t.shape[0] for t in d["k"])
        if have >= self.token_cap:
            return
        take = min(k.shape[0], self.token_cap - have)
        d["q"].append(q[:take].detach().float().reshape(take, num_heads, head_dim))
        d["k"].append(k[:take].detach().float().reshape(take, num_kv_heads, head_dim))
        d["v"].append(v[:take].detach().float().reshape(take, num_kv_heads, head_dim))

    def finalize(self) -> dict:
        """``{layer: {"q": {"cov", "count"}, "v": {"cov", "count"}}}`` on the CPU (fp32)."""
        out = {}
        for name, d in self.samples.items():
            if not d["k"]:
                continue
            q, k, v = (torch.cat(d[x], 0) for x in ("q", "k", "v"))
            cov_q, cov_s = layer_objectives(q, k, v)
            n = k.shape[0]
            out[name] = {"q": {"cov": cov_q.cpu(), "count": n}, "v": {"cov": cov_s.cpu(), "count": n}}
        return out


def _sym(x: torch.Tensor) -> torch.Tensor:
    return 0.5 * (x + x.transpose(-1, -2))


def layer_objectives(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Σ_Q and Σ_S for one layer from ``q [n,Hq,D]``, ``k/v [n,Hk,D]`` (fp32, on q's device)."""
    n, hq, D = q.shape
    hk = k.shape[1]
    if hq % hk:
        raise ValueError(f"Hq={hq} not divisible by Hk={hk}")
    g = hq // hk
    cov_q = torch.zeros(D, D, dtype=torch.float32, device=q.device)
    cov_s = torch.zeros_like(cov_q)
    for h in range(hk):
        qg = q[:, h * g:(h + 1) * g].reshape(-1, D).float()
        qq = _sym(qg.t() @ qg / qg.shape[0])
        cov_q += qq
        kh, vh = k[:, h].float(), v[:, h].float()
        w = ((kh @ qq) * kh).sum(-1)
        w = w / w.sum().clamp(min=1e-12) * n
        vw = vh * w.clamp(min=0).sqrt().unsqueeze(-1)
        cov_s += _sym(vw.t() @ vw / n)
    return cov_q / hk, cov_s / hk


def merge_rank_stats(per_rank: list[dict], D: int) -> dict:
    """Count-weighted sum of per-rank (already token-averaged) covariances."""
    merged: dict = {}
    for stats in per_rank:
        for layer, st in stats.items():
            for kind in ("q", "v"):
                agg = merged.setdefault(layer, {}).setdefault(kind, {"cov_sum": torch.zeros(D, D), "count": 0})
                agg["cov_sum"] = agg["cov_sum"] + st[kind]["cov"].float() * st[kind]["count"]
                agg["count"] += int(st[kind]["count"])
    return merged


def hadamard(n: int) -> torch.Tensor:
    """Normalised Sylvester Hadamard matrix (fp64); ``n`` must be a power of two."""
    if n < 1 or n & (n - 1):
        raise ValueError(f"Hadamard size must be a power of two, got {n}")
    h = torch.ones(1, 1, dtype=torch.float64)
    while h.shape[0] < n:
        h = torch.cat([torch.cat([h, h], 1), torch.cat([h, -h], 1)], 0)
    return h / math.sqrt(n)


def bit_reverse(d: int) -> torch.Tensor:
    if d < 1 or d & (d - 1):
        raise ValueError(f"Bit-reversal size must be a power of two, got {d}")
    bits = d.bit_length() - 1
    idx = torch.arange(d)
    rev = torch.zeros(d, dtype=torch.long)
    for b in range(bits):
        rev |= ((idx >> b) & 1) << (bits - 1 - b)
    return rev


def br_permutation(eigenvalues: torch.Tensor) -> torch.Tensor:
    """``P_br``: column ``br[i]`` of the result selects the i-th largest eigen-direction."""
    d = eigenvalues.numel()
    order = torch.argsort(eigenvalues, descending=True)
    perm = torch.empty(d, dtype=torch.long)
    perm[bit_reverse(d)] = order
    return torch.eye(d, dtype=torch.float64)[:, perm]


def compose_rotation(u: torch.Tensor, eigenvalues: torch.Tensor) -> torch.Tensor:
    D = u.shape[0]
    return u.double() @ hadamard(D) @ br_permutation(eigenvalues)


def rotation_from_stats(stats: dict, D: int) -> tuple[torch.Tensor, torch.Tensor]:
    """Merged ``{"cov_sum", "count"}`` -> (``R = U·H·P_br`` fp32, eigenvalues fp32)."""
    c = max(1, int(stats["count"]))
    cov = stats["cov_sum"].double() / c
    cov = 0.5 * (cov + cov.t()) + 1e-6 * torch.eye(D, dtype=torch.float64)
    evals, evecs = torch.linalg.eigh(cov)
    rot = compose_rotation(evecs, evals)
    err = (rot @ rot.t() - torch.eye(D, dtype=torch.float64)).abs().max().item()
    if err > 1e-6:
        print(f"[oscar] composed rotation orthogonality error {err:.2e}")
    return rot.float().contiguous(), evals.float().contiguous()


def build_checkpoint(merged: dict, D: int, path: str | None = None) -> dict[int, dict[str, torch.Tensor]]:
    """Turn merged statistics into the per-layer table and optionally save it (v2)."""
    from .rotation import layer_index_from_name

    layers: dict[int, dict[str, torch.Tensor]] = {}
    for name, st in sorted(merged.items()):
        lid = layer_index_from_name(name) if isinstance(name, str) else int(name)
        if lid is None:
            continue
        rk, ek = rotation_from_stats(st["q"], D)
        rv, ev = rotation_from_stats(st["v"], D)
        layers[lid] = {"rotation": rk, "rotation_v": rv, "eigenvalues": ek, "eigenvalues_v": ev}
    if path:
        save_rotations(path, layers)
    return layers
