"""Per-layer orthogonal K/V rotations in the ``oscar_rotations.pt`` format.

Accepted checkpoint structures (same as the reference reader,
``oscar_ascend/rotation.py:44-90``):

* v2: ``{"format_version": 2, "objective": "...r_h_pbr...", "layers": {"<lid>":
  {"rotation", "rotation_v", "eigenvalues", "eigenvalues_v", "layer_id"}}}``;
* ``{lid: matrix}`` or ``{lid: {"rotation": ...}}``;
* a stacked ``[L, D, D]`` tensor.

Layer keys may be ints, digit strings or module names (``...layers.11.self_attn``).
A missing path or layer gives the identity (plain clipped INT2) unless ``strict``;
strict mode rejects a missing layer and non-finite or non-orthogonal matrices
(atol 1e-3), as ``rotation.py:112-128`` does.
"""
from __future__ import annotations

import re
import warnings
from functools import lru_cache
from pathlib import Path

import torch

_LAYER_RE = re.compile(r"\.layers\.(\d+)\.")
FORMAT_VERSION = 2
OBJECTIVE = "qqt_r_h_pbr_k / sst_r_h_pbr_v"


def layer_index_from_name(name: str) -> int | None:
    m = _LAYER_RE.search(name)
    if m is not None:
        return int(m.group(1))
    nums = re.findall(r"\d+", name)
    return int(nums[-1]) if nums else None


def _key_to_layer(key) -> int | None:
    if isinstance(key, int):
        return key
    if isinstance(key, str):
        if key.strip().lstrip("-").isdigit():
            return int(key)
        return layer_index_from_name(key)
    return None


def _tensors(entry: dict) -> dict[str, torch.Tensor]:
    return {k: v.float().contiguous() for k, v in entry.items() if isinstance(v, torch.Tensor)}


def parse_checkpoint(obj) -> dict[int, dict[str, torch.Tensor]]:
    """Normalise any accepted structure to ``{layer_id: {"rotation": R, ...}}``."""
    table: dict[int, dict[str, torch.Tensor]] = {}
    if isinstance(obj, dict) and "layers" in obj:
        items = obj["layers"].items()
    elif isinstance(obj, dict):
        items = ((k, v) for k, v in obj.items() if k not in ("format_version", "objective", "source_grouping"))
    elif torch.is_tensor(obj) and obj.dim() == 3:
        return {i: {"rotation": obj[i].float().contiguous()} for i in range(obj.shape[0])}
    else:
        raise ValueError(f"Unrecognized OSCAR rotation checkpoint structure: {type(obj)}")
    for key, entry in items:
        lid = _key_to_layer(key)
        if lid is None:
            continue
        if isinstance(entry, dict) and "rotation" in entry:
            table[lid] = _tensors(entry)
        elif torch.is_tensor(entry):
            table[lid] = {"rotation": entry.float().contiguous()}
    return table


def is_v2(obj) -> bool:
    return (isinstance(obj, dict) and obj.get("format_version", 0) >= FORMAT_VERSION
            and "r_h_pbr" in str(obj.get("objective", "")))


@lru_cache(maxsize=8)
def load_checkpoint(path: str) -> dict[int, dict[str, torch.Tensor]]:
    obj = torch.load(path, map_location="cpu", weights_only=False)
    if not is_v2(obj):
        warnings.warn(
            f"[oscar] rotation checkpoint {path!r} is not a v2 U·H·P_br checkpoint; "
            "per-vector INT2 accuracy will degrade. Re-run calibration.", stacklevel=2)
    return parse_checkpoint(obj)


def get_layer_rotation(path: str, layer_name: str | int, head_dim: int,
                       device="cpu", dtype=torch.float32, mode: str = "k",
                       strict: bool = False) -> torch.Tensor:
    """``[D, D]`` rotation for one layer; ``mode="v"`` prefers ``rotation_v``."""
    eye = lambda: torch.eye(head_dim, device=device, dtype=dtype)  # noqa: E731
    if not path:
        return eye()
    table = load_checkpoint(path)
    lid = layer_name if isinstance(layer_name, int) else layer_index_from_name(layer_name)
    entry = table.get(lid) if lid is not None else None
    if entry is None:
        if strict:
            raise ValueError(f"Rotation checkpoint {path!r} is missing layer {layer_name}")
        return eye()
    rot = entry.get("rotation_v") if mode == "v" else None
    if rot is None:
        rot = entry.get("rotation")
    if rot is None:
        return eye()
    if tuple(rot.shape) != (head_dim, head_dim):
        raise ValueError(f"OSCAR rotation for layer {lid} has shape {tuple(rot.shape)}, "
                         f"expected ({head_dim}, {head_dim}).")
    if strict:
        ok = torch.isfinite(rot).all() and torch.allclose(
            rot @ rot.t(), torch.eye(head_dim), atol=1e-3, rtol=1e-3)
        if not ok:
            raise ValueError(f"Rotation checkpoint {path!r} layer {lid} is not finite/orthogonal")
    return rot.to(device=device, dtype=dtype).contiguous()


def save_rotations(path: str | Path, layers: dict[int, dict[str, torch.Tensor]],
                   objective: str = OBJECTIVE) -> None:
    """Write a v2 checkpoint readable by both this framework and the reference."""
    out = {
        "format_version": FORMAT_VERSION,
        "objective": objective,
        "source_grouping": "layer",
        "layers": {
            str(lid): {"layer_id": int(lid),
                       **{k: v.detach().float().cpu().contiguous() for k, v in e.items()}}
            for lid, e in sorted(layers.items())
        },
    }
    Path(path).parent.mkdir(parents=True, exist_ok=True)
    torch.save(out, str(path))
    load_checkpoint.cache_clear()


def random_orthogonal(D: int, seed: int) -> torch.Tensor:
    """Seeded random orthogonal matrix (QR of a Gaussian), as the benchmarks use."""
    g = torch.Generator().manual_seed(seed)
    return torch.linalg.qr(torch.randn(D, D, generator=g)).Q.contiguous()
