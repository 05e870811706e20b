"""KV memory budget, layer verification and the per-rank READY manifest.

The reference wraps the worker's ``determine_available_memory`` and
``initialize_kv_cache_tensors`` (``oscar_ascend/integration.py:17-187``).  Here the
engine owns its cache, so the same seam is a pair of plain functions called before
and after the cache is allocated:

* :func:`memory_budget` - ``blocks = (avail - fixed) // (native + shadow)``, budget
  ``blocks * native`` (``integration.py:17-23``).  ``native`` is the INT2 page bytes
  of every FULL layer for one 128-token block (plus the GDN state is fixed per slot
  and counted in ``fixed``), ``shadow`` the BF16 K+V of the MTP draft layer for one
  block, ``fixed`` the rotations (four D x D fp32 per FULL layer, as the reference
  counts R_k, R_v and their transposes), the staging arenas with their owner tags and
  any other per-model constant;
* :func:`verify_layers` - the FULL-attention layer ids must equal the expected set
  (``integration.py:35-44``);
* :func:`source_fingerprint` - sha256 over the package's source files
  (``integration.py:26-32``);
* :func:`ready_manifest` / :func:`validate` - the ``READY`` JSON line each rank prints
  and the check that all tensor-parallel ranks are present, agree on the layer set and
  run the same source (``delivery/check_ready.py:8-29``).

Pipeline parallelism is rejected like the reference (``integration.py:77-78``); data
parallelism is supported here (one budget per replica), unlike the reference, which
rejects DP != 1.
"""
from __future__ import annotations

import hashlib
import json
import os
from dataclasses import asdict, dataclass, field
from pathlib import Path

PAGE = 128


class BudgetError(RuntimeError):
    pass


@dataclass
class CacheGeometry:
    """Per-rank cache geometry of a hybrid model."""

    full_layers: int          # FULL-attention layers with INT2 KV on this rank
    kv_heads: int             # KV heads per rank
    head_dim: int = 256
    page_bytes: int = 17408   # one (block, KV head) INT2 page
    shadow_layers: int = 1    # MTP draft layers with BF16 KV
    stage_rows: int = 64      # staging arena rows (x 128 tokens) per FULL layer, 0 = off
    #                           (window layout: max_slots x (sink pages + ring); hashed: staging_tokens / 128)
    gdn_bytes_per_slot: int = 0
    max_slots: int = 0

    @property
    def native_per_block(self) -> int:
        return self.full_layers * self.kv_heads * self.page_bytes

    @property
    def shadow_per_block(self) -> int:
        return self.shadow_layers * 2 * PAGE * self.kv_heads * self.head_dim * 2

    @property
    def fixed_bytes(self) -> int:
        D = self.head_dim
        rot = self.full_layers * 4 * D * D * 4
        stage = self.full_layers * 2 * self.stage_rows * PAGE * self.kv_heads * D * 4
        owner = self.stage_rows * PAGE * 4
        return rot + stage + owner + self.gdn_bytes_per_slot * self.max_slots


@dataclass
class Budget:
    blocks: int
    native_bytes: int
    shadow_bytes: int
    fixed_bytes: int

    @property
    def total(self) -> int:
        return self.native_bytes + self.shadow_bytes + self.fixed_bytes


def memory_budget(avail_bytes: int, geo: CacheGeometry, pp: int = 1,
                  num_blocks_override: int | None = None) -> Budget:
    """Number of KV blocks that fit in ``avail_bytes`` and the bytes they take."""
    if pp != 1:
        raise BudgetError("pipeline parallelism is not supported (pp must be 1)")
    if num_blocks_override is not None:
        raise BudgetError("num_gpu_blocks_override is not supported: the budget is derived from memory")
    native, shadow, fixed = geo.native_per_block, geo.shadow_per_block, geo.fixed_bytes
    per = native + shadow
    if per <= 0:
        raise BudgetError("cache geometry has no per-block bytes")
    blocks = (avail_bytes - fixed) // per
    if blocks <= 0:
        raise BudgetError(f"not enough memory for one KV block: avail {avail_bytes} B, fixed {fixed} B, "
                          f"per block {per} B")
    return Budget(int(blocks), int(blocks * native), int(blocks * shadow), int(fixed))


def memory_line(rank: int, budget: Budget, geo: CacheGeometry, avail_bytes: int, allocated: dict,
                device=None) -> str:
    """``[oscar-b200] MEMORY {json}``: the budget derived from free memory and what the
    allocation took (the reference prints the same line from its budget seam)."""
    rec = {"rank": rank, "avail_bytes": int(avail_bytes), "fixed_bytes": geo.fixed_bytes,
           "native_per_block": geo.native_per_block, "shadow_per_block": geo.shadow_per_block,
           "blocks": budget.blocks, "native_bytes": budget.native_bytes, "shadow_bytes": budget.shadow_bytes,
           "budget_bytes": budget.total, "allocated": {k: int(v) for k, v in allocated.items()},
           "allocated_bytes": int(sum(allocated.values()))}
    if device is not None and getattr(device, "type", "cpu") == "cuda":
        import torch
        free, total = torch.cuda.mem_get_info(device)
        rec.update(gpu_free_bytes=int(free), gpu_total_bytes=int(total),
                   allocator_peak_bytes=int(torch.cuda.max_memory_allocated(device)))
    return "[oscar-b200] MEMORY " + json.dumps(rec, sort_keys=True)


def check_allocation(actual_bytes: int, budget: Budget, slack: float = 0.0) -> None:
    """The allocated cache must not exceed the budget it was sized from."""
    if actual_bytes > budget.total * (1.0 + slack):
        raise BudgetError(f"allocated cache {actual_bytes} B exceeds the budget {budget.total} B")


def verify_layers(expected: list[int] | set[int], actual: list[int] | set[int]) -> None:
    exp, act = set(int(x) for x in expected), set(int(x) for x in actual)
    if exp != act:
        missing, extra = sorted(exp - act), sorted(act - exp)
        raise BudgetError(f"FULL-attention layer set mismatch: missing {missing}, unexpected {extra}")


def source_fingerprint(root: str | Path | None = None) -> str:
    """sha256 over (relative path, bytes) of every .py/.cu/.cuh/.cpp/.h file of the package."""
    root = Path(root) if root is not None else Path(__file__).resolve().parents[1]
    h = hashlib.sha256()
    exts = {".py", ".cu", ".cuh", ".cpp", ".h"}
    files = sorted(p for p in root.rglob("*") if p.suffix in exts and p.is_file() and "__pycache__" not in p.parts)
    csrc = root.parent / "csrc"
    if csrc.is_dir():
        files += sorted(p for p in csrc.rglob("*") if p.suffix in exts and p.is_file())
    for p in files:
        rel = p.relative_to(root.parent).as_posix()
        h.update(rel.encode())
        h.update(b"\0")
        h.update(p.read_bytes())
        h.update(b"\0")
    return h.hexdigest()


@dataclass
class ReadyManifest:
    rank: int
    world_size: int
    layers: int
    layer_ids: list[int]
    shadow_layers: list[int]
    bytes: dict
    source: str
    sha256: str
    dp_rank: int = 0
    extra: dict = field(default_factory=dict)

    def line(self) -> str:
        return "[oscar-b200] READY " + json.dumps(asdict(self), sort_keys=True)


def ready_manifest(model, rank: int, world: int, budget: Budget | None = None, dp_rank: int = 0,
                   sha256: str | None = None) -> ReadyManifest:
    """Manifest of a model whose cache is allocated (``model.cache_bytes()``)."""
    full_ids = [m.layer_id for m in model.full_layers]
    shadow = [model.mtp.layer.layer_id] if getattr(model, "mtp", None) is not None else []
    by = dict(model.cache_bytes())
    if budget is not None:
        by["budget"] = budget.total
        by["blocks"] = budget.blocks
    src = str(Path(__file__).resolve().parents[1])
    return ReadyManifest(rank, world, len(full_ids), full_ids, shadow, by, src,
                         sha256 or source_fingerprint(), dp_rank)


def parse_ready_lines(text: str) -> list[dict]:
    out = []
    for line in text.splitlines():
        i = line.find("READY ")
        if i >= 0 and "[oscar-b200]" in line:
            out.append(json.loads(line[i + len("READY "):]))
    return out


def validate(manifests: list[dict], world_size: int | None = None, sha256: str | None = None) -> None:
    """All tensor-parallel ranks present (per data-parallel replica), identical layer
    sets, one source fingerprint (and the expected one when given)."""
    if not manifests:
        raise BudgetError("no READY manifest found")
    world = world_size or manifests[0]["world_size"]
    by_rep: dict[int, dict[int, dict]] = {}
    for m in manifests:
        if m["world_size"] != world:
            raise BudgetError(f"rank {m['rank']} reports world size {m['world_size']} != {world}")
        by_rep.setdefault(m.get("dp_rank", 0), {})[m["rank"]] = m
    for rep, ranks in by_rep.items():
        missing = sorted(set(range(world)) - set(ranks))
        if missing:
            raise BudgetError(f"replica {rep}: no READY manifest from ranks {missing}")
    ref = manifests[0]
    for m in manifests[1:]:
        if sorted(m["layer_ids"]) != sorted(ref["layer_ids"]):
            raise BudgetError(f"rank {m['rank']} layer ids {m['layer_ids']} != {ref['layer_ids']}")
        if m["sha256"] != ref["sha256"]:
            raise BudgetError(f"rank {m['rank']} runs different source ({m['sha256'][:12]} != {ref['sha256'][:12]})")
    if sha256 is not None and ref["sha256"] != sha256:
        raise BudgetError(f"source fingerprint {ref['sha256'][:12]} != expected {sha256[:12]}")


def geometry_of(model, max_slots: int = 0) -> CacheGeometry:
    """Cache geometry of a (not yet allocated) :class:`HybridModel`."""
    full = model.full_layers
    gdn = model.gdn_layers
    hk = full[0].Hk if full else 0
    D = full[0].D if full else 256
    o = model.oscar
    from ..kv.oracle import arena_rows
    int2 = bool(full) and full[0].kv_mode == 0
    rows = arena_rows(o.sink_tokens, o.recent_tokens, o.staging_tokens, o.staging_layout, max(1, max_slots)) if (
        o.window_enabled and int2) else 0
    from ..models.qwen35 import P_MAX
    per_slot = 0
    for g in gdn:  # bf16 state, two conv windows, two pending-token buffers, pending b/a
        per_slot += (g.Hv * g.dk * g.dv + 2 * g.conv_dim * 3 + 2 * P_MAX * g.conv_dim + P_MAX * 2 * g.Hv) * 2
    return CacheGeometry(full_layers=len(full), kv_heads=hk, head_dim=D,
                         page_bytes=17408 if int2 else 2 * PAGE * D * 2,
                         shadow_layers=1 if getattr(model, "mtp", None) is not None else 0,
                         stage_rows=rows, gdn_bytes_per_slot=per_slot, max_slots=max_slots)


def available_memory(device, utilization: float = 0.9, reserve_bytes: int = 0) -> int:
    """Bytes the cache may take on ``device``: free memory after the weights, capped at
    ``utilization`` of the total."""
    import torch
    free, total = torch.cuda.mem_get_info(device)
    used = total - free
    return max(0, int(total * utilization) - used - reserve_bytes)


def env_utilization() -> float:
    return float(os.environ.get("OSCAR_GPU_MEMORY_UTILIZATION", "0.9"))
