"""Memory-budget seam, layer verification and READY manifests (reference intent:
``tests/test_integration_budget.py``, ``tests/test_check_ready.py``)."""
import json

import pytest

from oscar_b200.engine import budget as B
from oscar_b200.models.config import tiny
from oscar_b200.models.qwen35 import HybridModel


def test_budget_math_matches_formula():
    geo = B.CacheGeometry(full_layers=16, kv_heads=1, head_dim=256, shadow_layers=1, stage_rows=64)
    avail = 80 * 2**30
    b = B.memory_budget(avail, geo)
    per = geo.native_per_block + geo.shadow_per_block
    assert b.blocks == (avail - geo.fixed_bytes) // per
    assert b.native_bytes == b.blocks * 16 * 17408
    assert b.shadow_bytes == b.blocks * 2 * 128 * 256 * 2
    # fixed = 4 DxD fp32 rotations + fp32 staging K/V + owner tags
    assert geo.fixed_bytes == 16 * 4 * 256 * 256 * 4 + 16 * 2 * 64 * 128 * 256 * 4 + 64 * 128 * 4


def test_budget_rejects():
    geo = B.CacheGeometry(full_layers=1, kv_heads=1)
    with pytest.raises(B.BudgetError):
        B.memory_budget(10, geo)
    with pytest.raises(B.BudgetError):
        B.memory_budget(2**34, geo, pp=2)
    with pytest.raises(B.BudgetError):
        B.memory_budget(2**34, geo, num_blocks_override=10)
    b = B.memory_budget(2**30, geo)
    B.check_allocation(b.total, b)
    with pytest.raises(B.BudgetError):
        B.check_allocation(b.total + 1, b)


def test_geometry_matches_allocation():
    m = HybridModel(tiny(num_layers=8), device="cpu", seed=0)
    geo = B.geometry_of(m, max_slots=4)
    b = B.memory_budget(256 * 2**20, geo)
    m.allocate_cache(b.blocks, 4)
    by = m.cache_bytes()
    pools = sum(l.pool.numel() for l in m.full_layers)
    stage = sum(l.stage_k.numel() * 8 for l in m.full_layers if l.stage_k is not None)
    assert pools == b.native_bytes
    assert by["full_kv"] == pools + stage
    assert by["mtp_shadow"] == b.shadow_bytes
    rot = len(m.full_layers) * 4 * 256 * 256 * 4
    assert by["gdn_state"] + by["owner"] + stage + rot == geo.fixed_bytes
    B.check_allocation(by["full_kv"] + by["mtp_shadow"] + by["gdn_state"] + by["owner"] + rot, b)


def test_verify_layers():
    B.verify_layers([3, 7, 11], {11, 7, 3})
    with pytest.raises(B.BudgetError, match="missing"):
        B.verify_layers([3, 7, 11], [3, 7])


def test_fingerprint_stable_and_sensitive(tmp_path):
    (tmp_path / "pkg").mkdir()
    (tmp_path / "pkg" / "a.py").write_text("x = 1\n")
    h1 = B.source_fingerprint(tmp_path / "pkg")
    assert h1 == B.source_fingerprint(tmp_path / "pkg")
    (tmp_path / "pkg" / "a.py").write_text("x = 2\n")
    assert B.source_fingerprint(tmp_path / "pkg") != h1


def _manifests(world=2, sha="ab" * 32, ids=(3, 7)):
    return [dict(rank=r, world_size=world, layers=len(ids), layer_ids=list(ids), shadow_layers=[8], bytes={},
                 source="x", sha256=sha, dp_rank=0, extra={}) for r in range(world)]


def test_ready_validate():
    B.validate(_manifests())
    with pytest.raises(B.BudgetError, match="ranks"):
        B.validate(_manifests()[:1], world_size=2)
    bad = _manifests()
    bad[1]["layer_ids"] = [3]
    with pytest.raises(B.BudgetError, match="layer ids"):
        B.validate(bad)
    bad = _manifests()
    bad[1]["sha256"] = "cd" * 32
    with pytest.raises(B.BudgetError, match="different source"):
        B.validate(bad)
    with pytest.raises(B.BudgetError, match="expected"):
        B.validate(_manifests(), sha256="ef" * 32)


def test_ready_line_roundtrip():
    m = HybridModel(tiny(num_layers=4), device="cpu", seed=0)
    m.allocate_cache(8, 2)
    man = B.ready_manifest(m, rank=0, world=1, sha256="00" * 32)
    parsed = B.parse_ready_lines("noise\n" + man.line() + "\nmore noise")
    assert parsed[0]["layer_ids"] == [m.full_layers[0].layer_id]
    assert parsed[0]["shadow_layers"] == [4]
    B.validate(parsed, world_size=1)
    json.dumps(parsed)


def test_budget_terms_equal_the_allocation():
    """The budget's per-block and fixed terms are the bytes the engine allocates: the INT2
    pool, the BF16 shadow pool, and the staging arena, owner tags and GDN state slots (the
    fixed term also counts the rotation matrices, which live with the weights)."""
    import json

    from oscar_b200.engine import budget as B
    from oscar_b200.engine.engine import LLMEngine
    from oscar_b200.models.config import tiny
    from oscar_b200.models.qwen35 import HybridModel

    m = HybridModel(tiny(num_layers=8), device="cpu")
    geo = B.geometry_of(m, max_slots=3)
    budget = B.memory_budget(64 * 2**20, geo)
    LLMEngine(m, num_blocks=budget.blocks, max_slots=3, max_batched_tokens=256)
    full = m.full_layers
    pools = sum(x.pool.numel() for x in full)
    staging = sum(x.stage_k.numel() * 4 + x.stage_v.numel() * 4 for x in full)
    alloc = m.cache_bytes()
    assert pools == budget.native_bytes
    assert alloc["mtp_shadow"] == budget.shadow_bytes
    rot = len(full) * 4 * 256 * 256 * 4
    assert staging + alloc["owner"] + alloc["gdn_state"] == geo.fixed_bytes - rot
    B.check_allocation(sum(alloc.values()), budget)
    line = B.memory_line(0, budget, geo, 64 * 2**20, alloc)
    rec = json.loads(line.split("MEMORY ", 1)[1])
    assert rec["blocks"] == budget.blocks and rec["allocated_bytes"] == sum(alloc.values())
