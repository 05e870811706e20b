"""OSCAR layer selection (reference intent: ``tests/test_plugin_selection.py``)."""
from types import SimpleNamespace

from oscar_b200.models import selection as S
from oscar_b200.models.config import tiny
from oscar_b200.models.qwen35 import HybridModel


def test_rules(monkeypatch):
    monkeypatch.delenv("OSCAR_ASCEND_ENABLE", raising=False)
    hyb = tiny()
    assert S.is_hybrid_config(hyb)
    assert S.is_hybrid_config(SimpleNamespace(model_type="qwen3_next", layer_types=[]))
    assert not S.is_hybrid_config(SimpleNamespace(layer_types=["full_attention"] * 4))
    assert S.should_oscar(S.AttentionSpec(3), hyb)
    assert not S.should_oscar(S.AttentionSpec(3, is_mtp=True), hyb)
    assert not S.should_oscar(S.AttentionSpec(3, attn_type="encoder"), hyb)
    assert not S.should_oscar(S.AttentionSpec(3, sliding_window=4096), hyb)
    assert not S.should_oscar(S.AttentionSpec(3, has_sinks=True), hyb)
    monkeypatch.setenv("OSCAR_ASCEND_ENABLE", "0")
    assert not S.should_oscar(S.AttentionSpec(3), hyb)


def test_model_uses_rules(monkeypatch):
    monkeypatch.setenv("OSCAR_ASCEND_ENABLE", "0")
    m = HybridModel(tiny(num_layers=4), device="cpu")
    assert all(l.kv_mode == 1 for l in m.full_layers)
    m.allocate_cache(8, 2)
    assert m.stage_rows == 0
    monkeypatch.setenv("OSCAR_ASCEND_ENABLE", "auto")
    m = HybridModel(tiny(num_layers=4), device="cpu")
    assert all(l.kv_mode == 0 for l in m.full_layers) and m.mtp.layer.kv_mode == 1
