"""PERF capture (reference intent: ``tests/test_diagnostics.py``): disabled means no
wrappers; bounded, filtered capture; sort attribution; exceptions propagate and the
capture context is reset."""
import json

import pytest
import torch

from oscar_b200.engine.engine import LLMEngine
from oscar_b200.models.config import tiny
from oscar_b200.models.qwen35 import HybridModel
from oscar_b200.utils import diagnostics as Dg


def _engine():
    m = HybridModel(tiny(num_layers=4), device="cpu", seed=2)
    return LLMEngine(m, num_blocks=32, max_slots=4, max_batched_tokens=256)


def test_disabled_installs_nothing(monkeypatch):
    monkeypatch.delenv("OSCAR_ASCEND_PROFILE_STEPS", raising=False)
    eng = _engine()
    assert Dg.install(eng) is None
    assert "step" not in vars(eng) and "forward" not in vars(eng.model)


def test_bounded_capture_with_stages(monkeypatch):
    monkeypatch.setenv("OSCAR_ASCEND_PROFILE_STEPS", "2")
    lines = []
    eng = _engine()
    d = Dg.install(eng, Dg.Diagnostics.from_env(sink=lines.append))
    eng.generate([list(range(3, 100)), list(range(9, 40))], 5)
    assert len(lines) == 2 and d.captured == 2 and d.seen > 2
    rec = json.loads(lines[0][len(Dg.PREFIX):])
    assert {"step", "forward", "full_attention", "gdn", "sample"} <= set(rec["stages"])
    assert rec["shape"]["requests"] == 2 and rec["code_sha256"]
    assert rec["stages"]["gdn"]["count"] == 3


def test_filters(monkeypatch):
    monkeypatch.setenv("OSCAR_ASCEND_PROFILE_STEPS", "5")
    monkeypatch.setenv("OSCAR_ASCEND_PROFILE_MIN_REQUESTS", "3")
    lines = []
    eng = _engine()
    Dg.install(eng, Dg.Diagnostics.from_env(sink=lines.append))
    eng.generate([list(range(3, 100)), list(range(9, 40))], 3)
    assert lines == []
    d = Dg.Diagnostics(steps=5, max_tokens_per_request=4)
    assert not d.matches({"requests": 2, "max_tokens_per_request": 97})
    assert d.matches({"requests": 2, "max_tokens_per_request": 4})


def test_sort_trace_and_exceptions():
    d = Dg.Diagnostics(steps=3, sink=lambda s: None)

    def step():
        torch.argsort(torch.tensor([3, 1, 2]))
        torch.sort(torch.tensor([0.5, 0.1]))
        return 7

    assert d.capture_step(step, {"requests": 1, "max_tokens_per_request": 1}) == 7
    rec = json.loads(d.lines[-1][len(Dg.PREFIX):])
    assert rec["sorts"] == 2 and rec["int_sorts"] == 1 and "argsort" in rec["int_sort_stacks"][0]

    def bad():
        raise ValueError("boom")

    with pytest.raises(ValueError, match="boom"):
        d.capture_step(bad, {"requests": 1, "max_tokens_per_request": 1})
    assert d._stages is None
    with d.timed("outside"):  # no capture active: no record
        pass
