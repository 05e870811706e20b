"""A/B harness semantics (reference intent: ``tests/test_benchmark_utils.py``): first
call separated, alternating order, numeric match first, shared output buffers caught.
Runs on the CPU with the timer replaced."""
import pytest
import torch

from oscar_b200.bench import harness as H


def test_compare_calls_semantics(monkeypatch):
    calls = []
    monkeypatch.setattr(H, "time_call", lambda fn, flush=True: (fn(), 1.0 if calls[-1] == "a" else 2.0)[1])
    x = torch.ones(4)

    def a():
        calls.append("a")
        return x * 2

    def b():
        calls.append("b")
        return x * 2 + 1e-6

    res = H.compare_calls({"a": a, "b": b}, iters=4)
    # numeric check (a, b), first calls (a, b), then alternating a b | b a | a b | b a
    assert calls == ["a", "b", "a", "b", "a", "b", "b", "a", "a", "b", "b", "a"]
    assert res["a"].median_ms == 1.0 and res["b"].median_ms == 2.0 and len(res["a"].samples) == 4


def test_compare_calls_rejects_mismatch_and_shared_buffers(monkeypatch):
    monkeypatch.setattr(H, "time_call", lambda fn, flush=True: 0.0)
    buf = torch.ones(4)
    with pytest.raises(AssertionError, match="differs"):
        H.compare_calls({"a": lambda: buf, "b": lambda: buf * 3})
    with pytest.raises(AssertionError, match="share one output buffer"):
        H.compare_calls({"a": lambda: buf, "b": lambda: buf})
