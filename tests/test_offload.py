"""Host KV offload (swap-based preemption): with a block pool too small for every
request at once, requests are swapped out to host memory and back, and the outputs
equal those of an engine that never preempts."""
import pytest
import torch

from oscar_b200.engine.engine import LLMEngine
from oscar_b200.models.config import tiny
from oscar_b200.models.qwen35 import HybridModel

PROMPTS = [list(range(3, 3 + 120)), list(range(40, 40 + 250)), list(range(7, 7 + 126))]


def _run(num_blocks, offload, device="cpu", n=60):
    m = HybridModel(tiny(num_layers=4), device=device, seed=6)
    eng = LLMEngine(m, num_blocks=num_blocks, max_slots=4, max_batched_tokens=512, offload=offload)
    out = eng.generate(PROMPTS, n)
    return out, eng


def _check(device):
    ref, _ = _run(64, False, device)
    out, eng = _run(6, True, device)  # the three requests grow to 7 blocks together
    assert eng.stats.get("preempted", 0) > 0
    assert eng.offload.stats.swapped_in == eng.offload.stats.swapped_out
    assert out == ref


def test_swap_preemption_matches_cpu():
    _check("cpu")


@pytest.mark.gpu
def test_swap_preemption_matches_gpu():
    _check("cuda")
