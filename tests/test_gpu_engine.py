"""Engine-level GPU checks: CUDA-graph replay equals eager execution (greedy and seeded
sampling), and speculative decoding with a perfect drafter reproduces plain greedy
decoding."""
import pytest
import torch

from oscar_b200.engine.engine import LLMEngine
from oscar_b200.models.config import tiny
from oscar_b200.models.qwen35 import HybridModel
from oscar_b200.ops.sampling import SamplingParams

pytestmark = pytest.mark.gpu


def _run(use_graphs: bool, num_spec: int = 3, steps_out: int = 12, sampling=None):
    torch.manual_seed(0)
    model = HybridModel(tiny(num_layers=4), device="cuda", seed=3)
    eng = LLMEngine(model, num_blocks=64, max_slots=8, max_batched_tokens=1024, num_spec=num_spec)
    eng.use_graphs = use_graphs
    prompts = [list(range(5, 300)), list(range(40, 170)), list(range(7, 520, 3))]
    out = eng.generate(prompts, max_new_tokens=steps_out, sampling=sampling)
    return out, eng


def test_graph_replay_matches_eager():
    eager, _ = _run(False)
    graph, eng = _run(True)
    assert eng._graphs, "no CUDA graph was captured"
    assert graph == eager


def test_spec_decode_matches_greedy_on_gpu():
    greedy, _ = _run(True, num_spec=0)
    spec, _ = _run(True, num_spec=3)
    assert spec == greedy


def test_sampled_graph_replay_matches_eager():
    """Steps with sampled requests (the sampler's per-row arrays ride in the graph's static
    metadata buffer) replay to the same tokens as eager steps."""
    sp = [SamplingParams(temperature=0.8, top_k=40, seed=1), SamplingParams(temperature=1.0, top_p=0.9, seed=2),
          None]
    eager, _ = _run(False, sampling=sp)
    graph, eng = _run(True, sampling=sp)
    assert any("samp_t" in str(k) for k in eng._graphs), "no sampling step was captured"
    assert graph == eager
