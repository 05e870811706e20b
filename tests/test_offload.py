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


def test_abort_of_a_swapped_out_request():
    """Aborting a request while it sits in host memory drops its host copy; the others
    finish as without preemption and every block comes back."""
    ref, _ = _run(64, False)
    m = HybridModel(tiny(num_layers=4), device="cpu", seed=6)
    eng = LLMEngine(m, num_blocks=6, max_slots=4, max_batched_tokens=512, offload=True)
    rids = [eng.add_request(p, 60) for p in PROMPTS]
    victim = None
    while eng.has_work():
        eng.step()
        if victim is None and eng.swapped_q:
            victim = eng.swapped_q[0]
            eng.abort(victim)
            assert victim not in eng.offload.swapped and eng.requests[victim].finish_reason == "abort"
    assert victim is not None
    for rid, want in zip(rids, ref):
        if rid != victim:
            assert eng.requests[rid].output == want
    assert eng.bm.free_blocks == 6 and not eng.offload.swapped


def test_pinned_pool_reuses_its_buffers():
    """Swaps take byte ranges of the pool and give them back; memory is allocated from the
    system only when the pool is created or when a request does not fit."""
    from oscar_b200.kv.offload import PinnedPool

    pool = PinnedPool(initial_bytes=1 << 20, chunk_bytes=1 << 20, pin=False)
    assert pool.allocations == 1 and pool.capacity == 1 << 20
    a, ha = pool.alloc(1000)
    b, hb = pool.alloc(300_000)
    assert a.numel() == 1000 and b.numel() == 300_000 and a.data_ptr() % 256 == 0 and b.data_ptr() % 256 == 0
    pool.release(ha)
    pool.release(hb)
    assert pool.used() == 0 and len(pool.free) == 1  # coalesced back into one range
    for _ in range(10):  # repeated swaps of the same size reuse the same range
        x, hx = pool.alloc(500_000)
        pool.release(hx)
    assert pool.allocations == 1
    big, hbig = pool.alloc(3 << 20)  # does not fit: one new chunk of at least that size
    assert pool.allocations == 2 and big.numel() == 3 << 20
    pool.release(hbig)
    assert pool.used() == 0
