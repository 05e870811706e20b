"""Engine behaviour on CPU (pure-torch op references): speculative decoding, chunked
prefill, continuous batching and tensor parallelism must not change greedy outputs.

Mirrors the reference's end-to-end serving checks (``tests/test_e2e_serving.py``,
``tests/test_mtp_acceptance.py``) with the tiny hybrid config instead of a checkpoint.
"""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from oscar_b200.engine.engine import LLMEngine, SeededAcceptance
from oscar_b200.models.config import tiny
from oscar_b200.models.qwen35 import HybridModel

PROMPTS = [[1, 2, 3, 4, 5] * 40, [7, 8, 9] * 30, list(range(11, 140))]


def _gen(num_spec=3, max_batched=512, prompts=PROMPTS, n=6, acceptance=None, tp=None, layers=4):
    m = HybridModel(tiny(num_layers=layers), tp=tp, device="cpu", seed=1)
    eng = LLMEngine(m, num_blocks=64, max_slots=4, max_batched_tokens=max_batched, num_spec=num_spec,
                    acceptance=acceptance)
    return eng.generate(prompts, n), eng


def test_spec_decode_matches_greedy():
    spec, eng = _gen(num_spec=3)
    greedy, _ = _gen(num_spec=0)
    assert spec == greedy
    assert eng.stats["drafts_proposed"] > 0


def test_chunked_prefill_matches_whole_prefill():
    whole, _ = _gen(max_batched=1024)
    chunked, _ = _gen(max_batched=48)
    assert chunked == whole


def test_batching_does_not_change_outputs():
    together, _ = _gen()
    alone = [_gen(prompts=[p])[0][0] for p in PROMPTS]
    assert together == alone


def _gen_static(lookahead: bool, prompts, n, acceptance=None):
    """The graph-form (static metadata) step path on CPU, with or without building the next
    step's metadata while the drafts are computed."""
    m = HybridModel(tiny(num_layers=4), device="cpu", seed=1)
    eng = LLMEngine(m, num_blocks=64, max_slots=4, max_batched_tokens=512, num_spec=3, acceptance=acceptance)
    eng.use_graphs = True
    eng.lookahead = lookahead
    ids = [eng.add_request(p, k) for p, k in zip(prompts, n)]
    while eng.has_work():
        eng.step()
    return [eng.requests[i].output for i in ids], eng


def test_lookahead_metadata_gives_the_same_tokens():
    # requests of different lengths: one finishes early, which invalidates a prepared batch
    n = [9, 4, 7]
    want, _ = _gen_static(False, PROMPTS, n)
    got, eng = _gen_static(True, PROMPTS, n)
    assert got == want
    assert eng.stats.get("lookahead_steps", 0) > 0
    want2, _ = _gen_static(False, PROMPTS, n, acceptance=SeededAcceptance(3, 2.0, seed=3))
    got2, _ = _gen_static(True, PROMPTS, n, acceptance=SeededAcceptance(3, 2.0, seed=3))
    assert got2 == want2


def test_seeded_acceptance_mean():
    acc = SeededAcceptance(3, 2.0, seed=0)  # 2 of 3 drafts accepted on average
    draws = [acc(0) for _ in range(3000)]
    assert all(0 <= d <= 3 for d in draws)
    assert abs(sum(draws) / len(draws) - 2.0) < 0.1


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _first_step_hidden(tp=None):
    m = HybridModel(tiny(num_layers=4), tp=tp, device="cpu", seed=1)
    eng = LLMEngine(m, num_blocks=64, max_slots=4, max_batched_tokens=512)
    for p in PROMPTS:
        eng.add_request(p, 4)
    eng.step()  # one prefill step of all prompts
    return eng.last[0].float().clone()


def _tp_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    from oscar_b200.parallel.groups import init_distributed, make_groups
    import torch.distributed as dist
    init_distributed("gloo", timeout_s=120)
    try:
        tp = make_groups(world)
        out, _ = _gen(tp=tp)
        q.put((rank, out, _first_step_hidden(tp).numpy()))
    finally:
        dist.destroy_process_group()


def test_tensor_parallel_matches_single_rank():
    """TP=2 ranks hold slices of the same logical model: they agree with each other
    exactly and with TP=1 up to the per-shard activation quantisation of the
    row-parallel inputs (per-token int8 scales are taken over each rank's shard; on
    this random-init model one such quantisation alone is ~3 % relative error, so four
    layers stay within 15 %)."""
    single_hid = _first_step_hidden()
    single, _ = _gen()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_tp_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {r: (out, torch.from_numpy(hid)) for r, out, hid in (q.get(timeout=300) for _ in procs)}
    for p in procs:
        p.join(60)
    assert res[0][0] == res[1][0]
    assert torch.equal(res[0][1], res[1][1])
    err = (res[0][1] - single_hid).norm() / single_hid.norm()
    assert err < 0.15, err
    assert [o[0] for o in res[0][0]] == [o[0] for o in single]


# Four ranks with more query heads than KV heads per rank and fewer KV heads than ranks:
# each rank holds 3 query heads and a replica of its group's KV head, and 1 GDN key head
# with its 3 value heads - the head layout of the target model at TP8.
_TP4_CFG = dict(num_layers=4, num_attention_heads=12, num_key_value_heads=2, linear_num_key_heads=4,
                linear_num_value_heads=12)


def _tp4_hidden(tp=None):
    m = HybridModel(tiny(**_TP4_CFG), tp=tp, device="cpu", seed=2)
    eng = LLMEngine(m, num_blocks=64, max_slots=4, max_batched_tokens=512)
    for p in PROMPTS:
        eng.add_request(p, 4)
    eng.step()  # one prefill step
    out = [eng.requests[r].output[:1] for r in sorted(eng.requests)]
    return eng.last[0].float().clone(), out


def _tp4_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    from oscar_b200.parallel.groups import init_distributed, make_groups
    import torch.distributed as dist
    init_distributed("gloo", timeout_s=180)
    try:
        hid, out = _tp4_hidden(make_groups(world))
        q.put((rank, hid.numpy(), out))
    finally:
        dist.destroy_process_group()


def test_tp4_with_replicated_kv_heads_matches_single_rank():
    """TP=4 over 2 KV heads (replicated, two ranks per KV head) and 4 GDN key heads:
    the ranks agree exactly and match TP=1 up to the per-shard activation quantisation
    (same bound as the TP=2 test above)."""
    single_hid, single_out = _tp4_hidden()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_tp4_worker, args=(r, 4, port, q)) for r in range(4)]
    for p in procs:
        p.start()
    res = {r: (torch.from_numpy(h), o) for r, h, o in (q.get(timeout=600) for _ in procs)}
    for p in procs:
        p.join(60)
    for r in (1, 2, 3):
        assert torch.equal(res[0][0], res[r][0])
        assert res[0][1] == res[r][1]
    err = (res[0][0] - single_hid).norm() / single_hid.norm()
    assert err < 0.15, err


def _dp_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    from oscar_b200.parallel.groups import init_distributed, make_groups
    import torch.distributed as dist
    init_distributed("gloo", timeout_s=180)
    try:
        tp = make_groups(tp=2, dp=2)
        mine = PROMPTS[:2] if tp.dp_rank == 0 else PROMPTS[2:]  # the request split of ``bench.py --dp``
        out, _ = _gen(tp=tp, prompts=mine)
        q.put((rank, tp.dp_rank, tp.rank, out))
    finally:
        dist.destroy_process_group()


def test_dp2_tp2_replicas_serve_their_own_requests():
    """DP2 x TP2 on four ranks: two replicas of two consecutive ranks, each running its own
    requests with its TP collectives on its own subgroup at the same time.  The two ranks of
    a replica agree exactly, and each replica's first tokens match TP=1 on the same prompts
    (later tokens may differ by the per-shard activation quantisation, as in the TP=2 test)."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_dp_worker, args=(r, 4, port, q)) for r in range(4)]
    for p in procs:
        p.start()
    res = {r: (d, t, out) for r, d, t, out in (q.get(timeout=600) for _ in procs)}
    for p in procs:
        p.join(60)
    assert [(res[r][0], res[r][1]) for r in range(4)] == [(0, 0), (0, 1), (1, 0), (1, 1)]
    assert res[0][2] == res[1][2] and res[2][2] == res[3][2]
    single, _ = _gen()
    assert [o[0] for o in res[0][2] + res[2][2]] == [o[0] for o in single]


def test_reused_state_slot_starts_from_zero_state():
    """A request that takes over a freed GDN state slot starts from a zero recurrent
    state and conv window, not from the previous occupant's: with one slot, requests
    run one after another give what each gives on a fresh engine."""
    m = HybridModel(tiny(num_layers=4), device="cpu", seed=1)
    eng = LLMEngine(m, num_blocks=64, max_slots=1, max_batched_tokens=512)
    seq = [eng.generate([p], 5)[0] for p in (PROMPTS[0], PROMPTS[1], PROMPTS[0])]
    fresh = [_gen(prompts=[p], n=5)[0][0] for p in (PROMPTS[0], PROMPTS[1])]
    assert seq == [fresh[0], fresh[1], fresh[0]]
