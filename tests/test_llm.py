"""Offline generation API (CPU): ``LLM.generate`` over a config name or a Hugging Face
checkpoint directory gives the engine's tokens, with max_tokens, stop ids, EOS and
seeded sampling taken from ``SamplingParams``."""
from __future__ import annotations

import json

import torch

import oscar_b200
from oscar_b200.engine.engine import LLMEngine
from oscar_b200.models import loader as L
from oscar_b200.models.config import tiny
from oscar_b200.models.qwen35 import HybridModel

KW = dict(device="cpu", num_blocks=64, max_num_seqs=4, max_batched_tokens=512)


def test_generate_matches_the_engine():
    llm = oscar_b200.LLM("qwen35-tiny", **KW)
    SP = oscar_b200.SamplingParams
    outs = llm.generate(["hello there", list(range(5, 40))], SP(max_tokens=6))
    eng = LLMEngine(HybridModel(tiny(), device="cpu", seed=0), num_blocks=64, max_slots=4, max_batched_tokens=512)
    want = eng.generate([[b + 3 for b in b"hello there"], list(range(5, 40))], 6)
    assert [o.outputs[0].token_ids for o in outs] == want
    assert outs[0].prompt == "hello there" and outs[1].prompt is None
    assert all(o.outputs[0].finish_reason == "length" for o in outs)
    # stop ids, EOS (none for the byte tokenizer) and seeded sampling
    stop = want[1][2]
    o = llm.generate(list(range(5, 40)), SP(max_tokens=6, stop_token_ids=[stop]))[0].outputs[0]
    assert o.token_ids == want[1][:want[1].index(stop) + 1] and o.finish_reason == "stop"
    a = llm.generate(list(range(5, 40)), SP(temperature=0.9, seed=3, max_tokens=6))[0].outputs[0].token_ids
    b = llm.generate(list(range(5, 40)), SP(temperature=0.9, seed=3, max_tokens=6))[0].outputs[0].token_ids
    assert a == b and len(a) == 6
    assert not llm.engine.requests  # released


def test_checkpoint_directory(tmp_path):
    m = HybridModel(tiny(), device="cpu", seed=4)
    L.save_hf_checkpoint(m, str(tmp_path), dtype=torch.float32)
    want = LLMEngine(L.from_pretrained(str(tmp_path), device="cpu"), num_blocks=64, max_slots=4,
                     max_batched_tokens=512).generate([list(range(9, 50))], 5)[0]
    (tmp_path / "generation_config.json").write_text(json.dumps({"eos_token_id": want[3]}))
    llm = oscar_b200.LLM(str(tmp_path), **KW)
    assert llm.eos_token_ids == [want[3]]
    o = llm.generate([list(range(9, 50))], oscar_b200.SamplingParams(max_tokens=5))[0].outputs[0]
    assert o.token_ids == want[:want.index(want[3]) + 1] and o.finish_reason == "stop"
    o = llm.generate([list(range(9, 50))], oscar_b200.SamplingParams(max_tokens=5, ignore_eos=True))[0].outputs[0]
    assert o.token_ids == want and o.finish_reason == "length"


def _rank(rank, port, q):
    import os

    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE="2",
                      LOCAL_RANK=str(rank))
    try:
        llm = oscar_b200.LLM("qwen35-tiny", **KW)
        outs = llm.generate([list(range(5, 40)), "hi"], oscar_b200.SamplingParams(max_tokens=5, temperature=0.8,
                                                                                  seed=2))
        q.put((rank, llm.world, [o.outputs[0].token_ids for o in outs]))
        llm.close()
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def test_every_rank_of_a_tp_launch_returns_the_same_outputs():
    import socket

    import torch.multiprocessing as mp

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_rank, args=(r, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = {r: (w, o) for r, w, o in (q.get(timeout=300) for _ in ps)}
    for p in ps:
        p.join(60)
    assert res[0][0] == res[1][0] == 2
    assert res[0][1] == res[1][1] and all(len(o) == 5 for o in res[0][1])


def test_stop_strings_cut_the_text_and_end_the_request():
    llm = oscar_b200.LLM("qwen35-tiny", **KW)
    full = llm.generate([list(range(5, 40))], oscar_b200.SamplingParams(max_tokens=12))[0].outputs[0]
    stop = full.text[3:5]
    assert stop and stop in full.text
    got = llm.generate([list(range(5, 40))], oscar_b200.SamplingParams(max_tokens=12, stop=[stop]))[0].outputs[0]
    assert got.text == full.text[:full.text.find(stop)] and got.finish_reason == "stop"
    assert len(got.token_ids) < len(full.token_ids)  # the engine stopped generating
    assert full.token_ids[:len(got.token_ids)] == got.token_ids
