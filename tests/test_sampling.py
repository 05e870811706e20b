"""Sampling and draft verification (CPU): the Gumbel-max sampler draws from the truncated
softmax, draft verification emits tokens distributed exactly as the target distribution,
a vocabulary split over ranks draws the same tokens as one rank, and the engine and the
HTTP server pass per-request sampling parameters through."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oscar_b200.ops import sampling as S


def _lowbias32(x: int) -> int:
    x &= 0xFFFFFFFF
    x ^= x >> 16
    x = (x * 0x7FEB352D) & 0xFFFFFFFF
    x ^= x >> 15
    x = (x * 0x846CA68B) & 0xFFFFFFFF
    return x ^ (x >> 16)


def test_hash_matches_plain_integer_arithmetic():
    xs = [0, 1, 2, 0xFFFF, 0x10000, 123456789, 0x7FFFFFFF, 0x80000000, 0xFFFFFFFF, 0xDEADBEEF]
    got = S.hash32(torch.tensor(xs, dtype=torch.int64)).tolist()
    assert got == [_lowbias32(x) for x in xs]


def _rows(n, temperature=1.0, top_k=0, top_p=1.0, seed=7, pos=None, draft=None):
    return S.SampleRows(torch.full((n,), float(temperature)), torch.full((n,), top_k, dtype=torch.int32),
                        torch.full((n,), float(top_p)), torch.full((n,), seed, dtype=torch.int32),
                        torch.arange(n, dtype=torch.int32) if pos is None else pos,
                        torch.full((n,), -1, dtype=torch.int32) if draft is None else draft)


def _freq(tokens, V):
    return np.bincount(tokens.numpy(), minlength=V) / len(tokens)


LOGITS = torch.randn(64, generator=torch.Generator().manual_seed(3)) * 2.0


@pytest.mark.parametrize("params", [
    S.SamplingParams(temperature=1.0),
    S.SamplingParams(temperature=0.6),
    S.SamplingParams(temperature=1.3, top_k=5),
    S.SamplingParams(temperature=0.9, top_p=0.7),
    S.SamplingParams(temperature=1.0, top_k=20, top_p=0.8),
])
def test_samples_follow_the_truncated_distribution(params):
    N, V = 40000, LOGITS.numel()
    logits = LOGITS.unsqueeze(0).expand(N, V).contiguous()
    rows = _rows(N, params.temperature, params.top_k, params.top_p)  # one position per draw
    tok = S.sample(logits, 0, rows)
    p = S.probabilities(LOGITS, params).numpy()
    f = _freq(tok, V)
    assert np.all(f[p == 0] == 0), "sampled a truncated token"
    assert 0.5 * np.abs(f - p).sum() < 0.02


@pytest.mark.parametrize("params", [S.SamplingParams(temperature=0.8), S.SamplingParams(temperature=1.0, top_k=8),
                                    S.SamplingParams(temperature=1.0, top_p=0.9)])
@pytest.mark.parametrize("draft", [0, 1, 63])
def test_draft_verification_is_exact(params, draft):
    """Accept-with-p(d) / resample-without-d emits tokens distributed as p for any draft,
    likely or not (token 0 is the most likely after sorting the test logits)."""
    N, V = 40000, LOGITS.numel()
    order = torch.argsort(LOGITS, descending=True)
    d = int(order[draft])
    logits = LOGITS.unsqueeze(0).expand(N, V).contiguous()
    rows = _rows(N, params.temperature, params.top_k, params.top_p, draft=torch.full((N,), d, dtype=torch.int32))
    tok = S.sample(logits, 0, rows)
    p = S.probabilities(LOGITS, params).numpy()
    f = _freq(tok, V)
    assert 0.5 * np.abs(f - p).sum() < 0.02
    assert abs(f[d] - p[d]) < 0.01  # acceptance rate = p(d)


def test_greedy_rows_take_the_argmax_and_ignore_drafts():
    logits = torch.randn(6, 100)
    rows = _rows(6, temperature=0.0, draft=torch.full((6,), 3, dtype=torch.int32))
    assert torch.equal(S.sample(logits, 0, rows), logits.argmax(1))


def test_vocab_split_over_ranks_draws_the_same_tokens():
    """Phase statistics of two vocabulary shards, gathered, give the tokens of one shard."""
    g = torch.Generator().manual_seed(5)
    n, V = 48, 3000
    logits = torch.randn(n, V, generator=g) * 3
    temps = torch.tensor([0.0, 0.7, 1.0, 1.5] * 12)
    rows = S.SampleRows(temps, torch.tensor([0, 0, 7, 2000] * 12, dtype=torch.int32),
                        torch.tensor([1.0, 0.85, 1.0, 0.6] * 12), torch.arange(n, dtype=torch.int32) * 31,
                        torch.arange(n, dtype=torch.int32) + 100,
                        torch.randint(-1, V, (n,), generator=g, dtype=torch.int32))
    want = S.sample(logits, 0, rows)
    for cut in (1000, 1500, 2999):
        shards = [(logits[:, :cut], 0), (logits[:, cut:], cut)]
        st = torch.stack([S.phase1(sh, rows) for sh, _ in shards])
        m, tau = S.combine1(st, rows)
        parts = torch.stack([S.phase2(sh, b, rows, m, tau) for sh, b in shards])
        assert torch.equal(S.combine2(parts, rows), want), cut


def test_samples_depend_only_on_seed_and_position():
    logits = torch.randn(1, 500).expand(8, 500).contiguous()
    pos = torch.tensor([5, 6, 7, 8, 5, 6, 7, 8], dtype=torch.int32)
    rows = _rows(8, 1.0, pos=pos)
    tok = S.sample(logits, 0, rows)
    assert torch.equal(tok[:4], tok[4:])
    other = S.sample(logits, 0, _rows(8, 1.0, seed=8, pos=pos))
    assert not torch.equal(tok, other)


def test_params_validation():
    with pytest.raises(ValueError):
        S.SamplingParams(temperature=-1).validate()
    with pytest.raises(ValueError):
        S.SamplingParams(top_k=S.MAX_TOP_K + 1).validate()
    with pytest.raises(ValueError):
        S.SamplingParams(top_p=0.0).validate()
    assert S.SamplingParams(temperature=0.0).greedy


# ----------------------------------------------------------------------------- engine
import os  # noqa: E402
import socket  # noqa: E402

import torch.multiprocessing as mp  # noqa: E402

from oscar_b200.engine.engine import LLMEngine  # noqa: E402
from oscar_b200.models.config import tiny  # noqa: E402
from oscar_b200.models.qwen35 import HybridModel  # noqa: E402

PROMPTS = [[1, 2, 3, 4, 5] * 12, [7, 8, 9] * 10, list(range(11, 60))]


def _engine(num_spec=3, tp=None, seed=0):
    m = HybridModel(tiny(num_layers=4), tp=tp, device="cpu", seed=1)
    return LLMEngine(m, num_blocks=64, max_slots=4, max_batched_tokens=512, num_spec=num_spec, seed=seed)


def test_temperature_zero_is_greedy():
    greedy = _engine().generate(PROMPTS, 6)
    assert _engine().generate(PROMPTS, 6, S.SamplingParams(temperature=0.0, top_k=3)) == greedy


def test_sampled_generation_is_seeded_and_batch_invariant():
    sp = [S.SamplingParams(temperature=1.0, seed=11), S.SamplingParams(temperature=0.8, top_p=0.9, seed=12),
          None]
    a = _engine().generate(PROMPTS, 8, sp)
    assert _engine().generate(PROMPTS, 8, sp) == a
    alone = [_engine().generate([p], 8, [s])[0] for p, s in zip(PROMPTS, sp)]
    assert alone == a  # the greedy request is unchanged by sharing a sampling batch
    assert a[2] == _engine().generate([PROMPTS[2]], 8)[0]
    other = _engine().generate(PROMPTS, 8, [S.SamplingParams(temperature=1.0, seed=99)] * 3)
    assert other[:2] != a[:2]
    # no seed: derived from the engine seed and the request id
    b1 = _engine(seed=5).generate(PROMPTS[:1], 8, S.SamplingParams(temperature=1.0))
    assert b1 == _engine(seed=5).generate(PROMPTS[:1], 8, S.SamplingParams(temperature=1.0))


def test_verify_rows_carry_their_drafts_and_positions(monkeypatch):
    """Each verify row samples position ``num_computed + i + 1`` and verifies draft ``i``."""
    eng = _engine()
    sp = S.SamplingParams(temperature=0.7, seed=3)
    for p in PROMPTS:
        eng.add_request(p, 10, sp)
    seen = []
    real = S.sample

    def spy(logits, vocab_begin, rows, tp=None):
        seen.append((rows.pos.tolist(), rows.draft.tolist()))
        return real(logits, vocab_begin, rows, tp)

    monkeypatch.setattr(S, "sample", spy)
    checked = 0
    while eng.has_work():
        want_pos, want_draft = [], []
        decoding = [eng.requests[r] for r in eng.running if eng.requests[r].prefill_done]
        for r in decoding:
            n = 1 + len(r.drafts)
            want_pos += [r.num_computed + i + 1 for i in range(n)]
            want_draft += [r.drafts[i] if i < len(r.drafts) else -1 for i in range(n)]
        seen.clear()
        eng.step()
        if decoding and not eng.waiting and all(eng.requests[r].prefill_done for r in eng.running):
            pos, draft = seen[0]
            if len(pos) == len(want_pos):
                assert pos == want_pos and draft == want_draft
                checked += 1
    assert checked >= 2
    assert eng.stats["drafts_proposed"] > 0


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _tp_rank(rank, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE="2",
                      LOCAL_RANK=str(rank))
    import torch.distributed as dist
    from oscar_b200.parallel.groups import init_distributed, make_groups
    init_distributed("gloo", timeout_s=120)
    try:
        out = _engine(tp=make_groups(2)).generate(PROMPTS, 6, S.SamplingParams(temperature=0.9, top_k=50, seed=4))
        q.put((rank, out))
    finally:
        dist.destroy_process_group()


def test_tensor_parallel_ranks_draw_the_same_tokens():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_tp_rank, args=(r, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = dict(q.get(timeout=300) for _ in ps)
    for p in ps:
        p.join(60)
    assert res[0] == res[1]
    assert all(len(o) == 6 for o in res[0])


def test_http_sampling_parameters():
    from fastapi.testclient import TestClient

    from oscar_b200.serve.server import create_app
    from oscar_b200.serve.worker import EngineWorker

    eng = _engine()
    w = EngineWorker(eng).start()
    try:
        c = TestClient(create_app(w, vocab_size=eng.model.cfg.vocab_size))
        body = {"prompt": PROMPTS[0], "max_tokens": 5, "temperature": 0.9, "top_k": -1, "top_p": 0.95, "seed": 21}
        a = c.post("/v1/completions", json=body).json()["choices"][0]["token_ids"]
        b = c.post("/v1/completions", json=body).json()["choices"][0]["token_ids"]
        assert a == b and len(a) == 5
        assert c.post("/v1/completions", json={**body, "top_p": 0.0}).status_code == 400
        assert c.post("/v1/completions", json={**body, "temperature": -1}).status_code == 400
        g = c.post("/v1/completions", json={"prompt": PROMPTS[0], "max_tokens": 5}).json()["choices"][0]["token_ids"]
        assert g == _engine().generate([PROMPTS[0]], 5)[0]
    finally:
        w.stop()


def test_static_metadata_form_samples_the_same_tokens():
    """The graph form of a decode step's metadata (bucketed block tables, padded owner
    updates, the sampler's rows) gives the same sampled tokens; on CPU it runs eagerly."""
    sp = [S.SamplingParams(temperature=0.8, top_k=40, seed=1), S.SamplingParams(temperature=1.0, top_p=0.9, seed=2),
          None]
    plain = _engine().generate(PROMPTS, 10, sp)
    eng = _engine()
    eng.use_graphs = True  # static metadata; _run_phase runs it eagerly off the GPU
    assert eng.generate(PROMPTS, 10, sp) == plain


def test_logprobs_over_vocab_shards_and_through_the_engine():
    """Token and top-k log-probabilities: equal to log_softmax on one shard, the same when
    the vocabulary is split over ranks (emulated), and attached to every output token by
    the engine, the offline API and the server."""
    g = torch.Generator().manual_seed(1)
    logits = torch.randn(5, 300, generator=g) * 2
    tok = torch.tensor([3, 299, 150, 0, 77])
    tl, ti, tv = S.logprobs(logits, 0, tok, 4)
    ref = torch.log_softmax(logits.double(), 1)
    assert torch.allclose(tl.double(), ref.gather(1, tok[:, None]).squeeze(1), atol=1e-5)
    rv, ri = ref.topk(4, dim=1)
    assert torch.equal(ti, ri) and torch.allclose(tv.double(), rv, atol=1e-5)

    class Recorder:  # rank 1: remembers the pack it would contribute to the all-gather
        world = 2

        def all_gather(self, x):
            self.pack = x
            return x

    rec = Recorder()
    S.logprobs(logits[:, 120:], 120, tok, 4, rec)

    class WithPeer:  # rank 0: its own pack, then rank 1's
        world = 2

        def all_gather(self, x):
            return torch.cat([x, rec.pack])

    sl, si, sv = S.logprobs(logits[:, :120], 0, tok, 4, WithPeer())
    assert torch.allclose(sl, tl, atol=1e-5) and torch.equal(si, ti) and torch.allclose(sv, tv, atol=1e-5)
    # engine: greedy and sampled requests, with and without MTP
    for num_spec in (0, 3):
        eng = _engine(num_spec=num_spec)
        rid = eng.add_request(PROMPTS[0], 6, logprobs=2)
        rid2 = eng.add_request(PROMPTS[1], 6, S.SamplingParams(temperature=0.8, seed=5), logprobs=0)
        while eng.has_work():
            eng.step()
        r, r2 = eng.requests[rid], eng.requests[rid2]
        assert len(r.lp) == len(r.output) == 6 and len(r2.lp) == 6
        for t, (lp, top) in zip(r.output, r.lp):
            assert len(top) == 2 and top[0][0] == t and abs(top[0][1] - lp) < 1e-5  # greedy: the argmax
            assert lp <= 0 and top[0][1] >= top[1][1]
        assert all(top == [] and lp <= 0 for lp, top in r2.lp)
    # the outputs do not change when logprobs are requested
    assert _engine().generate([PROMPTS[0]], 6)[0] == r.output


def test_logprobs_in_the_api_and_server():
    import oscar_b200
    from fastapi.testclient import TestClient

    from oscar_b200.serve.server import create_app
    from oscar_b200.serve.worker import EngineWorker

    llm = oscar_b200.LLM("qwen35-tiny", device="cpu", num_blocks=64, max_num_seqs=4, max_batched_tokens=512)
    o = llm.generate([PROMPTS[2]], S.SamplingParams(max_tokens=4, logprobs=3))[0].outputs[0]
    assert len(o.logprobs) == 4 and all(t in d and len(d) >= 3 for t, d in zip(o.token_ids, o.logprobs))
    eng = _engine()
    w = EngineWorker(eng).start()
    try:
        c = TestClient(create_app(w, vocab_size=eng.model.cfg.vocab_size))
        got = c.post("/v1/completions", json={"prompt": PROMPTS[0], "max_tokens": 5, "logprobs": 2}).json()
        lp = got["choices"][0]["logprobs"]
        assert len(lp["token_logprobs"]) == 5 and all(len(d) >= 1 for d in lp["top_logprobs"])
        assert c.post("/v1/completions", json={"prompt": PROMPTS[0], "max_tokens": 5, "logprobs": 50}).status_code == 400
    finally:
        w.stop()


def test_chat_logprobs():
    from fastapi.testclient import TestClient

    from oscar_b200.serve.server import create_app
    from oscar_b200.serve.worker import EngineWorker

    eng = _engine()
    w = EngineWorker(eng).start()
    try:
        c = TestClient(create_app(w, vocab_size=eng.model.cfg.vocab_size))
        body = {"messages": [{"role": "user", "content": "hi"}], "max_tokens": 4, "logprobs": True, "top_logprobs": 2}
        got = c.post("/v1/chat/completions", json=body).json()["choices"][0]
        content = got["logprobs"]["content"]
        assert len(content) == 4 and all(len(x["top_logprobs"]) == 2 and x["logprob"] <= 0 for x in content)
        plain = c.post("/v1/chat/completions", json={**body, "logprobs": False}).json()["choices"][0]
        assert "logprobs" not in plain and plain["message"] == got["message"]
    finally:
        w.stop()


def test_streamed_logprobs_match_the_plain_response():
    import json as _json

    from fastapi.testclient import TestClient

    from oscar_b200.serve.server import create_app
    from oscar_b200.serve.worker import EngineWorker

    def sse(resp):
        ev = [ln[6:] for ln in resp.iter_lines() if ln.startswith("data: ")]
        assert ev[-1] == "[DONE]"
        return [_json.loads(e) for e in ev[:-1]]

    eng = _engine()
    w = EngineWorker(eng).start()
    try:
        c = TestClient(create_app(w, vocab_size=eng.model.cfg.vocab_size))
        body = {"prompt": PROMPTS[1], "max_tokens": 7, "logprobs": 2}
        plain = c.post("/v1/completions", json=body).json()["choices"][0]["logprobs"]
        with c.stream("POST", "/v1/completions", json={**body, "stream": True}) as r:
            chunks = sse(r)
        got = sum((ch["choices"][0]["logprobs"]["token_logprobs"] for ch in chunks), [])
        assert got == plain["token_logprobs"] and len(got) == 7
        cb = {"messages": [{"role": "user", "content": "hi"}], "max_tokens": 5, "logprobs": True,
              "top_logprobs": 1, "stream": True}
        with c.stream("POST", "/v1/chat/completions", json=cb) as r:
            chunks = sse(r)
        content = sum((ch["choices"][0]["logprobs"]["content"] for ch in chunks), [])
        assert len(content) == 5 and all(len(x["top_logprobs"]) == 1 for x in content)
    finally:
        w.stop()


def test_n_choices():
    from fastapi.testclient import TestClient

    from oscar_b200.serve.server import create_app
    from oscar_b200.serve.worker import EngineWorker

    eng = _engine()
    w = EngineWorker(eng).start()
    try:
        c = TestClient(create_app(w, vocab_size=eng.model.cfg.vocab_size))
        body = {"prompt": PROMPTS[2], "max_tokens": 5, "temperature": 1.0, "seed": 40, "n": 3}
        got = c.post("/v1/completions", json=body).json()
        toks = [ch["token_ids"] for ch in got["choices"]]
        assert [ch["index"] for ch in got["choices"]] == [0, 1, 2] and got["usage"]["completion_tokens"] == 15
        one = c.post("/v1/completions", json={**body, "n": 1, "seed": 41}).json()["choices"][0]["token_ids"]
        assert toks[1] == one and len({tuple(t) for t in toks}) > 1  # choice i is seed + i
        chat = c.post("/v1/chat/completions", json={"messages": [{"role": "user", "content": "x"}], "max_tokens": 3,
                                                    "n": 2}).json()
        assert len(chat["choices"]) == 2
        assert c.post("/v1/completions", json={**body, "stream": True}).status_code == 400
    finally:
        w.stop()
