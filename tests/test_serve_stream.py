"""Stop conditions, aborts and streaming (CPU): stop token ids end a request (also in
the middle of an accepted MTP draft run), an abort frees a request's blocks between
steps on every rank, the worker reports tokens step by step, and the HTTP server
streams server-sent events, cuts stop strings and honours EOS / ``ignore_eos``."""
from __future__ import annotations

import json
import os
import socket

import pytest
import torch.multiprocessing as mp

from oscar_b200.engine.engine import LLMEngine
from oscar_b200.models.config import tiny
from oscar_b200.models.qwen35 import HybridModel
from oscar_b200.serve.worker import EngineWorker

PROMPTS = [[1, 2, 3, 4, 5] * 12, [7, 8, 9] * 10, list(range(11, 60))]


def _engine(num_spec=3, tp=None):
    m = HybridModel(tiny(num_layers=4), tp=tp, device="cpu", seed=1)
    return LLMEngine(m, num_blocks=64, max_slots=4, max_batched_tokens=512, num_spec=num_spec)


@pytest.mark.parametrize("num_spec", [0, 3])
def test_stop_token_ends_the_request(num_spec):
    full = _engine(num_spec).generate(PROMPTS, 12)
    eng = _engine(num_spec)
    stop = {full[0][4], full[1][2]}
    rids = [eng.add_request(p, 12, stop_ids=stop) for p in PROMPTS]
    while eng.has_work():
        eng.step()
    for rid, want in zip(rids, full):
        r = eng.requests[rid]
        cut = next((i for i, t in enumerate(want) if t in stop), None)
        if cut is None:
            assert r.output == want and r.finish_reason == "length"
        else:
            assert r.output == want[:cut + 1] and r.finish_reason == "stop"
    assert eng.bm.free_blocks == 64


def test_abort_frees_blocks_and_leaves_the_others_unchanged():
    want = _engine().generate(PROMPTS, 10)
    eng = _engine()
    rids = [eng.add_request(p, 10) for p in PROMPTS]
    for _ in range(3):
        eng.step()
    eng.abort(rids[1])
    r = eng.requests[rids[1]]
    assert r.finished and r.finish_reason == "abort" and r.output == want[1][:len(r.output)]
    while eng.has_work():
        eng.step()
    assert [eng.requests[i].output for i in (rids[0], rids[2])] == [want[0], want[2]]
    assert eng.bm.free_blocks == 64 and eng.slots.free_slots == 4
    eng.abort(rids[0])  # finished: no effect
    assert eng.requests[rids[0]].finish_reason == "length"


def test_worker_streams_tokens_and_aborts():
    want = _engine().generate(PROMPTS[:1], 8)[0]
    w = EngineWorker(_engine()).start()
    try:
        seen = []
        fut = w.submit(PROMPTS[0], 8, on_tokens=lambda new, reason: seen.append((list(new), reason)))
        assert fut.result(timeout=120) == want
        assert fut.finish_reason == "length"
        assert sum((n for n, _ in seen), []) == want
        assert [r for _, r in seen][-1] == "length" and all(r is None for _, r in seen[:-1])
        hits = []

        def stop_early(new, reason):
            hits.append(len(new))
            if len(hits) == 1:
                w.abort(f2)

        f2 = w.submit(PROMPTS[1], 400, on_tokens=stop_early)
        out = f2.result(timeout=120)
        assert f2.finish_reason == "abort" and 0 < len(out) < 400
    finally:
        w.stop()


class _SpaceTokenizer:
    """Token ids as space-separated numbers: stop strings are easy to place."""

    eos_token_id = None

    def encode(self, text):
        return [int(x) for x in text.split()]

    def decode(self, ids, skip_special_tokens=True):
        return "".join(f" {i}" for i in ids)


def _client(eos=None, tokenizer=None):
    from fastapi.testclient import TestClient

    from oscar_b200.serve.server import create_app

    eng = _engine()
    w = EngineWorker(eng).start()
    app = create_app(w, tokenizer, vocab_size=eng.model.cfg.vocab_size, eos_token_ids=eos, max_model_len=8192)
    return TestClient(app), w


def _sse(resp):
    events = [ln[len("data: "):] for ln in resp.iter_lines() if ln.startswith("data: ")]
    assert events[-1] == "[DONE]"
    return [json.loads(e) for e in events[:-1]]


def test_http_streaming_matches_the_plain_response():
    c, w = _client()
    try:
        body = {"prompt": PROMPTS[2], "max_tokens": 9}
        plain = c.post("/v1/completions", json=body).json()["choices"][0]
        with c.stream("POST", "/v1/completions", json={**body, "stream": True}) as resp:
            chunks = _sse(resp)
        ids = sum((ch["choices"][0]["token_ids"] for ch in chunks), [])
        assert ids == plain["token_ids"]
        assert "".join(ch["choices"][0]["text"] for ch in chunks) == plain["text"]
        assert chunks[-1]["choices"][0]["finish_reason"] == "length" == plain["finish_reason"]
        assert all(ch["choices"][0]["finish_reason"] is None for ch in chunks[:-1])
        assert c.get("/v1/models").json()["data"][0]["max_model_len"] == 8192
    finally:
        w.stop()


def test_http_stop_strings_stop_ids_and_eos():
    c, w = _client(tokenizer=_SpaceTokenizer())
    try:
        prompt = " ".join(map(str, PROMPTS[2]))
        full = c.post("/v1/completions", json={"prompt": prompt, "max_tokens": 10}).json()["choices"][0]
        ids = full["token_ids"]
        stop = f" {ids[3]}"
        for stream in (False, True):
            body = {"prompt": prompt, "max_tokens": 10, "stop": [stop, " never"], "stream": stream}
            if stream:
                with c.stream("POST", "/v1/completions", json=body) as resp:
                    chunks = _sse(resp)
                text = "".join(ch["choices"][0]["text"] for ch in chunks)
                reason = chunks[-1]["choices"][0]["finish_reason"]
            else:
                got = c.post("/v1/completions", json=body).json()["choices"][0]
                text, reason = got["text"], got["finish_reason"]
            assert text == full["text"][:full["text"].find(stop)] and reason == "stop"
        got = c.post("/v1/completions", json={"prompt": prompt, "max_tokens": 10,
                                              "stop_token_ids": [ids[5]]}).json()["choices"][0]
        assert got["token_ids"] == ids[:ids.index(ids[5]) + 1] and got["finish_reason"] == "stop"
    finally:
        w.stop()
    c, w = _client(eos=[ids[2]], tokenizer=_SpaceTokenizer())
    try:
        got = c.post("/v1/completions", json={"prompt": prompt, "max_tokens": 10}).json()["choices"][0]
        assert got["token_ids"] == ids[:ids.index(ids[2]) + 1] and got["finish_reason"] == "stop"
        got = c.post("/v1/completions", json={"prompt": prompt, "max_tokens": 10,
                                              "ignore_eos": True}).json()["choices"][0]
        assert got["token_ids"] == ids and got["finish_reason"] == "length"
    finally:
        w.stop()


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _lockstep_abort(rank, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE="2",
                      LOCAL_RANK=str(rank))
    import torch.distributed as dist
    from oscar_b200.parallel.groups import init_distributed, make_groups
    from oscar_b200.serve.worker import ControlChannel, follower_loop
    init_distributed("gloo", timeout_s=120)
    try:
        eng = _engine(tp=make_groups(2))
        ctl = ControlChannel.create([0, 1])
        if rank == 0:
            w = EngineWorker(eng, ctl, heartbeat_s=0.2).start()
            hits = []

            def stop_early(new, reason):
                hits.append(len(new))
                if len(hits) == 2:
                    w.abort(f2)

            f1 = w.submit(PROMPTS[0], 6)
            f2 = w.submit(PROMPTS[1], 300, on_tokens=stop_early)
            outs = [f1.result(timeout=240), f2.result(timeout=240)]
            w.stop()
            q.put((0, [len(o) for o in outs], f2.finish_reason, eng.stats["steps"], eng.bm.free_blocks))
        else:
            follower_loop(eng, ctl)
            q.put((1, None, None, eng.stats["steps"], eng.bm.free_blocks))
    finally:
        dist.destroy_process_group()


def test_abort_reaches_every_rank():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_lockstep_abort, args=(r, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = {r[0]: r[1:] for r in (q.get(timeout=300) for _ in ps)}
    for p in ps:
        p.join(60)
    lens, reason, steps0, free0 = res[0]
    assert lens[0] == 6 and 0 < lens[1] < 300 and reason == "abort"
    assert res[1][2] == steps0 and res[1][3] == free0 == 64


class _TemplateTokenizer(_SpaceTokenizer):
    """A tokenizer with a chat template that returns a BatchEncoding-like dict."""

    def apply_chat_template(self, messages, add_generation_prompt=True, tokenize=True):
        ids = [len(m["content"]) + 3 for m in messages] + ([9] if add_generation_prompt else [])
        return {"input_ids": ids}


def test_chat_completions():
    from oscar_b200.serve.server import chat_prompt

    msgs = [{"role": "system", "content": "be brief"}, {"role": "user", "content": "hi"}]
    assert chat_prompt(_TemplateTokenizer(), msgs) == [11, 5, 9]
    c, w = _client()
    try:
        body = {"messages": msgs, "max_tokens": 6}
        got = c.post("/v1/chat/completions", json=body).json()
        assert got["object"] == "chat.completion" and got["choices"][0]["message"]["role"] == "assistant"
        assert got["usage"]["completion_tokens"] == 6 and got["choices"][0]["finish_reason"] == "length"
        # the fallback template, tokenised as text, is the prompt of a plain completion
        from oscar_b200.serve.server import ByteTokenizer
        plain = c.post("/v1/completions", json={"prompt": chat_prompt(ByteTokenizer(), msgs),
                                                "max_tokens": 6}).json()["choices"][0]
        assert got["choices"][0]["message"]["content"] == plain["text"]
        with c.stream("POST", "/v1/chat/completions", json={**body, "stream": True}) as resp:
            chunks = _sse(resp)
        assert all(ch["object"] == "chat.completion.chunk" for ch in chunks)
        assert chunks[0]["choices"][0]["delta"]["role"] == "assistant"
        assert "".join(ch["choices"][0]["delta"]["content"] for ch in chunks) == plain["text"]
    finally:
        w.stop()


def test_router_streams_through():
    import httpx
    from fastapi.testclient import TestClient

    from oscar_b200.serve.router import create_router_app

    sse = b'data: {"choices": [{"text": "a"}]}\n\ndata: {"choices": [{"text": "b"}]}\n\ndata: [DONE]\n\n'
    seen = []

    def handler(request: httpx.Request):
        if request.url.path == "/v1/models":
            return httpx.Response(200, json={"object": "list", "data": [{"id": "m"}]})
        seen.append((str(request.url), json.loads(request.content)))
        return httpx.Response(200, content=sse, headers={"content-type": "text/event-stream"})

    app = create_router_app(["http://r0", "http://r1"], transport=httpx.MockTransport(handler))
    with TestClient(app) as cl:
        with cl.stream("POST", "/v1/chat/completions",
                       json={"messages": [{"role": "user", "content": "x"}], "stream": True}) as resp:
            body = b"".join(resp.iter_bytes())
            assert resp.headers["x-replica"] == "0"
        assert body == sse
        assert cl.get("/health").json()["load"] == [0, 0]  # released when the stream ended
        assert cl.get("/v1/models").json()["data"][0]["id"] == "m"
    assert seen[0][0] == "http://r0/v1/chat/completions" and seen[0][1]["stream"] is True


def test_serving_benchmark_client_against_a_live_server():
    """The serving benchmark client drives a real uvicorn server on localhost."""
    import asyncio
    import threading
    import time

    import uvicorn

    from oscar_b200.bench import serve_client as SC
    from oscar_b200.serve.server import create_app

    eng = _engine()
    w = EngineWorker(eng).start()
    port = _port()
    server = uvicorn.Server(uvicorn.Config(create_app(w, vocab_size=eng.model.cfg.vocab_size), host="127.0.0.1",
                                           port=port, log_level="warning"))
    th = threading.Thread(target=server.run, daemon=True)
    th.start()
    try:
        t0 = time.time()
        while not server.started and time.time() - t0 < 30:
            time.sleep(0.05)
        prompts = SC.make_prompts(5, 40, 1024, seed=1)
        out = asyncio.run(SC.run(f"http://127.0.0.1:{port}", prompts, output_len=7, concurrency=3))
        assert out["completed"] == 5 and out["failed"] == 0 and out["output_tokens"] == 35
        assert out["ttft_ms"]["mean"] > 0 and out["tpot_ms"]["mean"] > 0 and out["output_tok_per_s"] > 0
        assert out["itl_ms"]["p99"] is not None
    finally:
        server.should_exit = True
        th.join(30)
        w.stop()


def test_requests_the_engine_cannot_run_are_rejected_up_front():
    """Too long for the RoPE tables or the KV pool, out-of-vocabulary ids, empty prompts:
    rejected when submitted (HTTP 400), and the engine thread keeps serving."""
    eng = _engine()
    cap = eng.max_request_tokens()
    assert cap == min(eng.model.cfg.max_position, 64 * 128) - 8
    for prompt, n in (([1] * (cap - 3), 4), ([], 3), ([1, 2, 5000], 3), ([1, 2], 0), ([-1, 2], 3)):
        with pytest.raises(ValueError):
            eng.add_request(prompt, n)
    eng.add_request([1] * (cap - 4), 4)  # exactly at the limit
    c, w = _client()
    try:
        r = c.post("/v1/completions", json={"prompt": [1] * cap, "max_tokens": 4})
        assert r.status_code == 400 and "exceeds" in r.json()["detail"]
        ok = c.post("/v1/completions", json={"prompt": PROMPTS[0], "max_tokens": 3})
        assert ok.status_code == 200 and len(ok.json()["choices"][0]["token_ids"]) == 3
        assert w.error is None
    finally:
        w.stop()


def test_metrics_histograms_and_finish_reasons():
    from oscar_b200.serve.worker import Histogram

    h = Histogram((0.1, 1.0))
    for v in (0.05, 0.5, 0.7, 3.0):
        h.observe(v)
    assert h.lines("x")[1:4] == ['x_bucket{le="0.1"} 1', 'x_bucket{le="1.0"} 3', 'x_bucket{le="+Inf"} 4']
    assert h.count == 4 and abs(h.sum - 4.25) < 1e-12
    c, w = _client()
    try:
        c.post("/v1/completions", json={"prompt": PROMPTS[0], "max_tokens": 4})
        c.post("/v1/completions", json={"prompt": PROMPTS[1], "max_tokens": 4, "stop_token_ids": list(range(1024))})
        text = c.get("/metrics").text
        assert 'oscar_finish_reason_total{reason="length"} 1' in text
        assert 'oscar_finish_reason_total{reason="stop"} 1' in text
        assert 'oscar_ttft_seconds_bucket{le="+Inf"} 2' in text and "oscar_tpot_seconds_count 1" in text
        assert "oscar_finished 2.0" in text
        verify = [ln for ln in text.splitlines() if ln.startswith("oscar_verify_steps_total")]
        assert verify and all(0 <= int(ln.split('"')[1]) <= 3 for ln in verify)
    finally:
        w.stop()


def test_longbench_style_eval_client(tmp_path):
    """Prompt template, middle truncation, answer extraction and scoring against a mock
    server; then the whole path against the real app (random weights: only completion is
    checked)."""
    import asyncio

    import httpx

    from oscar_b200.bench import longbench as LB

    assert LB.extract("The correct answer is (C).") == "C"
    assert LB.extract("Hmm... B or maybe D") == "D" and LB.extract("no idea") is None
    assert LB.middle_truncate("abcdefghij", 4) == "abij"
    recs = [{"_id": str(i), "context": "x" * 50, "question": f"q{i}", "choice_A": "a", "choice_B": "b",
             "choice_C": "c", "choice_D": "d", "answer": "ABCD"[i % 4], "difficulty": ["easy", "hard"][i % 2]}
            for i in range(8)]
    data = tmp_path / "lb.jsonl"
    data.write_text("\n".join(json.dumps(r) for r in recs))
    assert LB.load(str(data), limit=5) == recs[:5]
    prompt = LB.prompt_of(recs[1], max_chars=10)
    assert "x" * 10 in prompt and "x" * 11 not in prompt and "(B) b" in prompt

    def handler(request: httpx.Request):
        body = json.loads(request.content)
        q = body["messages"][0]["content"].split("question: ")[1].split("\n")[0]
        i = int(q[1:])
        if i == 7:
            return httpx.Response(500, text="boom")
        guess = "ABCD"[i % 4] if i < 4 else "A"  # right on 0-3 and on 4; wrong on 5, 6; 7 fails
        return httpx.Response(200, json={"choices": [{"message": {"content": f"The correct answer is ({guess})"}}],
                                         "usage": {"completion_tokens": 6}})

    out = asyncio.run(LB.run("http://mock", recs, concurrency=3, transport=httpx.MockTransport(handler)))
    assert out["cases"] == 8 and out["failed"] == 1 and out["accuracy"] == 5 / 8
    assert out["accuracy_by"] == {"difficulty=easy": 3 / 4, "difficulty=hard": 2 / 4}
    # the real server end to end
    from oscar_b200.serve.server import create_app

    eng = _engine()
    w = EngineWorker(eng).start()
    try:
        app = create_app(w, vocab_size=eng.model.cfg.vocab_size)
        out = asyncio.run(LB.run("http://app", recs[:3], concurrency=2, max_tokens=4,
                                 transport=httpx.ASGITransport(app=app)))
        assert out["completed"] == 3 and out["completion_tokens"] == 12
    finally:
        w.stop()


def test_launcher_gates_and_ready_check(tmp_path, monkeypatch):
    """The one-shot launcher on CPU: self-check, fingerprint, a v2 rotation checkpoint
    reused, the serve process up, every READY manifest validated, /health answered."""
    import subprocess
    import sys

    from oscar_b200.kv.gen_rotations import main as gen_main

    rot = tmp_path / "rot.pt"
    monkeypatch.setenv("OSCAR_ASCEND_CALIB_TOKEN_CAP", "64")
    assert gen_main(["--out", str(rot), "--model", "qwen35-tiny", "--layers", "4", "--num-prompts", "1",
                     "--prompt-len", "64", "--device", "cpu"]) == 0
    logf = tmp_path / "serve.log"
    cmd = [sys.executable, "-m", "oscar_b200.serve.launch", "--device", "cpu", "--model", "qwen35-tiny",
           "--rotations", str(rot), "--skip-probes", "--port", str(_port()), "--log", str(logf),
           "--ready-timeout", "240", "--exit-after-ready", "--num-blocks", "16", "--max-num-seqs", "2",
           "--max-batched-tokens", "256"]
    p = subprocess.run(cmd, capture_output=True, text=True, timeout=400)
    assert p.returncode == 0, p.stdout[-3000:] + p.stderr[-3000:]
    assert "reusing v2 checkpoint" in p.stdout and "LAUNCH OK: 1 rank(s)" in p.stdout
    assert "READY" in logf.read_text()
    # a checkpoint that is not v2, without calibration: random rotations, still ready
    bad = tmp_path / "old.pt"
    import torch
    torch.save({"3": torch.eye(256)}, bad)
    cmd[cmd.index(str(rot))] = str(bad)
    p = subprocess.run(cmd + ["--no-calibrate"], capture_output=True, text=True, timeout=400)
    assert p.returncode == 0 and "not a v2 checkpoint" in p.stdout and "seeded random rotations" in p.stdout


def test_sampling_defaults_fill_omitted_fields(tmp_path):
    """A checkpoint's generation_config.json recommendation applies to requests that leave
    the sampling fields out; explicit fields win."""
    from fastapi.testclient import TestClient

    from oscar_b200.models.loader import generation_defaults
    from oscar_b200.serve.server import create_app

    (tmp_path / "generation_config.json").write_text(json.dumps({"temperature": 0.9, "top_k": 20, "top_p": 0.95}))
    d = generation_defaults(str(tmp_path))
    assert d == {"temperature": 0.9, "top_k": 20, "top_p": 0.95}
    (tmp_path / "generation_config.json").write_text(json.dumps({"do_sample": False, "temperature": 0.9}))
    assert generation_defaults(str(tmp_path)) == {"temperature": 0.0}
    greedy = _engine().generate([PROMPTS[2]], 6)[0]
    eng = _engine()
    w = EngineWorker(eng).start()
    try:
        c = TestClient(create_app(w, vocab_size=eng.model.cfg.vocab_size, sampling_defaults=d))
        body = {"prompt": PROMPTS[2], "max_tokens": 6, "seed": 3}
        a = c.post("/v1/completions", json=body).json()["choices"][0]["token_ids"]
        assert a == c.post("/v1/completions", json=body).json()["choices"][0]["token_ids"]  # seeded
        assert a != greedy  # sampled with the defaults
        g = c.post("/v1/completions", json={**body, "temperature": 0}).json()["choices"][0]["token_ids"]
        assert g == greedy
    finally:
        w.stop()


def test_stream_usage_chunk():
    c, w = _client()
    try:
        body = {"prompt": PROMPTS[0], "max_tokens": 6, "stream": True, "stream_options": {"include_usage": True}}
        with c.stream("POST", "/v1/completions", json=body) as resp:
            chunks = _sse(resp)
        assert chunks[-1]["choices"] == [] and chunks[-1]["usage"] == {
            "prompt_tokens": len(PROMPTS[0]), "completion_tokens": 6, "total_tokens": len(PROMPTS[0]) + 6}
        assert sum(len(ch["choices"][0]["token_ids"]) for ch in chunks[:-1]) == 6
        with c.stream("POST", "/v1/completions", json={**body, "stream_options": None}) as resp:
            assert all(ch["choices"] for ch in _sse(resp))
    finally:
        w.stop()


def test_chat_max_completion_tokens():
    c, w = _client()
    try:
        got = c.post("/v1/chat/completions", json={"messages": [{"role": "user", "content": "x"}], "max_tokens": 9,
                                                   "max_completion_tokens": 3}).json()
        assert got["usage"]["completion_tokens"] == 3
    finally:
        w.stop()


def test_failed_choice_aborts_its_siblings():
    """With ``n`` choices, a choice whose engine request fails ends the response with an
    error and aborts the other choices' requests (they would otherwise run to max_tokens)."""
    from concurrent.futures import Future

    c, w = _client()
    real_submit, real_abort = w.submit, w.abort
    subs, aborted = [], []

    def submit(*a, **k):
        if len(subs) == 1:  # the second choice fails at once
            f = Future()
            f.set_exception(RuntimeError("injected engine failure"))
            subs.append(f)
            return f
        f = real_submit(*a, **k)
        subs.append(f)
        return f

    def abort(f):
        aborted.append(f)
        return real_abort(f)

    w.submit, w.abort = submit, abort
    try:
        r = c.post("/v1/completions", json={"prompt": PROMPTS[0], "max_tokens": 400, "n": 3, "seed": 1,
                                            "temperature": 0.8})
        assert r.status_code == 500
        others = [f for i, f in enumerate(subs) if i != 1]
        assert len(others) == 2 and all(f in aborted for f in others)
    finally:
        w.submit, w.abort = real_submit, real_abort
        w.stop()
