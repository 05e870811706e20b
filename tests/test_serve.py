"""Serving front end on CPU: HTTP completions through the engine worker, READY
validation from a log, and tensor-parallel lockstep of the worker and its followers
(gloo ranks)."""
import os
import socket

import pytest
import torch.multiprocessing as mp
from fastapi.testclient import TestClient

from oscar_b200.engine import budget as B
from oscar_b200.engine.engine import LLMEngine
from oscar_b200.models.config import tiny
from oscar_b200.models.qwen35 import HybridModel
from oscar_b200.serve.check_ready import main as check_ready_main
from oscar_b200.serve.server import ByteTokenizer, create_app
from oscar_b200.serve.worker import EngineWorker


def _engine(seed=4, tp=None):
    m = HybridModel(tiny(num_layers=4), tp=tp, device="cpu", seed=seed)
    return LLMEngine(m, num_blocks=64, max_slots=4, max_batched_tokens=256)


def test_http_completions_match_engine():
    direct = _engine().generate([list(range(5, 80)), list(range(30, 60))], 5)
    eng = _engine()
    w = EngineWorker(eng).start()
    try:
        app = create_app(w, manifests=[{"rank": 0}], vocab_size=eng.model.cfg.vocab_size)
        with TestClient(app) as c:
            r1 = c.post("/v1/completions", json={"prompt": list(range(5, 80)), "max_tokens": 5}).json()
            r2 = c.post("/v1/completions", json={"prompt": list(range(30, 60)), "max_tokens": 5}).json()
            assert r1["choices"][0]["token_ids"] == direct[0]
            assert r2["choices"][0]["token_ids"] == direct[1]
            assert r1["usage"]["completion_tokens"] == 5
            t = c.post("/v1/completions", json={"prompt": "hello", "max_tokens": 3}).json()
            assert len(t["choices"][0]["token_ids"]) == 3
            assert c.post("/v1/completions", json={"prompt": [5000], "max_tokens": 3}).status_code == 400
            assert c.get("/health").json() == {"ok": True}
            assert "oscar_finished 3.0" in c.get("/metrics").text
            assert c.get("/ready").json()["manifests"] == [{"rank": 0}]
        assert not eng.requests  # finished requests were released
    finally:
        w.stop()


def test_byte_tokenizer_roundtrip():
    t = ByteTokenizer()
    assert t.decode(t.encode("héllo")) == "héllo"


def test_check_ready_cli(tmp_path, capsys):
    m = HybridModel(tiny(num_layers=4), device="cpu")
    m.allocate_cache(8, 2)
    log = tmp_path / "serve.log"
    log.write_text("boot\n" + B.ready_manifest(m, 0, 1, sha256="aa" * 32).line() + "\n")
    assert check_ready_main([str(log), "--world", "1"]) == 0
    assert check_ready_main([str(log), "--world", "2"]) == 1
    assert check_ready_main([str(log), "--sha256", "bb" * 32]) == 1


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _lockstep(rank, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE="2",
                      LOCAL_RANK=str(rank))
    import torch.distributed as dist
    from oscar_b200.parallel.groups import init_distributed, make_groups
    from oscar_b200.serve.worker import ControlChannel, follower_loop
    init_distributed("gloo", timeout_s=120)
    try:
        tp = make_groups(2)
        eng = _engine(tp=tp)
        ctl = ControlChannel.create([0, 1])
        if rank == 0:
            w = EngineWorker(eng, ctl, heartbeat_s=0.2).start()
            outs = [f.result(timeout=240) for f in [w.submit(list(range(5, 90)), 4), w.submit(list(range(9, 33)), 6)]]
            w.stop()
            q.put((0, outs, eng.stats["steps"]))
        else:
            follower_loop(eng, ctl)
            q.put((1, None, eng.stats["steps"]))
    finally:
        dist.destroy_process_group()


def test_tp_lockstep_worker():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_lockstep, args=(r, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = {r: (o, s) for r, o, s in (q.get(timeout=300) for _ in ps)}
    for p in ps:
        p.join(60)
    outs, steps0 = res[0]
    assert [len(o) for o in outs] == [4, 6]
    assert res[1][1] == steps0  # the follower ran exactly the same steps


def test_dp_router_policy_and_proxy():
    import httpx

    from oscar_b200.serve.router import DPRouter, create_router_app

    r = DPRouter(2)
    a = r.acquire(100)
    b = r.acquire(10)
    c = r.acquire(10)
    assert (a, b, c) == (0, 1, 1)
    r.release(0, 100)
    assert r.acquire(5) == 0

    seen = []

    def handler(request: httpx.Request):
        seen.append(str(request.url))
        return httpx.Response(200, json={"choices": [{"token_ids": [1, 2]}]})

    app = create_router_app(["http://r0", "http://r1"], transport=httpx.MockTransport(handler))
    with TestClient(app) as cl:
        out = [cl.post("/v1/completions", json={"prompt": [1] * 10, "max_tokens": 2}).json() for _ in range(3)]
        assert [o["replica"] for o in out] == [0, 0, 0]  # each finished before the next: least loaded = 0
        assert cl.get("/health").json()["sent"] == [3, 0]
    assert seen[0] == "http://r0/v1/completions"
