"""Failure detection, injected on the host (no GPU fault): a missing extension fails
loudly, a dead tensor-parallel peer ends the survivor's collective with an error
within the process-group timeout instead of hanging it, the serving worker turns
that error into failed requests, an allocator out-of-memory error inside a step fails
the pending requests and the health check, and a kernel status code ends the step with
an error naming it."""
import os
import socket
import time

import pytest
import torch
import torch.multiprocessing as mp

from oscar_b200.ops import _ext


def test_missing_extension_fails_loudly(monkeypatch):
    monkeypatch.setattr(_ext, "_EXT", None)
    monkeypatch.setattr(_ext, "_ERR", None)

    def boom(name):
        raise ImportError("simulated: no such .so")

    monkeypatch.setattr(_ext.importlib, "import_module", boom)
    with pytest.raises(RuntimeError, match="not built"):
        _ext.ext()
    assert not _ext.available()


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, port, q, mode):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE="2",
                      LOCAL_RANK=str(rank))
    import torch
    import torch.distributed as dist
    from oscar_b200.parallel.groups import init_distributed
    init_distributed("gloo", timeout_s=6)
    if rank == 1:
        os._exit(0)  # the peer dies between steps, with nothing in flight
    t0 = time.time()
    try:
        if mode == "collective":
            dist.all_reduce(torch.ones(4))
            q.put(("no error", time.time() - t0))
        else:
            from oscar_b200.engine.engine import LLMEngine
            from oscar_b200.models.config import tiny
            from oscar_b200.models.qwen35 import HybridModel
            from oscar_b200.serve.worker import ControlChannel, EngineWorker
            eng = LLMEngine(HybridModel(tiny(num_layers=4), device="cpu"), num_blocks=16, max_slots=2,
                            max_batched_tokens=128)
            w = EngineWorker(eng, ControlChannel(None, 0), heartbeat_s=0.1).start()
            fut = w.submit(list(range(3, 40)), 4)
            try:
                fut.result(timeout=60)
                q.put(("no error", time.time() - t0))
            except Exception as e:  # noqa: BLE001
                q.put((type(e).__name__, time.time() - t0))
    except Exception as e:  # noqa: BLE001
        q.put((type(e).__name__, time.time() - t0))
    q.close()
    q.join_thread()  # the result must leave this process before it ends abruptly
    os._exit(0)


@pytest.mark.parametrize("mode", ["collective", "worker"])
def test_dead_peer_is_detected(mode):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_rank, args=(r, port, q, mode)) for r in range(2)]
    for p in ps:
        p.start()
    kind, dt = q.get(timeout=120)
    for p in ps:
        p.join(30)
        if p.is_alive():
            p.kill()
    assert kind != "no error", "the survivor did not notice the dead peer"
    assert dt < 60


def _engine_cpu():
    from oscar_b200.engine.engine import LLMEngine
    from oscar_b200.models.config import tiny
    from oscar_b200.models.qwen35 import HybridModel
    return LLMEngine(HybridModel(tiny(num_layers=4), device="cpu"), num_blocks=16, max_slots=2,
                     max_batched_tokens=128)


def test_allocator_oom_in_a_step_fails_requests_and_health(monkeypatch):
    """An out-of-memory error raised inside a step (host-side injection at the GEMM wrapper)
    reaches every pending request, /health turns 503, and new submissions are refused."""
    from fastapi.testclient import TestClient

    from oscar_b200.ops import functional as F
    from oscar_b200.serve.server import create_app
    from oscar_b200.serve.worker import EngineWorker

    real = F.linear_i8
    calls = {"n": 0}

    def flaky(*a, **k):
        calls["n"] += 1
        if calls["n"] == 40:
            raise torch.OutOfMemoryError("simulated: allocator out of memory")
        return real(*a, **k)

    monkeypatch.setattr(F, "linear_i8", flaky)
    w = EngineWorker(_engine_cpu()).start()
    try:
        futs = [w.submit(list(range(3, 30)), 20), w.submit(list(range(5, 50)), 20)]
        for f in futs:
            with pytest.raises(torch.OutOfMemoryError, match="simulated"):
                f.result(timeout=120)
        c = TestClient(create_app(w))
        assert c.get("/health").status_code == 503
        with pytest.raises(RuntimeError, match="engine worker failed"):
            w.submit([1, 2, 3], 2)
    finally:
        w.stop()


def test_kernel_status_word_ends_the_step_with_a_clear_error(monkeypatch):
    """A kernel that gives up a bounded wait (or finds a bad index) records a code in the
    model's status word; the engine reads it after the step and raises, naming the code."""
    from oscar_b200.ops import functional as F

    eng = _engine_cpu()
    eng.model.status = torch.zeros(1, dtype=torch.int32)
    real = F.rmsnorm_quant

    def reports(*a, **k):
        st = k.get("status")
        if st is not None:
            st.fill_(5)  # kTimeoutPeerFlag: what a timed-out peer-flag wait records
        return real(*a, **{kk: v for kk, v in k.items()})

    monkeypatch.setattr(F, "rmsnorm_quant", reports)
    eng.add_request(list(range(3, 30)), 4)
    with pytest.raises(RuntimeError, match="status 5"):
        eng.step()
