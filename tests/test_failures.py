"""Failure detection, injected on the host (no GPU fault): a missing extension fails
loudly, a dead tensor-parallel peer ends the survivor's collective with an error
within the process-group timeout instead of hanging it, and the serving worker turns
that error into failed requests."""
import os
import socket
import time

import pytest
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
