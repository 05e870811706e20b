"""Multi-GPU tensor parallelism on NCCL (2 ranks as child processes).

The fused row-parallel GEMM + NVLS all-reduce must give the same tokens as the
GEMM + NCCL all-reduce baseline, and the ranks must agree with each other.  NVLS is
a property of the machine: when the group has no multicast support the fused run
falls back to NCCL and the test still checks rank agreement.
"""
import os
import socket
import subprocess
import sys
import textwrap

import pytest

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]

WORKER = textwrap.dedent('''
    import json, os, sys, torch
    import torch.distributed as dist
    from oscar_b200.engine.engine import LLMEngine
    from oscar_b200.models.config import tiny
    from oscar_b200.models.qwen35 import HybridModel
    from oscar_b200.parallel.groups import init_distributed, make_groups
    rank, world, local = init_distributed("nccl", timeout_s=120)
    tp = make_groups(world)
    res = {}
    for mode in ("0", "1"):
        os.environ["OSCAR_FUSED_AR"] = mode if mode == "0" else "auto"
        model = HybridModel(tiny(num_layers=4), tp=tp, device=torch.device("cuda", local), seed=5)
        eng = LLMEngine(model, num_blocks=64, max_slots=4, max_batched_tokens=512, num_spec=3)
        out = eng.generate([list(range(5, 300)), list(range(40, 170)), list(range(7, 520, 3))], 10)
        res[mode] = {"out": out, "fused": bool(getattr(model.row_reduce, "fused", False))}
        eng.close()
        torch.cuda.synchronize()
    if rank == 0:
        print("RESULT " + json.dumps(res), flush=True)
    dist.barrier()
    dist.destroy_process_group()
''')


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_tp2_fused_allreduce_matches_nccl(tmp_path):
    script = tmp_path / "worker.py"
    script.write_text(WORKER)
    env = dict(os.environ, NCCL_NVLS_ENABLE=os.environ.get("NCCL_NVLS_ENABLE", "1"),
               PYTHONPATH=os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    cmd = ["timeout", "-k", "30", "400", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node", "2", "--master-addr", "127.0.0.1", "--master-port", str(_port()), str(script)]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=460)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    line = [x for x in r.stdout.splitlines() if x.startswith("RESULT ")][-1]
    import json
    res = json.loads(line[len("RESULT "):])
    assert res["0"]["out"] == res["1"]["out"], res
    print("fused path active:", res["1"]["fused"])
