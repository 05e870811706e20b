"""GDN layer-core microbench on the target model's shapes (one TP rank).

Times ``gdn_step`` (conv1d + delta rule + gated RMSNorm) with CUDA events, median of
``--iters`` after warm-up, for a prefill step of ``--tokens`` tokens split into
``--requests`` equal requests, with the chunked tensor-core path (default) and, with
``--compare``, the per-token chunk kernel (``OSCAR_GDN_CHUNKED=0`` in a child process).
Reported: microseconds per call and new tokens per second.

    python -m oscar_b200.bench.gdn [--tp 1] [--tokens 15360] [--requests 1,32] [--compare]
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys

import torch

from ..ops.gdn import gdn_step
from .harness import time_call


def run(tp: int, tokens: int, requests: int, iters: int) -> dict:
    Hk, Hv, dk, dv = 16 // tp, 48 // tp, 128, 128
    r = Hv // Hk
    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(0)
    n_qkvz = Hk * (2 * dk + 2 * r * dv)
    proj = torch.randn(tokens, n_qkvz + 2 * Hv, device=dev, generator=g).to(torch.bfloat16)
    qkvz, ba = proj[:, :n_qkvz], proj[:, n_qkvz:]
    conv_dim = 2 * Hk * dk + Hv * dv
    slots, P = requests, 4
    st = (torch.randn(slots, Hv, dk, dv, device=dev, generator=g) * 0.1).to(torch.bfloat16)
    cs = torch.zeros(2, slots, conv_dim, 3, dtype=torch.bfloat16, device=dev)
    px = torch.zeros(2, slots, P, conv_dim, dtype=torch.bfloat16, device=dev)
    pb = torch.zeros(slots, P, 2 * Hv, dtype=torch.bfloat16, device=dev)
    per = tokens // requests
    q_start = torch.arange(0, requests + 1, device=dev, dtype=torch.int32) * per
    zeros = torch.zeros(requests, dtype=torch.int32, device=dev)
    w = dict(conv_w=torch.randn(conv_dim, 4, device=dev, generator=g) * 0.5,
             A_log=torch.log(torch.rand(Hv, device=dev, generator=g) * 15 + 1), dt_bias=torch.ones(Hv, device=dev),
             norm_w=torch.ones(dv, device=dev))
    out = torch.empty(per * requests, Hv * dv, dtype=torch.bfloat16, device=dev)

    def call():
        gdn_step(qkvz[:per * requests], ba[:per * requests], Hk=Hk, Hv=Hv, dk=dk, dv=dv, eps=1e-6, state=st,
                 conv_state=cs, pend_x=px, pend_ba=pb, parity=zeros, req_slot=torch.arange(requests, device=dev,
                 dtype=torch.int32), q_start=q_start, n_commit=zeros, keep_pending=zeros, out=out, smem_state=True,
                 **w)

    for _ in range(2):
        call()
    t = sorted(time_call(call) for _ in range(iters))[iters // 2]
    return {"tp": tp, "tokens": per * requests, "requests": requests, "us": round(t * 1e3, 1),
            "tok_per_s": round(per * requests / (t * 1e-3), 1),
            "path": "per-token" if os.environ.get("OSCAR_GDN_CHUNKED") == "0" else "chunked"}


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--tp", type=int, default=1)
    ap.add_argument("--tokens", type=int, default=15360)
    ap.add_argument("--requests", default="1,32")
    ap.add_argument("--iters", type=int, default=5)
    ap.add_argument("--compare", action="store_true")
    args = ap.parse_args(argv)
    for R in map(int, args.requests.split(",")):
        print(json.dumps(run(args.tp, args.tokens, R, args.iters)), flush=True)
    if args.compare and os.environ.get("OSCAR_GDN_CHUNKED") != "0":
        env = dict(os.environ, OSCAR_GDN_CHUNKED="0")
        subprocess.run([sys.executable, "-m", "oscar_b200.bench.gdn", "--tp", str(args.tp), "--tokens",
                        str(args.tokens), "--requests", args.requests, "--iters", str(max(2, args.iters // 2))],
                       env=env, check=True)


if __name__ == "__main__":
    main()
