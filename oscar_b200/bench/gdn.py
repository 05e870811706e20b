"""GDN layer-core microbench on the target model's shapes (one TP rank).

Times ``gdn_step`` (conv1d + delta rule + gated RMSNorm) with CUDA events, median of
``--iters`` after warm-up, for a prefill step of ``--tokens`` tokens split into
``--requests`` equal requests, with the chunked tensor-core path (default) and, with
``--compare``, the per-token chunk kernel (``OSCAR_GDN_CHUNKED=0`` in a child process).
``--decode`` times the decode / MTP-verify step instead: every request verifies
``--qlen`` tokens after committing ``--commit`` accepted ones (the serving step).
Reported: microseconds per call, new tokens per second and, for decode, the state bytes
moved per second against the measured copy bandwidth.

    python -m oscar_b200.bench.gdn [--tp 1] [--tokens 15360] [--requests 1,32] [--compare]
    python -m oscar_b200.bench.gdn --decode [--requests 32] [--qlen 4] [--commit 3]
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys

import torch

from ..ops.gdn import gdn_step
from .harness import time_call, peak_hbm_gbs


def run(tp: int, tokens: int, requests: int, iters: int, decode: bool = False, qlen: int = 4,
        commit: int = 3, trace: bool = False) -> dict:
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
    per = qlen if decode else tokens // requests
    q_start = torch.arange(0, requests + 1, device=dev, dtype=torch.int32) * per
    zeros = torch.zeros(requests, dtype=torch.int32, device=dev)
    n_commit = torch.full((requests,), commit if decode else 0, dtype=torch.int32, device=dev)
    keep = torch.full((requests,), 1 if decode else 0, dtype=torch.int32, device=dev)
    w = dict(conv_w=torch.randn(conv_dim, 4, device=dev, generator=g) * 0.5,
             A_log=torch.log(torch.rand(Hv, device=dev, generator=g) * 15 + 1), dt_bias=torch.ones(Hv, device=dev),
             norm_w=torch.ones(dv, device=dev))
    out = torch.empty(per * requests, Hv * dv, dtype=torch.bfloat16, device=dev)

    def call():
        gdn_step(qkvz[:per * requests], ba[:per * requests], Hk=Hk, Hv=Hv, dk=dk, dv=dv, eps=1e-6, state=st,
                 conv_state=cs, pend_x=px, pend_ba=pb, parity=zeros, req_slot=torch.arange(requests, device=dev,
                 dtype=torch.int32), q_start=q_start, n_commit=n_commit, keep_pending=keep, out=out,
                 smem_state=not decode, **w)

    for _ in range(2):
        call()
    t = sorted(time_call(call) for _ in range(iters))[iters // 2]
    phases = None
    if decode and trace:
        phases = _trace(call, requests * Hv)
    res = {"tp": tp, "tokens": per * requests, "requests": requests, "us": round(t * 1e3, 1),
           "tok_per_s": round(per * requests / (t * 1e-3), 1),
           "path": "decode" if decode else ("per-token" if os.environ.get("OSCAR_GDN_CHUNKED") == "0" else "chunked")}
    if decode:  # the recurrent state is read and written once per step
        state_bytes = 2 * requests * Hv * dk * dv * 2
        res["state_gbs"] = round(state_bytes / (t * 1e-3) / 1e9, 1)
        res["frac_hbm_of_measured"] = round(res["state_gbs"] / _peak_gbs(), 3)
    if phases is not None:
        res["trace"] = phases
    return res


# phase marks of the decode kernel's timeline (slots 0-9)
PHASES = ["inputs+conv", "norm", "kk/kq", "state wait", "pass1", "solve", "out", "pass2", "store"]


def _trace(call, n_cta: int) -> dict:
    """One traced launch: kernel span, CTA durations and the median time of every phase (µs)."""
    import numpy as np
    from ..ops._ext import ext
    buf = torch.zeros(n_cta * 16, dtype=torch.int64, device="cuda")
    ext().gdn_trace(buf.data_ptr())
    try:
        call()
        torch.cuda.synchronize()
    finally:
        ext().gdn_trace(0)
    t = buf.view(n_cta, 16)[:, :10].cpu().numpy().astype(np.float64)
    t0 = t[:, 0].min()
    dur = (t[:, 9] - t[:, 0]) / 1e3
    out = {"span_us": round(float((t[:, 9].max() - t0) / 1e3), 2),
           "cta_us_min_med_max": [round(float(x), 2) for x in (dur.min(), np.median(dur), dur.max())],
           "start_us_max": round(float((t[:, 0].max() - t0) / 1e3), 2)}
    out["phase_us_median"] = {name: round(float(np.median(t[:, k + 1] - t[:, k])) / 1e3, 2)
                              for k, name in enumerate(PHASES)}
    return out


def _peak_gbs() -> float:
    return peak_hbm_gbs()


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--tp", type=int, default=1)
    ap.add_argument("--tokens", type=int, default=15360)
    ap.add_argument("--requests", default="1,32")
    ap.add_argument("--iters", type=int, default=5)
    ap.add_argument("--compare", action="store_true")
    ap.add_argument("--decode", action="store_true")
    ap.add_argument("--qlen", type=int, default=4)
    ap.add_argument("--commit", type=int, default=3)
    ap.add_argument("--trace", action="store_true", help="with --decode: per-phase timeline of the kernel")
    args = ap.parse_args(argv)
    for R in map(int, args.requests.split(",")):
        print(json.dumps(run(args.tp, args.tokens, R, args.iters, args.decode, args.qlen, args.commit, args.trace)), flush=True)
    if args.decode:
        return
    if args.compare and os.environ.get("OSCAR_GDN_CHUNKED") != "0":
        env = dict(os.environ, OSCAR_GDN_CHUNKED="0")
        subprocess.run([sys.executable, "-m", "oscar_b200.bench.gdn", "--tp", str(args.tp), "--tokens",
                        str(args.tokens), "--requests", args.requests, "--iters", str(max(2, args.iters // 2))],
                       env=env, check=True)


if __name__ == "__main__":
    main()
