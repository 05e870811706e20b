"""W8A8 GEMM microbench on the decode / prefill shapes of the target model.

For each (name, M, N, K): ``linear_i8`` (the tcgen05 kernel, bf16 output or fp32
accumulate for the row-parallel projections) timed with CUDA events, L2 flushed before
every sample, median of ``--iters``; reported as achieved weight-streaming bandwidth
(the weights dominate the bytes at decode sizes) against the measured HBM copy peak,
and as int8 TOPS against twice the measured bf16 GEMM peak.  ``torch._int_mm``
(cuBLASLt int8) is timed on the same operands as a library reference.

    python -m oscar_b200.bench.gemm [--tp 1] [--m 128] [--iters 20]
"""
from __future__ import annotations

import argparse
import json
import os

import torch

from ..ops import functional as F
from .harness import time_call


def _peaks() -> tuple[float, float]:
    here = os.path.dirname(os.path.abspath(__file__))
    try:
        with open(os.path.join(here, "..", "..", "MEASURED_PEAKS.json")) as f:
            j = json.load(f)
        return float(j.get("hbm_gbs", 6650.0)), float(j.get("bf16_tflops", 1590.0))
    except (OSError, ValueError):
        return 6650.0, 1590.0


def shapes(tp: int, H: int = 5120, I: int = 17408):
    return [
        ("gdn_in", 16 * 1024 // tp + 96 // tp, H, False),
        ("gdn_out", H, 6144 // tp, True),
        ("attn_qkv", (24 * 512 + 8 * 256) // tp, H, False),
        ("attn_o", H, 6144 // tp, True),
        ("gate_up", 2 * I // tp, H, False),
        ("down", H, I // tp, True),
        ("lm_head", 248320 // tp, H, False),
    ]


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--tp", type=int, default=1)
    ap.add_argument("--m", default="128")
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--only", default=None)
    args = ap.parse_args(argv)
    dev = torch.device("cuda")
    hbm, bf16 = _peaks()
    g = torch.Generator(device=dev).manual_seed(0)
    for M in map(int, args.m.split(",")):
        for name, N, K, acc in shapes(args.tp):
            if args.only and name not in args.only.split(","):
                continue
            wq = torch.randint(-127, 128, (N, K), dtype=torch.int8, device=dev, generator=g)
            ws = torch.rand(N, device=dev, generator=g) * 0.01
            x = torch.randn(M, K, device=dev, generator=g).to(torch.bfloat16)
            xq, xs = F.act_quant(x)
            out = torch.zeros(M, N, dtype=torch.float32, device=dev) if acc else None

            def ours():
                if acc:
                    out.zero_()
                    return F.linear_i8(xq, xs, wq, ws, out=out, accumulate=True)
                return F.linear_i8(xq, xs, wq, ws)

            for _ in range(3):
                ours()
            t = sorted(time_call(ours) for _ in range(args.iters))[args.iters // 2]
            lib = None
            if M >= 17:  # cuBLASLt int8 needs M > 16
                wt = wq.t()
                for _ in range(3):
                    torch._int_mm(xq, wt)
                lib = sorted(time_call(lambda: torch._int_mm(xq, wt)) for _ in range(args.iters))[args.iters // 2]
            by = N * K + M * K + M * N * (4 if acc else 2)
            gbs = by / (t * 1e-3) / 1e9
            tops = 2.0 * M * N * K / (t * 1e-3) / 1e12
            print(json.dumps({"gemm": name, "M": M, "N": N, "K": K, "accumulate": acc, "us": round(t * 1e3, 2),
                              "gbs": round(gbs, 1), "frac_hbm_of_measured": round(gbs / hbm, 3),
                              "int8_tops": round(tops, 1), "frac_int8_of_measured_bf16x2": round(tops / (2 * bf16), 3),
                              "cublaslt_int_mm_us": None if lib is None else round(lib * 1e3, 2)}), flush=True)


if __name__ == "__main__":
    main()
