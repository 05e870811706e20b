"""W8A8 GEMM microbench on the decode / prefill shapes of the target model.

For each (name, M, N, K): ``linear_i8`` (the tcgen05 kernel, bf16 output or fp32
accumulate for the row-parallel projections) timed with CUDA events around ``--reps``
back-to-back calls that cycle through enough weight copies to exceed the L2 cache (so
every call streams its weights from HBM and host launch latency is hidden, as in the
model's step), median of ``--iters`` such samples; reported as achieved weight-streaming
bandwidth (the weights dominate the bytes at decode sizes) against the measured HBM copy
peak, and as int8 TOPS against twice the measured bf16 GEMM peak.  With ``--lib``,
``torch._int_mm`` (cuBLASLt int8) is timed the same way on the same operands.

    python -m oscar_b200.bench.gemm [--tp 1] [--m 128] [--iters 10] [--lib]
"""
from __future__ import annotations

import argparse
import json
import os

import torch

from ..ops import functional as F
from .harness import peak_bf16_tflops, peak_hbm_gbs, time_call


def _peaks() -> tuple[float, float]:
    return peak_hbm_gbs(), peak_bf16_tflops()


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
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--reps", type=int, default=8)
    ap.add_argument("--only", default=None)
    ap.add_argument("--lib", action="store_true", help="also time torch._int_mm (cuBLASLt int8)")
    args = ap.parse_args(argv)
    dev = torch.device("cuda")
    hbm, bf16 = _peaks()
    g = torch.Generator(device=dev).manual_seed(0)
    l2 = 126 * 2**20
    for M in map(int, args.m.split(",")):
        for name, N, K, acc in shapes(args.tp):
            if args.only and name not in args.only.split(","):
                continue
            copies = max(2, min(args.reps, -(-3 * l2 // (N * K))))  # > 3x L2 of weights in rotation
            wqs = [torch.randint(-127, 128, (N, K), dtype=torch.int8, device=dev, generator=g) for _ in range(copies)]
            ws = torch.rand(N, device=dev, generator=g) * 0.01
            x = torch.randn(M, K, device=dev, generator=g).to(torch.bfloat16)
            xq, xs = F.act_quant(x)
            out = torch.zeros(M, N, dtype=torch.float32, device=dev) if acc else None

            def ours():
                for i in range(args.reps):
                    if acc:
                        F.linear_i8(xq, xs, wqs[i % copies], ws, out=out, accumulate=True)
                    else:
                        F.linear_i8(xq, xs, wqs[i % copies], ws)

            ours()
            t = sorted(time_call(ours, flush=False) for _ in range(args.iters))[args.iters // 2] / args.reps
            lib = None
            if args.lib and M >= 17:  # cuBLASLt int8 needs M > 16
                wts = [w.t() for w in wqs]

                def theirs():
                    for i in range(args.reps):
                        torch._int_mm(xq, wts[i % copies])

                theirs()
                lib = sorted(time_call(theirs, flush=False) for _ in range(args.iters))[args.iters // 2] / args.reps
            by = N * K + M * K + M * N * (4 if acc else 2)
            gbs = by / (t * 1e-3) / 1e9
            tops = 2.0 * M * N * K / (t * 1e-3) / 1e12
            print(json.dumps({"gemm": name, "M": M, "N": N, "K": K, "accumulate": acc, "us": round(t * 1e3, 2),
                              "gbs": round(gbs, 1), "frac_hbm_of_measured": round(gbs / hbm, 3),
                              "int8_tops": round(tops, 1), "frac_int8_of_measured_bf16x2": round(tops / (2 * bf16), 3),
                              "cublaslt_int_mm_us": None if lib is None else round(lib * 1e3, 2)}), flush=True)
            del wqs


if __name__ == "__main__":
    main()
