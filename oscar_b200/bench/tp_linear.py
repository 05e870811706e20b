"""Tensor-parallel fused-collective microbench.

Row-parallel W8A8 projections of the target model (hidden 5120, intermediate 17408):
``down_proj`` (K = 17408 / tp -> N = 5120) and ``o_proj`` (K = 6144 / tp -> N = 5120)
for M = 32, 128, 2048 and 16384 tokens, int8 weights uniform in [-127, 127] with
per-channel fp32 scales, activations from N(0, 1) quantised per token.  Two paths
produce the all-reduced fp32 residual delta:

* ``nccl``  - tcgen05 GEMM into a local fp32 buffer, then ``dist.all_reduce`` (NCCL),
* ``fused`` - the same GEMM whose epilogue reduces through NVLS multicast
  (``multimem.red``) into every rank's buffer, completion signalled peer to peer,
  consumed by the RMSNorm that waits on the flags (included in both timings: the
  consumer RMSNorm + residual add runs after either path).

Each configuration is checked first (fused == nccl, rtol 1e-4), then timed on the
device with CUDA events over ``--iters`` back-to-back calls after warm-up; the
reported time is the max over ranks.  Roofline for the fused path: the slower of
(GEMM FLOPs / measured bf16 GEMM peak x 2 for int8) and (bytes each rank must send
over NVLink / 770 GB/s measured peer bandwidth); reported as achieved / roofline.

    torchrun --nproc-per-node N -m oscar_b200.bench.tp_linear [--m 32,128,2048,16384]
"""
from __future__ import annotations

import argparse
import json
import os

import torch
import torch.distributed as dist

from ..ops import functional as F
from ..parallel.fused import FusedRowReduce, NcclRowReduce
from ..parallel.groups import init_distributed, make_groups

NVLINK_GBS = 770.0  # measured peer copy bandwidth per direction on this pool


def _peaks():
    here = os.path.dirname(os.path.abspath(__file__))
    try:
        with open(os.path.join(here, "..", "..", "MEASURED_PEAKS.json")) as f:
            j = json.load(f)
        return float(j.get("bf16_tflops", 1590.0))
    except (OSError, ValueError):
        return 1590.0


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--m", default="32,128,2048,16384")
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--proj", default="down,o")
    args = ap.parse_args(argv)
    rank, world, local = init_distributed("nccl", timeout_s=120)
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    tp = make_groups(world)
    H = 5120
    Ms = [int(x) for x in args.m.split(",")]
    max_m = max(Ms)
    fused = FusedRowReduce(tp, max_m, H, dev)
    nccl = NcclRowReduce(tp)
    bf16_peak = _peaks()
    g = torch.Generator(device=dev).manual_seed(1234 + rank)
    projs = {"down": 17408 // world, "o": 6144 // world}
    w_norm = torch.zeros(H, device=dev)
    for proj in args.proj.split(","):
        K = projs[proj]
        wq = torch.randint(-127, 128, (H, K), dtype=torch.int8, device=dev, generator=g)
        ws = (torch.rand(H, device=dev, generator=g) * 0.5 + 0.75) / (73.3 * K ** 0.5)

        class W:
            q, s = wq, ws

        for M in Ms:
            x = torch.randn(M, K, device=dev, generator=g).to(torch.bfloat16)
            xq, xs = F.act_quant(x)
            res = {}
            outs = {}
            for name, red in (("nccl", nccl), ("fused", fused)):
                resid = torch.zeros(M, H, device=dev)

                def step():
                    red.begin(M, H, dev)
                    kw = red.gemm(xq, xs, W, 0)
                    F.rmsnorm_quant(resid, w_norm, 1e-6, **kw)
                    red.begin(M, H, dev)
                    kw = red.gemm(xq, xs, W, 1)
                    F.rmsnorm_quant(resid, w_norm, 1e-6, **kw)

                step()
                torch.cuda.synchronize()
                outs[name] = resid.clone()
                for _ in range(args.warmup):
                    step()
                dist.barrier()
                torch.cuda.synchronize()
                s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                s.record()
                for _ in range(args.iters):
                    step()
                e.record()
                torch.cuda.synchronize()
                t = torch.tensor([s.elapsed_time(e) / (2 * args.iters)], device=dev)
                dist.all_reduce(t, op=dist.ReduceOp.MAX)
                res[name] = float(t.item())
            err = float((outs["fused"] - outs["nccl"]).norm() / outs["nccl"].norm())
            flops = 2.0 * M * K * H
            t_gemm = flops / (2 * bf16_peak * 1e12)  # int8 dense peak = 2 x bf16
            bytes_nv = M * H * 4 * (world - 1) / world * 2  # all-reduce volume per rank
            t_link = bytes_nv / (NVLINK_GBS * 1e9)
            roof_ms = max(t_gemm, t_link) * 1e3
            if rank == 0:
                print(json.dumps({"proj": proj, "tp": world, "M": M, "K": K, "N": H,
                                  "nccl_ms": round(res["nccl"], 4), "fused_ms": round(res["fused"], 4),
                                  "speedup": round(res["nccl"] / res["fused"], 3), "rel_err": err,
                                  "roofline_ms": round(roof_ms, 4),
                                  "fused_frac_of_roofline": round(roof_ms / res["fused"], 3)}), flush=True)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
