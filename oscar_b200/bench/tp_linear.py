"""Tensor-parallel fused-collective microbench.

One half of a decoder layer of the target model (hidden 5120, intermediate 17408)
at ``W`` ranks, for M = 32, 128, 2048 and 16384 tokens; int8 weights uniform in
[-127, 127] with per-channel fp32 scales, activations from N(0, 1) quantised per token:

* ``rs``    row-parallel ``down_proj`` (K = 17408 / W -> N = 5120) whose result is
  reduce-scattered so that each rank holds its ``M / W`` token rows, added into the
  residual and normalised there;
* ``ag``    those normalised int8 rows all-gathered to every rank and fed to the
  column-parallel ``gate_up`` projection (K = 5120 -> N = 2 x 17408 / W);
* ``chain`` both back to back (what the model runs between two layers).

Two implementations of each:

* ``fused``  - this package's sequence-parallel path: the tcgen05 GEMM's epilogue stores
  every fp32 row straight into the owning rank's buffer over NVLink (reduce-scatter),
  the RMSNorm kernel pushes its int8 rows into every rank's activation buffer
  (all-gather) and the next GEMM, a programmatic dependent of a one-warp flag wait,
  streams its weights while the rows arrive;
* ``lib``    - the library path: cuBLASLt int8 GEMM (``torch._int_mm``) + scale,
  NCCL ``reduce_scatter_tensor`` (fp32), the RMSNorm kernel on the owned rows, NCCL
  ``all_gather_into_tensor`` of the int8 rows and scales, cuBLASLt int8 GEMM + scale.

Each case is first checked (fused vs lib gathered activations and GEMM outputs), then
timed on the device with CUDA events over ``--iters`` back-to-back calls after
warm-up, the max over ranks.  Roofline of the fused path: the slower of the GEMM
FLOPs at the int8 peak (twice the measured bf16 GEMM peak, ``--bf16-tflops``) and the
bytes each rank must move over NVLink at the measured 770 GB/s per direction
(``--nvlink-gbs``): ``(W-1)/W * M * 5120 * 4`` for the fp32 reduce-scatter and
``(W-1)/W * M * 5120`` for the int8 all-gather.  ``roofline_hbm_ms`` also counts the
int8 weights each rank streams from HBM at the measured copy bandwidth (``--hbm-gbs``),
the bound that decides the small-M cases.

    torchrun --nproc-per-node W -m oscar_b200.bench.tp_linear [--m 32,128,2048,16384]
"""
from __future__ import annotations

import argparse
import json

import torch
import torch.distributed as dist

from ..ops import functional as F
from ..parallel.groups import init_distributed, make_groups
from ..parallel.seqpar import SeqParallelTP


class _W:
    def __init__(self, q, s):
        self.q, self.s = q, s


def _int_mm_scaled(xq, xs, w_t, ws):
    """cuBLASLt int8 GEMM (int32 out) and the per-token x per-channel dequantisation."""
    M = xq.shape[0]
    if M <= 16:  # cuBLASLt int8 needs M > 16: pad the rows
        xp = torch.zeros(17, xq.shape[1], dtype=xq.dtype, device=xq.device)
        xp[:M] = xq
        return (torch._int_mm(xp, w_t)[:M].float() * xs[:, None]) * ws[None, :]
    return (torch._int_mm(xq, w_t).float() * xs[:, None]) * ws[None, :]


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--m", default="32,128,2048,16384")
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--bf16-tflops", type=float, default=1661.4,
                    help="measured bf16 GEMM peak (the int8 peak is taken as twice this)")
    ap.add_argument("--nvlink-gbs", type=float, default=770.0, help="measured peer bandwidth per direction")
    ap.add_argument("--hbm-gbs", type=float, default=6554.9, help="measured HBM copy bandwidth")
    args = ap.parse_args(argv)
    rank, world, local = init_distributed("nccl", timeout_s=120)
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    tp = make_groups(world)
    H, I = 5120, 17408
    Ms = [int(x) for x in args.m.split(",")]
    sp = SeqParallelTP(tp, max(Ms), H, dev)
    g = torch.Generator(device=dev).manual_seed(1234 + rank)
    Kd, Ngu = I // world, 2 * I // world
    down = _W(torch.randint(-127, 128, (H, Kd), dtype=torch.int8, device=dev, generator=g),
              (torch.rand(H, device=dev, generator=g) * 0.5 + 0.75) / (73.3 * Kd ** 0.5))
    gate_up = _W(torch.randint(-127, 128, (Ngu, H), dtype=torch.int8, device=dev, generator=g),
                 (torch.rand(Ngu, device=dev, generator=g) * 0.5 + 0.75) / (73.3 * H ** 0.5))
    down_t, gu_t = down.q.t(), gate_up.q.t()
    w_norm = torch.zeros(H, device=dev)
    for M in Ms:
        x = torch.randn(M, Kd, device=dev, generator=g).to(torch.bfloat16)
        xq, xs = F.act_quant(x)
        sp.begin(M, H, dev)
        Tl, own, row0 = sp.Tl, sp.own, sp.row0
        base = torch.randn(Tl, H, device=dev, generator=g)
        resid_lib = torch.zeros(Tl, H, device=dev)
        part = torch.zeros(Tl * world, H, device=dev)
        recv = torch.zeros(Tl, H, device=dev)
        q_full = torch.zeros(Tl * world, H, dtype=torch.int8, device=dev)
        s_full = torch.zeros(Tl * world, device=dev)

        def lib_rs():
            part[:M] = _int_mm_scaled(xq, xs, down_t, down.s)
            dist.reduce_scatter_tensor(recv, part, group=tp.group)
            return F.rmsnorm_quant(resid_lib, w_norm, 1e-6, delta=recv)

        def lib_ag(q, s):
            dist.all_gather_into_tensor(q_full, q, group=tp.group)
            dist.all_gather_into_tensor(s_full, s, group=tp.group)
            return _int_mm_scaled(q_full[:M], s_full[:M], gu_t, gate_up.s)

        def lib_chain():
            q, s, _ = lib_rs()
            return lib_ag(q, s)

        def fused_rs():
            sp.gemm(xq, xs, down)
            return sp.norm(sp.residual[:Tl], w_norm, 1e-6, {"rs": True})

        def fused_ag():
            q, s, _ = sp.norm(sp.residual[:Tl], w_norm, 1e-6, None)
            return F.linear_i8(q, s, gate_up.q, gate_up.s)

        def fused_chain():
            q, s, _ = fused_rs()
            return F.linear_i8(q, s, gate_up.q, gate_up.s)

        # correctness: the same residual rows in both, then one chain each
        resid_lib.copy_(base)
        sp.residual[:Tl].copy_(base)
        y_lib = lib_chain().float()
        y_fused = fused_chain().float()
        torch.cuda.synchronize()
        err_gemm = float((y_fused - y_lib).norm() / y_lib.norm())
        err_res = float((sp.residual[:own] - resid_lib[:own]).norm() / resid_lib[:own].norm().clamp(min=1e-30)) \
            if own else 0.0
        res = {}
        for name, fn in (("lib_rs", lib_rs), ("fused_rs", fused_rs),
                         ("lib_ag", lambda: lib_ag(*F.rmsnorm_quant(resid_lib, w_norm, 1e-6)[:2])),
                         ("fused_ag", fused_ag), ("lib_chain", lib_chain), ("fused_chain", fused_chain)):
            for _ in range(args.warmup):
                fn()
            dist.barrier()
            torch.cuda.synchronize()
            s_ev, e_ev = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s_ev.record()
            for _ in range(args.iters):
                fn()
            e_ev.record()
            torch.cuda.synchronize()
            t = torch.tensor([s_ev.elapsed_time(e_ev) / args.iters], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            res[name] = float(t.item())
        int8_peak = 2 * args.bf16_tflops * 1e12
        f_rs, f_ag = 2.0 * M * Kd * H, 2.0 * M * H * Ngu
        b_rs = (world - 1) / world * M * H * 4
        b_ag = (world - 1) / world * M * H
        link = args.nvlink_gbs * 1e9
        hbm = args.hbm_gbs * 1e9
        w_rs, w_ag = H * Kd, Ngu * H  # int8 weight bytes streamed per rank
        roof = {"rs": max(f_rs / int8_peak, b_rs / link), "ag": max(f_ag / int8_peak, b_ag / link),
                "chain": max((f_rs + f_ag) / int8_peak, (b_rs + b_ag) / link)}
        roof_hbm = {"rs": max(roof["rs"], w_rs / hbm), "ag": max(roof["ag"], w_ag / hbm),
                    "chain": max(roof["chain"], (w_rs + w_ag) / hbm)}
        if rank == 0:
            line = {"tp": world, "M": M, "down_K": Kd, "gate_up_N": Ngu, "rel_err_gemm": err_gemm,
                    "rel_err_residual": err_res}
            for op in ("rs", "ag", "chain"):
                lib_ms, fused_ms = res[f"lib_{op}"], res[f"fused_{op}"]
                line[op] = {"lib_ms": round(lib_ms, 4), "fused_ms": round(fused_ms, 4),
                            "speedup": round(lib_ms / fused_ms, 3), "roofline_ms": round(roof[op] * 1e3, 4),
                            "fused_frac_of_roofline": round(roof[op] * 1e3 / fused_ms, 3),
                            "roofline_hbm_ms": round(roof_hbm[op] * 1e3, 4),
                            "fused_frac_of_roofline_hbm": round(roof_hbm[op] * 1e3 / fused_ms, 3)}
            print(json.dumps(line), flush=True)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
