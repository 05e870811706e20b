"""Headline benchmark: output tok/s, TPOT and TTFT of the Qwen3.5-27B-shaped hybrid model
with INT2 KV + MTP (3 drafts) at 32 concurrent 16K-token requests.

    python bench.py --gpus N --steps K --warmup W          (N > 1: under torchrun, one rank per GPU)
    python bench.py --impl reference ...                   (the reference arm)

Synthetic data: uniform-random prompt tokens (seeded), random-init weights of the
model's shape, a seeded draft-acceptance pattern with mean 2 of 3 drafts accepted.
Timed region: exactly K engine steps (each a verify step of every request plus its
MTP drafting) bracketed by a barrier and a device synchronisation on both sides.
``value`` uses the device-busy time of the model's GPU work (CUDA events around every
GPU segment, max over ranks); ``e2e`` is the wall clock of the same K calls of the
public ``LLMEngine.step`` API, which includes building the step's metadata on the
host, its host-to-device copies from pinned memory and the device-to-host read of
the sampled tokens.  Every step streams all weights (27 GB at TP1), far more than
the 126 MB L2, so no L2 flush is needed between steps.
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import time

METRIC = "output tok/s @32 conc, TPOT, TTFT: Qwen3.5-27B-shape TP4 INT2-KV+MTP"
# Closest published reference figure: OSCAR generation throughput after the 8.5x
# step fix, Qwen3.5-27B W8A8 + MTP, TP4 on 4x Ascend 910B4
# (plan/audits/PERFORMANCE-20260908.md:76).
BASELINE_TOK_S = 11.3


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=4)
    ap.add_argument("--impl", choices=["oscar", "reference"], default="oscar")
    ap.add_argument("--model", default="qwen35-27b")
    ap.add_argument("--layers", type=int, default=None, help="override layer count (debug only; invalid for the headline)")
    ap.add_argument("--requests", type=int, default=32)
    ap.add_argument("--prompt-len", type=int, default=16384)
    ap.add_argument("--output-len", type=int, default=1024)
    ap.add_argument("--num-spec", type=int, default=3)
    ap.add_argument("--accept-mean", type=float, default=2.0)
    ap.add_argument("--kv", choices=["int2", "bf16"], default="int2")
    ap.add_argument("--prefill-policy", choices=["fcfs", "wide"], default="fcfs",
                    help="fcfs: prompts are prefilled in arrival order (15,360 tokens per step) and each request "
                         "starts decoding when its prompt is done, so TTFT is per request; wide: every prompt "
                         "advances together (every first token waits for the whole prefill)")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--dp", type=int, default=1,
                    help="data-parallel replicas, each TP over gpus/dp ranks (BASELINE config 5: DP2 x TP4)")
    ap.add_argument("--offload", action="store_true", help="swap-based host KV offload when the block pool runs out")
    ap.add_argument("--num-blocks", type=int, default=None,
                    help="KV blocks per rank (default: every request of the replica fits)")
    ap.add_argument("--kernel-profile", default=None, metavar="PREFIX",
                    help="after the timed region (untimed), run 2 more steps under torch.profiler and write "
                         "each rank's per-kernel device time to PREFIX.rank<r>.json")
    return ap.parse_args()


def reference_arm(args):
    """The reference is installed unmodified in baseline/_ref (pip --no-deps; its
    declared dependencies vllm==0.23.0 and vllm-ascend are not in the offline
    wheelhouse).  Its only public entry point is the vLLM general plugin
    ``oscar_ascend.plugin:load_plugin``, which forces the Ascend NPU platform and
    imports vllm_ascend / torch_npu on the serving path; none of that exists for CUDA,
    so the reference's own stock path cannot produce this metric on a B200."""
    import importlib.util
    ref = os.path.join(os.path.dirname(os.path.abspath(__file__)), "baseline", "_ref")
    missing = [m for m in ("vllm_ascend", "torch_npu") if importlib.util.find_spec(m) is None]
    if not os.path.isdir(os.path.join(ref, "oscar_ascend")):
        why = "reference not installed in baseline/_ref (offline pip install failed)"
    else:
        why = ("reference (oscar-ascend 0.2.0, installed in baseline/_ref) is a vLLM-Ascend plugin whose serving "
               f"path needs {', '.join(missing) or 'an Ascend NPU'} on Ascend NPUs; it has no CUDA path to run on B200")
    if int(os.environ.get("RANK", "0")) == 0:
        print(json.dumps({"impl": "reference", "unavailable": why, "metric": METRIC, "n_gpus": args.gpus}))
    return 0


def main():
    args = parse()
    if args.impl == "reference":
        return reference_arm(args)
    import numpy as np
    import torch
    import torch.distributed as dist

    from oscar_b200.config import OscarConfig
    from oscar_b200.engine.engine import LLMEngine, SeededAcceptance
    from oscar_b200.models.config import CONFIGS
    from oscar_b200.models.qwen35 import HybridModel
    from oscar_b200.parallel.groups import init_distributed, make_groups
    from oscar_b200.utils import launches
    from oscar_b200.utils.clocks import ClockSampler

    rank, world, local = init_distributed(timeout_s=600)
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if args.dp < 1 or world % args.dp or args.requests % args.dp:
        raise SystemExit(f"--dp {args.dp} must divide the GPU count ({world}) and --requests ({args.requests})")
    tp = make_groups(tp=world // args.dp, dp=args.dp)
    overrides = {} if args.layers is None else {"num_layers": args.layers}
    cfg = CONFIGS[args.model](**overrides)
    oscar = OscarConfig.from_env(head_dim=cfg.head_dim)
    t0 = time.perf_counter()
    model = HybridModel(cfg, tp, device=dev, seed=args.seed, oscar=oscar, kv_mode=args.kv, rotation="random")
    torch.cuda.synchronize()
    t_init = time.perf_counter() - t0
    R = args.requests // args.dp  # requests of this rank's replica
    per_req = args.prompt_len + args.output_len + 16 * (args.num_spec + 2)
    num_blocks = args.num_blocks or R * ((per_req + 127) // 128) + 64
    acc = SeededAcceptance(args.num_spec, args.accept_mean, seed=args.seed + 1)
    eng = LLMEngine(model, num_blocks=num_blocks, max_slots=R, num_spec=args.num_spec, acceptance=acc,
                    prefill_policy=args.prefill_policy, offload=args.offload)
    rng = np.random.default_rng(args.seed + tp.dp_rank)
    prompts = rng.integers(0, cfg.vocab_size, size=(R, args.prompt_len)).tolist()
    ids = [eng.add_request(p, args.output_len) for p in prompts]

    def barrier_sync():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    # ---------------- prefill (TTFT), untimed for the throughput metric
    barrier_sync()
    tp0 = time.perf_counter()
    for r in eng.requests.values():
        r.arrival = tp0
    prof_prefill = os.environ.get("OSCAR_PROFILE_RANGE") == "prefill"
    if prof_prefill:
        torch.cuda.cudart().cudaProfilerStart()
    while any(not eng.requests[i].output for i in ids):
        eng.step()
    barrier_sync()
    if prof_prefill:
        torch.cuda.cudart().cudaProfilerStop()
    t_prefill = time.perf_counter() - tp0
    ttft = [eng.requests[i].first_token_time - eng.requests[i].arrival for i in ids]

    # ---------------- warm-up decode steps
    for _ in range(args.warmup):
        eng.step()
    barrier_sync()

    # ---------------- timed region: exactly K steps
    out0 = eng.stats["tokens_out"]
    h2d0, d2h0 = eng.stats.get("h2d_bytes", 0), eng.stats.get("d2h_bytes", 0)
    eng.record_device_time = True
    eng.device_ms()
    if eng.host_profile is not None:
        eng.host_profile.clear()
    launches.reset()
    gpu_ids = None
    try:
        gpu_ids = [str(torch.cuda.get_device_properties(local).uuid)]
        gpu_ids = ["GPU-" + g if not g.startswith("GPU-") else g for g in gpu_ids]
    except Exception:
        gpu_ids = None
    sampler = ClockSampler(gpu_ids if local == 0 else None)
    with (sampler if local == 0 else _Null()):
        barrier_sync()
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        w0 = time.perf_counter()
        prof = os.environ.get("OSCAR_PROFILE_RANGE") == "1"
        if prof:
            torch.cuda.cudart().cudaProfilerStart()
        start.record()
        for _ in range(args.steps):
            eng.step()
        end.record()
        if prof:
            torch.cuda.cudart().cudaProfilerStop()
        barrier_sync()
        wall = time.perf_counter() - w0
    span_ms = start.elapsed_time(end)
    busy_ms = eng.device_ms()
    n_launch = launches.count()
    tokens = eng.stats["tokens_out"] - out0
    h2d_step = (eng.stats.get("h2d_bytes", 0) - h2d0) // args.steps
    d2h_step = (eng.stats.get("d2h_bytes", 0) - d2h0) // args.steps
    # max over ranks of the timed quantities
    t = torch.tensor([busy_ms, span_ms, wall], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    busy_ms, span_ms, wall = t.tolist()
    mem = torch.cuda.max_memory_allocated(dev) / 2**30
    if world > 1 and (args.dp > 1 or args.offload):
        # every replica's tokens (each TP rank holds its replica's count), peak HBM of any GPU
        tt = torch.tensor([tokens / tp.world, mem], device=dev, dtype=torch.float64)
        dist.all_reduce(tt[:1])
        dist.all_reduce(tt[1:], op=dist.ReduceOp.MAX)
        tokens, mem = int(round(tt[0].item())), float(tt[1].item())
    if eng.host_profile is not None and rank == 0:  # OSCAR_HOST_PROFILE=1: host ms per step phase
        print(json.dumps({"host_ms_per_step": {k: round(v * 1e3 / args.steps, 3)
                                               for k, v in eng.host_profile.items()}}), file=sys.stderr, flush=True)
    value = tokens / (busy_ms / 1e3)
    e2e = tokens / wall
    steps_tok = tokens / args.steps / (R * args.dp)  # output tokens per request per step
    tpot = (busy_ms / args.steps) / steps_tok
    if rank == 0:
        clocks = sampler.summary() if local == 0 else {}
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "tok/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(busy_ms / args.steps, 3), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": round(value / BASELINE_TOK_S, 2), "dtype": "bf16",
            "data": "synthetic (uniform-random prompt tokens, random-init weights, seeded acceptance pattern)",
            "config": {"model": cfg.name, "layers": cfg.num_layers, "global_batch": R * args.dp,
                       "seq_len": args.prompt_len, "output_len": args.output_len,
                       "parallelism": f"tp{world}" if args.dp == 1 else f"dp{args.dp}xtp{world // args.dp}",
                       "kv": args.kv,
                       "quantization": "W8A8 int8 linear layers, INT2 KV (FULL layers), BF16 MTP shadow KV",
                       "mtp_drafts": args.num_spec, "accept_mean": args.accept_mean,
                       "l2": "inputs larger than L2 (all weights streamed every step)",
                       "baseline_value_tok_s": BASELINE_TOK_S,
                       "baseline_source": "plan/audits/PERFORMANCE-20260908.md:76 (910B4 x4)"},
            "tpot_ms": round(tpot, 3), "ttft_ms_mean": round(1e3 * float(np.mean(ttft)), 1),
            "ttft_ms_p50": round(1e3 * float(np.median(ttft)), 1),
            "ttft_ms_max": round(1e3 * float(np.max(ttft)), 1), "prefill_s": round(t_prefill, 2),
            "prefill_policy": args.prefill_policy,
            "span_ms_per_step": round(span_ms / args.steps, 3), "tokens_timed": tokens,
            "e2e": {"value": round(e2e, 2), "unit": "tok/s", "h2d_bytes_per_step": int(h2d_step),
                    "d2h_bytes_per_step": int(d2h_step),
                    "path": "LLMEngine.step(): host scheduling + metadata from pinned memory (H2D) + "
                            "verify/draft + sampled tokens and drafts read back (D2H)"},
            "gpu_launches": n_launch, "clocks": clocks, "peak_hbm_gib": round(mem, 2),
            "init_s": round(t_init, 1),
        }
        if args.offload or args.num_blocks:
            off = eng.offload.stats if eng.offload is not None else None
            line["config"]["kv_blocks_per_rank"] = num_blocks
            line["offload"] = {"enabled": bool(args.offload), "preempted": eng.stats.get("preempted", 0),
                               "swapped_out_gib": round(off.bytes_out / 2**30, 3) if off else 0.0,
                               "swapped_in_gib": round(off.bytes_in / 2**30, 3) if off else 0.0}
        print(json.dumps(line), flush=True)
    if args.kernel_profile:
        from oscar_b200.utils.kernel_profile import profile_steps
        eng.use_graphs = False  # same kernels, launched eagerly (see profile_steps)
        profile_steps(eng.step, 2, args.kernel_profile, rank)
        barrier_sync()
    eng.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


class _Null:
    def __enter__(self):
        return self

    def __exit__(self, *a):
        return False


if __name__ == "__main__":
    sys.exit(main())
