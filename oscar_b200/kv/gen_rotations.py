"""Offline rotation generator: ``python -m oscar_b200.kv.gen_rotations --out oscar_rotations.pt``.

Same procedure as the reference's ``tools/gen_rotations.py:73-245``:

1. build the model with identity rotations (calibration mode, every rank of a TP
   launch when run under torchrun),
2. run a prefill over calibration prompts while each FULL-attention layer captures up
   to ``OSCAR_ASCEND_CALIB_TOKEN_CAP`` tokens of unquantised Q/K/V,
3. reduce the per-layer objectives (Σ_Q for K, score-weighted Σ_S for V) on each
   rank, gather them on rank 0 and merge them count-weighted,
4. eigen-decompose in fp64 on the CPU and compose ``R = U · H · P_br``,
5. check orthogonality (1e-6) and save the v2 ``oscar_rotations.pt``.

Weights: ``--weights DIR`` loads a Hugging Face checkpoint (the calibration then sees
the real model's activations), else seeded random weights (``--weights-seed``).

Prompts: ``--prompts FILE`` (one prompt per line, whitespace-separated token ids), or
seeded random tokens (``--num-prompts``, ``--prompt-len``) for the random-weight
models.  ``OSCAR_ASCEND_GEN_MAXLEN`` caps the prompt length like the reference.
"""
from __future__ import annotations

import argparse
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

from .calib import CalibrationCapture, build_checkpoint, merge_rank_stats


def calibrate(model, prompts: list[list[int]], token_cap: int | None = None, max_batched_tokens: int = 4096):
    """Prefill ``prompts`` through an engine of ``model`` (identity rotations) and return
    this rank's per-layer statistics."""
    from ..engine.engine import LLMEngine

    cap = CalibrationCapture(token_cap)
    for layer in model.full_layers:
        if layer.Rk is not None or layer.Rv is not None:
            raise ValueError("calibrate with rotation='identity': the capture must see unrotated q/k/v")
        layer.calib = cap
    total = sum(len(p) + 2 for p in prompts)
    eng = LLMEngine(model, num_blocks=total // 128 + 2 * len(prompts) + 8, max_slots=max(1, len(prompts)),
                    max_batched_tokens=max_batched_tokens, num_spec=0)
    eng.use_graphs = False
    try:
        eng.generate(prompts, max_new_tokens=1)
    finally:
        for layer in model.full_layers:
            layer.calib = None
        eng.close()
    return cap.finalize()


def merge_across_ranks(stats: dict, D: int) -> dict:
    """Gather every rank's statistics on all ranks and merge them count-weighted."""
    per_rank = [stats]
    if dist.is_initialized() and dist.get_world_size() > 1:
        per_rank = [None] * dist.get_world_size()
        dist.all_gather_object(per_rank, stats)
    return merge_rank_stats(per_rank, D)


def _prompts(args, vocab: int) -> list[list[int]]:
    maxlen = int(os.environ.get("OSCAR_ASCEND_GEN_MAXLEN", "0") or 0) or None
    if args.prompts:
        with open(args.prompts) as f:
            ps = [[int(t) for t in line.split()] for line in f if line.strip()]
    else:
        rng = np.random.default_rng(args.seed)
        ps = rng.integers(0, vocab, size=(args.num_prompts, args.prompt_len)).tolist()
    return [p[:maxlen] if maxlen else p for p in ps]


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="python -m oscar_b200.kv.gen_rotations")
    ap.add_argument("--out", default="oscar_rotations.pt")
    ap.add_argument("--model", default="qwen35-27b")
    ap.add_argument("--layers", type=int, default=None)
    ap.add_argument("--prompts", default=None)
    ap.add_argument("--num-prompts", type=int, default=4)
    ap.add_argument("--prompt-len", type=int, default=512)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--weights-seed", type=int, default=0)
    ap.add_argument("--weights", default=None,
                    help="Hugging Face model directory (config.json + safetensors); default: seeded random weights")
    ap.add_argument("--device", default=None, help="cpu: torch reference path")
    args = ap.parse_args(argv)

    from ..config import OscarConfig
    from ..models.config import CONFIGS
    from ..models.qwen35 import HybridModel
    from ..parallel.groups import init_distributed, make_groups

    rank, world, local = init_distributed(backend="gloo" if args.device == "cpu" else None)
    dev = torch.device("cpu") if args.device == "cpu" else torch.device("cuda", local)
    if dev.type == "cuda":
        torch.cuda.set_device(dev)
    if args.weights:
        from ..models.loader import config_from_hf, from_pretrained
        hd = config_from_hf(args.weights).head_dim
        model = from_pretrained(args.weights, make_groups(world), device=dev, oscar=OscarConfig.from_env(head_dim=hd),
                                rotation="identity", mtp=False, num_layers=args.layers)
        cfg = model.cfg
    else:
        cfg = CONFIGS[args.model](**({} if args.layers is None else {"num_layers": args.layers}))
        model = HybridModel(cfg, make_groups(world), device=dev, seed=args.weights_seed,
                            oscar=OscarConfig.from_env(head_dim=cfg.head_dim), rotation="identity", mtp=False)
    stats = calibrate(model, _prompts(args, cfg.vocab_size))
    merged = merge_across_ranks(stats, cfg.head_dim)
    if rank == 0:
        layers = build_checkpoint(merged, cfg.head_dim, args.out)
        print(f"[oscar-b200] wrote {args.out}: {len(layers)} layers {sorted(layers)}")
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
