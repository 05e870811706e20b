"""Serve CLI: ``python -m oscar_b200.serve`` (one process per GPU; torchrun for TP).

    torchrun --nproc-per-node 4 --master-addr 127.0.0.1 -m oscar_b200.serve \\
        --model qwen35-27b --port 8000

Equivalent of the reference's serve script (``delivery/serve_oscar.sh:64-99``):
TP over all ranks of the launch, 15,360 batched tokens per step, up to 128
concurrent sequences, MTP with 3 draft tokens, OSCAR INT2 KV for the FULL layers
(rotations from ``OSCAR_ASCEND_K_ROTATION_PATH`` / ``V_ROTATION_PATH`` when set, else
seeded random orthogonal), the cache sized from free memory by the budget seam.
Every rank prints its READY manifest; rank 0 serves HTTP, the others follow it in
lockstep.  ``--weights DIR`` serves a Hugging Face Qwen3.5 checkpoint (``config.json``
and safetensors, quantised to W8A8 at load, each rank reading its own slices; the
tokenizer is taken from the same directory when it has one), else the weights are
random (seeded) of the ``--model`` shape.
"""
from __future__ import annotations

import argparse
import json
import os
import sys

import torch
import torch.distributed as dist


def parse(argv=None):
    ap = argparse.ArgumentParser(prog="python -m oscar_b200.serve")
    ap.add_argument("--model", default="qwen35-27b")
    ap.add_argument("--layers", type=int, default=None)
    ap.add_argument("--host", default="127.0.0.1")
    ap.add_argument("--port", type=int, default=8000)
    ap.add_argument("--max-num-seqs", type=int, default=128)
    ap.add_argument("--max-batched-tokens", type=int,
                    default=int(os.environ.get("OSCAR_ASCEND_BATCHED_TOKENS", "15360") or 15360))
    ap.add_argument("--num-spec", type=int, default=3)
    ap.add_argument("--kv", choices=["int2", "bf16"], default="int2")
    ap.add_argument("--gpu-memory-utilization", type=float, default=0.9)
    ap.add_argument("--num-blocks", type=int, default=None, help="fixed block count (testing)")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--weights", default=None,
                    help="Hugging Face model directory (config.json + safetensors); default: random weights")
    ap.add_argument("--tokenizer", default=None, help="local HF tokenizer directory (optional)")
    ap.add_argument("--rope-scaling", default=None,
                    help='RoPE scaling override as JSON, e.g. \'{"rope_type": "yarn", "factor": 4.0, '
                         '"original_max_position_embeddings": 262144}\' (the reference serve script\'s override)')
    ap.add_argument("--generation-config", choices=["auto", "none"], default="auto",
                    help="auto: requests without temperature / top_k / top_p take the checkpoint's "
                         "generation_config.json values; none: greedy")
    ap.add_argument("--device", default=None, help="cpu runs the torch reference path (testing)")
    return ap.parse_args(argv)


def build(args):
    from ..engine import budget as B
    from ..llm import create_engine

    rank, world, model, eng, budget = create_engine(
        args.model, weights=args.weights, layers=args.layers, kv=args.kv, num_spec=args.num_spec,
        max_num_seqs=args.max_num_seqs, max_batched_tokens=args.max_batched_tokens,
        gpu_memory_utilization=args.gpu_memory_utilization, num_blocks=args.num_blocks, seed=args.seed,
        device=args.device, rope_scaling=args.rope_scaling)
    man = B.ready_manifest(model, rank, world, budget)
    print(man.line(), flush=True)
    mans = [None] * world
    if world > 1:
        dist.all_gather_object(mans, json.loads(man.line().split("READY ", 1)[1]))
        B.validate(mans, world_size=world)
    else:
        mans = [json.loads(man.line().split("READY ", 1)[1])]
    return rank, world, model, eng, mans


def main(argv=None) -> int:
    args = parse(argv)
    rank, world, model, eng, mans = build(args)
    from .worker import ControlChannel, EngineWorker, follower_loop

    control = ControlChannel.create(list(range(world))) if world > 1 else None
    if rank != 0:
        follower_loop(eng, control)
        eng.close()
        dist.destroy_process_group()
        return 0
    import uvicorn

    from .server import create_app

    tok = None
    tok_dir = args.tokenizer
    if tok_dir is None and args.weights and os.path.exists(os.path.join(args.weights, "tokenizer_config.json")):
        tok_dir = args.weights
    if tok_dir:
        from transformers import AutoTokenizer
        tok = AutoTokenizer.from_pretrained(tok_dir, local_files_only=True)
    worker = EngineWorker(eng, control).start()
    eos = None
    if args.weights:
        from ..models.loader import eos_token_ids
        eos = eos_token_ids(args.weights) or None  # None: the tokenizer's, if any
    gen = None
    if args.weights and args.generation_config == "auto":
        from ..models.loader import generation_defaults
        gen = generation_defaults(args.weights) or None
    app = create_app(worker, tok, mans, model_name=model.cfg.name, vocab_size=model.cfg.vocab_size,
                     eos_token_ids=eos, max_model_len=model.cfg.max_position, sampling_defaults=gen)
    try:
        uvicorn.run(app, host=args.host, port=args.port, log_level="info")
    finally:
        worker.stop()
        eng.close()
        if world > 1:
            dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
