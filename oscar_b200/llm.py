"""Offline generation API and the engine construction shared with the serve CLI.

    from oscar_b200 import LLM, SamplingParams
    llm = LLM("/models/Qwen3.5-27B")                # a Hugging Face directory, or a config name
    outs = llm.generate(["Hello"], SamplingParams(temperature=0.7, max_tokens=64))
    print(outs[0].outputs[0].text)

The same surface as the offline API the reference's rotation tool drives
(``tools/gen_rotations.py:166-196``: ``LLM(...)``, ``SamplingParams(max_tokens=...,
temperature=...)``, ``llm.generate(prompt, params)``).  Under ``torchrun`` every rank
builds the ``LLM`` and calls ``generate`` with the same prompts: the engines run in
lockstep (one tensor-parallel group over all ranks) and every rank returns the outputs.
"""
from __future__ import annotations

import json
import os
from dataclasses import dataclass, field

import torch
import torch.distributed as dist

from .ops.sampling import SamplingParams


def create_engine(model: str = "qwen35-27b", *, weights: str | None = None, layers: int | None = None,
                  kv: str = "int2", num_spec: int = 3, max_num_seqs: int = 128, max_batched_tokens: int = 15360,
                  gpu_memory_utilization: float = 0.9, num_blocks: int | None = None, seed: int = 0,
                  device: str | None = None, rope_scaling: dict | str | None = None, offload: bool = False):
    """Builds this rank's model and engine: ``(rank, world, model, engine, budget)``.

    Tensor parallelism spans every rank of the launch (``torchrun``; one process is TP1).
    ``weights`` is a Hugging Face model directory, else ``model`` names a config with
    random (seeded) weights.  Without ``num_blocks`` the KV pool takes what the memory
    budget allows (every rank the smallest).  ``device="cpu"`` runs the torch reference
    path (testing)."""
    from .config import OscarConfig
    from .engine import budget as B
    from .engine.engine import LLMEngine
    from .models.config import CONFIGS
    from .models.qwen35 import HybridModel
    from .parallel.groups import init_distributed, make_groups

    rank, world, local = init_distributed(backend="gloo" if device == "cpu" else None)
    dev = torch.device("cpu") if device == "cpu" else torch.device("cuda", local)
    if dev.type == "cuda":
        torch.cuda.set_device(dev)
    tp = make_groups(tp=world)
    if weights:
        from .models.loader import config_from_hf
        cfg = config_from_hf(weights)
    else:
        cfg = CONFIGS[model](**({} if layers is None else {"num_layers": layers}))
    if rope_scaling:
        cfg.rope_scaling = json.loads(rope_scaling) if isinstance(rope_scaling, str) else dict(rope_scaling)
    oscar = OscarConfig.from_env(head_dim=cfg.head_dim)
    rot = oscar.k_rotation_path or "random"
    if weights:
        from .models.loader import from_pretrained
        m = from_pretrained(weights, tp, device=dev, oscar=oscar, kv_mode=kv, rotation=rot, num_layers=layers,
                            seed=seed, config=cfg)
    else:
        m = HybridModel(cfg, tp, device=dev, seed=seed, oscar=oscar, kv_mode=kv, rotation=rot)
    budget = geo = None
    avail = 0
    if num_blocks is None:
        geo = B.geometry_of(m, max_slots=max_num_seqs)
        avail = B.available_memory(dev, gpu_memory_utilization)
        budget = B.memory_budget(avail, geo)
        num_blocks = budget.blocks
        if world > 1:  # every rank uses the smallest budget
            t = torch.tensor([num_blocks], device=dev if dev.type == "cuda" else "cpu")
            dist.all_reduce(t, op=dist.ReduceOp.MIN)
            num_blocks = int(t.item())
    eng = LLMEngine(m, num_blocks=num_blocks, max_slots=max_num_seqs, max_batched_tokens=max_batched_tokens,
                    num_spec=num_spec, offload=offload, seed=seed)
    B.verify_layers(m.cfg.full_layer_ids, [x.layer_id for x in m.full_layers])
    if budget is not None:  # the allocation may not exceed the budget it was sized from
        alloc = m.cache_bytes()
        print(B.memory_line(rank, budget, geo, avail, alloc, dev), flush=True)
        B.check_allocation(sum(alloc.values()), budget)
    return rank, world, m, eng, budget


@dataclass
class CompletionOutput:
    index: int
    text: str
    token_ids: list
    finish_reason: str | None
    logprobs: list | None = None  # per token: {token id: logprob} of the token and the k most likely


@dataclass
class RequestOutput:
    request_id: int
    prompt: str | None
    prompt_token_ids: list
    outputs: list = field(default_factory=list)
    finished: bool = True


class LLM:
    """Offline batched generation over one engine (see the module docstring).

    ``model``: a Hugging Face model directory (weights, config, tokenizer when present) or a
    config name (random weights; the byte tokenizer).  Keyword arguments go to
    :func:`create_engine`; ``tokenizer`` names a local Hugging Face tokenizer directory."""

    def __init__(self, model: str = "qwen35-27b", tokenizer: str | None = None, **engine_kw):
        weights = model if os.path.isdir(model) else None
        self.rank, self.world, self.model, self.engine, self.budget = create_engine(
            "qwen35-27b" if weights else model, weights=weights, **engine_kw)
        tok_dir = tokenizer or (weights if weights and os.path.exists(
            os.path.join(weights, "tokenizer_config.json")) else None)
        if tok_dir:
            from transformers import AutoTokenizer
            self.tokenizer = AutoTokenizer.from_pretrained(tok_dir, local_files_only=True)
        else:
            from .serve.server import ByteTokenizer
            self.tokenizer = ByteTokenizer()
        eos = []
        if weights:
            from .models.loader import eos_token_ids
            eos = eos_token_ids(weights)
        if not eos:
            e = getattr(self.tokenizer, "eos_token_id", None)
            eos = [] if e is None else ([e] if isinstance(e, int) else list(e))
        self.eos_token_ids = [int(x) for x in eos]

    def _decode(self, ids) -> str:
        try:
            return self.tokenizer.decode(ids, skip_special_tokens=True)
        except TypeError:
            return self.tokenizer.decode(ids)

    def generate(self, prompts, sampling_params: SamplingParams | list | None = None) -> list[RequestOutput]:
        """``prompts``: a string, a list of token ids, or a list of either.  Runs them to
        completion and returns one :class:`RequestOutput` per prompt, in order."""
        if isinstance(prompts, str) or (isinstance(prompts, list) and prompts and isinstance(prompts[0], int)):
            prompts = [prompts]
        params = sampling_params if isinstance(sampling_params, (list, tuple)) else [sampling_params] * len(prompts)
        if len(params) != len(prompts):
            raise ValueError(f"{len(params)} sampling params for {len(prompts)} prompts")
        eng = self.engine
        reqs = []
        strings: dict = {}  # request id -> stop strings
        for p, sp in zip(prompts, params):
            sp = (sp or SamplingParams()).validate()
            ids = self.tokenizer.encode(p) if isinstance(p, str) else [int(t) for t in p]
            stop = list(sp.stop_token_ids or []) + ([] if sp.ignore_eos else self.eos_token_ids)
            rid = eng.add_request(ids, sp.max_tokens, None if sp.greedy else sp, stop, sp.logprobs)
            reqs.append((rid, p if isinstance(p, str) else None, ids))
            if sp.stop:
                strings[rid] = [x for x in ([sp.stop] if isinstance(sp.stop, str) else sp.stop) if x]
        cut: dict = {}  # request id -> text up to its first stop string
        while eng.has_work():
            eng.step()
            for rid, stops in strings.items():
                r = eng.requests[rid]
                if rid in cut or not r.output:
                    continue
                text = self._decode(list(r.output))
                hits = [text.find(x) for x in stops if x in text]
                if hits:
                    cut[rid] = text[:min(hits)]
                    eng.abort(rid)  # nothing past the stop string is generated
        out = []
        for rid, text, ids in reqs:
            r = eng.requests[rid]
            toks = list(r.output)
            body, reason = (cut[rid], "stop") if rid in cut else (self._decode(toks), r.finish_reason)
            lps = None
            if r.logprobs is not None:
                lps = [{t: lp, **dict(top)} for t, (lp, top) in zip(toks, r.lp)]
            out.append(RequestOutput(rid, text, ids, [CompletionOutput(0, body, toks, reason, lps)]))
            eng.release(rid)
        return out

    def close(self) -> None:
        self.engine.close()
