"""OpenAI-style HTTP front end of the engine (rank 0).

The reference serves through vLLM's OpenAI server (``delivery/serve_oscar.sh:64-99``);
this is the same surface for this framework's engine, kept minimal:

* ``POST /v1/completions`` - ``{"prompt": str | [int], "max_tokens": int, "temperature",
  "top_k", "top_p", "seed"}``; returns the generated token ids and, when a tokenizer is
  configured, the text.  Decoding is greedy unless ``temperature > 0`` (this server's
  default is greedy, the benchmarks' setting, where OpenAI's is 1.0); ``top_k`` 0 or -1
  and ``top_p`` 1 switch truncation off; a request without ``seed`` gets one derived from
  the engine seed and its id;
* ``GET /health``, ``GET /ready`` (the READY manifests), ``GET /metrics`` (Prometheus:
  requests, output tokens, TTFT / TPOT histograms, draft acceptance, free KV blocks).

Prompts given as text are tokenised with the configured tokenizer, or byte-level
(UTF-8 bytes + 3) for the random-weight models the benchmarks use.
"""
from __future__ import annotations

import asyncio
import itertools
import time

from fastapi import FastAPI, HTTPException
from fastapi.responses import PlainTextResponse
from pydantic import BaseModel

from ..ops.sampling import SamplingParams
from .worker import EngineWorker


class ByteTokenizer:
    """UTF-8 bytes shifted past 3 special ids; enough to drive random-weight models."""

    offset = 3

    def encode(self, text: str) -> list[int]:
        return [b + self.offset for b in text.encode("utf-8")]

    def decode(self, ids) -> str:
        return bytes(max(0, min(255, i - self.offset)) for i in ids).decode("utf-8", errors="replace")


class CompletionRequest(BaseModel):
    prompt: str | list[int]
    max_tokens: int = 16
    model: str | None = None
    temperature: float = 0.0
    top_k: int = 0
    top_p: float = 1.0
    seed: int | None = None


def create_app(worker: EngineWorker, tokenizer=None, manifests: list | None = None, model_name: str = "oscar-b200",
               vocab_size: int | None = None) -> FastAPI:
    app = FastAPI(title="oscar-b200")
    tok = tokenizer or ByteTokenizer()
    ids = itertools.count()

    @app.get("/health")
    def health():
        if worker.error is not None:
            raise HTTPException(503, f"engine failed: {worker.error!r}")
        return {"ok": True}

    @app.get("/ready")
    def ready():
        return {"manifests": manifests or []}

    @app.get("/metrics", response_class=PlainTextResponse)
    def metrics():
        m = worker.metrics.snapshot(worker.engine)
        lines = [f"oscar_{k} {float(v)}" for k, v in m.items() if v is not None]
        return "\n".join(lines) + "\n"

    @app.post("/v1/completions")
    async def completions(req: CompletionRequest):
        prompt = tok.encode(req.prompt) if isinstance(req.prompt, str) else list(req.prompt)
        if not prompt:
            raise HTTPException(400, "empty prompt")
        if vocab_size is not None and (min(prompt) < 0 or max(prompt) >= vocab_size):
            raise HTTPException(400, f"token ids must be in [0, {vocab_size})")
        if req.max_tokens < 1:
            raise HTTPException(400, "max_tokens must be >= 1")
        sp = None
        if req.temperature > 0:
            sp = SamplingParams(req.temperature, max(0, req.top_k), req.top_p, req.seed)
            try:
                sp.validate()
            except ValueError as e:
                raise HTTPException(400, str(e)) from e
        elif req.temperature < 0:
            raise HTTPException(400, "temperature must be >= 0")
        t0 = time.time()
        fut = worker.submit(prompt, req.max_tokens, sp)
        try:
            out = await asyncio.wrap_future(fut)
        except Exception as e:  # noqa: BLE001
            raise HTTPException(500, f"generation failed: {e!r}") from e
        return {"id": f"cmpl-{next(ids)}", "object": "text_completion", "created": int(t0), "model": model_name,
                "choices": [{"index": 0, "text": tok.decode(out), "token_ids": out, "finish_reason": "length"}],
                "usage": {"prompt_tokens": len(prompt), "completion_tokens": len(out),
                          "total_tokens": len(prompt) + len(out)}}

    return app
