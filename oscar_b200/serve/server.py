"""OpenAI-style HTTP front end of the engine (rank 0).

The reference serves through vLLM's OpenAI server (``delivery/serve_oscar.sh:64-99``);
this is the same surface for this framework's engine, kept minimal:

* ``POST /v1/completions`` - ``{"prompt": str | [int], "max_tokens": int, "temperature",
  "top_k", "top_p", "seed", "stream", "stop", "stop_token_ids", "ignore_eos"}``; returns
  the generated token ids, the text and the finish reason (``"stop"`` or ``"length"``).
  Decoding is greedy unless ``temperature > 0``; fields a request leaves out take the
  server's defaults: greedy (the benchmarks' setting, where OpenAI's is 1.0), or, when it
  serves a checkpoint, that checkpoint's ``generation_config.json`` recommendation (as
  vLLM does by default); ``top_k`` 0 or -1 and ``top_p`` 1 switch truncation off; a request without ``seed`` gets one derived from the engine seed and
  its id.  ``stream: true`` answers with server-sent events, one per engine step that
  produced tokens, then ``data: [DONE]``.  A stop string ends the request when it appears
  in the text (it is cut from the text, and the request is aborted in the engine); stop
  token ids and the model's EOS ids (unless ``ignore_eos``) end it in the engine.  A
  streaming client that disconnects aborts its request.  ``logprobs: k`` (0-20) returns the
  OpenAI ``logprobs`` object (token, its log-probability, the k most likely tokens), in the
  plain response or in every streamed chunk for that chunk's tokens;
  ``n`` (1-16, not with ``stream``) returns that many choices, sampled with seeds ``seed + i``;
  ``stream_options: {"include_usage": true}`` adds a last streamed chunk with the token counts;
* ``POST /v1/chat/completions`` - ``{"messages": [{"role", "content"}], ...}`` with the same
  generation fields; the prompt is the tokenizer's chat template (``<|role|>`` headers
  with the byte tokenizer), the answer a ``chat.completion`` (``chat.completion.chunk``
  events when streaming);
* ``GET /v1/models``;
* ``GET /health``, ``GET /ready`` (the READY manifests), ``GET /metrics`` (Prometheus:
  requests, output tokens, running / waiting / preempted, draft acceptance, free KV blocks
  as gauges; TTFT / TPOT histograms; finished requests per finish reason; verify steps per
  number of accepted drafts).

Prompts given as text are tokenised with the configured tokenizer, or byte-level
(UTF-8 bytes + 3) for the random-weight models the benchmarks use.
"""
from __future__ import annotations

import asyncio
import itertools
import json
import time

from fastapi import FastAPI, HTTPException
from fastapi.responses import PlainTextResponse, StreamingResponse
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
    temperature: float | None = None  # None: the server's default (greedy, or the checkpoint's)
    top_k: int | None = None
    top_p: float | None = None
    seed: int | None = None
    stream: bool = False
    stop: str | list[str] | None = None
    stop_token_ids: list[int] | None = None
    ignore_eos: bool = False
    logprobs: int | None = None
    n: int = 1
    stream_options: dict | None = None


class ChatMessage(BaseModel):
    role: str
    content: str


class ChatRequest(BaseModel):
    messages: list[ChatMessage]
    max_tokens: int = 16
    model: str | None = None
    temperature: float | None = None  # None: the server's default (greedy, or the checkpoint's)
    top_k: int | None = None
    top_p: float | None = None
    seed: int | None = None
    stream: bool = False
    stop: str | list[str] | None = None
    stop_token_ids: list[int] | None = None
    ignore_eos: bool = False
    logprobs: bool = False
    top_logprobs: int | None = None
    n: int = 1
    max_completion_tokens: int | None = None  # the newer name of max_tokens
    stream_options: dict | None = None


def chat_prompt(tok, messages: list[dict]) -> list[int]:
    """Token ids of a chat: the tokenizer's chat template with the assistant turn opened,
    or, for a tokenizer without one, ``<|role|>`` headers over the plain text."""
    if hasattr(tok, "apply_chat_template"):
        out = tok.apply_chat_template(messages, add_generation_prompt=True, tokenize=True)
        if hasattr(out, "keys"):  # a BatchEncoding
            out = out["input_ids"]
        return [int(t) for t in out]
    text = "".join(f"<|{m['role']}|>\n{m['content']}\n" for m in messages) + "<|assistant|>\n"
    return tok.encode(text)


def _decoder(tok):
    def decode(ids):
        try:
            return tok.decode(ids, skip_special_tokens=True)
        except TypeError:
            return tok.decode(ids)
    return decode


async def _events(aq: asyncio.Queue, decode, stops: list[str], on_stop):
    """Text deltas of one request from its ``(new_ids, finish_reason)`` updates.  A stop
    string ends the request (``on_stop`` aborts it) and is cut from the text; text that
    could still become a stop string, or ends in an incomplete character, is held back
    until the next update."""
    ids: list[int] = []
    sent = ""
    hold = max((len(x) for x in stops), default=1) - 1
    while True:
        new, reason = await aq.get()
        ids += new
        text = decode(ids)
        cuts = [text.find(x) for x in stops if x and x in text]
        if cuts:
            text = text[:min(cuts)]
            if reason is None:
                on_stop()
            reason = "stop"
        elif reason is None:
            end = len(text) - hold
            while end > len(sent) and text[end - 1:end] == "\ufffd":
                end -= 1
            text = text[:max(end, len(sent))]
        delta = text[len(sent):] if text.startswith(sent) else ""
        sent = text if text.startswith(sent) else sent
        yield delta, new, reason
        if reason is not None:
            return


def create_app(worker: EngineWorker, tokenizer=None, manifests: list | None = None, model_name: str = "oscar-b200",
               vocab_size: int | None = None, eos_token_ids=None, max_model_len: int | None = None,
               sampling_defaults: dict | None = None) -> FastAPI:
    """``eos_token_ids`` end every request that does not set ``ignore_eos`` (default: the
    tokenizer's ``eos_token_id``, if it has one); ``sampling_defaults`` (``temperature``,
    ``top_k``, ``top_p``) fill the fields a request leaves out (default: greedy)."""
    defaults = {"temperature": 0.0, "top_k": 0, "top_p": 1.0, **(sampling_defaults or {})}
    app = FastAPI(title="oscar-b200")
    tok = tokenizer or ByteTokenizer()
    decode = _decoder(tok)
    ids = itertools.count()
    if eos_token_ids is None:
        e = getattr(tokenizer, "eos_token_id", None)
        eos_token_ids = [] if e is None else ([e] if isinstance(e, int) else list(e))
    eos = [int(x) for x in eos_token_ids]

    @app.get("/health")
    def health():
        if worker.error is not None:
            raise HTTPException(503, f"engine failed: {worker.error!r}")
        return {"ok": True}

    @app.get("/ready")
    def ready():
        return {"manifests": manifests or []}

    @app.get("/v1/models")
    def models():
        return {"object": "list", "data": [{"id": model_name, "object": "model", "owned_by": "oscar-b200",
                                            "max_model_len": max_model_len}]}

    @app.get("/metrics", response_class=PlainTextResponse)
    def metrics():
        return worker.metrics.exposition(worker.engine)

    async def generate(prompt: list[int], req, cid: str, chunk, final, lp: int | None = None):
        """Runs one request: ``chunk(text, ids, reason, first)`` builds a streamed event,
        ``final(text, ids, reason, logprobs)`` the plain response (``logprobs``: per output
        token ``(logprob, [(id, logprob), ...])`` when ``lp`` asked for them)."""
        if not prompt:
            raise HTTPException(400, "empty prompt")
        if vocab_size is not None and (min(prompt) < 0 or max(prompt) >= vocab_size):
            raise HTTPException(400, f"token ids must be in [0, {vocab_size})")
        if req.max_tokens < 1:
            raise HTTPException(400, "max_tokens must be >= 1")
        temp = defaults["temperature"] if req.temperature is None else req.temperature
        top_k = defaults["top_k"] if req.top_k is None else req.top_k
        top_p = defaults["top_p"] if req.top_p is None else req.top_p
        sp = None
        if temp > 0:
            sp = SamplingParams(float(temp), max(0, int(top_k)), float(top_p), req.seed)
            try:
                sp.validate()
            except ValueError as e:
                raise HTTPException(400, str(e)) from e
        elif temp < 0:
            raise HTTPException(400, "temperature must be >= 0")
        stops = [req.stop] if isinstance(req.stop, str) else list(req.stop or [])
        stop_ids = list(req.stop_token_ids or []) + ([] if req.ignore_eos else eos)
        loop = asyncio.get_running_loop()
        aq: asyncio.Queue = asyncio.Queue()

        def on_tokens(new, reason):
            if not loop.is_closed():  # the handler may have returned (stop string) before the engine ended
                loop.call_soon_threadsafe(aq.put_nowait, (new, reason))

        if lp is not None and not 0 <= lp <= 20:
            raise HTTPException(400, "logprobs must be in [0, 20]")
        try:
            fut = worker.submit(prompt, req.max_tokens, sp, stop_ids, on_tokens=on_tokens, logprobs=lp)
        except ValueError as e:
            raise HTTPException(400, str(e)) from e
        ended = asyncio.Event()
        fut.add_done_callback(lambda _: None if loop.is_closed() else loop.call_soon_threadsafe(ended.set))

        async def failed():
            """The engine's error once the request's future resolved (None: no error).  The
            future is watched, never awaited: cancelling an awaiting task would cancel it."""
            await ended.wait()
            return None if fut.cancelled() else fut.exception()

        watch = asyncio.ensure_future(failed())
        events = _events(aq, decode, stops, lambda: worker.abort(fut))

        async def next_event():
            """The next text delta, or the engine's error if it failed first."""
            nxt = asyncio.ensure_future(events.__anext__())
            await asyncio.wait({nxt, watch}, return_when=asyncio.FIRST_COMPLETED)
            if not nxt.done():
                err = watch.result()
                if err is not None:
                    nxt.cancel()
                    raise RuntimeError(f"generation failed: {err!r}")
                await nxt  # the future resolved; its last update is already queued
            return nxt.result()

        if req.stream:
            async def sse():
                done = False
                try:
                    reason, first, n_sent = None, True, 0
                    usage = bool((req.stream_options or {}).get("include_usage"))
                    failed = False
                    while reason is None:
                        try:
                            text, new, reason = await next_event()
                        except RuntimeError as e:
                            yield f"data: {json.dumps({'error': str(e)})}\n\n"
                            failed = True
                            break
                        entries = None
                        if lp is not None:  # this chunk's tokens' logprobs, recorded before the update
                            entries = list(getattr(fut, "lp_live", None) or [])[n_sent:n_sent + len(new)]
                        n_sent += len(new)
                        yield f"data: {json.dumps(chunk(text, new, reason, first, entries))}\n\n"
                        first = False
                    if usage and not failed:  # a last chunk with no choices and the token counts
                        last = {**chunk("", [], None, False), "choices": []}
                        last["usage"] = {"prompt_tokens": len(prompt), "completion_tokens": n_sent,
                                         "total_tokens": len(prompt) + n_sent}
                        yield f"data: {json.dumps(last)}\n\n"
                    done = True
                    yield "data: [DONE]\n\n"
                finally:
                    if not done:
                        worker.abort(fut)  # the client went away

            return StreamingResponse(sse(), media_type="text/event-stream")

        text, out, reason = "", [], None
        try:
            while reason is None:
                try:
                    delta, new, reason = await next_event()
                except RuntimeError as e:
                    raise HTTPException(500, str(e)) from e
                text += delta
                out += new
        except asyncio.CancelledError:
            worker.abort(fut)  # the client went away, or a sibling choice failed
            raise
        entries = None
        if lp is not None:
            await watch  # the worker attaches the logprobs when it resolves the future
            entries = (fut.logprobs or [])[:len(out)] if not fut.cancelled() else []
        res = final(text, out, reason, entries)
        res["usage"] = {"prompt_tokens": len(prompt), "completion_tokens": len(out),
                        "total_tokens": len(prompt) + len(out)}
        return res

    async def generate_n(prompt: list[int], req, cid: str, chunk, final, lp: int | None = None):
        """``n`` choices of one prompt: ``n`` requests whose seeds differ (``seed + i``, or the
        per-request default), answered as one response (not with ``stream``)."""
        n = int(req.n or 1)
        if n == 1:
            return await generate(prompt, req, cid, chunk, final, lp)
        if not 1 <= n <= 16:
            raise HTTPException(400, "n must be in [1, 16]")
        if req.stream:
            raise HTTPException(400, "n > 1 is not supported with stream")
        reqs = [req.model_copy(update={"seed": None if req.seed is None else req.seed + i, "n": 1}) for i in range(n)]
        tasks = [asyncio.ensure_future(generate(prompt, r, cid, chunk, final, lp)) for r in reqs]
        try:
            res = await asyncio.gather(*tasks)
        except BaseException:
            # one choice failed or the client went away: the others stop too (their
            # cancellation aborts their engine requests)
            for t in tasks:
                t.cancel()
            raise
        choices = [{**x["choices"][0], "index": i} for i, x in enumerate(res)]
        done = sum(x["usage"]["completion_tokens"] for x in res)
        return {**res[0], "choices": choices,
                "usage": {"prompt_tokens": len(prompt), "completion_tokens": done, "total_tokens": len(prompt) + done}}

    @app.post("/v1/completions")
    async def completions(req: CompletionRequest):
        prompt = tok.encode(req.prompt) if isinstance(req.prompt, str) else list(req.prompt)
        cid, t0 = f"cmpl-{next(ids)}", int(time.time())
        head = {"id": cid, "object": "text_completion", "created": t0, "model": model_name}

        def lp_object(token_ids, entries):  # the completions logprobs object
            return {"tokens": [decode([t]) for t in token_ids[:len(entries)]],
                    "token_logprobs": [e[0] for e in entries],
                    "top_logprobs": [{decode([i]): v for i, v in e[1]} for e in entries]}

        def chunk(text, token_ids, reason, first, entries=None):
            return {**head, "choices": [{"index": 0, "text": text, "token_ids": token_ids,
                                         "logprobs": None if entries is None else lp_object(token_ids, entries),
                                         "finish_reason": reason}]}

        def final(text, token_ids, reason, entries):
            ch = {"index": 0, "text": text, "token_ids": token_ids, "finish_reason": reason}
            if entries is not None:
                ch["logprobs"] = lp_object(token_ids, entries)
            return {**head, "choices": [ch]}

        return await generate_n(prompt, req, cid, chunk, final, req.logprobs)

    @app.post("/v1/chat/completions")
    async def chat(req: ChatRequest):
        if req.max_completion_tokens is not None:
            req = req.model_copy(update={"max_tokens": req.max_completion_tokens})
        prompt = chat_prompt(tok, [m.model_dump() for m in req.messages])
        cid, t0 = f"chatcmpl-{next(ids)}", int(time.time())
        head = {"id": cid, "created": t0, "model": model_name}

        def lp_object(token_ids, entries):  # the chat logprobs object
            return {"content": [{"token": decode([t]), "logprob": e[0],
                                 "top_logprobs": [{"token": decode([i]), "logprob": v} for i, v in e[1]]}
                                for t, e in zip(token_ids, entries)]}

        def chunk(text, token_ids, reason, first, entries=None):
            delta = {"role": "assistant", "content": text} if first else {"content": text}
            ch = {"index": 0, "delta": delta, "finish_reason": reason}
            if entries is not None:
                ch["logprobs"] = lp_object(token_ids, entries)
            return {**head, "object": "chat.completion.chunk", "choices": [ch]}

        def final(text, token_ids, reason, entries):
            ch = {"index": 0, "message": {"role": "assistant", "content": text}, "finish_reason": reason}
            if entries is not None:
                ch["logprobs"] = lp_object(token_ids, entries)
            return {**head, "object": "chat.completion", "choices": [ch]}

        lp = (req.top_logprobs or 0) if req.logprobs else None
        return await generate_n(prompt, req, cid, chunk, final, lp)

    return app
