"""Serving benchmark client: the headline metric measured through the HTTP API.

``python -m oscar_b200.bench.serve_client --url http://127.0.0.1:8000 --concurrency 32
--num-requests 64 --input-len 16384 --output-len 1024``

Sends synthetic requests (uniform-random prompt token ids, seeded, ``ignore_eos`` so every
request produces ``--output-len`` tokens) to ``/v1/completions`` with ``stream: true``,
at most ``--concurrency`` in flight, and measures per request:

* TTFT - from sending the request to the first event that carries tokens;
* TPOT - ``(end - first token) / (output tokens - 1)``;
* ITL - the gaps between token-carrying events (one event per engine step, so with MTP
  a gap covers up to 1 + drafts tokens).

Output tokens are counted from each event's ``token_ids`` (one per text event when a
server sends none), and from the final usage chunk when the server sends one.

Prints one JSON line: output tok/s over the run's wall time, request rate, and mean /
median / p99 of TTFT, TPOT and ITL in milliseconds.  The same measurement the reference's
delivery runs with vLLM's serving benchmark against its OpenAI server (the north star
names output tok/s at 32 concurrent requests, TPOT and TTFT); it works against any
OpenAI-compatible server that streams completions.
"""
from __future__ import annotations

import argparse
import asyncio
import json
import sys
import time
from dataclasses import dataclass, field

import numpy as np


@dataclass
class Result:
    ok: bool = False
    sent: float = 0.0
    first: float | None = None
    end: float = 0.0
    tokens: int = 0
    gaps: list = field(default_factory=list)
    error: str | None = None


def make_prompts(n: int, input_len: int, vocab: int, seed: int) -> list[list[int]]:
    rng = np.random.default_rng(seed)
    return [rng.integers(10, vocab, size=input_len).tolist() for _ in range(n)]


async def _one(client, url: str, body: dict) -> Result:
    res = Result(sent=time.perf_counter())
    last = None
    try:
        async with client.stream("POST", url, json=body) as resp:
            if resp.status_code != 200:
                res.error = f"HTTP {resp.status_code}: {(await resp.aread())[:200]!r}"
                return res
            async for line in resp.aiter_lines():
                if not line.startswith("data: "):
                    continue
                data = line[len("data: "):]
                if data == "[DONE]":
                    break
                ev = json.loads(data)
                if "error" in ev:
                    res.error = str(ev["error"])
                    return res
                if not ev.get("choices"):  # the usage chunk: the server's own token count
                    if ev.get("usage"):
                        res.tokens = int(ev["usage"]["completion_tokens"])
                    continue
                ch = ev["choices"][0]
                n = len(ch.get("token_ids") or []) if "token_ids" in ch else (1 if ch.get("text") else 0)
                if n:
                    now = time.perf_counter()
                    if res.first is None:
                        res.first = now
                    else:
                        res.gaps.append(now - last)
                    last = now
                    res.tokens += n
        res.end = time.perf_counter()
        res.ok = res.first is not None
    except Exception as e:  # noqa: BLE001 - reported per request
        res.error = repr(e)
    return res


async def run(url: str, prompts: list, output_len: int, concurrency: int, temperature: float = 0.0,
              transport=None, timeout_s: float = 3600.0) -> dict:
    import httpx

    sem = asyncio.Semaphore(concurrency)
    endpoint = url.rstrip("/") + "/v1/completions"

    async with httpx.AsyncClient(transport=transport, timeout=timeout_s) as client:
        async def bounded(p):
            async with sem:
                body = {"prompt": p, "max_tokens": output_len, "stream": True, "ignore_eos": True,
                        "temperature": temperature, "stream_options": {"include_usage": True}}
                return await _one(client, endpoint, body)

        t0 = time.perf_counter()
        results = await asyncio.gather(*(bounded(p) for p in prompts))
        wall = time.perf_counter() - t0
    return summarize(results, wall, concurrency)


def _stats(xs) -> dict:
    if not len(xs):
        return {"mean": None, "median": None, "p99": None}
    a = np.asarray(xs) * 1e3
    return {"mean": round(float(a.mean()), 3), "median": round(float(np.median(a)), 3),
            "p99": round(float(np.percentile(a, 99)), 3)}


def summarize(results: list, wall: float, concurrency: int) -> dict:
    ok = [r for r in results if r.ok]
    out_tok = sum(r.tokens for r in ok)
    tpot = [(r.end - r.first) / (r.tokens - 1) for r in ok if r.tokens > 1]
    return {
        "metric": "output tok/s, TTFT, TPOT through the HTTP API", "concurrency": concurrency,
        "requests": len(results), "completed": len(ok), "failed": len(results) - len(ok),
        "errors": sorted({r.error for r in results if r.error})[:3],
        "wall_s": round(wall, 3), "output_tokens": out_tok,
        "output_tok_per_s": round(out_tok / wall, 2) if wall > 0 else None,
        "request_per_s": round(len(ok) / wall, 4) if wall > 0 else None,
        "ttft_ms": _stats([r.first - r.sent for r in ok]), "tpot_ms": _stats(tpot),
        "itl_ms": _stats([g for r in ok for g in r.gaps]),
    }


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="python -m oscar_b200.bench.serve_client")
    ap.add_argument("--url", default="http://127.0.0.1:8000")
    ap.add_argument("--concurrency", type=int, default=32)
    ap.add_argument("--num-requests", type=int, default=64)
    ap.add_argument("--input-len", type=int, default=16384)
    ap.add_argument("--output-len", type=int, default=1024)
    ap.add_argument("--vocab", type=int, default=248320, help="prompt token ids are drawn below this")
    ap.add_argument("--temperature", type=float, default=0.0)
    ap.add_argument("--seed", type=int, default=0)
    args = ap.parse_args(argv)
    prompts = make_prompts(args.num_requests, args.input_len, args.vocab, args.seed)
    out = asyncio.run(run(args.url, prompts, args.output_len, args.concurrency, args.temperature))
    out["config"] = {"input_len": args.input_len, "output_len": args.output_len, "seed": args.seed,
                     "data": "synthetic (uniform-random prompt token ids)"}
    print(json.dumps(out), flush=True)
    return 0 if out["failed"] == 0 else 1


if __name__ == "__main__":
    sys.exit(main())
