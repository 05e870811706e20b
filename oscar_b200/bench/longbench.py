"""Long-context multiple-choice evaluation through the chat API (LongBench v2 format).

``python -m oscar_b200.bench.longbench --data longbench_v2.jsonl --url http://127.0.0.1:8000
--concurrency 32``

The reference's end-to-end figures are an evaluation of this kind: LongBench v2 at 32
concurrent requests, reported as total wall time, seconds per case and accuracy
(``plan/audits/END_TO_END_SLOWNESS_AND_PLAN-20260908.md:13-22``).  Each record of
``--data`` (JSON lines or a JSON list) has the LongBench v2 fields ``context``,
``question``, ``choice_A`` .. ``choice_D`` and ``answer`` (optional: ``_id``,
``difficulty``, ``length``).  The prompt is the benchmark's zero-shot template (read the
text, answer the question, reply "The correct answer is (X)"); contexts longer than
``--max-context-chars`` keep their first and last halves.  Requests go to
``/v1/chat/completions`` greedily; the answer is the letter after "The correct answer
is", else the last standalone A-D in the reply.

Prints one JSON line: cases, completed, failed, wall seconds, seconds per case, accuracy
(over all cases; a failed request counts as wrong) and accuracy per difficulty / length.
"""
from __future__ import annotations

import argparse
import asyncio
import json
import re
import sys
import time

TEMPLATE = (
    "Please read the following text and answer the question below.\n\n<text>\n{context}\n</text>\n\n"
    "What is the correct answer to this question: {question}\nChoices:\n(A) {A}\n(B) {B}\n(C) {C}\n(D) {D}\n\n"
    'Format your response as follows: "The correct answer is (insert answer here)".')

_ANSWER = re.compile(r"The correct answer is \(?([A-D])\)?")
_LETTER = re.compile(r"\b([A-D])\b")


def load(path: str, limit: int | None = None) -> list[dict]:
    with open(path) as f:
        text = f.read()
    rows = json.loads(text) if text.lstrip().startswith("[") else [json.loads(ln) for ln in text.splitlines()
                                                                     if ln.strip()]
    return rows[:limit] if limit else rows


def middle_truncate(text: str, max_chars: int | None) -> str:
    if not max_chars or len(text) <= max_chars:
        return text
    half = max_chars // 2
    return text[:half] + text[len(text) - (max_chars - half):]


def prompt_of(rec: dict, max_chars: int | None = None) -> str:
    return TEMPLATE.format(context=middle_truncate(rec["context"], max_chars), question=rec["question"],
                           A=rec["choice_A"], B=rec["choice_B"], C=rec["choice_C"], D=rec["choice_D"])


def extract(reply: str) -> str | None:
    m = _ANSWER.search(reply)
    if m:
        return m.group(1)
    letters = _LETTER.findall(reply)
    return letters[-1] if letters else None


async def _ask(client, url: str, rec: dict, max_chars, max_tokens: int) -> dict:
    body = {"messages": [{"role": "user", "content": prompt_of(rec, max_chars)}], "max_tokens": max_tokens,
            "temperature": 0.0}
    t0 = time.perf_counter()
    try:
        r = await client.post(url, json=body)
        if r.status_code != 200:
            return {"ok": False, "error": f"HTTP {r.status_code}", "s": time.perf_counter() - t0}
        reply = r.json()["choices"][0]["message"]["content"]
        return {"ok": True, "pred": extract(reply), "s": time.perf_counter() - t0,
                "tokens": r.json().get("usage", {}).get("completion_tokens")}
    except Exception as e:  # noqa: BLE001 - counted as a failed case
        return {"ok": False, "error": repr(e), "s": time.perf_counter() - t0}


async def run(url: str, records: list[dict], concurrency: int = 32, max_chars: int | None = None,
              max_tokens: int = 128, transport=None, timeout_s: float = 3600.0) -> dict:
    import httpx

    sem = asyncio.Semaphore(concurrency)
    endpoint = url.rstrip("/") + "/v1/chat/completions"
    async with httpx.AsyncClient(transport=transport, timeout=timeout_s) as client:
        async def bounded(rec):
            async with sem:
                return await _ask(client, endpoint, rec, max_chars, max_tokens)

        t0 = time.perf_counter()
        res = await asyncio.gather(*(bounded(r) for r in records))
        wall = time.perf_counter() - t0
    return summarize(records, res, wall, concurrency)


def summarize(records: list[dict], results: list[dict], wall: float, concurrency: int) -> dict:
    n = len(records)
    right = [bool(res.get("ok") and res.get("pred") == rec.get("answer")) for rec, res in zip(records, results)]
    groups: dict = {}
    for key in ("difficulty", "length"):
        for rec, ok in zip(records, right):
            if key in rec:
                g = groups.setdefault(f"{key}={rec[key]}", [0, 0])
                g[0] += ok
                g[1] += 1
    tokens = [res["tokens"] for res in results if res.get("tokens") is not None]
    return {"metric": "long-context multiple-choice eval through the chat API", "concurrency": concurrency,
            "cases": n, "completed": sum(1 for r in results if r.get("ok")),
            "failed": sum(1 for r in results if not r.get("ok")), "wall_s": round(wall, 3),
            "s_per_case": round(wall / max(1, n), 3), "accuracy": round(sum(right) / max(1, n), 4),
            "accuracy_by": {k: round(a / b, 4) for k, (a, b) in sorted(groups.items())},
            "completion_tokens": sum(tokens) if tokens else None,
            "errors": sorted({r["error"] for r in results if r.get("error")})[:3]}


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="python -m oscar_b200.bench.longbench")
    ap.add_argument("--data", required=True, help="LongBench v2 records (JSON lines or a JSON list)")
    ap.add_argument("--url", default="http://127.0.0.1:8000")
    ap.add_argument("--concurrency", type=int, default=32)
    ap.add_argument("--limit", type=int, default=None)
    ap.add_argument("--max-context-chars", type=int, default=None, help="middle-truncate longer contexts")
    ap.add_argument("--max-tokens", type=int, default=128)
    args = ap.parse_args(argv)
    recs = load(args.data, args.limit)
    out = asyncio.run(run(args.url, recs, args.concurrency, args.max_context_chars, args.max_tokens))
    print(json.dumps(out), flush=True)
    return 0 if out["failed"] == 0 else 1


if __name__ == "__main__":
    sys.exit(main())
