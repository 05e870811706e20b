"""Data-parallel request router: one HTTP endpoint in front of several engine replicas.

BASELINE config 5 runs DP2 x TP4 on 8 GPUs; the reference rejects DP != 1
(``oscar_ascend/integration.py:75-76``).  Here every DP replica is an independent
TP serve group (``python -m oscar_b200.serve`` on its own port) and this router
forwards each completion or chat completion (streamed ones as a pass-through of the
replica's server-sent events) to the replica with the least outstanding work: prompt +
requested tokens of the requests it has sent there and not yet seen answered, ties
broken by replica index (deterministic, so a replayed trace lands identically).

    python -m oscar_b200.serve.router --backends http://127.0.0.1:8000,http://127.0.0.1:8001 --port 9000
"""
from __future__ import annotations

import argparse
import threading

import httpx
from fastapi import FastAPI, HTTPException, Request
from fastapi.responses import StreamingResponse


class DPRouter:
    """Least-outstanding-tokens assignment over ``n`` replicas."""

    def __init__(self, n: int):
        if n < 1:
            raise ValueError("need at least one replica")
        self.load = [0] * n
        self.sent = [0] * n
        self._lock = threading.Lock()

    def acquire(self, cost: int) -> int:
        with self._lock:
            i = min(range(len(self.load)), key=lambda j: (self.load[j], j))
            self.load[i] += cost
            self.sent[i] += 1
            return i

    def release(self, i: int, cost: int) -> None:
        with self._lock:
            self.load[i] -= cost


def request_cost(body: dict) -> int:
    if "messages" in body:
        n = sum(len(str(m.get("content", "")).encode()) for m in body["messages"])
    else:
        p = body.get("prompt", [])
        n = len(p) if isinstance(p, list) else len(str(p).encode())
    return n + int(body.get("max_tokens", 16)) * max(1, int(body.get("n", 1) or 1))


def create_router_app(backends: list[str], transport: httpx.AsyncBaseTransport | None = None,
                      timeout_s: float = 3600.0) -> FastAPI:
    app = FastAPI(title="oscar-b200 router")
    router = DPRouter(len(backends))
    client = httpx.AsyncClient(transport=transport, timeout=timeout_s)

    @app.get("/health")
    async def health():
        return {"ok": True, "replicas": len(backends), "load": router.load, "sent": router.sent}

    async def forward(path: str, req: Request):
        body = await req.json()
        cost = request_cost(body)
        i = router.acquire(cost)
        url = backends[i].rstrip("/") + path
        if body.get("stream"):
            # server-sent events pass through as they come; the replica's load is
            # released when the stream ends (or the client goes away)
            try:
                r = await client.send(client.build_request("POST", url, json=body), stream=True)
            except httpx.HTTPError as e:
                router.release(i, cost)
                raise HTTPException(502, f"replica {i} unreachable: {e!r}") from e
            if r.status_code != 200:
                text = (await r.aread()).decode(errors="replace")
                await r.aclose()
                router.release(i, cost)
                raise HTTPException(r.status_code, text)

            async def relay():
                try:
                    async for part in r.aiter_bytes():
                        yield part
                finally:
                    await r.aclose()
                    router.release(i, cost)

            return StreamingResponse(relay(), media_type="text/event-stream", headers={"x-replica": str(i)})
        try:
            r = await client.post(url, json=body)
        except httpx.HTTPError as e:
            raise HTTPException(502, f"replica {i} unreachable: {e!r}") from e
        finally:
            router.release(i, cost)
        if r.status_code != 200:
            raise HTTPException(r.status_code, r.text)
        out = r.json()
        out["replica"] = i
        return out

    @app.get("/v1/models")
    async def models():
        try:
            r = await client.get(backends[0].rstrip("/") + "/v1/models")
        except httpx.HTTPError as e:
            raise HTTPException(502, f"replica 0 unreachable: {e!r}") from e
        return r.json()

    @app.post("/v1/completions")
    async def completions(req: Request):
        return await forward("/v1/completions", req)

    @app.post("/v1/chat/completions")
    async def chat(req: Request):
        return await forward("/v1/chat/completions", req)

    app.state.router = router
    return app


def main(argv=None) -> int:
    import uvicorn

    ap = argparse.ArgumentParser(prog="python -m oscar_b200.serve.router")
    ap.add_argument("--backends", required=True)
    ap.add_argument("--host", default="127.0.0.1")
    ap.add_argument("--port", type=int, default=9000)
    args = ap.parse_args(argv)
    uvicorn.run(create_router_app(args.backends.split(",")), host=args.host, port=args.port)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
