"""Request balancer: one HTTP endpoint in front of several serving replicas (aggregated servers, or the
prefill/decode groups of a disaggregated deployment that each expose the serving API).

Each request goes to the backend with the fewest outstanding requests (ties rotate). A connection failure
before any response byte moves the request to the next backend (up to --retries); streaming responses
are passed through chunk by chunk. `/get_server_info` reports per-backend outstanding/served/failed counts.

    python -m sglang_neuron_b200.disaggregation.balancer --backends http://127.0.0.1:30000 \\
        http://127.0.0.1:30001 --port 8000

Parity: the reference's disaggregation/balancer.py (`Backends` :90, `_Attempt` :248): sends each request
to the prefill replica with the fewest outstanding requests, SSE pass-through, retries, trace.
"""

import argparse
import itertools
import logging
from typing import Dict, List, Optional

logger = logging.getLogger(__name__)


class Backends:
    def __init__(self, urls: List[str]):
        if not urls:
            raise ValueError("the balancer needs at least one backend")
        self.urls = [u.rstrip("/") for u in urls]
        self.outstanding: Dict[str, int] = {u: 0 for u in self.urls}
        self.served: Dict[str, int] = {u: 0 for u in self.urls}
        self.failed: Dict[str, int] = {u: 0 for u in self.urls}
        self._rr = itertools.count()

    def order(self) -> List[str]:
        """Backends by outstanding requests (fewest first), ties rotated."""
        k = next(self._rr)
        n = len(self.urls)
        rot = [self.urls[(k + i) % n] for i in range(n)]
        return sorted(rot, key=lambda u: self.outstanding[u])

    def info(self) -> Dict:
        return {u: {"outstanding": self.outstanding[u], "served": self.served[u], "failed": self.failed[u]}
                for u in self.urls}


def build_app(urls: List[str], retries: int = 2):
    import aiohttp
    from fastapi import FastAPI, Request
    from fastapi.responses import JSONResponse, Response, StreamingResponse

    app = FastAPI(title="sglang_neuron_b200 balancer")
    be = Backends(urls)
    state: Dict[str, Optional[aiohttp.ClientSession]] = {"session": None}

    def session():
        if state["session"] is None:
            state["session"] = aiohttp.ClientSession(timeout=aiohttp.ClientTimeout(total=None))
        return state["session"]

    @app.on_event("shutdown")
    async def _close():
        if state["session"] is not None:
            await state["session"].close()

    async def forward(path: str, body: dict):
        stream = bool(body.get("stream"))
        last_err = None
        for url in be.order()[: max(1, retries + 1)]:
            be.outstanding[url] += 1
            try:
                resp = await session().post(url + path, json=body)
            except aiohttp.ClientError as e:  # nothing was sent back: try the next backend
                be.outstanding[url] -= 1
                be.failed[url] += 1
                last_err = f"{url}: {e!r}"
                logger.warning("backend failed before responding: %s", last_err)
                continue
            if not stream:
                try:
                    data = await resp.read()
                    be.served[url] += 1
                    return Response(content=data, status_code=resp.status,
                                    media_type=resp.headers.get("content-type", "application/json"))
                finally:
                    resp.release()
                    be.outstanding[url] -= 1

            async def relay(resp=resp, url=url):
                try:
                    async for chunk in resp.content.iter_any():
                        yield chunk
                    be.served[url] += 1
                finally:
                    resp.release()
                    be.outstanding[url] -= 1
            return StreamingResponse(relay(), status_code=resp.status, media_type="text/event-stream")
        return JSONResponse({"error": f"no backend answered ({last_err})"}, status_code=503)

    @app.post("/generate")
    async def generate(req: Request):
        return await forward("/generate", await req.json())

    @app.post("/v1/completions")
    async def completions(req: Request):
        return await forward("/v1/completions", await req.json())

    @app.post("/v1/chat/completions")
    async def chat(req: Request):
        return await forward("/v1/chat/completions", await req.json())

    @app.get("/health")
    async def health():
        return Response(content="ok", media_type="text/plain")

    @app.get("/get_server_info")
    async def info():
        return {"backends": be.info()}

    app.state.backends = be
    return app


def main(argv=None):
    p = argparse.ArgumentParser("balancer")
    p.add_argument("--backends", nargs="+", required=True)
    p.add_argument("--host", default="127.0.0.1")
    p.add_argument("--port", type=int, default=8000)
    p.add_argument("--retries", type=int, default=2)
    a = p.parse_args(argv)
    import uvicorn
    uvicorn.run(build_app(a.backends, a.retries), host=a.host, port=a.port, log_level="info")


if __name__ == "__main__":
    main()
