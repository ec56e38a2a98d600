"""HTTP server: SGLang-native `/generate` plus the OpenAI-compatible `/v1/completions` and
`/v1/chat/completions` (streaming by server-sent events), model/server info, health, prefix-cache flush,
Prometheus `/metrics` and a profiler window (`/start_profile`, `/stop_profile`).

    python -m sglang_neuron_b200.entrypoints.http_server --model gpt-oss-120b --tp-size 1 --port 30000

Parity: the reference serves through SGLang's HTTP server (L7 of its layer map) with its platform plugged
in; this build owns that layer because it is a standalone engine.
"""
import argparse
import asyncio
import dataclasses
import json
import logging
import os
import time
import uuid
from typing import Any, Dict, List, Optional

from ..managers.schedule_batch import SamplingParams
from ..engine import trim_at_stop
from ..server_args import ServerArgs

try:  # FastAPI resolves handler annotations from module globals
    from fastapi import FastAPI, Request
    from fastapi.responses import JSONResponse, PlainTextResponse, StreamingResponse
except ImportError:  # pragma: no cover
    FastAPI = Request = None

logger = logging.getLogger(__name__)


def _sampling_from_openai(body: Dict[str, Any]) -> SamplingParams:
    return SamplingParams(
        max_new_tokens=int(body.get("max_tokens") or body.get("max_completion_tokens") or 128),
        temperature=float(body.get("temperature", 1.0) if body.get("temperature") is not None else 1.0),
        top_k=int(body.get("top_k") or 0), top_p=float(body.get("top_p") if body.get("top_p") is not None else 1.0),
        seed=body.get("seed"), stop_token_ids=body.get("stop_token_ids"), ignore_eos=bool(body.get("ignore_eos", False)),
        return_logprob=_openai_logprobs(body)[0], top_logprobs_num=_openai_logprobs(body)[1],
        stop=([body["stop"]] if isinstance(body.get("stop"), str) else (body.get("stop") or None)))


def _openai_logprobs(body: Dict[str, Any]):
    """(return_logprob, top-k) of an OpenAI request: completions take `logprobs: int` (top-k), chat takes
    `logprobs: bool` plus `top_logprobs: int`."""
    lp = body.get("logprobs")
    if isinstance(lp, bool):
        return lp, int(body.get("top_logprobs") or 0) if lp else 0
    if isinstance(lp, int):
        return True, lp
    return False, 0


def build_app(engine, loop_holder: Dict[str, Any]):
    from .engine_loop import EngineLoop
    from ..utils.metrics import Metrics

    app = FastAPI(title="sglang_neuron_b200")
    metrics = Metrics()
    state: Dict[str, Any] = {"profiler": None}

    def loop() -> EngineLoop:
        if "loop" not in loop_holder:
            loop_holder["loop"] = EngineLoop(engine)
        return loop_holder["loop"]

    def encode(prompt) -> List[int]:
        if isinstance(prompt, list):
            return [int(t) for t in prompt]
        if engine.tokenizer is None:
            raise ValueError("this server has no tokenizer; send token ids (input_ids / prompt as a list)")
        return engine.tokenizer.encode(prompt)

    def decode(ids: List[int]) -> str:
        if engine.tokenizer is None:
            return ""
        return engine.tokenizer.decode(ids)

    async def run(ids: List[int], sp: SamplingParams, rid: Optional[str] = None):
        if sp.stop and engine.tokenizer is None:
            raise ValueError("text stop sequences need a tokenizer; use stop_token_ids")
        rid, st = loop().submit(ids, sp, rid)
        metrics.requests_total.inc()
        t0 = time.perf_counter()
        first = True
        done = False
        try:
            while True:
                item = await st.queue.get()
                if "error" in item:
                    done = True
                    raise ValueError(item["error"])
                if first and item.get("new_ids"):
                    metrics.ttft.observe(time.perf_counter() - t0)
                    first = False
                metrics.tokens_total.inc(len(item.get("new_ids", [])))
                yield item
                if item.get("finished"):
                    done = True
                    metrics.e2e.observe(time.perf_counter() - t0)
                    return
        finally:
            if not done:  # the client went away (or the handler was cancelled): stop generating
                loop().abort(rid)

    @app.get("/health")
    async def health():
        return PlainTextResponse("ok")

    @app.get("/health_generate")
    async def health_generate():
        async for _ in run([1, 2, 3], SamplingParams(max_new_tokens=1)):
            pass
        return PlainTextResponse("ok")

    @app.get("/get_model_info")
    async def model_info():
        return {"model_path": engine.args.model, "architecture": engine.cfg.architecture,
                "is_generation": True, "config": engine.cfg.to_dict()}

    @app.get("/get_server_info")
    async def server_info():
        d = {k: v for k, v in vars(engine.args).items()}
        d["scheduler_stats"] = dict(engine.scheduler.stats)
        d["kv_pages"] = engine.runner.num_pages
        from .. import sglang_tree
        d["parallel"] = sglang_tree.parallel_of()
        d["rank_label"] = sglang_tree.rank_label()
        d["serving_policy"] = dataclasses.asdict(engine.policy) if getattr(engine, "policy", None) else None
        return d

    @app.get("/v1/models")
    async def models():
        return {"object": "list", "data": [{"id": engine.args.model, "object": "model", "owned_by": "sglang_neuron_b200"}]}

    @app.post("/flush_cache")
    async def flush_cache():
        engine.flush_cache()
        return PlainTextResponse("cache flushed")

    @app.get("/metrics")
    async def prom():
        metrics.update_from(engine)
        return PlainTextResponse(metrics.render(), media_type="text/plain; version=0.0.4")

    @app.post("/start_profile")
    async def start_profile(req: Request):
        body = await req.json() if (await req.body()) else {}
        from ..utils.profiling import ProfileWindow
        state["profiler"] = ProfileWindow(body.get("output_dir", "/tmp/snb_profile"), body.get("num_steps"))
        state["profiler"].start()
        return PlainTextResponse("profiling started")

    @app.post("/stop_profile")
    async def stop_profile():
        p = state.get("profiler")
        if p is None:
            return PlainTextResponse("no profile running", status_code=400)
        path = p.stop()
        state["profiler"] = None
        return {"trace": path}

    @app.post("/abort_request")
    async def abort_request(req: Request):
        body = await req.json()
        loop().abort(str(body["rid"]))
        return {"success": True}

    @app.post("/generate")
    async def generate(req: Request):
        body = await req.json()
        try:
            ids = encode(body["input_ids"] if "input_ids" in body else body["text"])
        except (KeyError, ValueError) as e:
            return JSONResponse({"error": str(e)}, status_code=400)
        sp = SamplingParams.from_dict(body.get("sampling_params"))
        if body.get("return_logprob"):  # SGLang puts these at the request level
            sp.return_logprob = True
            sp.top_logprobs_num = int(body.get("top_logprobs_num") or sp.top_logprobs_num or 0)

        def logprob_meta(lps, tops, toks):
            m = {"output_token_logprobs": [[lp, t, None] for lp, t in zip(lps, toks)]}
            if sp.top_logprobs_num > 0:
                m["output_top_logprobs"] = [[[lp, t, None] for lp, t in row] for row in tops]
            return m

        if body.get("stream"):
            async def sse():
                acc: List[int] = []
                lps, tops = [], []
                async for item in run(ids, sp, body.get("rid")):
                    acc += item["new_ids"]
                    lps += item.get("new_logprobs", [])
                    tops += item.get("new_top_logprobs", [])
                    meta = {"finish_reason": item["finish_reason"], "completion_tokens": item["completion_tokens"]}
                    if sp.return_logprob:
                        meta.update(logprob_meta(lps, tops, acc))
                    out = {"text": trim_at_stop(decode(acc), sp.stop), "output_ids": list(acc), "meta_info": meta}
                    yield f"data: {json.dumps(out)}\n\n"
                yield "data: [DONE]\n\n"
            return StreamingResponse(sse(), media_type="text/event-stream")
        acc: List[int] = []
        lps, tops = [], []
        last = None
        try:
            async for item in run(ids, sp, body.get("rid")):
                acc += item["new_ids"]
                lps += item.get("new_logprobs", [])
                tops += item.get("new_top_logprobs", [])
                last = item
        except ValueError as e:
            return JSONResponse({"error": str(e)}, status_code=400)
        meta = {"prompt_tokens": last["prompt_tokens"], "completion_tokens": last["completion_tokens"],
                "cached_tokens": last["cached_tokens"], "finish_reason": last["finish_reason"]}
        if sp.return_logprob:
            meta.update(logprob_meta(lps, tops, acc))
        return {"text": trim_at_stop(decode(acc), sp.stop), "output_ids": acc, "meta_info": meta}

    async def _openai(body, ids, chat: bool):
        sp = _sampling_from_openai(body)
        created = int(time.time())
        cid = ("chatcmpl-" if chat else "cmpl-") + uuid.uuid4().hex[:16]
        obj = "chat.completion" if chat else "text_completion"
        if body.get("stream"):
            async def sse():
                async for item in run(ids, sp):
                    text = decode(item["new_ids"])
                    if chat:
                        choice = {"index": 0, "delta": {"content": text}, "finish_reason": item["finish_reason"]}
                    else:
                        choice = {"index": 0, "text": text, "finish_reason": item["finish_reason"],
                                  "token_ids": item["new_ids"]}
                    yield "data: " + json.dumps({"id": cid, "object": obj + ".chunk", "created": created,
                                                 "model": engine.args.model, "choices": [choice]}) + "\n\n"
                yield "data: [DONE]\n\n"
            return StreamingResponse(sse(), media_type="text/event-stream")
        async def one(index: int, spi: SamplingParams):
            acc: List[int] = []
            lps, tops = [], []
            last = None
            async for item in run(ids, spi):
                acc += item["new_ids"]
                lps += item.get("new_logprobs", [])
                tops += item.get("new_top_logprobs", [])
                last = item
            text = trim_at_stop(decode(acc), spi.stop)
            choice = ({"index": index, "message": {"role": "assistant", "content": text},
                       "finish_reason": last["finish_reason"]}
                      if chat else {"index": index, "text": text, "finish_reason": last["finish_reason"],
                                    "token_ids": acc})
            if spi.return_logprob:
                tok = (lambda t: decode([t]) if engine.tokenizer is not None else str(t))
                if chat:
                    choice["logprobs"] = {"content": [
                        {"token": tok(t), "logprob": lp, "bytes": None,
                         "top_logprobs": [{"token": tok(tt), "logprob": tl}
                                          for tl, tt in (tops[i] if i < len(tops) else [])]}
                        for i, (lp, t) in enumerate(zip(lps, acc))]}
                else:
                    choice["logprobs"] = {"tokens": [tok(t) for t in acc], "token_logprobs": lps,
                                          "top_logprobs": [{tok(tt): tl for tl, tt in row} for row in tops] or None,
                                          "text_offset": None}
            return choice, last

        n = max(1, int(body.get("n") or 1))
        sps = []
        for i in range(n):  # n samples: distinct seeds (seed + i when a seed is given)
            spi = dataclasses.replace(sp)
            if sp.seed is not None:
                spi.seed = sp.seed + i
            sps.append(spi)
        results = await asyncio.gather(*[one(i, spi) for i, spi in enumerate(sps)])
        choices = [c for c, _ in results]
        last = results[0][1]
        completion = sum(l["completion_tokens"] for _, l in results)
        return {"id": cid, "object": obj, "created": created, "model": engine.args.model, "choices": choices,
                "usage": {"prompt_tokens": last["prompt_tokens"], "completion_tokens": completion,
                          "total_tokens": last["prompt_tokens"] + completion}}


    @app.post("/v1/completions")
    async def completions(req: Request):
        body = await req.json()
        try:
            ids = encode(body.get("prompt", ""))
            return await _openai(body, ids, chat=False)
        except ValueError as e:
            return JSONResponse({"error": {"message": str(e)}}, status_code=400)

    @app.post("/v1/chat/completions")
    async def chat(req: Request):
        body = await req.json()
        if engine.tokenizer is None:
            return JSONResponse({"error": {"message": "chat needs a tokenizer with a chat template"}}, status_code=400)
        try:
            ids = engine.tokenizer.apply_chat_template(body["messages"], add_generation_prompt=True)
            return await _openai(body, list(ids), chat=True)
        except ValueError as e:
            return JSONResponse({"error": {"message": str(e)}}, status_code=400)

    return app


def main(argv=None):
    p = argparse.ArgumentParser("sglang_neuron_b200 server")
    ServerArgs.add_cli_args(p)
    ns = p.parse_args(argv)
    args = ServerArgs.from_cli(ns)
    logging.basicConfig(level=getattr(logging, args.log_level.upper(), logging.INFO))
    from ..process_init import install_clean_exit
    install_clean_exit()
    from ..engine import Engine
    engine = Engine(args)
    if engine.rank != 0:
        # follower ranks of a TP group: run the scheduler in lockstep, rank 0 owns intake
        engine.scheduler.on_token = None
        while True:
            engine.scheduler.step()
    import uvicorn
    app = build_app(engine, {})
    uvicorn.run(app, host=args.host, port=args.port, log_level=args.log_level)


if __name__ == "__main__":
    main()
