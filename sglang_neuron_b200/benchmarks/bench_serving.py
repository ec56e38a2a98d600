"""Online serving benchmark: drives a running server over HTTP at a fixed concurrency and reports output
throughput, TTFT, TPOT and ITL (the metrics of the reference's headline table).

    python -m sglang_neuron_b200.benchmarks.bench_serving --base-url http://127.0.0.1:30000 \\
        --num-prompts 256 --concurrency 64 --input-len 1024 --output-len 1024 --output-file runs.jsonl

Requests are random token-id prompts sent to `/generate` with streaming on and `ignore_eos`, so every
request produces exactly its output length. Each server-sent chunk carries the tokens of one or more engine
steps; the arrival time of a chunk is attributed to every token in it (ITL = chunk gap / tokens in it).
One JSON line per run is printed and, with --output-file, appended to a JSONL file that
`benchmarks/bench_report.py` renders.

Parity: the reference benchmarks with upstream `sglang.bench_serving` and renders the JSONL with
tools/bench_report.py (output tok/s, TTFT and TPOT median/p99, ITL, versus concurrency).
"""
from __future__ import annotations

import argparse
import asyncio
import json
import random
import statistics
import time
from dataclasses import dataclass, field
from typing import Awaitable, Callable, Dict, List, Optional


@dataclass
class RequestResult:
    prompt_len: int
    output_len: int = 0
    ttft: Optional[float] = None          # seconds to the first generated token
    latency: float = 0.0                  # seconds to the last chunk
    itls: List[float] = field(default_factory=list)
    ok: bool = True
    error: str = ""


def percentile(xs: List[float], q: float) -> Optional[float]:
    if not xs:
        return None
    s = sorted(xs)
    k = (len(s) - 1) * q
    lo, hi = int(k), min(int(k) + 1, len(s) - 1)
    return s[lo] + (s[hi] - s[lo]) * (k - lo)


def summarize(results: List[RequestResult], duration: float, concurrency: int) -> Dict:
    ok = [r for r in results if r.ok]
    out_tok = sum(r.output_len for r in ok)
    in_tok = sum(r.prompt_len for r in ok)
    ttfts = [r.ttft * 1e3 for r in ok if r.ttft is not None]
    tpots = [(r.latency - r.ttft) / (r.output_len - 1) * 1e3 for r in ok
             if r.ttft is not None and r.output_len > 1]
    itls = [x * 1e3 for r in ok for x in r.itls]
    lat = [r.latency * 1e3 for r in ok]

    def rnd(v):
        return None if v is None else round(v, 3)

    return {
        "concurrency": concurrency, "completed": len(ok), "failed": len(results) - len(ok),
        "duration_s": round(duration, 3), "request_throughput": round(len(ok) / duration, 3),
        "input_tok_s": round(in_tok / duration, 1), "output_tok_s": round(out_tok / duration, 1),
        "total_output_tokens": out_tok,
        "ttft_ms_mean": rnd(statistics.fmean(ttfts)) if ttfts else None, "ttft_ms_p50": rnd(percentile(ttfts, 0.5)),
        "ttft_ms_p99": rnd(percentile(ttfts, 0.99)),
        "tpot_ms_p50": rnd(percentile(tpots, 0.5)), "tpot_ms_p99": rnd(percentile(tpots, 0.99)),
        "itl_ms_p50": rnd(percentile(itls, 0.5)), "itl_ms_p99": rnd(percentile(itls, 0.99)),
        "e2e_ms_p50": rnd(percentile(lat, 0.5)),
    }


def make_prompts(n: int, input_len: int, output_len: int, vocab: int, ratio: float, seed: int):
    """(prompt ids, output length) pairs; lengths uniform in [ratio * len, len]."""
    rng = random.Random(seed)
    out = []
    for _ in range(n):
        il = max(1, int(rng.uniform(ratio, 1.0) * input_len))
        ol = max(1, int(rng.uniform(ratio, 1.0) * output_len))
        out.append(([rng.randrange(1, vocab) for _ in range(il)], ol))
    return out


async def _stream_generate(session, url: str, ids: List[int], out_len: int) -> RequestResult:
    res = RequestResult(prompt_len=len(ids))
    body = {"input_ids": ids, "stream": True,
            "sampling_params": {"max_new_tokens": out_len, "temperature": 0.0, "ignore_eos": True}}
    t0 = time.perf_counter()
    last_t, seen = t0, 0
    try:
        async with session.post(url + "/generate", json=body) as resp:
            if resp.status != 200:
                res.ok, res.error = False, f"HTTP {resp.status}: {await resp.text()}"
                return res
            buf = b""
            async for chunk in resp.content.iter_any():
                buf += chunk
                while b"\n\n" in buf:
                    line, buf = buf.split(b"\n\n", 1)
                    line = line.strip()
                    if not line.startswith(b"data: ") or line == b"data: [DONE]":
                        continue
                    item = json.loads(line[6:])
                    now = time.perf_counter()
                    n = len(item.get("output_ids", []))
                    new = n - seen
                    if new > 0:
                        if seen == 0:
                            res.ttft = now - t0
                            new -= 1  # the first token's gap is the TTFT
                        if new > 0:
                            res.itls += [(now - last_t) / new] * new
                        seen, last_t = n, now
    except Exception as e:  # connection errors count as failed requests
        res.ok, res.error = False, repr(e)
    res.output_len = seen
    res.latency = time.perf_counter() - t0
    return res


async def run_benchmark(base_url: str, prompts, concurrency: int,
                        send: Optional[Callable[..., Awaitable[RequestResult]]] = None) -> Dict:
    import aiohttp
    send = send or _stream_generate
    sem = asyncio.Semaphore(concurrency)
    timeout = aiohttp.ClientTimeout(total=None)
    async with aiohttp.ClientSession(timeout=timeout) as session:
        async def one(ids, ol):
            async with sem:
                return await send(session, base_url, ids, ol)
        t0 = time.perf_counter()
        results = await asyncio.gather(*[one(ids, ol) for ids, ol in prompts])
        duration = time.perf_counter() - t0
    out = summarize(results, duration, concurrency)
    errs = [r.error for r in results if not r.ok]
    if errs:
        out["first_error"] = errs[0][:300]
    return out


def main(argv=None):
    p = argparse.ArgumentParser("bench_serving")
    p.add_argument("--base-url", default="http://127.0.0.1:30000")
    p.add_argument("--num-prompts", type=int, default=256)
    p.add_argument("--concurrency", type=int, default=64)
    p.add_argument("--input-len", type=int, default=1024)
    p.add_argument("--output-len", type=int, default=1024)
    p.add_argument("--random-range-ratio", type=float, default=1.0)
    p.add_argument("--vocab", type=int, default=32000)
    p.add_argument("--seed", type=int, default=1)
    p.add_argument("--tag", default="")
    p.add_argument("--output-file", default=None)
    a = p.parse_args(argv)
    prompts = make_prompts(a.num_prompts, a.input_len, a.output_len, a.vocab, a.random_range_ratio, a.seed)
    res = asyncio.run(run_benchmark(a.base_url, prompts, a.concurrency))
    res.update({"tag": a.tag, "input_len": a.input_len, "output_len": a.output_len, "num_prompts": a.num_prompts})
    line = json.dumps(res)
    print(line, flush=True)
    if a.output_file:
        with open(a.output_file, "a") as f:
            f.write(line + "\n")
    return res


if __name__ == "__main__":
    main()
