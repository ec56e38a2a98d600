"""Greedy-token parity between two servers (or one server against itself): the same fixed prompts are sent
one at a time (solo) and in concurrent waves, to A and to B, and the generated token ids are compared.
Solo-vs-wave on one server checks that batching does not change greedy results; A-vs-B compares two
builds or configurations.

    python -m sglang_neuron_b200.benchmarks.parity --a http://127.0.0.1:30000 --b http://127.0.0.1:30001

Parity: the reference's tools/parity_fixed_batches.py and tools/parity_compare.py (greedy token A/B, solo
and in waves of 8).
"""
from __future__ import annotations

import argparse
import asyncio
import json
import random
from typing import Dict, List


async def _generate(session, url: str, ids: List[int], n: int) -> List[int]:
    body = {"input_ids": ids, "sampling_params": {"max_new_tokens": n, "temperature": 0.0, "ignore_eos": True}}
    async with session.post(url + "/generate", json=body) as r:
        r.raise_for_status()
        return (await r.json())["output_ids"]


async def collect(url: str, prompts: List[List[int]], n: int, wave: int) -> List[List[int]]:
    """Generated ids per prompt; wave=1 sends them one at a time, else `wave` at once."""
    import aiohttp
    out: List[List[int]] = [None] * len(prompts)  # type: ignore
    async with aiohttp.ClientSession() as s:
        for i in range(0, len(prompts), wave):
            chunk = list(range(i, min(len(prompts), i + wave)))
            res = await asyncio.gather(*[_generate(s, url, prompts[j], n) for j in chunk])
            for j, r in zip(chunk, res):
                out[j] = r
    return out


def compare(a: List[List[int]], b: List[List[int]]) -> Dict:
    mism = [i for i, (x, y) in enumerate(zip(a, b)) if x != y]
    first = {}
    if mism:
        i = mism[0]
        k = next((t for t, (x, y) in enumerate(zip(a[i], b[i])) if x != y), min(len(a[i]), len(b[i])))
        first = {"prompt": i, "token": k}
    return {"prompts": len(a), "mismatched": len(mism), "first_divergence": first}


def run(a_url: str, b_url: str, num: int = 16, input_len: int = 32, output_len: int = 16, wave: int = 8,
        vocab: int = 32000, seed: int = 0) -> Dict:
    rng = random.Random(seed)
    prompts = [[rng.randrange(1, vocab) for _ in range(rng.randint(input_len // 2, input_len))] for _ in range(num)]
    a_solo = asyncio.run(collect(a_url, prompts, output_len, 1))
    a_wave = asyncio.run(collect(a_url, prompts, output_len, wave))
    b_wave = asyncio.run(collect(b_url, prompts, output_len, wave))
    return {"a_solo_vs_a_wave": compare(a_solo, a_wave), "a_wave_vs_b_wave": compare(a_wave, b_wave)}


def main(argv=None):
    p = argparse.ArgumentParser("parity")
    p.add_argument("--a", required=True)
    p.add_argument("--b", default=None)
    p.add_argument("--num", type=int, default=16)
    p.add_argument("--input-len", type=int, default=32)
    p.add_argument("--output-len", type=int, default=16)
    p.add_argument("--wave", type=int, default=8)
    p.add_argument("--vocab", type=int, default=32000)
    a = p.parse_args(argv)
    res = run(a.a, a.b or a.a, a.num, a.input_len, a.output_len, a.wave, a.vocab)
    print(json.dumps(res))
    return res


if __name__ == "__main__":
    main()
