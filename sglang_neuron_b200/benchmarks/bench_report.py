"""Render serving-benchmark JSONL (benchmarks/bench_serving.py output) as a markdown table: one row per run,
sorted by tag then concurrency, with output tok/s, TTFT, TPOT and ITL (median and p99), and the speed-up of
each run over the run of the same concurrency in a baseline file.

    python -m sglang_neuron_b200.benchmarks.bench_report runs.jsonl [--baseline ref.jsonl]

Parity: the reference's tools/bench_report.py (renders sglang.bench_serving JSONL versus concurrency).
"""
from __future__ import annotations

import argparse
import json
from typing import Dict, List, Optional

COLUMNS = [("tag", "run"), ("concurrency", "conc"), ("completed", "ok"), ("output_tok_s", "out tok/s"),
           ("ttft_ms_p50", "TTFT p50 ms"), ("ttft_ms_p99", "TTFT p99 ms"), ("tpot_ms_p50", "TPOT p50 ms"),
           ("tpot_ms_p99", "TPOT p99 ms"), ("itl_ms_p50", "ITL p50 ms")]


def load(path: str) -> List[Dict]:
    rows = []
    with open(path) as f:
        for line in f:
            line = line.strip()
            if line.startswith("{"):
                rows.append(json.loads(line))
    return rows


def render(rows: List[Dict], baseline: Optional[List[Dict]] = None) -> str:
    base = {r.get("concurrency"): r for r in (baseline or [])}
    cols = list(COLUMNS) + ([("speedup", "vs baseline")] if baseline else [])
    out = ["| " + " | ".join(h for _, h in cols) + " |", "|" + "---|" * len(cols)]
    for r in sorted(rows, key=lambda r: (str(r.get("tag", "")), r.get("concurrency", 0))):
        vals = []
        for key, _ in cols:
            if key == "speedup":
                b = base.get(r.get("concurrency"))
                v = (round(r["output_tok_s"] / b["output_tok_s"], 2)
                     if b and b.get("output_tok_s") else None)
            else:
                v = r.get(key)
            vals.append("-" if v is None or v == "" else str(v))
        out.append("| " + " | ".join(vals) + " |")
    return "\n".join(out)


def main(argv=None):
    p = argparse.ArgumentParser("bench_report")
    p.add_argument("files", nargs="+")
    p.add_argument("--baseline", default=None)
    a = p.parse_args(argv)
    rows = [r for f in a.files for r in load(f)]
    text = render(rows, load(a.baseline) if a.baseline else None)
    print(text)
    return text


if __name__ == "__main__":
    main()
