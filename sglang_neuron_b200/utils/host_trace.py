"""Per-rank host timeline as TSV rows (phase, start_ns, end_ns, step, batch, tokens).

Parity: the reference's host trace (sglang_neuron/model_executor/host_trace.py:54 `HostTrace`,
managers/host_loop.py:149): `SGLANG_NEURON_HOST_TRACE=<dir>` writes rows for recv/input/select/launch/result
phases in CLOCK_REALTIME ns. Here `SGLANG_B200_HOST_TRACE=<dir>` (or ServerArgs.host_trace_dir) does the same.
"""
from __future__ import annotations

import os
import threading
import time
from typing import Optional


class HostTrace:
    def __init__(self, directory: Optional[str], rank="0"):
        self.enabled = bool(directory)
        self.f = None
        self.lock = threading.Lock()
        if self.enabled:
            os.makedirs(directory, exist_ok=True)
            self.f = open(os.path.join(directory, f"host_trace_rank{rank}.tsv"), "a", buffering=1 << 16)
            self.f.write("phase\tstart_ns\tend_ns\tstep\tbatch\ttokens\n")

    def span(self, phase: str, step: int = -1, batch: int = 0, tokens: int = 0):
        return _Span(self, phase, step, batch, tokens)

    def write(self, phase, t0, t1, step, batch, tokens) -> None:
        if self.f is None:
            return
        with self.lock:
            self.f.write(f"{phase}\t{t0}\t{t1}\t{step}\t{batch}\t{tokens}\n")

    def close(self) -> None:
        if self.f is not None:
            self.f.flush()
            self.f.close()
            self.f = None


class _Span:
    def __init__(self, tr: HostTrace, phase, step, batch, tokens):
        self.tr, self.phase, self.step, self.batch, self.tokens = tr, phase, step, batch, tokens

    def __enter__(self):
        self.t0 = time.time_ns() if self.tr.enabled else 0
        return self

    def __exit__(self, *exc):
        if self.tr.enabled:
            self.tr.write(self.phase, self.t0, time.time_ns(), self.step, self.batch, self.tokens)
        return False
