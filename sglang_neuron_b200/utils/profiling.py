"""Bounded profiling windows.

Parity: the reference's device-profile window over decode steps (sglang_neuron/model_executor/profiling.py:108
`device_profile`, :211 `ServingCapture`) and the `/start_profile` route (sglang_patches/neuron_system_profile.py).
Here a window wraps torch.profiler (CUDA activity, exported as a Chrome trace) and NVTX ranges mark each step
for external tools; a step-bounded window stops itself after `num_steps` scheduler steps.
"""
from __future__ import annotations

import os
import time
from typing import Optional

import torch


class ProfileWindow:
    def __init__(self, output_dir: str, num_steps: Optional[int] = None):
        self.output_dir = output_dir
        self.num_steps = num_steps
        self.prof = None
        self.steps = 0
        self.last_path: Optional[str] = None

    def start(self) -> None:
        os.makedirs(self.output_dir, exist_ok=True)
        acts = [torch.profiler.ProfilerActivity.CPU]
        if torch.cuda.is_available():
            acts.append(torch.profiler.ProfilerActivity.CUDA)
        self.prof = torch.profiler.profile(activities=acts, record_shapes=False)
        self.prof.__enter__()

    def step(self) -> bool:
        """Count one scheduler step; returns True when the window closed itself."""
        self.steps += 1
        if self.num_steps is not None and self.steps >= self.num_steps:
            self.stop()
            return True
        return False

    def stop(self) -> Optional[str]:
        if self.prof is None:
            return None
        self.prof.__exit__(None, None, None)
        path = os.path.join(self.output_dir, f"trace-{int(time.time())}.json")
        self.prof.export_chrome_trace(path)
        self.prof = None
        self.last_path = path
        return path


class nvtx_range:
    """Context manager for an NVTX range (no-op without CUDA)."""

    def __init__(self, name: str):
        self.name = name

    def __enter__(self):
        if torch.cuda.is_available():
            torch.cuda.nvtx.range_push(self.name)
        return self

    def __exit__(self, *exc):
        if torch.cuda.is_available():
            torch.cuda.nvtx.range_pop()
        return False
