"""Toolchain pin: the CUDA, driver, NCCL and torch versions this build was made with, and a digest of the
kernel sources that keys the build cache.

Parity: sglang_neuron/release/neuron_sdk.toml + release/neuron_sdk.py:69-213 (SDK pin with file hashes) and
backend/compile_cache.py:149-222 (refuse a compiled-artifact cache built from other kernel sources).
"""
from __future__ import annotations

import glob
import hashlib
import json
import os
import subprocess
from typing import Dict, Optional

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PINS = {"cuda": "12.9", "torch_major_minor": "2.11", "arch": "sm_100a", "nccl_min": "2.27"}
STAMP = os.path.join(ROOT, "sglang_neuron_b200", ".kernel_digest.json")


def source_digest(root: str = ROOT) -> str:
    h = hashlib.sha256()
    for path in sorted(glob.glob(os.path.join(root, "csrc", "**", "*.*"), recursive=True)):
        if path.endswith((".cu", ".cuh", ".h", ".cpp")):
            h.update(os.path.relpath(path, root).encode())
            with open(path, "rb") as f:
                h.update(f.read())
    h.update(open(os.path.join(root, "setup.py"), "rb").read())
    return h.hexdigest()


def nvcc_version() -> Optional[str]:
    try:
        out = subprocess.run(["nvcc", "--version"], capture_output=True, text=True, timeout=30).stdout
        return out.strip().splitlines()[-1]
    except Exception:
        return None


def toolchain() -> Dict[str, Optional[str]]:
    import torch
    d = {"torch": torch.__version__, "torch_cuda": torch.version.cuda, "nvcc": nvcc_version()}
    try:
        d["nccl"] = ".".join(map(str, torch.cuda.nccl.version()))
    except Exception:
        d["nccl"] = None
    return d


def write_stamp() -> dict:
    stamp = {"digest": source_digest(), "toolchain": toolchain()}
    with open(STAMP, "w") as f:
        json.dump(stamp, f, indent=1)
    return stamp


def check_stamp() -> Optional[str]:
    """None if the built kernels match the sources, else a reason string."""
    if not os.path.exists(STAMP):
        return "no build stamp (extension built outside setup/build())"
    stamp = json.load(open(STAMP))
    if stamp.get("digest") != source_digest():
        return "kernel sources changed since the extension was built; rebuild"
    return None
