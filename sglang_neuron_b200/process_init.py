"""Per-process initialisation, once: CUDA device selection, NCCL environment and allocator settings.

Parity: sglang_neuron/process_init.py:14-55 (torch-neuronx init, device module, one shared gloo device).
"""
from __future__ import annotations

import os

_DONE = [False]


def init_process(local_rank=None) -> None:
    if _DONE[0]:
        return
    # expandable segments keep the pool's and the graphs' memory from fragmenting the caching allocator
    os.environ.setdefault("PYTORCH_CUDA_ALLOC_CONF", "expandable_segments:True")
    # NCCL: CUDA-graph-capturable collectives; NVLS (in-switch reduction) where the fabric has it
    os.environ.setdefault("NCCL_CUMEM_ENABLE", "1")
    os.environ.setdefault("TORCH_NCCL_ASYNC_ERROR_HANDLING", "1")
    import torch
    if torch.cuda.is_available():
        lr = int(os.environ.get("LOCAL_RANK", "0")) if local_rank is None else local_rank
        torch.cuda.set_device(lr)
        from . import env_registry
        if env_registry.get_bool("SGLANG_B200_NUMA_BIND", False):
            from .cpu_placement import bind_to_gpu
            bind_to_gpu(lr)
    _DONE[0] = True


def install_clean_exit() -> None:
    """SIGTERM raises SystemExit in the main thread, so `finally` blocks run (CUDA graphs released, process
    groups destroyed, shared buffers unmapped) instead of the process dying mid-collective.
    Parity: the reference's runtime_init install_clean_exit (sglang_neuron/model_executor/runtime_init.py:313)."""
    import signal

    def _handler(signum, frame):
        raise SystemExit(128 + signum)

    try:
        signal.signal(signal.SIGTERM, _handler)
    except ValueError:  # not the main thread: leave the default disposition
        pass
