"""Loader of the compiled sm_100a extension.

On a machine with a CUDA device the extension is mandatory: importing a CUDA op without it raises, so a
GPU run can never fall back silently to a PyTorch path. On CPU-only machines the ops use their PyTorch
reference implementations (the oracle path of the CPU test tier).
"""
import importlib

import torch  # noqa: F401  (loads libc10 / libtorch, which the extension links against)

_C = None
_runtime = None
_err = None
_rt_err = None

try:
    _C = importlib.import_module("sglang_neuron_b200._C")
except ImportError as e:  # pragma: no cover - depends on the build
    _err = e

try:
    _runtime = importlib.import_module("sglang_neuron_b200._runtime")
except ImportError as e:  # pragma: no cover
    _rt_err = e


_launches = [0]


def launch_count() -> int:
    """Kernels of this package launched so far (eager calls plus the kernels inside replayed graphs)."""
    return _launches[0]


def add_launches(n: int) -> None:
    _launches[0] += n


_HOST_ONLY = {"set_pdl", "get_pdl", "symm_alloc", "symm_open", "symm_close", "nvls_flag_bytes"}


class _CountingKernels:
    """Forwards to the compiled module and counts the kernels each call launches."""

    def __init__(self, mod):
        self._mod = mod
        self._cache = {}

    def __getattr__(self, name):
        fn = getattr(self._mod, name)
        if name == "decode_attention":
            def call(*a, **k):
                _launches[0] += 2 if (len(a) > 15 and int(a[15]) > 1) else 1
                return fn(*a, **k)
        elif name == "gemm_bf16":
            def call(*a, **k):
                _launches[0] += 2 if (len(a) > 8 and int(a[6]) > 1 and a[7] is not None and a[8]) else 1
                return fn(*a, **k)
        elif name in _HOST_ONLY:
            return fn
        else:
            def call(*a, **k):
                _launches[0] += 1
                return fn(*a, **k)
        return call


_counting = None


def kernels():
    """Return the kernel module or raise a clear error if it was not built."""
    global _counting
    if _C is None:
        raise RuntimeError(
            "sglang_neuron_b200._C is not built; run `python setup.py build_ext --inplace` "
            f"(import error: {_err})"
        )
    if _counting is None:
        _counting = _CountingKernels(_C)
    return _counting


def runtime():
    if _runtime is None:
        raise RuntimeError(
            "sglang_neuron_b200._runtime is not built; run `python setup.py build_ext --inplace` "
            f"(import error: {_rt_err})"
        )
    return _runtime


def available() -> bool:
    return _C is not None
