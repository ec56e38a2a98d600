"""Loader of the compiled sm_100a extension.

On a machine with a CUDA device the extension is mandatory: importing a CUDA op without it raises, so a
GPU run can never fall back silently to a PyTorch path. On CPU-only machines the ops use their PyTorch
reference implementations (the oracle path of the CPU test tier).
"""
import importlib

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


def kernels():
    """Return the kernel module or raise a clear error if it was not built."""
    if _C is None:
        raise RuntimeError(
            "sglang_neuron_b200._C is not built; run `python setup.py build_ext --inplace` "
            f"(import error: {_err})"
        )
    return _C


def runtime():
    if _runtime is None:
        raise RuntimeError(
            "sglang_neuron_b200._runtime is not built; run `python setup.py build_ext --inplace` "
            f"(import error: {_rt_err})"
        )
    return _runtime


def available() -> bool:
    return _C is not None
