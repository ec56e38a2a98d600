"""Kernel front ends. Each op runs its sm_100a kernel on CUDA tensors and its PyTorch reference on CPU
tensors (the CPU oracle path); the reference implementations double as the numerics oracle of the GPU
tests. Parity: the reference's op wrappers branch on `can_run_kernel` (sglang_neuron/utils/neuron_utils.py:9)
between NKI kernels and torch paths in the same way.
"""
from .norm import rmsnorm, fused_add_rmsnorm, head_rmsnorm  # noqa: F401
