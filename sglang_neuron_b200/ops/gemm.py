"""Dense linear layers: the tcgen05 bf16 GEMM on CUDA, torch matmul on CPU."""
from typing import Optional

import torch

from .._ext import kernels

_status = {}


def _status_buf(device) -> torch.Tensor:
    key = (device.type, device.index)
    buf = _status.get(key)
    if buf is None:
        buf = torch.zeros(4, dtype=torch.int32, device=device)
        _status[key] = buf
    return buf


def check_status(device) -> None:
    """Raise if a kernel recorded a bounded-wait timeout (reads device memory: call between steps)."""
    buf = _status.get((device.type, device.index))
    if buf is not None:
        code = int(buf[0].item())
        if code != 0:
            raise RuntimeError(f"sm_100a kernel reported status {code} (bounded wait expired)")


def linear(x: torch.Tensor, w: torch.Tensor, bias: Optional[torch.Tensor] = None, out=None,
           bn: int = 0) -> torch.Tensor:
    """y = x @ w.T (+ bias). x: [..., K], w: [F, K]."""
    if not x.is_cuda or x.dtype != torch.bfloat16:
        y = torch.nn.functional.linear(x, w, bias)
        if out is not None:
            out.copy_(y)
            return out
        return y
    shape = x.shape
    x2 = x.reshape(-1, shape[-1])
    if x2.stride(-1) != 1 or (x2.stride(0) * 2) % 16 != 0 or x2.data_ptr() % 16 != 0:
        x2 = x2.contiguous()
    F = w.shape[0]
    if out is None:
        out = torch.empty(x2.shape[0], F, dtype=x.dtype, device=x.device)
    kernels().gemm_bf16(out.view(-1, F), x2, w, bias, _status_buf(x.device), bn)
    return out.view(*shape[:-1], F)
