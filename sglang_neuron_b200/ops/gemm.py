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


def pick_splits(T: int, F: int, K: int, num_sms: int = 148) -> int:
    """Split K when the output tiles alone cannot occupy the SMs (decode-sized GEMMs)."""
    bn = 16 if T <= 16 else 32 if T <= 32 else 64 if T <= 64 else 128 if T <= 128 else 256
    ctas = ((F + 127) // 128) * ((T + bn - 1) // bn)
    nk = (K + 63) // 64
    if ctas >= num_sms:
        return 1
    # one CTA per SM (the kernel's pipeline takes ~200 KB of shared memory): stay within one wave
    return int(max(1, min(num_sms // ctas, nk // 2, 16)))


def linear(x: torch.Tensor, w: torch.Tensor, bias: Optional[torch.Tensor] = None, out=None,
           bn: int = 0, splits: Optional[int] = None) -> torch.Tensor:
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
    T = x2.shape[0]
    if out is None:
        out = torch.empty(T, F, dtype=x.dtype, device=x.device)
    if splits is None:
        splits = pick_splits(T, F, x2.shape[1])
    ws = torch.empty(splits * T * F, dtype=torch.float32, device=x.device) if splits > 1 else None
    kernels().gemm_bf16(out.view(-1, F), x2, w, bias, _status_buf(x.device), bn, splits, ws)
    return out.view(*shape[:-1], F)
