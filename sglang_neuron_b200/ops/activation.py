"""Gated activations."""
import torch

from .._ext import kernels


def silu_and_mul(x: torch.Tensor, out=None) -> torch.Tensor:
    I = x.shape[-1] // 2
    if not x.is_cuda or x.dtype != torch.bfloat16:
        r = torch.nn.functional.silu(x[..., :I].float()) * x[..., I:].float()
        r = r.to(x.dtype)
        if out is not None:
            out.copy_(r)
            return out
        return r
    x2 = x.reshape(-1, 2 * I)
    if out is None:
        out = torch.empty(x2.shape[0], I, dtype=x.dtype, device=x.device)
    kernels().silu_and_mul(out, x2)
    return out.view(*x.shape[:-1], I)
