"""RMSNorm ops (plain, fused residual add, per-head QK-norm)."""
import torch

from .._ext import kernels


def rmsnorm_ref(x: torch.Tensor, w: torch.Tensor, eps: float, plus_one: bool = False) -> torch.Tensor:
    xf = x.float()
    var = xf.pow(2).mean(-1, keepdim=True)
    wf = w.float() + 1.0 if plus_one else w.float()
    return (xf * torch.rsqrt(var + eps) * wf).to(x.dtype)


def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float, plus_one: bool = False, out=None) -> torch.Tensor:
    if not x.is_cuda:
        r = rmsnorm_ref(x, w, eps, plus_one)
        if out is not None:
            out.copy_(r)
            return out
        return r
    x2 = x.reshape(-1, x.shape[-1])
    o = torch.empty_like(x2) if out is None else out.reshape(-1, x.shape[-1])
    kernels().rmsnorm_out(o, x2, w, eps, plus_one)
    return o.view(x.shape)


def fused_add_rmsnorm(x: torch.Tensor, residual: torch.Tensor, w: torch.Tensor, eps: float,
                      plus_one: bool = False):
    """residual <- x + residual; x <- rmsnorm(residual). Returns (x, residual), both updated in place."""
    if not x.is_cuda:
        s = (x.float() + residual.float()).to(x.dtype)
        residual.copy_(s)
        x.copy_(rmsnorm_ref(s, w, eps, plus_one))
        return x, residual
    kernels().fused_add_rmsnorm(x.view(-1, x.shape[-1]), residual.view(-1, x.shape[-1]), w, eps, plus_one)
    return x, residual


def head_rmsnorm(x: torch.Tensor, w: torch.Tensor, heads: int, eps: float) -> torch.Tensor:
    """In-place per-head RMSNorm of a [T, heads*D] view."""
    if not x.is_cuda:
        T = x.shape[0]
        D = w.shape[0]
        v = x.view(T, heads, D) if x.is_contiguous() else x.reshape(T, heads, D)
        r = rmsnorm_ref(v, w, eps)
        x.copy_(r.view(T, heads * D))
        return x
    kernels().head_rmsnorm_(x, w, heads, eps)
    return x
