"""Dense linear layers: the tcgen05 bf16 GEMM on CUDA, torch matmul on CPU.

By default a decode-sized GEMM splits K across the CTAs of a thread-block cluster and reduces the partial
tiles through distributed shared memory inside the kernel; an explicit `splits` > 1 writes fp32 partials
that a second launch (or a fused consumer) sums."""
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


class TiledWeight:
    """A bf16 [F, K] weight re-laid out for the tcgen05 GEMM: every 128-row x 64-column tile is one contiguous
    16 KB block, `data` = [ceil(F/128) * ceil(K/64) * 128, 64] (tile (f, k) at rows ((f * nk) + k) * 128),
    zero padded. One TMA box then reads one contiguous DRAM stream instead of 128 strided 128-byte rows."""

    __slots__ = ("data", "F", "K", "rowmajor")

    def __init__(self, w: torch.Tensor, keep_rowmajor: bool = False):
        F, K = w.shape
        self.rowmajor = w if keep_rowmajor else None  # the nn.Linear copy, for plain GEMMs through cuBLAS
        ntf, nk = (F + 127) // 128, (K + 63) // 64
        pad = torch.zeros(ntf * 128, nk * 64, dtype=w.dtype, device=w.device)
        pad[:F, :K] = w
        self.data = pad.view(ntf, 128, nk, 64).permute(0, 2, 1, 3).contiguous().view(ntf * nk * 128, 64)
        self.F, self.K = F, K

    @property
    def shape(self):
        return (self.F, self.K)

    @property
    def dtype(self):
        return self.data.dtype

    @property
    def device(self):
        return self.data.device

    def untiled(self) -> torch.Tensor:
        ntf, nk = (self.F + 127) // 128, (self.K + 63) // 64
        full = self.data.view(ntf, nk, 128, 64).permute(0, 2, 1, 3).reshape(ntf * 128, nk * 64)
        return full[: self.F, : self.K]


def _weight_args(w):
    """(tensor handed to the kernel, logical F, tiled_f flag value)."""
    if isinstance(w, TiledWeight):
        return w.data, w.F, w.F
    return w, w.shape[0], 0


def pick_splits(T: int, F: int, K: int, num_sms: int = 148) -> int:
    """Split K when the output tiles alone cannot occupy the SMs (decode-sized GEMMs)."""
    bn = 16 if T <= 16 else 32 if T <= 32 else 64 if T <= 64 else 128 if T <= 128 else 256
    ctas = ((F + 127) // 128) * ((T + bn - 1) // bn)
    nk = (K + 63) // 64
    if ctas >= num_sms:
        return 1
    # one CTA per SM (the kernel's pipeline takes ~200 KB of shared memory): stay within one wave
    return int(max(1, min(num_sms // ctas, nk // 2, 16)))


def cublas_baseline() -> bool:
    """SGLANG_B200_BASELINE=nccl: the comparison build - dense GEMMs through cuBLAS (torch.matmul) and every
    collective through NCCL, the rest of the engine unchanged."""
    from .. import env_registry
    return (env_registry.get("SGLANG_B200_BASELINE", "") or "").strip().lower() == "nccl"


_CUBLAS = cublas_baseline()


def plain_gemm_backend() -> str:
    """Where a plain dense GEMM (no fused collective, no grouped layout) runs: "cublas" (default) or "tcgen05"
    (SGLANG_B200_DENSE_GEMM). Measured in CUDA graphs on a B200, cuBLAS is ahead of this package's tcgen05
    kernel on every dense shape of the served models (e.g. 64 x 5120 x 2880: 7.8 us against 13.4 us; the
    1087-token Qwen3-8B mixed step: 23.3 ms against 33.5 ms), so plain library GEMMs go to the library and the
    tcgen05 kernel serves the fused forms: split-K partials feeding the NVLink all-reduce, the GEMM with the
    all-reduce in its epilogue, the per-head grouped GEMMs of absorbed MLA."""
    from .. import env_registry
    v = (env_registry.get("SGLANG_B200_DENSE_GEMM", "cublas") or "cublas").strip().lower()
    if v not in ("cublas", "tcgen05"):
        raise ValueError(f"SGLANG_B200_DENSE_GEMM={v!r}: expected 'cublas' or 'tcgen05'")
    return v


_PLAIN_CUBLAS = plain_gemm_backend() == "cublas"


def linear(x: torch.Tensor, w: torch.Tensor, bias: Optional[torch.Tensor] = None, out=None,
           bn: int = 0, splits: Optional[int] = None) -> torch.Tensor:
    """y = x @ w.T (+ bias). x: [..., K], w: [F, K] tensor or TiledWeight."""
    cublas = _CUBLAS and not isinstance(w, TiledWeight)
    if (x.is_cuda and x.dtype == torch.bfloat16 and _PLAIN_CUBLAS and splits is None and bn == 0
            and isinstance(w, TiledWeight) and w.rowmajor is not None):
        w, cublas = w.rowmajor, True  # a layer's plain GEMM: the library path (see plain_gemm_backend)
    if not x.is_cuda or x.dtype != torch.bfloat16 or cublas:
        if isinstance(w, TiledWeight):
            w = w.untiled()
        y = torch.nn.functional.linear(x, w, bias)
        if out is not None:
            out.copy_(y)
            return out
        return y
    shape = x.shape
    x2 = x.reshape(-1, shape[-1])
    if x2.stride(-1) != 1 or (x2.stride(0) * 2) % 16 != 0 or x2.data_ptr() % 16 != 0:
        x2 = x2.contiguous()
    wk, F, tiled_f = _weight_args(w)
    T = x2.shape[0]
    if out is None:
        out = torch.empty(T, F, dtype=x.dtype, device=x.device)
    if splits is None:
        splits = 0  # automatic: K split inside a thread-block cluster where tiles < SMs
    ws = torch.empty(splits * T * F, dtype=torch.float32, device=x.device) if splits > 1 else None
    kernels().gemm_bf16(out.view(-1, F), x2, wk, bias, _status_buf(x.device), bn, splits, ws, True, tiled_f)
    return out.view(*shape[:-1], F)


def linear_partials(x2: torch.Tensor, w: torch.Tensor, splits: int) -> torch.Tensor:
    """Split-K fp32 partial products [splits, T, F] of x2 @ w.T, left unreduced (a fused reduce follows)."""
    wk, F, tiled_f = _weight_args(w)
    T = x2.shape[0]
    ws = torch.empty(splits * T * F, dtype=torch.float32, device=x2.device)
    dummy = torch.empty((0, F), dtype=x2.dtype, device=x2.device)
    kernels().gemm_bf16(dummy, x2, wk, None, _status_buf(x2.device), 0, splits, ws, False, tiled_f)
    return ws
