"""Symmetric device buffers over CUDA IPC and the one-shot NVLink all-reduce built on them.

Every rank of the TP group allocates one buffer, exports its IPC handle, gathers the others' handles over
the host (gloo) group and maps them, so a kernel on any rank can store into any peer's buffer over NVLink.
Parity: the reference lowers its TP all-reduce into the compiled graph over CCOM
(sglang_neuron/parallel/collectives.py:22-55); on B200 the equivalent low-latency path is peer memory.
"""
from __future__ import annotations

import logging
from typing import List, Optional

import torch
import torch.distributed as dist

from .._ext import kernels
from .state import get_state

logger = logging.getLogger(__name__)


class IpcAllReduce:
    def __init__(self, capacity_bytes: int = 8 << 20, max_ctas: int = 64):
        st = get_state()
        self.rank, self.world = st.tp_rank, st.tp_size
        self.capacity = capacity_bytes
        self.max_ctas = max_ctas
        k = kernels()
        ptr, handle = k.symm_alloc(capacity_bytes, self.world)
        self.own = ptr
        handles: List = [None] * self.world
        dist.all_gather_object(handles, (self.rank, handle), group=st.cpu_group)
        self.ptrs = [0] * self.world
        for r, h in handles:
            self.ptrs[r] = ptr if r == self.rank else k.symm_open(h)
        self.status = torch.zeros(4, dtype=torch.int32, device=st.device)

    def can_run(self, x: torch.Tensor) -> bool:
        return (x.is_cuda and x.dtype == torch.bfloat16 and x.is_contiguous() and x.numel() % 8 == 0
                and x.numel() * 2 <= self.capacity)

    def all_reduce(self, x: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        if out is None:
            out = torch.empty_like(x)
        nvec = x.numel() // 8
        ctas = max(1, min(self.max_ctas, (nvec + 255) // 256))  # ~4 KB per CTA: many SMs drive NVLink
        kernels().one_shot_allreduce(out, x, self.ptrs, self.rank, self.capacity, ctas, self.status)
        return out

    def combine_all_reduce(self, out: torch.Tensor, y: torch.Tensor, inv_map: torch.Tensor,
                           w: torch.Tensor) -> torch.Tensor:
        """MoE combine (weighted sum of this rank's expert rows per token) fused with the all-reduce."""
        nvec = out.numel() // 8
        ctas = max(1, min(self.max_ctas, (nvec + 255) // 256))
        kernels().moe_combine_allreduce(out, y, inv_map, w, self.ptrs, self.rank, self.capacity, ctas, self.status)
        return out

    def gemm_can_run(self, T: int, F: int, num_sms: int) -> bool:
        bn = 16 if T <= 16 else 32 if T <= 32 else 64 if T <= 64 else 128 if T <= 128 else 256
        tiles = ((F + 127) // 128) * ((T + bn - 1) // bn)
        return tiles <= min(num_sms, 1024) and T * F * 2 <= self.capacity

    def gemm_all_reduce(self, x: torch.Tensor, w: torch.Tensor, bias: Optional[torch.Tensor],
                        num_sms: int) -> torch.Tensor:
        """out = all_reduce(x @ w.T (+ bias on rank 0 only)) in one kernel: tcgen05 GEMM whose epilogue
        stores its tiles into every peer's buffer and reduces them."""
        from ..ops.gemm import _weight_args
        wk, F, tiled_f = _weight_args(w)
        out = torch.empty(x.shape[0], F, dtype=x.dtype, device=x.device)
        kernels().gemm_bf16_allreduce(out, x, wk, bias, self.status, self.ptrs, self.rank, self.capacity, num_sms,
                                      tiled_f)
        return out

    def splitk_all_reduce(self, partial: torch.Tensor, splits: int, T: int, F: int,
                          bias: Optional[torch.Tensor], out: torch.Tensor) -> torch.Tensor:
        """Sum split-K partials (+ bias), all-reduce over the group: one launch after the split-K GEMM."""
        nvec = T * F // 8
        ctas = max(1, min(self.max_ctas, (nvec + 255) // 256))
        kernels().splitk_allreduce(out, partial, splits, bias, self.ptrs, self.rank, self.capacity, ctas, self.status)
        return out

    def close(self) -> None:
        k = kernels()
        for r, p in enumerate(self.ptrs):
            if p:
                k.symm_close(p, r == self.rank)
        self.ptrs = []
