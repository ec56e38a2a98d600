"""Symmetric device buffers and the NVLink all-reduces built on them.

IpcAllReduce: buffers shared over CUDA IPC, one-shot all-reduce (every rank stores its message into every
peer's buffer, then reduces locally). NvlsAllReduce: a buffer bound to an NVSwitch multicast object
(PyTorch symmetric memory provides the allocation, mapping and rendezvous), reduced in the switch with
multimem.ld_reduce / multimem.st by this package's kernel (csrc/kernels/allreduce_nvls.cu).

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


class NvlsAllReduce:
    """Same interface as IpcAllReduce (all_reduce, combine_all_reduce, splitk_all_reduce), reduced through
    NVLink multicast. Raises at construction when the group has no multicast support."""

    def __init__(self, capacity_bytes: int = 8 << 20, max_ctas: int = 64):
        import torch.distributed._symmetric_memory as symm_mem
        st = get_state()
        self.rank, self.world = st.tp_rank, st.tp_size
        self.capacity = capacity_bytes
        self.max_ctas = max_ctas
        k = kernels()
        self.buf = symm_mem.empty(capacity_bytes + k.nvls_flag_bytes(), dtype=torch.uint8, device=st.device)
        self.buf.zero_()
        self.handle = symm_mem.rendezvous(self.buf, st.tp_group.group_name)
        mc = int(getattr(self.handle, "multicast_ptr", 0) or 0)
        if not mc:
            raise RuntimeError("no NVLink multicast for this group")
        off = self.buf.data_ptr() - int(self.handle.buffer_ptrs[self.rank])
        self.uc, self.mc = self.buf.data_ptr(), mc + off
        self.status = torch.zeros(4, dtype=torch.int32, device=st.device)
        torch.cuda.synchronize(st.device)
        dist.barrier(group=st.cpu_group)  # zeroed flags everywhere before the first call

    def can_run(self, x: torch.Tensor) -> bool:
        return (x.is_cuda and x.dtype == torch.bfloat16 and x.is_contiguous() and x.numel() % 8 == 0
                and x.numel() * 2 <= self.capacity)

    supports_norm = False  # the fused residual + RMSNorm epilogue is on the IPC kernels only

    def all_reduce(self, x: torch.Tensor, out: Optional[torch.Tensor] = None, norm=None) -> torch.Tensor:
        if out is None:
            out = torch.empty_like(x)
        kernels().nvls_allreduce(out, x, self.uc, self.mc, self.capacity, self.rank, self.world, self.max_ctas,
                                 self.status)
        return out

    def combine_all_reduce(self, out: torch.Tensor, y: torch.Tensor, inv_map: torch.Tensor,
                           w: torch.Tensor, norm=None) -> torch.Tensor:
        kernels().nvls_combine_allreduce(out, y, inv_map, w, self.uc, self.mc, self.capacity, self.rank,
                                         self.world, self.max_ctas, self.status)
        return out

    def gemm_can_run(self, T: int, F: int, num_sms: int) -> bool:
        return False

    def splitk_all_reduce(self, partial: torch.Tensor, splits: int, T: int, F: int,
                          bias: Optional[torch.Tensor], out: torch.Tensor, norm=None) -> torch.Tensor:
        kernels().nvls_splitk_allreduce(out, partial, splits, bias, self.uc, self.mc, self.capacity, self.rank,
                                        self.world, self.max_ctas, self.status)
        return out

    def close(self) -> None:
        self.handle = None
        self.buf = None


def make_tp_allreduce(capacity_bytes: int = 8 << 20):
    """The IPC one-shot all-reduce; the NVLS (multicast) one with SGLANG_B200_NVLS=1 where the fabric offers
    it. Measured at TP2 on a 368 KB decode message the one-shot is faster (16 us vs 26 us), so it is the
    default."""
    from .. import env_registry
    if env_registry.get_bool("SGLANG_B200_NVLS", False):
        try:
            return NvlsAllReduce(capacity_bytes)
        except Exception as e:  # no multicast on this fabric / driver
            logger.info("NVLS all-reduce unavailable (%s); using the IPC one-shot all-reduce", e)
    return IpcAllReduce(capacity_bytes)


class IpcAllReduce:
    """`wait_ns`: budget of every peer-flag wait in these kernels (0: the compiled default of 2 s). A wait that
    runs out records SNB_ERR_TIMEOUT_PEER in `status`, skips the reduce and returns; the engine raises at the
    next step boundary."""

    def __init__(self, capacity_bytes: int = 8 << 20, max_ctas: int = 64, wait_ns: int = 0, ptrs=None):
        self.capacity = capacity_bytes
        self.max_ctas = max_ctas
        self.wait_ns = wait_ns
        k = kernels()
        if ptrs is not None:
            # a caller-built peer table (tests: every slot a buffer of this GPU, rank 0)
            self.rank, self.world, self.own = 0, len(ptrs), ptrs[0]
            self.ptrs = list(ptrs)
            self._owned = set(range(len(ptrs)))
            self.status = torch.zeros(4, dtype=torch.int32, device=torch.device("cuda", torch.cuda.current_device()))
            return
        st = get_state()
        self.rank, self.world = st.tp_rank, st.tp_size
        ptr, handle = k.symm_alloc(capacity_bytes, self.world)
        self.own = ptr
        self._owned = {self.rank}
        handles: List = [None] * self.world
        dist.all_gather_object(handles, (self.rank, handle), group=st.cpu_group)
        self.ptrs = [0] * self.world
        for r, h in handles:
            self.ptrs[r] = ptr if r == self.rank else k.symm_open(h)
        self.status = torch.zeros(4, dtype=torch.int32, device=st.device)

    def can_run(self, x: torch.Tensor) -> bool:
        return (x.is_cuda and x.dtype == torch.bfloat16 and x.is_contiguous() and x.numel() % 8 == 0
                and x.numel() * 2 <= self.capacity)

    supports_norm = True

    @staticmethod
    def _norm_kw(norm):
        """Fused residual add + RMSNorm arguments (FusedNorm), marked as applied."""
        if norm is None:
            return {}
        norm.done = True
        return {"residual": norm.residual, "weight": norm.weight, "eps": norm.eps}

    def all_reduce(self, x: torch.Tensor, out: Optional[torch.Tensor] = None, norm=None) -> torch.Tensor:
        """norm (parallel.collectives.FusedNorm): out receives rmsnorm(sum + residual) and the residual is
        updated in place, in the same launch."""
        if out is None:
            out = torch.empty_like(x)
        nvec = x.numel() // 8
        ctas = max(1, min(self.max_ctas, (nvec + 255) // 256))  # ~4 KB per CTA: many SMs drive NVLink
        kernels().one_shot_allreduce(out, x, self.ptrs, self.rank, self.capacity, ctas, self.status,
                                     wait_ns=self.wait_ns, **self._norm_kw(norm))
        return out

    def combine_all_reduce(self, out: torch.Tensor, y: torch.Tensor, inv_map: torch.Tensor,
                           w: torch.Tensor, norm=None) -> torch.Tensor:
        """MoE combine (weighted sum of this rank's expert rows per token) fused with the all-reduce."""
        nvec = out.numel() // 8
        ctas = max(1, min(self.max_ctas, (nvec + 255) // 256))
        kernels().moe_combine_allreduce(out, y, inv_map, w, self.ptrs, self.rank, self.capacity, ctas, self.status,
                                        wait_ns=self.wait_ns, **self._norm_kw(norm))
        return out

    supports_sp = True

    def _sp_ctas(self, nvec: int) -> int:
        return max(1, min(148, (nvec + 511) // 512))

    def all_gather(self, x: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
        """Sequence-parallel all-gather of this rank's [rows, H] block into out [world * rows, H] (rank-major),
        one NVLink launch."""
        kernels().sp_allgather(out, x, self.ptrs, self.rank, self.capacity, self._sp_ctas(x.numel() // 8),
                               self.status, self.wait_ns)
        return out

    def reduce_scatter(self, x: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
        """Sequence-parallel reduce-scatter: x [world * rows, H] partial sums -> out [rows, H], this rank's
        block of the sums, one NVLink launch."""
        kernels().sp_reducescatter(out, x, self.ptrs, self.rank, self.capacity, self._sp_ctas(out.numel() // 8),
                                   self.status, self.wait_ns)
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
                          bias: Optional[torch.Tensor], out: torch.Tensor, norm=None) -> torch.Tensor:
        """Sum split-K partials (+ bias), all-reduce over the group: one launch after the split-K GEMM."""
        nvec = T * F // 8
        ctas = max(1, min(self.max_ctas, (nvec + 255) // 256))
        kernels().splitk_allreduce(out, partial, splits, bias, self.ptrs, self.rank, self.capacity, ctas, self.status,
                                   wait_ns=self.wait_ns, **self._norm_kw(norm))
        return out

    def close(self) -> None:
        k = kernels()
        for r, p in enumerate(self.ptrs):
            if p:
                k.symm_close(p, r in self._owned)
        self.ptrs = []
