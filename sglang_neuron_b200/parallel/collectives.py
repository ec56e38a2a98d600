"""Device collectives of the model forward.

The default path is NCCL through torch.distributed (graph-capturable). When a fused NVLink
communicator is registered for the TP group (parallel/symm_mem.py), all-reduce goes through it instead.
Parity: the reference's traced collectives (sglang_neuron/parallel/collectives.py:22-55).
"""
from __future__ import annotations

import contextlib
import os
from typing import Optional

import torch
import torch.distributed as dist

from .state import get_state

_custom_allreduce = None
_defer = [0]  # > 0 inside deferred_reduction(): TP reductions are left to the caller
_FUSED_NORM = os.environ.get("SGLANG_B200_FUSED_AR_NORM", "1") != "0"


def set_custom_allreduce(comm) -> None:
    global _custom_allreduce
    _custom_allreduce = comm


class FusedNorm:
    """The residual add + RMSNorm that follows a block's all-reduce, offered to the reduction: when the NVLink
    all-reduce kernel takes it (`done` becomes True) the reduced output comes back normalised and `residual`
    is updated in place, in the same launch; otherwise the caller applies the norm itself."""

    __slots__ = ("residual", "weight", "eps", "done")

    def __init__(self, residual: torch.Tensor, weight: torch.Tensor, eps: float):
        self.residual, self.weight, self.eps, self.done = residual, weight, eps, False

    @staticmethod
    def offer(residual: Optional[torch.Tensor], norm_module) -> Optional["FusedNorm"]:
        """A FusedNorm when the fused path can apply to rows like `residual`, else None."""
        st = get_state()
        ar = _custom_allreduce
        if (residual is None or not _FUSED_NORM or norm_module is None or st.tp_size == 1 or _defer[0] or ar is None
                or not getattr(ar, "supports_norm", False) or not residual.is_cuda
                or residual.dtype != torch.bfloat16 or not residual.is_contiguous()):
            return None
        w = norm_module.weight
        H = w.numel()
        if w.dtype != torch.bfloat16 or H % 8 or H > 8192 or residual.shape[-1] != H or residual.numel() * 2 > ar.capacity:
            return None
        return FusedNorm(residual, w, norm_module.eps)


def tp_all_reduce(x: torch.Tensor, norm: Optional[FusedNorm] = None) -> torch.Tensor:
    st = get_state()
    if st.tp_size == 1 or _defer[0]:
        return x
    if _custom_allreduce is not None and _custom_allreduce.can_run(x):
        return _custom_allreduce.all_reduce(x, norm=norm)
    dist.all_reduce(x, group=st.tp_group)
    return x


def fused_combine_all_reduce(out: torch.Tensor, y: torch.Tensor, inv_map: torch.Tensor, w: torch.Tensor,
                             norm: Optional[FusedNorm] = None) -> bool:
    """MoE combine + TP/EP all-reduce in one NVLink kernel; returns False when that path is unavailable."""
    st = get_state()
    if st.tp_size == 1 or _defer[0] or _custom_allreduce is None or not _custom_allreduce.can_run(out):
        return False
    _custom_allreduce.combine_all_reduce(out, y, inv_map, w, norm=norm)
    return True


_num_sms = {}


def fused_gemm_all_reduce(x: torch.Tensor, w: torch.Tensor, bias, norm: Optional[FusedNorm] = None):
    """Row-parallel GEMM + all-reduce over NVLink, or None when that path does not apply.

    Decode-sized GEMMs (split-K > 1) run as two launches: the split-K tcgen05 GEMM writes fp32 partials and
    one kernel sums them, adds the bias, pushes the tile to every peer and reduces; larger GEMMs run the
    GEMM then the one-shot all-reduce. (The tcgen05 GEMM with the all-reduce inside its epilogue,
    IpcAllReduce.gemm_all_reduce, covers one-wave grids but keeps only F/128 CTAs busy, so it loses to the
    split-K form at the shapes measured; it stays available.)"""
    st = get_state()
    if st.tp_size == 1 or _defer[0] or _custom_allreduce is None or not x.is_cuda or x.dtype != torch.bfloat16:
        return None
    from ..ops.gemm import linear, linear_partials, pick_splits
    x2 = x.reshape(-1, x.shape[-1])
    if x2.stride(-1) != 1 or (x2.stride(0) * 2) % 16 or x2.data_ptr() % 16:
        x2 = x2.contiguous()
    T, F = x2.shape[0], w.shape[0]
    if T * F * 2 > _custom_allreduce.capacity or F % 8:
        return None
    dev = x.device.index
    if dev not in _num_sms:
        _num_sms[dev] = torch.cuda.get_device_properties(x.device).multi_processor_count
    splits = pick_splits(T, F, x2.shape[1], _num_sms[dev])
    out = torch.empty(T, F, dtype=x.dtype, device=x.device)
    if splits > 1:
        part = linear_partials(x2, w, splits)
        _custom_allreduce.splitk_all_reduce(part, splits, T, F, bias, out, norm=norm)
    else:
        y = linear(x2, w, bias, splits=1)
        _custom_allreduce.all_reduce(y, out, norm=norm)
    return out.view(*x.shape[:-1], F)


def tp_all_gather(x: torch.Tensor, dim: int = -1) -> torch.Tensor:
    st = get_state()
    if st.tp_size == 1:
        return x
    parts = [torch.empty_like(x) for _ in range(st.tp_size)]
    dist.all_gather(parts, x.contiguous(), group=st.tp_group)
    return torch.cat(parts, dim=dim)


def tp_all_gather_into(out: torch.Tensor, x: torch.Tensor) -> torch.Tensor:
    """out: [tp_size * x.shape[0], ...] gathered along dim 0."""
    st = get_state()
    if st.tp_size == 1:
        out.copy_(x)
        return out
    dist.all_gather_into_tensor(out, x.contiguous(), group=st.tp_group)
    return out


def tp_reduce_scatter(x: torch.Tensor) -> torch.Tensor:
    st = get_state()
    if st.tp_size == 1:
        return x
    out = torch.empty((x.shape[0] // st.tp_size,) + tuple(x.shape[1:]), dtype=x.dtype, device=x.device)
    dist.reduce_scatter_tensor(out, x.contiguous(), group=st.tp_group)
    return out


def cpu_broadcast_object(obj, src: int = 0):
    """Broadcast a picklable object from replica rank `src` over the host (gloo) group of the DP replica
    (every TP rank of every pipeline stage)."""
    st = get_state()
    if st.replica_size == 1:
        return obj
    buf = [obj]
    dist.broadcast_object_list(buf, src=src + st.replica_base, group=st.replica_cpu_group)
    return buf[0]


def cpu_barrier() -> None:
    st = get_state()
    if st.replica_size > 1:
        dist.barrier(group=st.replica_cpu_group)


# ---- sequence parallelism between layers ----------------------------------------------------------------
# Prefill steps keep ceil(T / t) rows of the hidden state and residual per TP rank between layers: the norms
# and residual adds run on 1/t of the rows, an all-gather brings the normalised rows to every rank before
# attention and the MLP/MoE, and a reduce-scatter replaces the all-reduce after them (same bytes on the wire).
# Parity: the reference's GPT-OSS prefill graph (sglang_neuron/models/gpt_oss/mxfp4/model_prefill.py:32,111,
# 131,197) and the sampled-row gather (models/gpt_oss/sequence_parallel.py:23).

@contextlib.contextmanager
def deferred_reduction():
    """Inside this block a layer's TP reduction is left to the caller: tp_all_reduce returns the partial sum
    unchanged and the fused GEMM / MoE-combine all-reduce paths decline, so a sequence-parallel layer can
    reduce-scatter the partials instead."""
    _defer[0] += 1
    try:
        yield
    finally:
        _defer[0] -= 1


def sp_reduce_scatter(x: torch.Tensor, rows: int) -> torch.Tensor:
    """x: [T, H] partial sums (T <= rows * tp); returns this rank's [rows, H] block of the reduced rows."""
    st = get_state()
    tp = st.tp_size
    if x.shape[0] < rows * tp:
        x = torch.cat([x, x.new_zeros(rows * tp - x.shape[0], *x.shape[1:])])
    out = torch.empty((rows,) + tuple(x.shape[1:]), dtype=x.dtype, device=x.device)
    if _sp_native(out):
        return _custom_allreduce.reduce_scatter(x.contiguous(), out)
    dist.reduce_scatter_tensor(out, x.contiguous(), group=st.tp_group)
    return out


_SP_NVLINK = os.environ.get("SGLANG_B200_SP_NVLINK", "0") == "1"


def _sp_native(block: torch.Tensor) -> bool:
    """The NVLink all-gather / reduce-scatter kernels take bf16 blocks that fit one buffer slot
    (SGLANG_B200_SP_NVLINK=1; NCCL otherwise)."""
    ar = _custom_allreduce
    return (_SP_NVLINK and ar is not None and getattr(ar, "supports_sp", False) and block.is_cuda
            and block.dtype == torch.bfloat16 and block.numel() % 8 == 0 and block.numel() * 2 <= ar.capacity)


def sp_all_gather(x: torch.Tensor) -> torch.Tensor:
    """x: [rows, H] this rank's block; returns [rows * tp, H] (rank-major)."""
    st = get_state()
    out = torch.empty((x.shape[0] * st.tp_size,) + tuple(x.shape[1:]), dtype=x.dtype, device=x.device)
    if _sp_native(x):
        return _custom_allreduce.all_gather(x.contiguous(), out)
    dist.all_gather_into_tensor(out, x.contiguous(), group=st.tp_group)
    return out


def sp_gather_rows(x: torch.Tensor, idx: torch.Tensor, rows: int) -> torch.Tensor:
    """Rows `idx` (global row ids) of a row-sharded [rows, H] tensor, on every rank: each rank contributes
    the rows it holds (zeros elsewhere) and one all-reduce of [len(idx), H] merges them."""
    st = get_state()
    local = idx - st.tp_rank * rows
    mine = (local >= 0) & (local < rows)
    sel = x.index_select(0, local.clamp(0, rows - 1))
    sel = torch.where(mine.unsqueeze(1), sel, torch.zeros_like(sel))
    return tp_all_reduce(sel)


# ---- DP attention: token exchange around the MoE ------------------------------------------------------------
# Each attention group holds its own requests' rows; the experts are split over every rank. Before a MoE
# block the groups' rows (padded to the step's largest group, `rows`) are all-gathered so every rank routes
# every token through its experts; after it the partial outputs are summed over all ranks and each group
# keeps its own rows (a reduce-scatter when groups are single ranks). Parity: the reference's DP-attention
# decode (sglang_neuron/models/gpt_oss/mxfp4/model_decode.py:90-98: all-gather over the DP group, experts,
# wide all-reduce or reduce-scatter).

def dp_gather_rows(x: torch.Tensor, rows: int) -> torch.Tensor:
    """x: [T_g, H] (T_g <= rows) -> [D * rows, H], group-major, zero padding rows."""
    st = get_state()
    if x.shape[0] < rows:
        x = torch.cat([x, x.new_zeros(rows - x.shape[0], *x.shape[1:])])
    out = torch.empty((rows * st.attn_dp_size,) + tuple(x.shape[1:]), dtype=x.dtype, device=x.device)
    dist.all_gather_into_tensor(out, x.contiguous(), group=st.dp_cross_group)
    return out


def dp_scatter_rows(part: torch.Tensor, rows: int, n: int) -> torch.Tensor:
    """part: [D * rows, H] partial sums on every rank -> this group's first n rows of the total."""
    st = get_state()
    if st.tp_size == 1:  # one rank per group: a reduce-scatter over all ranks
        out = torch.empty((rows,) + tuple(part.shape[1:]), dtype=part.dtype, device=part.device)
        dist.reduce_scatter_tensor(out, part.contiguous(), group=st.moe_group)
        return out[:n]
    dist.all_reduce(part, group=st.moe_group)
    g = st.attn_dp_rank
    return part[g * rows:g * rows + n]


def dp_exchange(obj):
    """All-gather a host object over every rank of the DP-attention world (the per-step lockstep record)."""
    st = get_state()
    out = [None] * st.replica_size
    dist.all_gather_object(out, obj, group=st.replica_cpu_group)
    return out


# ---- pipeline parallelism -------------------------------------------------------------------------------
# Stage boundaries move (hidden, residual) of every token from stage s to stage s+1 (same TP rank) with one
# point-to-point send (NCCL on GPUs, gloo on the CPU tier); the last stage's sampled ids are broadcast to the
# whole replica so every rank's scheduler and token relay see them. Parity: the reference's PP seam moves the
# boundary HBM->HBM and relays tokens back to the first stage (sglang_neuron/distributed/pp_seam.py:306).

def pp_send_hidden(h: torch.Tensor, residual: torch.Tensor) -> None:
    st = get_state()
    dist.send(torch.stack([h, residual]).contiguous(), dst=st.stage_rank(st.pp_rank + 1))


def pp_isend_hidden(h: torch.Tensor, residual: torch.Tensor):
    """Non-blocking stage-boundary send: (work, buffer); the buffer must stay alive until work.wait()."""
    st = get_state()
    buf = torch.stack([h, residual]).contiguous()
    return dist.isend(buf, dst=st.stage_rank(st.pp_rank + 1)), buf


def pp_recv_hidden(num_tokens: int, hidden: int, dtype, device):
    st = get_state()
    buf = torch.empty(2, num_tokens, hidden, dtype=dtype, device=device)
    dist.recv(buf, src=st.stage_rank(st.pp_rank - 1))
    return buf[0], buf[1]


def pp_broadcast_ids(ids: torch.Tensor) -> torch.Tensor:
    """ids: [B] int64, valid on the last stage; returned on every rank of the replica."""
    st = get_state()
    if st.pp_size == 1:
        return ids
    dist.broadcast(ids, src=st.replica_base + (st.pp_size - 1) * st.tp_size, group=st.replica_group)
    return ids
