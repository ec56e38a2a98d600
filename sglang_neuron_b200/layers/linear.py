"""Tensor-parallel linear layers.

Parity: the reference's `ColumnParallelLinear` / `RowParallelLinear` (sglang_neuron/layers/linear.py:13,40)
and its QKV / gate_up sharding with KV-head replication when TP exceeds the KV head count
(models/transformer/weights.py:13-15). Weights live as [out, in] bf16 (nn.Linear layout) so the tcgen05
GEMM uses them as its 128-row operand directly.
"""
from __future__ import annotations

from typing import List, Optional

import torch
from torch import nn

from ..ops.gemm import TiledWeight, linear
from ..parallel.collectives import fused_gemm_all_reduce, tp_all_reduce
from ..parallel.state import get_state


def _param(shape, dtype, device) -> nn.Parameter:
    return nn.Parameter(torch.empty(shape, dtype=dtype, device=device), requires_grad=False)


class PackedWeight:
    """Mixin of the GEMM layers: after loading, `pack()` re-lays a CUDA bf16 weight out as contiguous
    128 x 64 tiles (ops/gemm.TiledWeight) and frees the row-major copy; `gemm_weight` is what forward() hands
    to the GEMM (the tiled weight when packed, else the parameter)."""

    _packed: Optional[TiledWeight] = None

    @property
    def gemm_weight(self):
        return self._packed if self._packed is not None else self.weight

    def pack(self) -> None:
        from ..ops.gemm import cublas_baseline
        w = self.weight
        if (self._packed is not None or not w.is_cuda or w.dtype != torch.bfloat16 or w.dim() != 2 or not w.numel()
                or cublas_baseline()):  # the cuBLAS comparison build keeps nn.Linear weights
            return
        from ..ops.gemm import plain_gemm_backend
        keep = plain_gemm_backend() == "cublas"  # plain GEMMs read the nn.Linear copy through cuBLAS
        self._packed = TiledWeight(w.data, keep_rowmajor=keep)
        if not keep:
            self.weight = nn.Parameter(torch.empty(0, dtype=w.dtype, device=w.device), requires_grad=False)

    def unpack(self) -> None:
        """Back to a row-major parameter (before loading new weights into a packed layer)."""
        if self._packed is not None:
            if self._packed.rowmajor is None:
                self.weight = nn.Parameter(self._packed.untiled().contiguous(), requires_grad=False)
            self._packed = None


def pack_linear_weights(model: nn.Module) -> int:
    """Pack every GEMM layer of `model`; returns how many were packed."""
    n = 0
    for m in model.modules():
        if isinstance(m, PackedWeight) and m._packed is None:
            m.pack()
            n += m._packed is not None
    return n


class ReplicatedLinear(PackedWeight, nn.Module):
    def __init__(self, in_features: int, out_features: int, bias: bool = False, dtype=torch.bfloat16, device=None):
        super().__init__()
        self.weight = _param((out_features, in_features), dtype, device)
        self.bias = _param((out_features,), dtype, device) if bias else None

    def forward(self, x):
        return linear(x, self.gemm_weight, self.bias)

    def load(self, w: torch.Tensor, b: Optional[torch.Tensor] = None):
        self.unpack()
        self.weight.data.copy_(w)
        if b is not None:
            self.bias.data.copy_(b)


class ColumnParallelLinear(PackedWeight, nn.Module):
    """Output features split over TP ranks; no communication."""

    def __init__(self, in_features: int, out_features: int, bias: bool = False, dtype=torch.bfloat16, device=None):
        super().__init__()
        st = get_state()
        assert out_features % st.tp_size == 0, f"{out_features} not divisible by tp {st.tp_size}"
        self.out_local = out_features // st.tp_size
        self.weight = _param((self.out_local, in_features), dtype, device)
        self.bias = _param((self.out_local,), dtype, device) if bias else None

    def forward(self, x):
        return linear(x, self.gemm_weight, self.bias)

    def shard(self, full: torch.Tensor, dim: int = 0) -> torch.Tensor:
        st = get_state()
        return full.narrow(dim, st.tp_rank * self.out_local, self.out_local)

    def load(self, w: torch.Tensor, b: Optional[torch.Tensor] = None):
        self.unpack()
        self.weight.data.copy_(self.shard(w))
        if b is not None:
            self.bias.data.copy_(self.shard(b))


class MergedColumnParallelLinear(ColumnParallelLinear):
    """Several column-parallel outputs fused into one GEMM (e.g. gate_up): each part is sharded separately
    and the local shards are concatenated."""

    def __init__(self, in_features: int, parts: List[int], bias: bool = False, dtype=torch.bfloat16, device=None):
        super().__init__(in_features, sum(parts), bias, dtype, device)
        st = get_state()
        self.parts_local = [p // st.tp_size for p in parts]

    def load_part(self, idx: int, w: torch.Tensor, b: Optional[torch.Tensor] = None):
        self.unpack()
        st = get_state()
        n = self.parts_local[idx]
        off = sum(self.parts_local[:idx])
        self.weight.data[off:off + n].copy_(w.narrow(0, st.tp_rank * n, n))
        if b is not None:
            self.bias.data[off:off + n].copy_(b.narrow(0, st.tp_rank * n, n))


class QKVParallelLinear(PackedWeight, nn.Module):
    """Fused Q/K/V projection with heads split over TP; KV heads are replicated when tp > num_kv_heads."""

    def __init__(self, hidden: int, head_dim: int, num_heads: int, num_kv_heads: int, bias: bool = False,
                 dtype=torch.bfloat16, device=None):
        super().__init__()
        st = get_state()
        tp = st.tp_size
        assert num_heads % tp == 0, "query heads must divide over TP"
        self.head_dim = head_dim
        self.num_heads = num_heads // tp
        if num_kv_heads >= tp:
            assert num_kv_heads % tp == 0
            self.num_kv_heads = num_kv_heads // tp
            self.kv_head_start = st.tp_rank * self.num_kv_heads
        else:
            assert tp % num_kv_heads == 0
            self.num_kv_heads = 1
            self.kv_head_start = st.tp_rank // (tp // num_kv_heads)
        self.q_size = self.num_heads * head_dim
        self.kv_size = self.num_kv_heads * head_dim
        out = self.q_size + 2 * self.kv_size
        self.weight = _param((out, hidden), dtype, device)
        self.bias = _param((out,), dtype, device) if bias else None

    def forward(self, x):
        return linear(x, self.gemm_weight, self.bias)

    def load(self, q, k, v, qb=None, kb=None, vb=None):
        self.unpack()
        st = get_state()
        D = self.head_dim
        qs = q.narrow(0, st.tp_rank * self.q_size, self.q_size)
        ks = k.narrow(0, self.kv_head_start * D, self.kv_size)
        vs = v.narrow(0, self.kv_head_start * D, self.kv_size)
        self.weight.data.copy_(torch.cat([qs, ks, vs], 0))
        if self.bias is not None and qb is not None:
            self.bias.data.copy_(torch.cat([qb.narrow(0, st.tp_rank * self.q_size, self.q_size),
                                            kb.narrow(0, self.kv_head_start * D, self.kv_size),
                                            vb.narrow(0, self.kv_head_start * D, self.kv_size)], 0))


class RowParallelLinear(PackedWeight, nn.Module):
    """Input features split over TP ranks; the partial outputs are summed with an all-reduce (unless
    reduce=False, when the caller fuses the reduction with a later one)."""

    def __init__(self, in_features: int, out_features: int, bias: bool = False, reduce: bool = True,
                 dtype=torch.bfloat16, device=None):
        super().__init__()
        st = get_state()
        assert in_features % st.tp_size == 0
        self.in_local = in_features // st.tp_size
        self.reduce = reduce
        self.weight = _param((out_features, self.in_local), dtype, device)
        self.bias = _param((out_features,), dtype, device) if bias else None

    def forward(self, x, norm=None):
        """norm: an optional parallel.collectives.FusedNorm folded into the all-reduce (see there)."""
        st = get_state()
        # the bias is added once (on rank 0) so the all-reduce sums it exactly once
        b = self.bias if (self.bias is not None and st.tp_rank == 0) else None
        if self.reduce and st.tp_size > 1:
            y = fused_gemm_all_reduce(x, self.gemm_weight, b, norm=norm)
            if y is not None:
                return y
        y = linear(x, self.gemm_weight, b)
        if self.reduce and st.tp_size > 1:
            y = tp_all_reduce(y, norm=norm)
        return y

    def load(self, w: torch.Tensor, b: Optional[torch.Tensor] = None):
        self.unpack()
        st = get_state()
        self.weight.data.copy_(w.narrow(1, st.tp_rank * self.in_local, self.in_local))
        if b is not None:
            self.bias.data.copy_(b)
