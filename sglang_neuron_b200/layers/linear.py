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

from ..ops.gemm import linear
from ..parallel.collectives import fused_gemm_all_reduce, tp_all_reduce
from ..parallel.state import get_state


def _param(shape, dtype, device) -> nn.Parameter:
    return nn.Parameter(torch.empty(shape, dtype=dtype, device=device), requires_grad=False)


class ReplicatedLinear(nn.Module):
    def __init__(self, in_features: int, out_features: int, bias: bool = False, dtype=torch.bfloat16, device=None):
        super().__init__()
        self.weight = _param((out_features, in_features), dtype, device)
        self.bias = _param((out_features,), dtype, device) if bias else None

    def forward(self, x):
        return linear(x, self.weight, self.bias)

    def load(self, w: torch.Tensor, b: Optional[torch.Tensor] = None):
        self.weight.data.copy_(w)
        if b is not None:
            self.bias.data.copy_(b)


class ColumnParallelLinear(nn.Module):
    """Output features split over TP ranks; no communication."""

    def __init__(self, in_features: int, out_features: int, bias: bool = False, dtype=torch.bfloat16, device=None):
        super().__init__()
        st = get_state()
        assert out_features % st.tp_size == 0, f"{out_features} not divisible by tp {st.tp_size}"
        self.out_local = out_features // st.tp_size
        self.weight = _param((self.out_local, in_features), dtype, device)
        self.bias = _param((self.out_local,), dtype, device) if bias else None

    def forward(self, x):
        return linear(x, self.weight, self.bias)

    def shard(self, full: torch.Tensor, dim: int = 0) -> torch.Tensor:
        st = get_state()
        return full.narrow(dim, st.tp_rank * self.out_local, self.out_local)

    def load(self, w: torch.Tensor, b: Optional[torch.Tensor] = None):
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
        st = get_state()
        n = self.parts_local[idx]
        off = sum(self.parts_local[:idx])
        self.weight.data[off:off + n].copy_(w.narrow(0, st.tp_rank * n, n))
        if b is not None:
            self.bias.data[off:off + n].copy_(b.narrow(0, st.tp_rank * n, n))


class QKVParallelLinear(nn.Module):
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
        return linear(x, self.weight, self.bias)

    def load(self, q, k, v, qb=None, kb=None, vb=None):
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


class RowParallelLinear(nn.Module):
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

    def forward(self, x):
        st = get_state()
        # the bias is added once (on rank 0) so the all-reduce sums it exactly once
        b = self.bias if (self.bias is not None and st.tp_rank == 0) else None
        if self.reduce and st.tp_size > 1:
            y = fused_gemm_all_reduce(x, self.weight, b)
            if y is not None:
                return y
        y = linear(x, self.weight, b)
        if self.reduce and st.tp_size > 1:
            y = tp_all_reduce(y)
        return y

    def load(self, w: torch.Tensor, b: Optional[torch.Tensor] = None):
        st = get_state()
        self.weight.data.copy_(w.narrow(1, st.tp_rank * self.in_local, self.in_local))
        if b is not None:
            self.bias.data.copy_(b)
