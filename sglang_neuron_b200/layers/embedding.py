"""Vocabulary-parallel embedding and LM head.

Parity: `VocabDimShardedEmbedding` (sglang_neuron/layers/embedding.py:13-41): masked local lookup over
this rank's vocabulary shard plus an all-reduce. The LM head keeps the same shard; sampling merges the
per-shard candidates (see layers/sampler.py) instead of gathering full logits.
"""
from __future__ import annotations

import torch
from torch import nn

from ..ops.gemm import linear
from .linear import PackedWeight
from ..parallel.collectives import tp_all_reduce
from ..parallel.state import get_state


def vocab_shard(vocab: int, tp: int, rank: int):
    per = (vocab + tp - 1) // tp
    per = ((per + 63) // 64) * 64  # keep shards 64-aligned
    start = min(vocab, rank * per)
    end = min(vocab, start + per)
    return start, end, per


class VocabParallelEmbedding(nn.Module):
    def __init__(self, vocab: int, hidden: int, dtype=torch.bfloat16, device=None):
        super().__init__()
        st = get_state()
        self.vocab = vocab
        self.start, self.end, self.per = vocab_shard(vocab, st.tp_size, st.tp_rank)
        self.weight = nn.Parameter(torch.zeros(self.per, hidden, dtype=dtype, device=device), requires_grad=False)

    def forward(self, ids: torch.Tensor) -> torch.Tensor:
        st = get_state()
        if st.tp_size == 1:
            # clamped: an id the scheduler refuses may already be the input of the overlapped next step
            return self.weight[ids.clamp(0, self.weight.shape[0] - 1)]
        local = ids - self.start
        mask = (local >= 0) & (local < (self.end - self.start))
        out = self.weight[local.clamp(0, self.per - 1)] * mask[:, None].to(self.weight.dtype)
        return tp_all_reduce(out)

    def load(self, w: torch.Tensor):
        n = self.end - self.start
        self.weight.data[:n].copy_(w[self.start:self.end])


class ParallelLMHead(PackedWeight, nn.Module):
    def __init__(self, vocab: int, hidden: int, dtype=torch.bfloat16, device=None):
        super().__init__()
        st = get_state()
        self.vocab = vocab
        self.start, self.end, self.per = vocab_shard(vocab, st.tp_size, st.tp_rank)
        self.weight = nn.Parameter(torch.zeros(self.per, hidden, dtype=dtype, device=device), requires_grad=False)

    def forward(self, h: torch.Tensor) -> torch.Tensor:
        """Local logits [B, per] (columns past the vocabulary end are masked by the sampler)."""
        return linear(h, self.gemm_weight)

    def load(self, w: torch.Tensor):
        self.unpack()
        n = self.end - self.start
        self.weight.data[:n].copy_(w[self.start:self.end])
