"""Device-side description of one forward step.

Parity: SGLang's ForwardBatch as the reference's graph runtime consumes it (block table, slot mapping,
cached sequence lengths; sglang_neuron/attention/backend.py:30 `NeuronForwardMetadata`). Everything a
captured CUDA graph reads lives in a tensor here, so replaying a graph only needs these buffers refreshed.
"""
from __future__ import annotations

import dataclasses
import enum
from typing import Optional

import torch


class ForwardMode(enum.IntEnum):
    EXTEND = 1   # prefill / chunked prefill (queries over a paged prior + causal chunk)
    DECODE = 2   # one new token per request
    IDLE = 3     # no local work (keeps collectives in lockstep)


@dataclasses.dataclass
class ForwardBatch:
    mode: ForwardMode
    batch_size: int
    num_tokens: int
    input_ids: torch.Tensor          # [T] int64
    positions: torch.Tensor          # [T] int64
    out_cache_loc: torch.Tensor      # [T] int64 slot = page * page_size + offset (-1: do not write)
    seq_lens: torch.Tensor           # [B] int32 KV length after this step
    block_table: torch.Tensor        # [B, W] int32 page ids
    logits_idx: torch.Tensor         # [B] int64 row of each request's last token
    qo_indptr: Optional[torch.Tensor] = None  # [B+1] int32 (extend)
    max_extend: int = 0
    max_seq_len: int = 0
    temperature: Optional[torch.Tensor] = None  # [B] fp32
    seeds: Optional[torch.Tensor] = None        # [B] int64
    top_k: Optional[torch.Tensor] = None        # [B] int64 (0 = off)
    top_p: Optional[torch.Tensor] = None        # [B] fp32 (1 = off)
    needs_topk_topp: bool = False
    decode_splits: int = 1
    # speculative decoding: number of query tokens per request in a verify step (1 = plain decode)
    spec_tokens: int = 1
    extra: dict = dataclasses.field(default_factory=dict)

    @property
    def is_decode(self) -> bool:
        return self.mode == ForwardMode.DECODE

    def slice_decode(self, b0: int, b1: int) -> "ForwardBatch":
        """Requests [b0, b1) of a plain decode step (one token per request, row i = request i) as a step of
        their own: the same split count and context bound, fresh per-step caches."""
        assert self.is_decode and self.spec_tokens == 1 and self.num_tokens == self.batch_size

        def sl(t):
            return None if t is None else t[b0:b1]

        extra = {k: self.extra[k] for k in ("logprob_k", "dp_rows") if k in self.extra}
        extra["num_decode"] = b1 - b0
        return dataclasses.replace(
            self, batch_size=b1 - b0, num_tokens=b1 - b0, input_ids=sl(self.input_ids), positions=sl(self.positions),
            out_cache_loc=sl(self.out_cache_loc), seq_lens=sl(self.seq_lens), block_table=sl(self.block_table),
            logits_idx=self.logits_idx[b0:b1] - b0, temperature=sl(self.temperature), seeds=sl(self.seeds),
            top_k=sl(self.top_k), top_p=sl(self.top_p), extra=extra)
