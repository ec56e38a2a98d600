"""Attention backend: runs the paged attention kernels for a layer from the step's ForwardBatch.

Parity: `NeuronAttnBackend` (sglang_neuron/attention/backend.py:41) builds exact block tables / slot
mappings and lets graphs run attention; here the backend owns the decode split policy and the split-K
scratch (sized once for the largest batch so every captured graph reuses it).
"""
from __future__ import annotations

import torch

from ..ops.attention import DecodeScratch, decode_attention, default_num_splits, extend_attention
from ..model_executor.forward_batch import ForwardBatch


class AttentionBackend:
    def __init__(self, max_batch: int, num_q_heads: int, head_dim: int, device, max_splits: int = 32,
                 num_sms: int = 148):
        self.num_sms = num_sms
        self.max_splits = max_splits
        self.scratch = None
        if torch.device(device).type == "cuda":
            self.scratch = DecodeScratch(max_batch, num_q_heads, head_dim, max_splits, device)

    def splits_for(self, batch: int, num_kv_heads: int, max_ctx: int) -> int:
        return min(self.max_splits, default_num_splits(batch, num_kv_heads, max_ctx, self.num_sms))

    def attend(self, q: torch.Tensor, layer, fb: ForwardBatch, out=None) -> torch.Tensor:
        parts = fb.extra.get("parts") if fb.extra else None
        if parts is not None:
            # mixed step: decode rows first (split-K decode kernel), then the extend rows
            D, dec, ext = parts
            o = torch.empty(q.shape[0], layer.num_heads * layer.head_dim, dtype=q.dtype, device=q.device)
            self.attend(q[:D], layer, dec, out=o[:D])
            self.attend(q[D:], layer, ext, out=o[D:])
            return o
        kc, vc = layer.kv_cache()
        pool = layer.kv_pool
        if fb.is_decode:
            return decode_attention(q, kc, vc, fb.block_table, fb.seq_lens, layer.num_heads, layer.num_kv_heads,
                                    layer.head_dim, pool.page_size, layer.window, layer.scaling, pool.k_scale,
                                    pool.v_scale, layer.sinks_f32(), num_splits=fb.decode_splits,
                                    scratch=self.scratch, out=out)
        return extend_attention(q, kc, vc, fb.block_table, fb.qo_indptr, fb.seq_lens, fb.max_extend, layer.num_heads,
                                layer.num_kv_heads, layer.head_dim, pool.page_size, layer.window, layer.scaling,
                                pool.k_scale, pool.v_scale, layer.sinks_f32(), out=out)
