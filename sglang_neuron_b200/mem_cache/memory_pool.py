"""KV pools.

Parity: `NeuronMHATokenToKVPool` (sglang_neuron/mem_cache/memory_pool.py:45) keeps per-layer K and V as
[num_blocks, kv_heads, page, head_dim] (head-major, page 0 reserved), bf16 or FP8; `NeuronMLATokenToKVPool`
(memory_pool.py:306, paged variant mla_pool.py:314) keeps one compact latent row (kv_lora + rope) per token.
The B200 pools use the same head-major paged layout, which is what the decode/extend kernels read, and
size themselves from free HBM (180 GB per GPU) instead of a fixed token count.
"""
from __future__ import annotations

from typing import Dict, List, Optional

import torch


class MHATokenToKVPool:
    """Per-layer paged K/V: [num_pages, num_kv_heads, page_size, head_dim]. Page 0 is a reserved dummy
    page that padding rows of a batch point at.

    With a hybrid sliding-window layout (`layer_pages`), the sliding layers' buffers have the window pool's
    page count and `swa` translates block tables and slots into it (mem_cache/hybrid_swa.py)."""

    def __init__(self, num_layers: int, num_pages: int, page_size: int, num_kv_heads: int, head_dim: int,
                 dtype: torch.dtype, device, k_scale: float = 1.0, v_scale: float = 1.0,
                 layer_ids: Optional[List[int]] = None, layer_pages: Optional[Dict[int, int]] = None):
        self.num_pages = num_pages
        self.page_size = page_size
        self.num_kv_heads = num_kv_heads
        self.head_dim = head_dim
        self.dtype = dtype
        self.k_scale = k_scale
        self.v_scale = v_scale
        self.layer_ids = list(range(num_layers)) if layer_ids is None else list(layer_ids)
        pages = {lid: (layer_pages or {}).get(lid, num_pages) for lid in self.layer_ids}
        self.hybrid = layer_pages is not None
        self.swa = None  # SwaTranslate when hybrid
        self.k_buffers = [torch.zeros((pages[l], num_kv_heads, page_size, head_dim), dtype=dtype, device=device)
                          for l in self.layer_ids]
        self.v_buffers = [torch.zeros((pages[l], num_kv_heads, page_size, head_dim), dtype=dtype, device=device)
                          for l in self.layer_ids]
        self._index = {lid: i for i, lid in enumerate(self.layer_ids)}

    def kv(self, layer_id: int):
        i = self._index[layer_id]
        return self.k_buffers[i], self.v_buffers[i]

    @staticmethod
    def bytes_per_page(num_layers, page_size, num_kv_heads, head_dim, dtype) -> int:
        el = torch.empty(0, dtype=dtype).element_size()
        return 2 * num_layers * page_size * num_kv_heads * head_dim * el

    def copy_pages(self, src: torch.Tensor, dst: torch.Tensor) -> None:
        """Copy whole pages (all layers): used by PD transfer and by copy-on-write of shared pages."""
        if self.hybrid:
            raise RuntimeError("whole-page copies are not defined for the hybrid sliding-window pool")
        for k, v in zip(self.k_buffers, self.v_buffers):
            k[dst] = k[src]
            v[dst] = v[src]


class MLATokenToKVPool:
    """Per-layer paged latent rows: [num_pages, 1, page_size, kv_lora_rank + rope_dim]."""

    def __init__(self, num_layers: int, num_pages: int, page_size: int, kv_lora_rank: int, rope_dim: int,
                 dtype: torch.dtype, device, layer_ids: Optional[List[int]] = None):
        self.num_pages = num_pages
        self.page_size = page_size
        self.kv_lora_rank = kv_lora_rank
        self.rope_dim = rope_dim
        self.dtype = dtype
        self.k_scale = 1.0
        self.v_scale = 1.0
        shape = (num_pages, 1, page_size, kv_lora_rank + rope_dim)
        self.layer_ids = list(range(num_layers)) if layer_ids is None else list(layer_ids)
        self.buffers = [torch.zeros(shape, dtype=dtype, device=device) for _ in self.layer_ids]
        self._index = {lid: i for i, lid in enumerate(self.layer_ids)}
        self.dcp = None  # parallel.dcp.DcpView when the context's pages are split over DCP ranks

    def kv(self, layer_id: int):
        b = self.buffers[self._index[layer_id]]
        return b, b

    @staticmethod
    def bytes_per_page(num_layers, page_size, kv_lora_rank, rope_dim, dtype) -> int:
        el = torch.empty(0, dtype=dtype).element_size()
        return num_layers * page_size * (kv_lora_rank + rope_dim) * el

    def copy_pages(self, src: torch.Tensor, dst: torch.Tensor) -> None:
        for b in self.buffers:
            b[dst] = b[src]


class ReqToPagePool:
    """Device block tables: one row of page ids per request slot (the attention kernels' block table)."""

    def __init__(self, max_reqs: int, max_pages_per_req: int, device):
        self.max_reqs = max_reqs
        self.max_pages = max_pages_per_req
        self.table = torch.zeros(max_reqs, max_pages_per_req, dtype=torch.int32, device=device)
        self.free_slots = list(range(max_reqs - 1, -1, -1))

    def alloc(self) -> Optional[int]:
        return self.free_slots.pop() if self.free_slots else None

    def free(self, idx: int) -> None:
        self.free_slots.append(idx)

    def available(self) -> int:
        return len(self.free_slots)
