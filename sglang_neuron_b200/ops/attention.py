"""Paged attention ops over the KV pool: decode (one query per request) and extend (chunk of queries over
a paged prior). Both support GQA, learned per-head sinks, a sliding window and bf16 or fp8-e4m3 caches.

KV cache layout: [num_pages, num_kv_heads, page_size, head_dim].
"""
from typing import Optional

import torch

from .._ext import kernels


def _gather_kv(cache: torch.Tensor, block_row: torch.Tensor, n_tok: int, page_size: int, scale: float):
    """Return [n_tok, Hkv, D] fp32 for the first n_tok positions of one request."""
    if n_tok == 0:
        return cache.new_zeros((0, cache.shape[1], cache.shape[3]), dtype=torch.float32)
    n_pages = (n_tok + page_size - 1) // page_size
    pages = block_row[:n_pages].long()
    kv = cache[pages].float()  # [n_pages, Hkv, page, D]
    kv = kv.permute(0, 2, 1, 3).reshape(n_pages * page_size, cache.shape[1], cache.shape[3])
    return kv[:n_tok] * scale


def _attend_ref(q, k, v, q_pos, k_pos, sm_scale, window, sinks):
    """q: [Tq, Hq, D], k/v: [Tk, Hkv, D] fp32; positions absolute. Returns [Tq, Hq, D] fp32."""
    Hq, Hkv = q.shape[1], k.shape[1]
    G = Hq // Hkv
    k = k.repeat_interleave(G, dim=1)
    v = v.repeat_interleave(G, dim=1)
    s = torch.einsum("qhd,khd->hqk", q.float(), k) * sm_scale
    allowed = k_pos[None, :] <= q_pos[:, None]
    if window and window > 0:
        allowed &= (q_pos[:, None] - k_pos[None, :]) < window
    s = s.masked_fill(~allowed[None], float("-inf"))
    if sinks is not None:
        sink = sinks.float()[:, None, None].expand(Hq, q.shape[0], 1)
        s = torch.cat([s, sink], dim=-1)
    m = s.amax(-1, keepdim=True)
    m = torch.where(torch.isfinite(m), m, torch.zeros_like(m))
    p = torch.exp(s - m)
    denom = p.sum(-1, keepdim=True)
    p = p / torch.where(denom > 0, denom, torch.ones_like(denom))
    if sinks is not None:
        p = p[..., :-1]
    return torch.einsum("hqk,khd->qhd", p, v)


def decode_attention_ref(q, k_cache, v_cache, block_table, seq_lens, num_q_heads, num_kv_heads, head_dim,
                         page_size, window=0, sm_scale=None, k_scale=1.0, v_scale=1.0, sinks=None):
    B = q.shape[0]
    sm_scale = head_dim ** -0.5 if sm_scale is None else sm_scale
    out = torch.zeros(B, num_q_heads, head_dim, dtype=torch.float32, device=q.device)
    qv = q.reshape(B, num_q_heads, head_dim)
    for b in range(B):
        L = int(seq_lens[b])
        if L == 0:
            continue
        k = _gather_kv(k_cache, block_table[b], L, page_size, k_scale)
        v = _gather_kv(v_cache, block_table[b], L, page_size, v_scale)
        pos = torch.arange(L, device=q.device)
        out[b] = _attend_ref(qv[b:b + 1].float(), k, v, pos[-1:], pos, sm_scale, window, sinks)[0]
    return out.reshape(B, num_q_heads * head_dim)


def extend_attention_ref(q, k_cache, v_cache, block_table, qo_indptr, kv_lens, num_q_heads, num_kv_heads,
                         head_dim, page_size, window=0, sm_scale=None, k_scale=1.0, v_scale=1.0, sinks=None):
    sm_scale = head_dim ** -0.5 if sm_scale is None else sm_scale
    Tq = q.shape[0]
    out = torch.zeros(Tq, num_q_heads, head_dim, dtype=torch.float32, device=q.device)
    qv = q.reshape(Tq, num_q_heads, head_dim)
    for b in range(kv_lens.shape[0]):
        s0, s1 = int(qo_indptr[b]), int(qo_indptr[b + 1])
        ext = s1 - s0
        if ext == 0:
            continue
        L = int(kv_lens[b])
        k = _gather_kv(k_cache, block_table[b], L, page_size, k_scale)
        v = _gather_kv(v_cache, block_table[b], L, page_size, v_scale)
        kpos = torch.arange(L, device=q.device)
        qpos = torch.arange(L - ext, L, device=q.device)
        out[s0:s1] = _attend_ref(qv[s0:s1].float(), k, v, qpos, kpos, sm_scale, window, sinks)
    return out.reshape(Tq, num_q_heads * head_dim)


def default_num_splits(batch: int, num_kv_heads: int, max_ctx: int, num_sms: int = 148) -> int:
    """Flash-decoding split count: as many context splits as keep (batch x kv heads x splits) CTAs within one
    resident wave (4 CTAs per SM), at least 128 tokens per split. Measured at 64 x 8 x 1536 (fp8 KV, token-major
    kernel, in a CUDA graph): one split 23.5 us, two 41.9 us: beyond one wave the extra CTAs and the merge cost
    more than they hide."""
    ctas = max(1, batch * num_kv_heads)
    want = max(1, (4 * num_sms) // ctas)
    cap = max(1, (max_ctx + 127) // 128)
    return int(min(want, cap, 32))


class DecodeScratch:
    """fp32 scratch for split partials, sized once for a maximum batch (CUDA-graph friendly)."""

    def __init__(self, max_batch: int, num_q_heads: int, head_dim: int, max_splits: int, device):
        self.max_splits = max_splits
        self.o = torch.empty(max_batch * num_q_heads * max_splits * head_dim, dtype=torch.float32, device=device)
        self.lse = torch.empty(max_batch * num_q_heads * max_splits, dtype=torch.float32, device=device)
        # arrival counters of the in-kernel split merge (FP8 kernel): zero between calls, re-armed by the kernel
        self.merge_cnt = torch.zeros(max_batch * num_q_heads, dtype=torch.int32, device=device)


def decode_attention(q, k_cache, v_cache, block_table, seq_lens, num_q_heads, num_kv_heads, head_dim,
                     page_size, window=0, sm_scale=None, k_scale=1.0, v_scale=1.0,
                     sinks: Optional[torch.Tensor] = None, num_splits: int = 1,
                     scratch: Optional[DecodeScratch] = None, out=None):
    sm_scale = head_dim ** -0.5 if sm_scale is None else sm_scale
    if not q.is_cuda:
        r = decode_attention_ref(q, k_cache, v_cache, block_table, seq_lens, num_q_heads, num_kv_heads, head_dim,
                                 page_size, window, sm_scale, k_scale, v_scale, sinks).to(q.dtype)
        if out is not None:
            out.copy_(r)
            return out
        return r
    B = q.shape[0]
    if out is None:
        out = torch.empty(B, num_q_heads * head_dim, dtype=q.dtype, device=q.device)
    cnt = None
    if num_splits > 1:
        if scratch is None:
            scratch = DecodeScratch(B, num_q_heads, head_dim, num_splits, q.device)
        assert num_splits <= scratch.max_splits
        o_part, lse_part, cnt = scratch.o, scratch.lse, scratch.merge_cnt
    else:
        o_part = lse_part = torch.empty(0, dtype=torch.float32, device=q.device)
    from .gemm import _status_buf
    kernels().decode_attention(out, q, k_cache, v_cache, block_table, seq_lens, num_q_heads, num_kv_heads,
                               head_dim, page_size, window, sm_scale, k_scale, v_scale, sinks, num_splits,
                               o_part, lse_part, _status_buf(q.device), cnt)
    return out


def extend_attention(q, k_cache, v_cache, block_table, qo_indptr, kv_lens, max_extend, num_q_heads,
                     num_kv_heads, head_dim, page_size, window=0, sm_scale=None, k_scale=1.0, v_scale=1.0,
                     sinks=None, out=None):
    sm_scale = head_dim ** -0.5 if sm_scale is None else sm_scale
    if not q.is_cuda:
        r = extend_attention_ref(q, k_cache, v_cache, block_table, qo_indptr, kv_lens, num_q_heads, num_kv_heads,
                                 head_dim, page_size, window, sm_scale, k_scale, v_scale, sinks).to(q.dtype)
        if out is not None:
            out.copy_(r)
            return out
        return r
    if out is None:
        out = torch.empty(q.shape[0], num_q_heads * head_dim, dtype=q.dtype, device=q.device)
    kernels().extend_attention(out, q, k_cache, v_cache, block_table, qo_indptr, kv_lens, int(max_extend),
                               num_q_heads, num_kv_heads, head_dim, page_size, window, sm_scale, k_scale,
                               v_scale, sinks)
    return out
