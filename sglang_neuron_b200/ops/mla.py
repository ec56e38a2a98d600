"""Absorbed multi-head latent attention over the paged latent pool ([pages, 1, page, r + rope]).

q rows carry [q_nope . W_UK (r values) || rope(q_pe)] per head; every head attends the same latent rows, the
value is the first r values of each row. Parity: the reference's `paged_absorbed_mla` decode and
`prefill_absorbed_mla_cte` (sglang_neuron/nki/deepseek_mla_decode.py:510, deepseek_mla_prefill.py:437) and
their torch twins (ops/attention/mla.py:32,56).
"""
from __future__ import annotations

import torch

from ..model_executor.forward_batch import ForwardBatch


def mla_write_rows(cache: torch.Tensor, rows: torch.Tensor, slots: torch.Tensor, page_size: int) -> None:
    """Write latent rows at their slots; rows with slot < 0 (batch padding) land in the reserved page 0
    (no host synchronisation: the write is capturable in a CUDA graph)."""
    s = torch.where(slots >= 0, slots, torch.zeros_like(slots))
    cache[s // page_size, 0, s % page_size] = rows.to(cache.dtype)


def mla_kernel_ok(q: torch.Tensor, cache: torch.Tensor, r: int) -> bool:
    return (q.is_cuda and cache.dtype == torch.bfloat16 and q.dtype == torch.bfloat16 and r == 512
            and q.shape[-1] == 576)


def mla_num_splits(batch: int, heads: int, max_ctx: int, num_sms: int = 148) -> int:
    """Context splits so that batch x head groups x splits CTAs fill about two waves (1 CTA of 85 KB smem
    per SM slot pair), at least 64 tokens per split."""
    ctas = max(1, batch * ((heads + 15) // 16))
    return int(max(1, min(2 * num_sms // ctas, (max_ctx + 63) // 64, 16)))


def mla_decode(q: torch.Tensor, cache: torch.Tensor, block_table: torch.Tensor, seq_lens: torch.Tensor,
               page_size: int, scale: float, num_splits: int) -> torch.Tensor:
    """Tensor-core absorbed-MLA decode (csrc/kernels/mla_decode.cu): q [B, H, 576] -> [B, H, 512]."""
    from .._ext import kernels
    B, H, _ = q.shape
    out = torch.empty(B, H, 512, dtype=q.dtype, device=q.device)
    S = max(1, int(num_splits))
    o_part = torch.empty(B * H * S * 512 if S > 1 else 1, dtype=torch.float32, device=q.device)
    lse = torch.empty(B * H * S if S > 1 else 1, dtype=torch.float32, device=q.device)
    kernels().mla_decode(out, q.contiguous(), cache, block_table, seq_lens, page_size, scale, S, o_part, lse)
    return out


def mla_extend(q: torch.Tensor, cache: torch.Tensor, block_table: torch.Tensor, seq_lens: torch.Tensor,
               qo_indptr: torch.Tensor, max_extend: int, page_size: int, scale: float, dcp=(1, 0),
               lse_out=None) -> torch.Tensor:
    """Prefill / chunked-prefill absorbed MLA on tensor cores: q [T, H, 576] of the new tokens (their latent
    rows already written) -> [T, H, 512]; causal within each request's chunk, full over its prefix.
    dcp = (D, rank): block_table lists this rank's pages of a DCP-interleaved context (parallel/dcp.py);
    lse_out [T, H] fp32 receives each row's log2-sum-exp.
    Parity: the reference's `prefill_absorbed_mla_cte` (sglang_neuron/nki/deepseek_mla_prefill.py:437)."""
    from .._ext import kernels
    out = torch.empty(q.shape[0], q.shape[1], 512, dtype=q.dtype, device=q.device)
    kernels().mla_extend(out, q.contiguous(), cache, block_table, seq_lens, qo_indptr, int(max_extend), page_size,
                         scale, int(dcp[0]), int(dcp[1]), lse_out)
    return out


def _one(q, cache, bt_row, L, q_pos, r, scale, page_size):
    n_pages = (L + page_size - 1) // page_size
    kv = cache[bt_row[:n_pages].long(), 0].reshape(n_pages * page_size, -1)[:L].float()  # [L, r+rope]
    s = torch.einsum("qhd,kd->hqk", q.float(), kv) * scale
    kpos = torch.arange(L, device=q.device)
    s = s.masked_fill(kpos[None, None, :] > q_pos[None, :, None], float("-inf"))
    p = torch.softmax(s, dim=-1)
    return torch.einsum("hqk,kr->qhr", p, kv[:, :r])


def mla_attention(q: torch.Tensor, cache: torch.Tensor, fb: ForwardBatch, r: int, scale: float,
                  page_size: int) -> torch.Tensor:
    """q: [T, H, r + rope] -> [T, H, r]."""
    out = torch.empty(q.shape[0], q.shape[1], r, dtype=q.dtype, device=q.device)
    parts = fb.extra.get("parts") if fb.extra else None
    if parts is not None:
        D, dec, ext = parts
        out[:D] = mla_attention(q[:D], cache, dec, r, scale, page_size)
        out[D:] = mla_attention(q[D:], cache, ext, r, scale, page_size)
        return out
    if fb.is_decode and mla_kernel_ok(q, cache, r):
        splits = fb.decode_splits or mla_num_splits(q.shape[0], q.shape[1], fb.max_seq_len or 4096)
        return mla_decode(q, cache, fb.block_table, fb.seq_lens, page_size, scale, splits)
    if not fb.is_decode and mla_kernel_ok(q, cache, r) and fb.qo_indptr is not None and fb.max_extend > 0:
        return mla_extend(q, cache, fb.block_table, fb.seq_lens, fb.qo_indptr, fb.max_extend, page_size, scale)
    seq = fb.seq_lens.tolist()
    if fb.is_decode:
        for b, L in enumerate(seq):
            if L == 0:
                out[b] = 0
                continue
            out[b] = _one(q[b:b + 1], cache, fb.block_table[b], L, torch.tensor([L - 1], device=q.device), r, scale,
                          page_size)[0].to(q.dtype)
        return out
    qo = fb.qo_indptr.tolist()
    for b, L in enumerate(seq):
        s0, s1 = qo[b], qo[b + 1]
        if s1 == s0:
            continue
        qpos = torch.arange(L - (s1 - s0), L, device=q.device)
        out[s0:s1] = _one(q[s0:s1], cache, fb.block_table[b], L, qpos, r, scale, page_size).to(q.dtype)
    return out
