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
    keep = slots >= 0
    s = slots.clamp(min=0)
    page = s // page_size
    off = s % page_size
    vals = rows.to(cache.dtype)
    if bool(keep.all()):
        cache[page, 0, off] = vals
    else:
        cache[page[keep], 0, off[keep]] = vals[keep]


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
