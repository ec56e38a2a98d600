"""Decode context parallelism (DCP) for the latent (MLA) KV pool.

Under tensor parallelism every rank of an MLA model holds the same latent rows (one 576-wide row per token,
shared by all heads), so the pool is replicated t times. With DCP of size D, the D ranks of a DCP group
(consecutive TP ranks) split each request's pages instead: logical page j lives on DCP rank j % D, so each
rank stores 1/D of the context. Per attention layer:

  1. the D ranks all-gather their query heads (each rank then holds the group's D x h heads),
  2. each rank attends those heads over its own pages (keys walked in local order, causal limits checked
     against logical positions) and keeps each row's log-sum-exp,
  3. the partial outputs and log-sum-exps are all-gathered and every rank merges the D partials of its own
     heads (exact: softmax over the union of the key sets).

Pages: the scheduler's allocator hands out global page ids g = local * D + owner from D per-owner pools
(`DcpPageAllocator`), choosing the owner from the page's logical index; each rank's pool holds its local
pages, and `DcpView` turns a step's block table and write slots into this rank's local ones on the device.

Parity: the reference's DCP layout and decode (sglang_neuron/distributed/decode_context_parallel.py:26
`DcpLayout`, :74 `decode_context`, :98 `group_sinks`; ops/attention/attention_decode.py:76-133) and the
exact log-sum-exp merge of partial attention (parallel/context_parallel.py:66 `merge_partials`).
"""
from __future__ import annotations

from typing import List

import torch
import torch.distributed as dist

from ..mem_cache.allocator import make_page_allocator
from .state import get_state


class DcpPageAllocator:
    """D per-owner page pools behind one allocator interface; global id = local id * D + owner."""

    def __init__(self, local_pages: int, page_size: int, dcp_size: int, reserved: int = 1):
        self.D = dcp_size
        self.pools = [make_page_allocator(local_pages, page_size, reserved) for _ in range(dcp_size)]

    def available(self) -> int:
        return min(p.available() for p in self.pools) * self.D

    def alloc_at(self, start: int, n: int) -> List[int]:
        """n pages for logical page indices start .. start + n - 1 (owner = index % D), or [] if any owner
        is out of pages."""
        want = [0] * self.D
        for j in range(start, start + n):
            want[j % self.D] += 1
        got = []
        for o in range(self.D):
            pages = list(self.pools[o].alloc(want[o])) if want[o] else []
            if len(pages) != want[o]:
                for oo, pp in enumerate(got):
                    if pp:
                        self.pools[oo].free(pp)
                if pages:
                    self.pools[o].free(pages)
                return []
            got.append(pages)
        out = []
        for j in range(start, start + n):
            o = j % self.D
            out.append(got[o].pop(0) * self.D + o)
        return out

    def alloc(self, n: int) -> List[int]:
        return self.alloc_at(0, n)

    def _split(self, pages):
        by = [[] for _ in range(self.D)]
        for g in pages:
            by[g % self.D].append(g // self.D)
        return by

    def free(self, pages) -> None:
        for o, pp in enumerate(self._split(pages)):
            if pp:
                self.pools[o].free(pp)

    def free_after(self, pages, epoch: int) -> None:
        for o, pp in enumerate(self._split(pages)):
            if pp:
                self.pools[o].free_after(pp, epoch)

    def retire(self, epoch: int) -> int:
        return sum(p.retire(epoch) for p in self.pools)

    def reset(self) -> None:
        for p in self.pools:
            p.reset()


class DcpView:
    """Device side: this rank's local block table and write slots for a step (cached on the ForwardBatch)."""

    def __init__(self, page_size: int):
        st = get_state()
        self.D, self.d, self.P = st.dcp_size, st.dcp_rank, page_size

    def local(self, fb):
        got = fb.extra.get("dcp_local")
        if got is not None:
            return got
        D, d, P = self.D, self.d, self.P
        bt = torch.div(fb.block_table[:, d::D], D, rounding_mode="floor").contiguous()
        loc = fb.out_cache_loc
        page = torch.div(loc.clamp(min=0), P, rounding_mode="floor")
        mine = (loc >= 0) & (page % D == d)
        lloc = torch.where(mine, torch.div(page, D, rounding_mode="floor") * P + loc.clamp(min=0) % P,
                           torch.full_like(loc, -1))
        fb.extra["dcp_local"] = (bt, lloc)
        return bt, lloc


def _gather_heads(x: torch.Tensor) -> torch.Tensor:
    """[T, h, ...] on each DCP rank -> [T, D * h, ...] (heads of rank 0 first)."""
    st = get_state()
    D = st.dcp_size
    out = torch.empty((D * x.shape[0],) + tuple(x.shape[1:]), dtype=x.dtype, device=x.device)
    dist.all_gather_into_tensor(out, x.contiguous(), group=st.dcp_group)
    out = out.view((D,) + tuple(x.shape))
    return out.movedim(0, 1).reshape(x.shape[0], D * x.shape[1], *x.shape[2:])


def merge_partials(o: torch.Tensor, lse2: torch.Tensor) -> torch.Tensor:
    """o: [D, T, h, V] normalised partials, lse2: [D, T, h] log2-sum-exp (-inf: no keys) -> [T, h, V]."""
    m = lse2.amax(0, keepdim=True)
    m = torch.where(torch.isfinite(m), m, torch.zeros_like(m))
    w = torch.exp2(lse2 - m)                      # -inf -> 0
    tot = w.sum(0)
    out = (w.unsqueeze(-1) * o.float()).sum(0) / tot.clamp(min=1e-30).unsqueeze(-1)
    return out


def partial_ref(q, cache, bt, seq_lens, qo, P, scale, D, d, r=512):
    """PyTorch twin of the DCP kernel path: q [T, H, r+rope] over this rank's local pages -> (o [T, H, r],
    lse2 [T, H]); causal limits on logical positions."""
    T, H = q.shape[0], q.shape[1]
    o = torch.zeros(T, H, r, dtype=torch.float32, device=q.device)
    lse = torch.full((T, H), float("-inf"), dtype=torch.float32, device=q.device)
    seq = seq_lens.tolist()
    qo = qo.tolist()
    ln2 = 0.6931471805599453
    for b, L in enumerate(seq):
        s0, s1 = qo[b], qo[b + 1]
        if s1 == s0:
            continue
        nl = bt.shape[1]
        kv = cache[bt[b, :nl].long(), 0].reshape(nl * P, -1).float()
        v = torch.arange(nl * P, device=q.device)
        logical = ((v // P) * D + d) * P + v % P
        qpos = torch.arange(L - (s1 - s0), L, device=q.device)
        s = torch.einsum("qhd,kd->hqk", q[s0:s1].float(), kv) * scale
        bad = (logical[None, None, :] > qpos[None, :, None]) | (logical[None, None, :] >= L)
        s = s.masked_fill(bad, float("-inf"))
        m = s.amax(-1, keepdim=True)
        has = torch.isfinite(m)
        p = torch.where(has, torch.exp(s - torch.where(has, m, torch.zeros_like(m))), torch.zeros_like(s))
        den = p.sum(-1, keepdim=True)
        ob = torch.einsum("hqk,kr->qhr", p / den.clamp(min=1e-30), kv[:, :r])
        o[s0:s1] = ob
        l2 = torch.where(has, (m + torch.log(den.clamp(min=1e-30))) / ln2, torch.full_like(m, float("-inf")))
        lse[s0:s1] = l2.squeeze(-1).transpose(0, 1)
    return o, lse


def dcp_mla_attention(q: torch.Tensor, cache: torch.Tensor, fb, r: int, scale: float, page_size: int,
                      view: DcpView) -> torch.Tensor:
    """q: [T, h, r + rope] of this rank's heads -> [T, h, r], over the DCP group's distributed pages."""
    from ..ops.mla import mla_extend, mla_kernel_ok
    parts = fb.extra.get("parts")
    if parts is not None:  # mixed step: decode rows, then the extend rows, each with its own tables
        nd, dec, ext = parts
        return torch.cat([dcp_mla_attention(q[:nd], cache, dec, r, scale, page_size, view),
                          dcp_mla_attention(q[nd:], cache, ext, r, scale, page_size, view)])
    st = get_state()
    D, d = st.dcp_size, st.dcp_rank
    T, h = q.shape[0], q.shape[1]
    bt, _ = view.local(fb)
    if fb.is_decode:
        qo = torch.arange(fb.batch_size + 1, dtype=torch.int32, device=q.device)
        max_ext = 1
    else:
        qo, max_ext = fb.qo_indptr, fb.max_extend
    qa = _gather_heads(q)                                   # [T, D*h, r+rope]
    if mla_kernel_ok(qa, cache, r):
        lse = torch.empty(T, D * h, dtype=torch.float32, device=q.device)
        o = mla_extend(qa, cache, bt, fb.seq_lens, qo, max_ext, page_size, scale, dcp=(D, d), lse_out=lse)
    else:
        o, lse = partial_ref(qa, cache, bt, fb.seq_lens, qo, page_size, scale, D, d, r)
        o = o.to(q.dtype)
    # every rank's partials for every head of the group; keep this rank's heads from each source rank
    og = _gather_ranks(o)[:, :, d * h:(d + 1) * h]         # [D, T, h, r]
    lg = _gather_ranks(lse)[:, :, d * h:(d + 1) * h]       # [D, T, h]
    return merge_partials(og, lg).to(q.dtype)


def _gather_ranks(x: torch.Tensor) -> torch.Tensor:
    st = get_state()
    out = torch.empty((st.dcp_size * x.shape[0],) + tuple(x.shape[1:]), dtype=x.dtype, device=x.device)
    dist.all_gather_into_tensor(out, x.contiguous(), group=st.dcp_group)
    return out.view((st.dcp_size,) + tuple(x.shape))
