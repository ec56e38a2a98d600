"""Hybrid sliding-window KV: the sliding-attention layers of a model keep their K/V in a small window pool.

Full-attention layers keep every page of a request in the main pool. A sliding layer only ever reads the
last `window` keys, so its K/V lives in a second pool that holds, per request, just the pages that still
intersect the window (plus the pages of the chunk being prefilled). The two pools share one page index:
a request's logical page j is main-pool page `pages[j]`, and the window pool keeps a device map
`swa_map[main page] -> window page` (0 = none; page 0 is the reserved dummy page of both pools). Each step
translates the block table and the write slots of the sliding layers through that map with two gathers
(captured with the decode graph), so the attention kernels and the KV-write kernel run unchanged.

Pages whose last token is older than the window of the next step are returned to the window pool through
the same retire-aware frees as the main pool (the step in flight may still read them).

Sizing (the pool must never be the reason a running request stalls): every running request holds at most
ceil(window / page) + 2 window pages between steps, and one prefill chunk adds ceil(chunk / page) pages plus
one partial page per request it touches; with one step in flight the chunk term counts twice.

Parity: the reference's hybrid SWA pool (sglang_neuron/mem_cache/hybrid_swa.py: `configure` :163, the
full->swa index translation of slots and tables per step, the window-pool sizing proof
`check_window_pool` :234, `window_blocks` :279).
"""
from __future__ import annotations

import dataclasses
from typing import List, Optional

import torch


def window_blocks(window: int, page_size: int) -> int:
    """Window pages one request holds between steps: the pages of keys [L - window, L) plus the page being
    written, plus one page of slack for the conservative free rule."""
    return -(-window // page_size) + 2


def window_pool_pages(max_running: int, window: int, page_size: int, chunk: int) -> int:
    """Smallest window pool (pages, including the reserved page 0) that can never run out."""
    per_chunk = -(-chunk // page_size) + max_running
    return max_running * window_blocks(window, page_size) + 2 * per_chunk + 1


def check_window_pool(num_pages: int, max_running: int, window: int, page_size: int, chunk: int) -> None:
    need = window_pool_pages(max_running, window, page_size, chunk)
    if num_pages < need:
        raise ValueError(f"window KV pool of {num_pages} pages is below the {need} pages that "
                         f"{max_running} running requests with a {window}-token window and {chunk}-token prefill "
                         f"chunks need (page {page_size})")


class SwaPageTracker:
    """Host side (scheduler): window-pool pages of each request, allocation alongside the main pool and
    release of pages that left the window. Map updates travel in the step's page-update stream as
    (-1, main page, window page) triples."""

    def __init__(self, alloc, window: int, page_size: int):
        self.alloc = alloc
        self.window = window
        self.P = page_size

    def available(self) -> int:
        return self.alloc.available()

    def alloc_for(self, n: int) -> Optional[List[int]]:
        if n <= 0:
            return []
        pages = self.alloc.alloc(n)
        if len(pages) != n:
            if pages:
                self.alloc.free(list(pages))
            return None
        return list(pages)

    def undo(self, pages: List[int]) -> None:
        """Give back pages that no step has used."""
        if pages:
            self.alloc.free(list(pages))

    @staticmethod
    def bind(r, main_pages: List[int], swa_pages: List[int], upd: List[int]) -> None:
        for m, s in zip(main_pages, swa_pages):
            upd += [-1, m, s]
            r.swa_pages.append(s)

    def trim(self, r, kv_len: int) -> None:
        """Free the window pages of logical pages whose tokens every later query is past: a query at
        position >= kv_len attends keys > kv_len - window, so pages ending at or before kv_len - window - P
        are never read again (one page of slack)."""
        keep_from = (kv_len - self.window) // self.P - 1
        if keep_from <= r.swa_freed:
            return
        upto = min(keep_from, len(r.swa_pages))
        freed = [p for p in r.swa_pages[r.swa_freed:upto] if p]
        for j in range(r.swa_freed, upto):
            r.swa_pages[j] = 0
        r.swa_freed = upto
        if freed:
            self.alloc.free_after(freed, r.last_step)

    def release(self, r) -> None:
        freed = [p for p in r.swa_pages[r.swa_freed:] if p]
        if freed:
            self.alloc.free_after(freed, r.last_step)
        r.swa_pages, r.swa_freed = [], 0

    def retire(self, epoch: int) -> None:
        self.alloc.retire(epoch)

    def reset(self) -> None:
        self.alloc.reset()


class SwaTranslate:
    """Device side: the main->window page map and the per-step translation of block tables and slots."""

    def __init__(self, num_main_pages: int, page_size: int, device):
        self.map = torch.zeros(num_main_pages, dtype=torch.int32, device=device)
        self.P = page_size

    def apply(self, u: torch.Tensor) -> torch.Tensor:
        """u: [U, 3] int64 update triples; applies the (-1, main, window) ones to the map and returns a mask
        of them (the caller routes the others to the block table)."""
        m = u[:, 0] < 0
        self.map[torch.where(m, u[:, 1], torch.zeros_like(u[:, 1]))] = torch.where(
            m, u[:, 2], torch.zeros_like(u[:, 2])).to(torch.int32)
        return m

    def batch(self, fb):
        """The ForwardBatch the sliding layers see (cached on fb): block table and write slots in window
        pages; mixed steps translate their decode and extend parts too."""
        got = fb.extra.get("swa_fb")
        if got is not None:
            return got
        out = self._translate(fb)
        parts = fb.extra.get("parts")
        if parts is not None:
            D, dec, ext = parts
            out.extra = dict(fb.extra)
            out.extra["parts"] = (D, self._translate(dec), self._translate(ext))
        fb.extra["swa_fb"] = out
        return out

    def _translate(self, fb):
        bt = self.map[fb.block_table.clamp(min=0).long()]
        loc = fb.out_cache_loc
        P = self.P
        page = torch.div(loc.clamp(min=0), P, rounding_mode="floor")
        sloc = torch.where(loc >= 0, self.map[page].long() * P + loc.clamp(min=0) % P, torch.full_like(loc, -1))
        return dataclasses.replace(fb, block_table=bt, out_cache_loc=sloc, extra={})
