"""Hierarchical KV cache: a host-memory tier below the device prefix cache (HiCache).

Pages that enter the device radix tree are also written to a pinned host pool (write-through), indexed by
a page-granular hash chain of the token prefix (hash of page i covers tokens [0, (i+1) * page)). When the
device tree has evicted a prefix, a new request whose prompt continues past the device match looks the
following pages up on the host and loads them into freshly allocated device pages instead of recomputing
them. Host slots are recycled least-recently-used first.

Ordering on a GPU: writes are issued on a copy stream after an event recorded on the compute stream when
the pages were inserted (the steps that wrote them come first); the pages of an eviction are handed back
to the allocator only after pending writes finished (`sync_writes`). Loads are issued on the copy stream
and the compute stream waits on their event before the next step (`wait_loads`). The copies themselves are
one launch per batch of pages (csrc/kernels/kv_page_copy.cu reads/writes pinned host memory directly).

Parity: the reference's HiCache L2 host pools (sglang_neuron/mem_cache/host_pool.py:233 TransferEngine,
hicache_hold.py, host_budget.py): a pinned layer-first host mirror with batched DMA on store and load.
"""
from __future__ import annotations

from collections import OrderedDict
from typing import List, Optional, Sequence, Tuple

import torch


def chain_hashes(tokens: Sequence[int], page_size: int, n_pages: int) -> List[int]:
    """Hash of every full page's prefix: h_i = hash((h_{i-1}, tokens of page i))."""
    out, h = [], 0
    for i in range(n_pages):
        h = hash((h, tuple(tokens[i * page_size:(i + 1) * page_size])))
        out.append(h)
    return out


class HostKVPool:
    """Host mirror of a device KV pool: one [num_host_pages, ...page shape...] tensor per device buffer."""

    def __init__(self, device_buffers: List[torch.Tensor], num_host_pages: int, pin: bool):
        self.device_buffers = device_buffers
        self.buffers = [torch.zeros((num_host_pages,) + tuple(b.shape[1:]), dtype=b.dtype, pin_memory=pin)
                        for b in device_buffers]
        self.num_pages = num_host_pages
        self.page_bytes = device_buffers[0][0].numel() * device_buffers[0].element_size() if device_buffers else 0


def _pool_buffers(pool) -> List[torch.Tensor]:
    if hasattr(pool, "k_buffers"):
        return list(pool.k_buffers) + list(pool.v_buffers)
    return list(pool.buffers)


class HiCache:
    def __init__(self, device_pool, page_size: int, num_host_pages: int, device: torch.device):
        self.page_size = page_size
        self.device = torch.device(device)
        self.cuda = self.device.type == "cuda"
        self.host = HostKVPool(_pool_buffers(device_pool), num_host_pages, pin=self.cuda)
        self.index: "OrderedDict[int, int]" = OrderedDict()  # chain hash -> host slot, LRU first
        self.free_slots = list(range(num_host_pages - 1, -1, -1))
        self.stream = torch.cuda.Stream(self.device) if self.cuda else None
        self._write_ev: Optional[torch.cuda.Event] = None
        self._load_evs: List[torch.cuda.Event] = []
        self.stats = {"written_pages": 0, "loaded_pages": 0, "host_evictions": 0}
        if self.cuda:
            self._dev_bases = torch.tensor([b.data_ptr() for b in self.host.device_buffers], dtype=torch.int64,
                                           device=self.device)
            self._host_bases = torch.tensor([b.data_ptr() for b in self.host.buffers], dtype=torch.int64,
                                            device=self.device)

    # ---- copies ------------------------------------------------------------------------------------
    def _copy(self, to_host: bool, dev_pages: List[int], host_slots: List[int]) -> None:
        if not dev_pages:
            return
        if not self.cuda:
            di, hi = torch.tensor(dev_pages), torch.tensor(host_slots)
            for d, h in zip(self.host.device_buffers, self.host.buffers):
                if to_host:
                    h.index_copy_(0, hi, d.index_select(0, di))
                else:
                    d.index_copy_(0, di, h.index_select(0, hi))
            return
        from .._ext import kernels
        dp = torch.tensor(dev_pages, dtype=torch.int32).pin_memory().to(self.device, non_blocking=True)
        hp = torch.tensor(host_slots, dtype=torch.int32).pin_memory().to(self.device, non_blocking=True)
        if to_host:
            kernels().kv_page_copy(self._dev_bases, self._host_bases, dp, hp, self.host.page_bytes)
        else:
            kernels().kv_page_copy(self._host_bases, self._dev_bases, hp, dp, self.host.page_bytes)

    def _take_slot(self) -> Optional[int]:
        if self.free_slots:
            return self.free_slots.pop()
        if not self.index:
            return None
        _, slot = self.index.popitem(last=False)  # least recently used
        self.stats["host_evictions"] += 1
        return slot

    # ---- write-through ---------------------------------------------------------------------------
    def write_through(self, tokens: Sequence[int], device_pages: Sequence[int]) -> int:
        """Back up the full pages of a prefix (page i of `device_pages` holds tokens of page i). Returns the
        number of pages written (pages already on the host are only refreshed in the LRU order)."""
        n = min(len(device_pages), len(tokens) // self.page_size)
        hashes = chain_hashes(tokens, self.page_size, n)
        dev, slots = [], []
        for h, p in zip(hashes, device_pages[:n]):
            if h in self.index:
                self.index.move_to_end(h)
                continue
            s = self._take_slot()
            if s is None:
                break
            self.index[h] = s
            dev.append(int(p))
            slots.append(s)
        if not dev:
            return 0
        if self.cuda:
            ev = torch.cuda.Event()
            ev.record()  # after every step that wrote these pages
            with torch.cuda.stream(self.stream):
                self.stream.wait_event(ev)
                self._copy(True, dev, slots)
                self._write_ev = torch.cuda.Event()
                self._write_ev.record(self.stream)
        else:
            self._copy(True, dev, slots)
        self.stats["written_pages"] += len(dev)
        return len(dev)

    def sync_writes(self) -> None:
        """Block until every issued write finished (before device pages they read are reused)."""
        if self._write_ev is not None:
            self._write_ev.synchronize()
            self._write_ev = None

    # ---- lookup and load -------------------------------------------------------------------------
    def match(self, tokens: Sequence[int], start_page: int, max_pages: int) -> List[int]:
        """Host slots of pages start_page, start_page + 1, ... while they are all on the host."""
        n = min(start_page + max_pages, len(tokens) // self.page_size)
        hashes = chain_hashes(tokens, self.page_size, n)
        out = []
        for h in hashes[start_page:]:
            s = self.index.get(h)
            if s is None:
                break
            self.index.move_to_end(h)
            out.append(s)
        return out

    def load(self, host_slots: List[int], device_pages: List[int]) -> None:
        if not host_slots:
            return
        if self.cuda:
            with torch.cuda.stream(self.stream):
                self._copy(False, list(device_pages), list(host_slots))
                ev = torch.cuda.Event()
                ev.record(self.stream)
            self._load_evs.append(ev)
        else:
            self._copy(False, list(device_pages), list(host_slots))
        self.stats["loaded_pages"] += len(host_slots)

    def wait_loads(self) -> None:
        """Make the compute stream wait for issued loads (call before launching the next step)."""
        if self.cuda:
            cur = torch.cuda.current_stream(self.device)
            for ev in self._load_evs:
                cur.wait_event(ev)
        self._load_evs.clear()

    def reset(self) -> None:
        self.sync_writes()
        self.index.clear()
        self.free_slots = list(range(self.host.num_pages - 1, -1, -1))
