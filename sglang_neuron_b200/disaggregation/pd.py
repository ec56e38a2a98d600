"""Disaggregated prefill/decode on one box: a prefill TP group and a decode TP group inside one process
world, KV pages moved rank-to-rank (prefill tp_rank i -> decode tp_rank i, same head shard) by P2P copies
over NVLink (NCCL send/recv on a dedicated stream; gloo on the CPU tier), with the control plane on the
process group's store.

Parity: the reference's PD path (sglang_neuron/disaggregation/*, sglang_patches/nixl_*, pd_*): the decode
side pre-allocates pages and publishes where the KV must land (TransferInfo), the prefill side writes the
pool pages and the first token, then posts a status; failures are contained per request (peer refusal,
status lock, settle-then-ack, decode KV quarantine: a page that a transfer may still write is never reused).
NIXL/EFA becomes P2P inside one NVLink domain.

Protocol for request `rid` (sequence number n):
  1. prefill leader, after the prompt's first token is known: store["pd/hdr/n"] = (rid, prompt, first_token,
     params, n_pages) and marks the request's pages "sending".
  2. decode leader polls the store, broadcasts the header to its group; every decode rank allocates
     n_pages, posts irecv from its prefill peer on the transfer stream, then the leader sets store["pd/ready/n"].
  3. prefill ranks poll "ready", post isend of [layers, K|V, n_pages, ...] from the pool, and free the pages
     once the send's event completed.
  4. decode ranks, once their recv event completed (the leader decides, followers wait), insert the request
     with kv_len = prompt length and the first token in the relay, and decode it like any other request.
  A header whose ready flag does not appear within `timeout_s` is aborted on the prefill side (pages freed);
  a receive that does not complete within `timeout_s` is aborted on the decode side and its pages are
  quarantined (never freed) because the peer may still write them.
"""
from __future__ import annotations

import dataclasses
import logging
import pickle
import time
from typing import Dict, List, Optional, Tuple

import torch
import torch.distributed as dist

from ..managers.schedule_batch import Req, SamplingParams
from ..parallel.state import get_state

logger = logging.getLogger(__name__)

POLL_WIDTH = 64  # transfers whose state one poll reduce carries (later ones wait for the next poll)


@dataclasses.dataclass
class Header:
    seq: int
    rid: str
    prompt: List[int]
    first_token: int
    params: SamplingParams
    n_pages: int


def gather_pages(pool, pages: torch.Tensor) -> torch.Tensor:
    """Pack the given pages of every layer into one contiguous buffer [L, 2, n, ...]."""
    ks = [k.index_select(0, pages) for k in _k_buffers(pool)]
    vs = [v.index_select(0, pages) for v in _v_buffers(pool)]
    return torch.stack([torch.stack([k, v]) for k, v in zip(ks, vs)]).contiguous()


def scatter_pages(pool, pages: torch.Tensor, buf: torch.Tensor) -> None:
    for li, (k, v) in enumerate(zip(_k_buffers(pool), _v_buffers(pool))):
        k.index_copy_(0, pages, buf[li, 0])
        v.index_copy_(0, pages, buf[li, 1])


def _k_buffers(pool):
    return pool.k_buffers if hasattr(pool, "k_buffers") else pool.buffers


def _v_buffers(pool):
    return pool.v_buffers if hasattr(pool, "v_buffers") else pool.buffers


def page_buffer_shape(pool, n: int) -> Tuple[int, ...]:
    k0 = _k_buffers(pool)[0]
    return (len(_k_buffers(pool)), 2, n) + tuple(k0.shape[1:])


class Transfer:
    """One posted point-to-point transfer (the torch Work plus its completion state)."""

    __slots__ = ("work", "completed")

    def __init__(self, work):
        self.work = work
        self.completed = False


class PDLink:
    """Store-based control plane + rank-to-rank data plane between the two groups."""

    def __init__(self, role: str, tp_size: int, store, timeout_s: float = 60.0):
        st = get_state()
        self.role = role
        self.tp = tp_size
        self.store = store
        self.timeout_s = timeout_s
        self.peer = (st.tp_rank + tp_size) if role == "prefill" else st.tp_rank
        self.is_leader = st.tp_rank == 0
        self.device = st.device
        self.stream = torch.cuda.Stream(device=self.device) if self.device.type == "cuda" else None

    def put(self, key: str, obj) -> None:
        self.store.set(key, pickle.dumps(obj))

    def has(self, key: str) -> bool:
        return self.store.check([key])

    def get(self, key: str):
        return pickle.loads(self.store.get(key))

    def send(self, buf: torch.Tensor):
        if self.stream is None:
            return Transfer(dist.isend(buf, self.peer))
        self.stream.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(self.stream):
            work = dist.isend(buf, self.peer)
        return Transfer(work)

    def done(self, work) -> bool:
        """Has a posted transfer completed? NCCL work reports its CUDA event; gloo point-to-point work only
        completes through wait(), which on the CPU tier blocks until the matching peer call arrived."""
        if work.completed:
            return True
        if self.stream is None:
            # gloo point-to-point work only completes through wait(), and a wait that times out closes the
            # pair, so wait without a short limit: the protocol has already posted the matching call (decode
            # posts its receive before acknowledging; prefill sends only after the acknowledgement), and the
            # process group's timeout bounds it
            work.work.wait()
            work.completed = True
            return True
        work.completed = work.work.is_completed()
        return work.completed

    def finish(self, work) -> None:
        """Block until a transfer that done() reported (or is about to report) completed."""
        if self.stream is None:
            while not self.done(work):
                pass
        else:
            work.work.wait()
            work.completed = True

    def recv(self, buf: torch.Tensor):
        if self.stream is None:
            return Transfer(dist.irecv(buf, self.peer))
        with torch.cuda.stream(self.stream):
            work = dist.irecv(buf, self.peer)
        return Transfer(work)


class PrefillSide:
    """Wraps a prefill-role Engine: every request is prefilled (first token only) and handed to decode."""

    def __init__(self, engine, link: PDLink):
        self.engine = engine
        self.link = link
        self.seq = 0
        self.pending: Dict[int, Tuple[Req, List[int], float]] = {}   # seq -> (req, pages, t_published)
        self.sending: List[Tuple[int, object, torch.Tensor, List[int]]] = []
        self.aborted: List[str] = []
        self.sent = 0
        self.user_params: Dict[str, SamplingParams] = {}
        sched = engine.scheduler
        self._orig_finish = sched._finish
        sched._finish = self._on_finish  # keep pages of finished prefills until their KV left

    def submit(self, rid: str, prompt: List[int], params: SamplingParams):
        self.user_params[rid] = params  # the decode side serves the request with these
        p = dataclasses.replace(params, max_new_tokens=1)
        self.engine.scheduler.add_request(rid, prompt, p)

    def _on_finish(self, r: Req, reason: str) -> None:
        sched = self.engine.scheduler
        r.finished = True
        r.finish_reason = reason
        if r in sched.running:
            sched.running.remove(r)
        n_pages = (r.prompt_len + sched.P - 1) // sched.P
        pages = list(r.pages[:n_pages])
        seq = self.seq
        self.seq += 1
        if self.link.is_leader:
            params = self.user_params.pop(r.rid, r.params)
            self.link.put(f"pd/hdr/{seq}", Header(seq, r.rid, r.origin_input_ids, r.output_ids[0], params, n_pages))
        else:
            self.user_params.pop(r.rid, None)
        self.pending[seq] = (r, pages, time.time())
        sched.finished_reqs.append(r)
        sched.finished_by_rid[r.rid] = r

    def _release(self, r: Req) -> None:
        self.engine.scheduler._release(r)

    def poll(self) -> None:
        """Post sends for headers the decode side acknowledged; free pages of completed sends."""
        sched = self.engine.scheduler
        for seq in sorted(self.pending):
            r, pages, t0 = self.pending[seq]
            key = f"pd/ready/{seq}"
            if self.link.has(key):
                status = self.link.get(key)
                del self.pending[seq]
                if status != "ready":
                    self._release(r)
                    self.aborted.append(r.rid)
                    continue
                idx = torch.tensor(pages, dtype=torch.long, device=self.link.device)
                buf = gather_pages(self.engine.runner.kv_pool, idx)
                work = self.link.send(buf)
                self.sending.append((seq, work, buf, r))
            elif time.time() - t0 > self.link.timeout_s:
                # peer never acknowledged: abort and free (nothing was sent, nothing can land)
                del self.pending[seq]
                self._release(r)
                self.aborted.append(r.rid)
                if self.link.is_leader:
                    self.link.put(f"pd/abort/{seq}", "prefill-timeout")
        still = []
        for seq, work, buf, r in self.sending:
            if self.link.done(work):
                self._release(r)
                self.sent += 1
            else:
                still.append((seq, work, buf, r))
        self.sending = still

    def step(self) -> None:
        self.engine.scheduler.step()
        self.poll()


class DecodeSide:
    """Wraps a decode-role Engine: receives prefilled requests and decodes them."""

    def __init__(self, engine, link: PDLink):
        self.engine = engine
        self.link = link
        self.next_seq = 0
        self.receiving: List[Tuple[Header, object, torch.Tensor, List[int], int, float]] = []
        self.quarantined: List[int] = []
        self.aborted: List[str] = []
        # poll reduce: the MIN over the group's ranks of each transfer's state (2 received, 1 waiting,
        # 0 timed out) through node shared memory; None (one rank, or no shared memory) keeps the leader's
        # decision broadcast over gloo. Parity: the reference's poll reduce over node shm
        # (sglang_neuron/disaggregation/poll_reduce.py:68-108).
        from ..managers.scheduler import _make_shm
        self._poll = _make_shm(get_state(), POLL_WIDTH, "pdpoll")

    def poll(self) -> None:
        sched = self.engine.scheduler
        st = get_state()
        # 1. leader discovers new headers; the group learns them through the broadcast below
        new: List[Header] = []
        if self.link.is_leader:
            while self.link.has(f"pd/hdr/{self.next_seq}"):
                new.append(self.link.get(f"pd/hdr/{self.next_seq}"))
                self.next_seq += 1
        if st.tp_size > 1:
            from ..parallel.collectives import cpu_broadcast_object
            new = cpu_broadcast_object(new, src=0)
            if not self.link.is_leader:
                self.next_seq += len(new)
        for h in new:
            if not sched.free_slots:
                if self.link.is_leader:
                    self.link.put(f"pd/ready/{h.seq}", "refused: no request slot")
                self.aborted.append(h.rid)
                continue
            pages = sched._alloc_pages(h.n_pages)
            if pages is None:
                if self.link.is_leader:
                    self.link.put(f"pd/ready/{h.seq}", "refused: no KV pages")
                self.aborted.append(h.rid)
                continue
            buf = torch.empty(page_buffer_shape(self.engine.runner.kv_pool, h.n_pages),
                              dtype=self.engine.runner.kv_pool.dtype, device=self.link.device)
            work = self.link.recv(buf)
            if self.link.is_leader:
                self.link.put(f"pd/ready/{h.seq}", "ready")
            self.receiving.append((h, work, buf, pages, sched.epoch, time.time()))
        # 2. completed receives become running requests: every rank's own transfer state, MIN-reduced (or the
        #    leader decides and followers wait for their own)
        done_seqs: List[int] = []
        if self._poll is not None:
            items = self.receiving[:POLL_WIDTH]
            now = time.time()
            states = [2 if self.link.done(work) else (0 if now - t0 > self.link.timeout_s else 1)
                      for _h, work, _b, _p, _e, t0 in items]
            red = self._poll.min(states + [2] * (POLL_WIDTH - len(states)), timeout_s=1800.0)
            for (h, *_rest), s in zip(items, red):
                if s == 2:
                    done_seqs.append(h.seq)
                elif s == 0:
                    done_seqs.append(-h.seq - 1)  # abort marker
        elif self.link.is_leader:
            for h, work, buf, pages, _e, t0 in self.receiving:
                if self.link.done(work):
                    done_seqs.append(h.seq)
                elif time.time() - t0 > self.link.timeout_s:
                    done_seqs.append(-h.seq - 1)  # abort marker
        if st.tp_size > 1 and self._poll is None:
            from ..parallel.collectives import cpu_broadcast_object
            done_seqs = cpu_broadcast_object(done_seqs, src=0)
        keep = []
        for item in self.receiving:
            h, work, buf, pages, _e, _t = item
            if h.seq in done_seqs:
                self.link.finish(work)
                self._admit(h, buf, pages)
            elif (-h.seq - 1) in done_seqs:
                self.quarantined += pages  # the peer may still write them: never reuse
                self.aborted.append(h.rid)
            else:
                keep.append(item)
        self.receiving = keep

    def _admit(self, h: Header, buf: torch.Tensor, pages: List[int]) -> None:
        sched = self.engine.scheduler
        runner = self.engine.runner
        idx = torch.tensor(pages, dtype=torch.long, device=self.link.device)
        if self.link.stream is not None:
            torch.cuda.current_stream(self.link.device).wait_stream(self.link.stream)
        scatter_pages(runner.kv_pool, idx, buf)
        r = Req(h.rid, h.prompt, h.params, eos_ids=[] if h.params.ignore_eos else sched.eos)
        r.slot = sched.free_slots.pop()
        r.pages = list(pages)
        r.kv_len = len(h.prompt)
        r.prefill_target = len(h.prompt)
        r.output_ids = [h.first_token]
        r.scheduled_outputs = 1
        r.first_token_time = time.perf_counter()
        r.token_times.append(r.first_token_time)
        row = torch.tensor(pages, dtype=torch.int32, device=runner.device)
        runner.req_to_page.table[r.slot, : len(pages)] = row
        runner.relay[r.slot] = h.first_token
        sched.reqs_by_rid[r.rid] = r
        if len(r.output_ids) >= r.params.max_new_tokens:
            sched._finish(r, "length")
        else:
            sched.running.append(r)

    def step(self) -> None:
        self.poll()
        self.engine.scheduler.step()
