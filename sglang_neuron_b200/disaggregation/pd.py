"""Disaggregated prefill/decode on one box: a prefill TP group and a decode TP group inside one process
world, with the control plane on the process group's store.

Data plane on GPUs (P2P): every decode rank exports its KV pool buffers over CUDA IPC once; a prefill rank
maps them and, when a request's destination pages are known, one copy kernel writes the request's pages of
every layer straight from its own pool into the decode pool's pages over NVLink (plain 16-byte peer stores,
no staging on either side). Head-major slicing: each rank's pool holds a contiguous range of KV heads, and a
page's heads are contiguous, so a prefill rank copies exactly the overlap of its head range with each decode
rank's (any TP sizes on the two sides; a head held by several prefill ranks is sent by the lowest of them).
Settle-then-ack: a prefill rank posts pd/done/<seq>/<src>/<dst> only after its copy kernel completed, and a
decode rank admits the request once every done key it expects exists. On the CPU tier the data plane is
gloo send/recv of packed head slices along the same plan (whole pages rank to rank when both groups shard
alike). The two groups may differ in TP size: launch them as DP replicas with `replica_tp_sizes` (prefill first)
and give each PDLink the other group's size.

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


def _is_mha(pool) -> bool:
    return hasattr(pool, "k_buffers")


def head_slice(pool, buf: torch.Tensor, off_bytes: int, nbytes: int) -> torch.Tensor:
    """The heads [off, off + n) of a packed [L, 2, n_pages, heads, page, D] buffer (byte offsets within a page,
    as slice_plan gives them), contiguous; the whole buffer when the slice covers every head (and for latent
    pools, whose page is one 'head')."""
    geo = pool_geometry(pool, 0)
    h0, nh = off_bytes // geo["head_bytes"], nbytes // geo["head_bytes"]
    if not _is_mha(pool) or (h0 == 0 and nh == geo["heads"]):
        return buf
    return buf[:, :, :, h0:h0 + nh].contiguous()


def scatter_head_slice(pool, pages: torch.Tensor, buf: torch.Tensor, off_bytes: int, nbytes: int) -> None:
    """Write a packed head slice (head_slice's layout) into the given pages at heads [off, off + n)."""
    geo = pool_geometry(pool, 0)
    h0, nh = off_bytes // geo["head_bytes"], nbytes // geo["head_bytes"]
    if not _is_mha(pool) or (h0 == 0 and nh == geo["heads"]):
        scatter_pages(pool, pages, buf)
        return
    for li, (k, v) in enumerate(zip(_k_buffers(pool), _v_buffers(pool))):
        for src, dst in ((buf[li, 0], k), (buf[li, 1], v)):
            rows = dst.index_select(0, pages)
            rows[:, h0:h0 + nh] = src
            dst.index_copy_(0, pages, rows)


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


class DoneKeys:
    """A P2P transfer as the decode side sees it: complete once every expected done key is in the store."""

    __slots__ = ("keys", "completed")

    def __init__(self, keys: List[str]):
        self.keys = keys
        self.completed = False


def _pool_buffers(pool) -> List[torch.Tensor]:
    """Every layer buffer of a pool, in a fixed order (MHA: K buffers then V buffers; MLA: latent buffers)."""
    if hasattr(pool, "k_buffers"):
        return list(pool.k_buffers) + list(pool.v_buffers)
    return list(pool.buffers)


def pool_geometry(pool, head_start: int) -> Dict:
    """Page and head-slice sizes of a pool: [pages, heads, page, D] for MHA (a head's slice of a page is
    contiguous), [pages, page, width] for MLA (one 'head')."""
    b0 = _pool_buffers(pool)[0]
    page_bytes = b0[0].numel() * b0.element_size()
    heads = b0.shape[1] if hasattr(pool, "k_buffers") else 1
    return {"page_bytes": page_bytes, "heads": heads, "head_start": head_start, "head_bytes": page_bytes // heads,
            "buffers": len(_pool_buffers(pool))}


def export_pool(pool, head_start: int) -> Dict:
    """IPC handles of the pool's buffers (allocation handle + byte offset of the buffer inside it)."""
    out = []
    for b in _pool_buffers(pool):
        info = b.untyped_storage()._share_cuda_()
        handle, off = bytes(info[1]), info[3]
        # the caching allocator prefixes the 64-byte cudaIpcMemHandle with its segment kind ('c': cudaMalloc);
        # expandable (virtual-memory) segments have no IPC handle of this kind
        if len(handle) == 65:
            if handle[:1] != b"c":
                raise RuntimeError("PD P2P needs cudaMalloc-backed KV pools (expandable segments are not shareable)")
            handle = handle[1:]
        out.append((handle, int(off) + b.storage_offset() * b.element_size()))
    return {"bufs": out, **pool_geometry(pool, head_start)}


def slice_plan(src_geo: List[Dict], dst_geo: List[Dict]) -> List[Tuple[int, int, int, int, int]]:
    """(src rank, dst rank, src byte offset, dst byte offset, bytes) per page for every overlap of a source
    rank's head range with a destination rank's; each head comes from the lowest source rank holding it."""
    plan = []
    for j, d in enumerate(dst_geo):
        d0, d1 = d["head_start"], d["head_start"] + d["heads"]
        covered = set()
        for i, s_ in enumerate(src_geo):
            s0, s1 = s_["head_start"], s_["head_start"] + s_["heads"]
            lo, hi = max(s0, d0), min(s1, d1)
            heads = [h for h in range(lo, hi) if h not in covered]
            if not heads:
                continue
            if s_["head_bytes"] != d["head_bytes"]:
                raise ValueError("PD: prefill and decode pools differ in page size, head dim or KV dtype")
            lo, hi = heads[0], heads[-1] + 1
            covered.update(range(lo, hi))
            plan.append((i, j, (lo - s0) * s_["head_bytes"], (lo - d0) * d["head_bytes"], (hi - lo) * d["head_bytes"]))
        if covered != set(range(d0, d1)):
            raise ValueError(f"PD: decode rank {j} heads {d0}..{d1} not all held by the prefill group")
    return plan


class PeerPools:
    """The decode group's pools mapped into this prefill rank (one IPC open per allocation)."""

    def __init__(self, metas: List[Dict], device):
        from .._ext import kernels
        self.k = kernels()
        self.opened: Dict[bytes, int] = {}
        self.geo = metas
        self.bases = []
        for m in metas:
            ptrs = []
            for handle, off in m["bufs"]:
                if handle not in self.opened:
                    self.opened[handle] = self.k.symm_open(handle)
                ptrs.append(self.opened[handle] + off)
            self.bases.append(torch.tensor(ptrs, dtype=torch.int64, device=device))

    def close(self) -> None:
        for p in self.opened.values():
            self.k.symm_close(p, False)
        self.opened = {}


class PDLink:
    """Store-based control plane + rank-to-rank data plane between the two groups."""

    def __init__(self, role: str, tp_size: int, store, timeout_s: float = 60.0, peer_tp: Optional[int] = None):
        """tp_size: this group's TP size; peer_tp: the other group's (default: the same). The prefill group holds
        global ranks [0, n_prefill), the decode group the n_decode ranks after it."""
        st = get_state()
        self.role = role
        self.tp = tp_size
        other = tp_size if peer_tp is None else int(peer_tp)
        self.n_prefill = tp_size if role == "prefill" else other
        self.n_decode = tp_size if role == "decode" else other
        self.store = store
        self.timeout_s = timeout_s
        self.peer = (st.tp_rank + tp_size) if role == "prefill" else st.tp_rank
        self.tp_rank = st.tp_rank
        self.is_leader = st.tp_rank == 0
        self.device = st.device
        self.stream = torch.cuda.Stream(device=self.device) if self.device.type == "cuda" else None
        self.p2p = self.device.type == "cuda"  # CUDA IPC page copies; gloo send/recv on the CPU tier

    def wait_keys(self, keys: List[str], timeout_s: float = 600.0) -> None:
        t0 = time.time()
        while not self.store.check(keys):
            if time.time() - t0 > timeout_s:
                raise TimeoutError(f"PD: store keys {keys} never appeared")
            time.sleep(0.001)


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
        if isinstance(work, DoneKeys):
            work.completed = self.store.check(work.keys)
            return work.completed
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
        if isinstance(work, DoneKeys):
            return
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

    def prefill_rank(self, i: int) -> int:
        return i

    def decode_rank(self, j: int) -> int:
        return self.n_prefill + j

    def send_to(self, buf: torch.Tensor, dst: int):
        peer, self.peer = self.peer, dst
        try:
            return self.send(buf)
        finally:
            self.peer = peer

    def recv_from(self, buf: torch.Tensor, src: int):
        peer, self.peer = self.peer, src
        try:
            return self.recv(buf)
        finally:
            self.peer = peer

    def done_all(self, works) -> bool:
        return all(self.done(w) for w in works)

    def finish_all(self, works) -> None:
        for w in works:
            self.finish(w)


def _head_start(engine) -> int:
    a = engine.runner.model.attention_layers()[0]
    return int(getattr(getattr(a, "qkv_proj", None), "kv_head_start", 0))


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
        self.on_send = None  # test seam: called with (rid, pages) when a request's pages are handed off
        sched = engine.scheduler
        self._orig_finish = sched._finish
        sched._finish = self._on_finish  # keep pages of finished prefills until their KV left
        self.peers: Optional[PeerPools] = None
        self.plan: Optional[List[Tuple[int, int, int, int, int]]] = None
        pool = engine.runner.kv_pool
        self.geo = pool_geometry(pool, _head_start(engine))
        link.put(f"pd/pgeo/{link.tp_rank}", self.geo)
        if link.p2p:
            self.src_bases = torch.tensor([b.data_ptr() for b in _pool_buffers(pool)], dtype=torch.int64,
                                          device=link.device)

    def _ensure_peers(self) -> None:
        """Keep this rank's rows of the head-slice plan (once every decode rank published its pool) and, on
        GPUs, map the decode group's pools."""
        if self.plan is not None:
            return
        link = self.link
        n_dec, n_pre = link.n_decode, link.n_prefill
        link.wait_keys([f"pd/ipc/{j}" for j in range(n_dec)] + [f"pd/pgeo/{i}" for i in range(n_pre)])
        metas = [link.get(f"pd/ipc/{j}") for j in range(n_dec)]
        pgeo = [link.get(f"pd/pgeo/{i}") for i in range(n_pre)]
        self.plan = [p for p in slice_plan(pgeo, metas) if p[0] == link.tp_rank]
        if link.p2p:
            self.peers = PeerPools(metas, link.device)

    def _send_p2p(self, seq: int, pages: List[int], dst_pages: List[int]):
        """One copy launch per destination rank on the transfer stream; returns (event, done keys)."""
        from .._ext import kernels
        self._ensure_peers()
        link = self.link
        src = torch.tensor(pages, dtype=torch.int32, device=link.device)
        dst = torch.tensor(dst_pages, dtype=torch.int32, device=link.device)
        link.stream.wait_stream(torch.cuda.current_stream(link.device))
        keys = []
        with torch.cuda.stream(link.stream):
            for i, j, so, do, nb in self.plan:
                kernels().kv_page_slice_copy(self.src_bases, self.peers.bases[j], src, dst, self.geo["page_bytes"],
                                             self.peers.geo[j]["page_bytes"], so, do, nb)
                keys.append(f"pd/done/{seq}/{i}/{j}")
            ev = torch.cuda.Event()
            ev.record(link.stream)
        return ev, keys, (src, dst)

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
                ok = status == "ready" or (isinstance(status, tuple) and status[0] == "ready")
                if not ok:
                    self._release(r)
                    self.aborted.append(r.rid)
                    continue
                if self.on_send is not None:
                    self.on_send(r.rid, pages)
                if self.link.p2p:
                    ev, keys, keep = self._send_p2p(seq, pages, list(status[1]))
                    self.sending.append((seq, (ev, keys), keep, r))
                    continue
                # packed transfer (CPU tier): this rank's head slice of the pages to every decode rank that holds
                # those heads (the whole pages rank to rank when both groups shard alike)
                self._ensure_peers()
                pool = self.engine.runner.kv_pool
                idx = torch.tensor(pages, dtype=torch.long, device=self.link.device)
                buf = gather_pages(pool, idx)
                works, keep = [], []
                for _i, j, so, _do, nb in self.plan:
                    piece = head_slice(pool, buf, so, nb)
                    works.append(self.link.send_to(piece, self.link.decode_rank(j)))
                    keep.append(piece)
                self.sending.append((seq, works, keep, r))
            elif time.time() - t0 > self.link.timeout_s:
                # peer never acknowledged: abort and free (nothing was sent, nothing can land)
                del self.pending[seq]
                self._release(r)
                self.aborted.append(r.rid)
                if self.link.is_leader:
                    self.link.put(f"pd/abort/{seq}", "prefill-timeout")
        still = []
        for seq, work, buf, r in self.sending:
            if isinstance(work, tuple):  # P2P: settle (copy kernel complete), then acknowledge, then free
                ev, keys = work
                if ev.query():
                    for k in keys:
                        self.link.put(k, "ok")
                    self._release(r)
                    self.sent += 1
                else:
                    still.append((seq, work, buf, r))
            elif self.link.done_all(work):
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
        self._rows: Optional[List[Tuple[int, int, int, int, int]]] = None  # plan rows feeding this rank
        self.on_admit = None  # test seam: called with (header, pages) when a request's KV has landed
        pool = engine.runner.kv_pool
        link.put(f"pd/ipc/{link.tp_rank}", export_pool(pool, _head_start(engine)) if link.p2p
                 else pool_geometry(pool, _head_start(engine)))

    def _plan_rows(self) -> List[Tuple[int, int, int, int, int]]:
        """The head-slice plan rows whose destination is this rank (once both groups published their pools)."""
        if self._rows is None:
            link = self.link
            link.wait_keys([f"pd/ipc/{j}" for j in range(link.n_decode)] +
                           [f"pd/pgeo/{i}" for i in range(link.n_prefill)])
            metas = [link.get(f"pd/ipc/{j}") for j in range(link.n_decode)]
            pgeo = [link.get(f"pd/pgeo/{i}") for i in range(link.n_prefill)]
            self._rows = [p for p in slice_plan(pgeo, metas) if p[1] == link.tp_rank]
        return self._rows

    def _done_keys(self, seq: int) -> List[str]:
        return [f"pd/done/{seq}/{i}/{j}" for i, j, *_ in self._plan_rows()]

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
            if self.link.p2p:
                # the prefill ranks write straight into these pages; they are identical on every decode rank
                work, buf = DoneKeys(self._done_keys(h.seq)), None
                if self.link.is_leader:
                    self.link.put(f"pd/ready/{h.seq}", ("ready", list(pages)))
            else:
                # packed transfer (CPU tier): one receive per prefill rank holding some of this rank's heads
                pool = self.engine.runner.kv_pool
                shape = page_buffer_shape(pool, h.n_pages)
                head_bytes = pool_geometry(pool, 0)["head_bytes"]
                work, buf = [], []
                for i, _j, _so, do, nb in self._plan_rows():
                    shp = shape[:3] + (nb // head_bytes,) + shape[4:] if _is_mha(pool) else shape
                    b = torch.empty(shp, dtype=pool.dtype, device=self.link.device)
                    work.append(self.link.recv_from(b, self.link.prefill_rank(i)))
                    buf.append((do, nb, b))
                if self.link.is_leader:
                    self.link.put(f"pd/ready/{h.seq}", "ready")
            self.receiving.append((h, work, buf, pages, sched.epoch, time.time()))
        # 2. completed receives become running requests: every rank's own transfer state, MIN-reduced (or the
        #    leader decides and followers wait for their own)
        done_seqs: List[int] = []
        if self._poll is not None:
            items = self.receiving[:POLL_WIDTH]
            now = time.time()
            states = [2 if self._done(work) else (0 if now - t0 > self.link.timeout_s else 1)
                      for _h, work, _b, _p, _e, t0 in items]
            red = self._poll.min(states + [2] * (POLL_WIDTH - len(states)), timeout_s=1800.0)
            for (h, *_rest), s in zip(items, red):
                if s == 2:
                    done_seqs.append(h.seq)
                elif s == 0:
                    done_seqs.append(-h.seq - 1)  # abort marker
        elif self.link.is_leader:
            for h, work, buf, pages, _e, t0 in self.receiving:
                if self._done(work):
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
                if isinstance(work, list):
                    self.link.finish_all(work)
                else:
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
        if buf is not None:  # packed head slices (CPU tier); P2P copies already landed in the pages
            idx = torch.tensor(pages, dtype=torch.long, device=self.link.device)
            if self.link.stream is not None:
                torch.cuda.current_stream(self.link.device).wait_stream(self.link.stream)
            for do, nb, b in buf:
                scatter_head_slice(runner.kv_pool, idx, b, do, nb)
        if self.on_admit is not None:
            self.on_admit(h, pages)
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

    def _done(self, work) -> bool:
        return self.link.done_all(work) if isinstance(work, list) else self.link.done(work)

    def step(self) -> None:
        self.poll()
        self.engine.scheduler.step()
