"""Continuous-batching scheduler with chunked prefill, mixed prefill+decode steps, a page-granular prefix
cache, retire-aware page frees and an overlapped (one step ahead) launch loop.

Parity:
  * scheduling loop and prefill chunking: SGLang's Scheduler + PrefillAdder as the reference runs them
    (sglang_neuron/general_plugin.py:870 one request per prefill, sglang_patches/prefill_chunk_grid.py);
    here several requests may share a chunk and decode rows ride along (mixed step).
  * overlap: the reference's async execution (model_executor/async_execution.py: TokenRelay, PendingSample,
    CompletionEvent) launches step N+1 before reading step N's tokens; results are read after the launch.
  * frees held until the launches that read them retire (mem_cache/allocator.py:172).
  * SPMD ranks: every TP rank runs this scheduler on the same request stream (rank 0 broadcasts arrivals),
    so all ranks build identical batches and their collectives stay in lockstep (parity: DP identity /
    lockstep plan_step, graph_runner.py:822-869).
"""
from __future__ import annotations

import collections
import logging
import time
from typing import Callable, Deque, Dict, List, Optional, Tuple

import numpy as np

from ..mem_cache.allocator import RadixCacheHandle, make_page_allocator
from ..model_executor.forward_batch import ForwardMode
from ..parallel.collectives import cpu_broadcast_object
from ..parallel.state import get_state
from .schedule_batch import Req, SamplingParams, StepInput

logger = logging.getLogger(__name__)


class Scheduler:
    def __init__(self, args, cfg, runner):
        self.args = args
        self.cfg = cfg
        self.runner = runner
        self.P = args.page_size
        if get_state().dcp_size > 1:
            from ..parallel.dcp import DcpPageAllocator
            self.alloc = DcpPageAllocator(runner.num_pages, self.P, get_state().dcp_size)
        else:
            self.alloc = make_page_allocator(runner.num_pages, self.P, reserved=1)
        self.radix = None if args.disable_radix_cache else RadixCacheHandle(self.P)
        self.swa = None
        if getattr(runner, "swa_num_pages", 0):
            from ..mem_cache.hybrid_swa import SwaPageTracker
            self.swa = SwaPageTracker(make_page_allocator(runner.swa_num_pages, self.P, reserved=1),
                                      runner.swa_window, self.P)
        self.hicache = None
        if args.enable_hierarchical_cache and self.radix is not None:
            from ..mem_cache.hicache import HiCache
            n_host = args.hicache_host_pages or int(runner.num_pages * args.hicache_ratio)
            self.hicache = HiCache(runner.kv_pool, self.P, max(1, n_host), runner.device)
        self.waiting: Deque[Req] = collections.deque()
        self.running: List[Req] = []
        self.inflight: Deque[Tuple[StepInput, object, object]] = collections.deque()
        self.free_slots = list(range(runner.max_reqs - 1, -1, -1))
        self.epoch = 0
        from .. import serving_policy
        pol = serving_policy.current()
        # overlap depth from the launch's serving policy: steps launched before the oldest one is processed
        self.overlap = (pol.async_execution if pol is not None else not args.disable_overlap_schedule)
        self.inflight_depth = max(1, pol.max_inflight_launches if pol is not None else 2)
        if args.disable_overlap_schedule:
            self.overlap = False
        self.eos = set(cfg.eos_token_id or [])
        self.pending_arrivals: List[Req] = []
        self.pending_aborts: List[str] = []
        self.stop_checker = None  # callable(req) -> bool: a text stop sequence appeared (set with a tokenizer)
        self.finished_reqs: List[Req] = []
        self.finished_by_rid: Dict[str, Req] = {}
        self.reqs_by_rid: Dict[str, Req] = {}
        self.on_token: Optional[Callable[[Req], None]] = None
        self.stats = collections.Counter()
        self.step_times: List[Tuple[int, float, int, int]] = []
        # device time of recent steps: (0 decode / 1 prefill or mixed, ms), from the runner's step timer
        self.device_ms: Deque[Tuple[int, float]] = collections.deque(maxlen=2048)
        # DP attention: this rank's attention group serves every D-th arrival; the others' requests are
        # mirrored from the per-step exchange (tokens and finish state published by each group's rank 0)
        st = get_state()
        self.dp_groups, self.dp_group = st.attn_dp_size, st.attn_dp_rank
        self.dp_leader = st.tp_rank == 0
        self._arrival_seq = 0
        self._remote: Dict[str, Req] = {}
        self._outbox: List[Tuple] = []
        self._global_busy = False
        if self.dp_groups > 1:
            self.overlap = False  # results are published once per step, right after the step
        self._arrival_flag = _make_shm(st, 1, "arr")
        # optional program fence: ranks check that they launch the same step program (debug; one shared-memory
        # reduce per step). Parity: the reference's ProgramSwitchFence (model_executor/program_fence.py:69).
        import os
        self._fence = (_make_shm(st, 2, "fence") if os.environ.get("SGLANG_B200_STEP_FENCE") == "1"
                       and self.dp_groups == 1 else None)
        # host timeline (select / launch / result spans per step), one TSV per rank label
        from .. import sglang_tree
        from ..utils.host_trace import HostTrace
        self.trace = HostTrace(args.host_trace_dir or os.environ.get("SGLANG_B200_HOST_TRACE"),
                               sglang_tree.rank_label())

    # ------------------------------------------------------------------------------------------
    # request intake
    def add_request(self, rid: str, input_ids: List[int], params: SamplingParams) -> Req:
        req = Req(rid, input_ids, params, eos_ids=[] if params.ignore_eos else self.eos)
        if len(input_ids) + params.max_new_tokens > self.args.context_length:
            raise ValueError(f"request {rid}: prompt {len(input_ids)} + max_new_tokens {params.max_new_tokens} "
                             f"exceeds context length {self.args.context_length}")
        self.pending_arrivals.append(req)
        return req

    def _sync_arrivals(self) -> None:
        st = get_state()
        if st.replica_size > 1 and self._arrival_flag is not None:
            # shared-memory MAX of rank 0's arrival + abort count: the object broadcast only when it has some
            n = len(self.pending_arrivals) + len(self.pending_aborts) if st.replica_rank == 0 else 0
            # (never tighter than a gloo collective: 1800 s, as the reference's node-shm reduce)
            if self._arrival_flag.max([n], timeout_s=1800.0)[0] == 0:
                self.pending_arrivals, self.pending_aborts = [], []
                return
        if st.replica_size > 1:
            payload = (([(r.rid, r.origin_input_ids, r.params) for r in self.pending_arrivals], self.pending_aborts)
                       if st.replica_rank == 0 else None)
            payload = cpu_broadcast_object(payload, src=0)
            if st.replica_rank != 0:
                self.pending_arrivals = [Req(rid, ids, p, eos_ids=[] if p.ignore_eos else self.eos)
                                         for rid, ids, p in payload[0]]
                self.pending_aborts = list(payload[1])
        for r in self.pending_arrivals:
            self.reqs_by_rid[r.rid] = r
        if self.dp_groups > 1:
            for r in self.pending_arrivals:
                g = self._arrival_seq % self.dp_groups
                self._arrival_seq += 1
                if g == self.dp_group:
                    self.waiting.append(r)
                else:
                    self._remote[r.rid] = r
        else:
            self.waiting.extend(self.pending_arrivals)
        self.pending_arrivals = []
        aborts, self.pending_aborts = self.pending_aborts, []
        for rid in aborts:
            self._abort(rid)

    def abort(self, rid: str) -> None:
        """Abort a request (queued or running) at the next step boundary; every rank applies it at the same
        point of the request stream."""
        self.pending_aborts.append(rid)

    def _abort(self, rid: str) -> None:
        r = self.reqs_by_rid.get(rid)
        if r is None or r.finished:
            return
        if r in self.waiting:
            self.waiting.remove(r)
            r.finished, r.finish_reason = True, "abort"
            self.finished_reqs.append(r)
            self.finished_by_rid[r.rid] = r
        else:
            self._finish(r, "abort")
        if self.on_token is not None:
            self.on_token(r)

    def has_work(self) -> bool:
        return bool(self.waiting or self.running or self.inflight or self.pending_arrivals or self._global_busy)

    # ------------------------------------------------------------------------------------------
    # page management
    def _alloc_pages(self, n: int, start: int = 0) -> Optional[List[int]]:
        """n pages for a request's logical pages start .. start + n - 1 (the index picks the owner rank under
        decode context parallelism)."""
        if n <= 0:
            return []
        dcp = hasattr(self.alloc, "alloc_at")
        pages = self.alloc.alloc_at(start, n) if dcp else self.alloc.alloc(n)
        if len(pages) == n:
            return list(pages)
        if self.radix is not None:
            freed = self.radix.evict(max(n - self.alloc.available(), n if dcp else 0))
            if freed:
                if self.hicache is not None:
                    self.hicache.sync_writes()  # host copies of these pages must land before reuse
                self.alloc.free(list(freed))
            pages = self.alloc.alloc_at(start, n) if dcp else self.alloc.alloc(n)
            if len(pages) == n:
                return list(pages)
        return None

    def _ensure_pages(self, r: Req, upto_tokens: int, upd: List[int]) -> bool:
        if self.swa is not None:
            self.swa.trim(r, r.kv_len)
        need = (upto_tokens + self.P - 1) // self.P - len(r.pages)
        if need <= 0:
            return True
        swa = None
        if self.swa is not None:
            swa = self.swa.alloc_for(need)
            if swa is None:
                return False
        pages = self._alloc_pages(need, len(r.pages))
        if pages is None:
            if swa:
                self.swa.undo(swa)
            return False
        if swa is not None:
            self.swa.bind(r, pages, swa, upd)
        for p in pages:
            upd += [r.slot, len(r.pages), p]
            r.pages.append(p)
        return True

    def _release(self, r: Req) -> None:
        """Return a finished (or retracted) request's pages: full pages go to the prefix cache."""
        owned = r.pages[r.owned_from:]
        if self.radix is not None and not r.retracted_flag():
            ids = r.all_ids()
            n_tok = (min(r.kv_len, len(ids)) // self.P) * self.P
            n_pages = n_tok // self.P
            if n_pages > 0:
                dup = self.radix.insert(ids[:n_tok], r.pages[:n_pages])
                to_free = list(dup) + r.pages[max(n_pages, r.owned_from):]
                if self.hicache is not None:
                    # write-through from the tree's own pages (duplicates are freed right below)
                    _, canon, _ = self.radix.match_prefix(ids[:n_tok])
                    self.hicache.write_through(ids[:n_tok], list(canon)[:n_pages])
            else:
                to_free = owned
            if r.prefix_node is not None:
                self.radix.dec_lock(r.prefix_node)
        else:
            to_free = owned
            if self.radix is not None and r.prefix_node is not None:
                self.radix.dec_lock(r.prefix_node)
        if to_free:
            self.alloc.free_after(list(to_free), r.last_step)
        if self.swa is not None:
            self.swa.release(r)
        r.pages, r.owned_from, r.prefix_node = [], 0, None
        if r.slot is not None:
            self.free_slots.append(r.slot)
            r.slot = None

    # ------------------------------------------------------------------------------------------
    def _admit(self) -> None:
        while self.waiting and self.free_slots:
            r = self.waiting[0]
            ids = r.all_ids()
            prefix_len, prefix_pages, node = 0, [], None
            if self.radix is not None:
                matched, pages, node = self.radix.match_prefix(ids[:-1] if len(ids) > 1 else [])
                grid = self.args.prefill_chunk_grid or self.P  # chunk-keyed reuse: whole grid chunks only
                prefix_len = (matched // grid) * grid
                prefix_pages = list(pages)[: prefix_len // self.P]
            need = (len(ids) + 1 + self.P - 1) // self.P - len(prefix_pages)
            if self.alloc.available() + (self.radix.evictable_pages() if self.radix else 0) < need:
                break
            self.waiting.popleft()
            r.slot = self.free_slots.pop()
            if self.radix is not None and node is not None:
                self.radix.inc_lock(node)
                r.prefix_node = node
            tree_pages = len(prefix_pages)  # pages of the device tree: shared, not owned by the request
            if self.hicache is not None:
                # pages past the device match that the host tier still holds: load instead of recompute
                room = (len(ids) - 1) // self.P - tree_pages
                slots = self.hicache.match(ids, tree_pages, room) if room > 0 else []
                if slots and self.args.prefill_chunk_grid:  # keep the reused prefix on the chunk grid
                    gp = self.args.prefill_chunk_grid // self.P
                    slots = slots[: max(0, ((tree_pages + len(slots)) // gp) * gp - tree_pages)]
                # logical pages tree_pages.. onward (the start picks each page's owner under DCP; DCP with the
                # host tier is refused at launch, so this start only matters if that refusal is lifted)
                new = self._alloc_pages(len(slots), tree_pages) if slots else None
                if new:
                    self.hicache.load(slots, new)
                    prefix_pages = prefix_pages + new
                    prefix_len = len(prefix_pages) * self.P
                    self.stats["host_hit_tokens"] = self.stats.get("host_hit_tokens", 0) + len(new) * self.P
            r.pages = prefix_pages
            r.owned_from = tree_pages
            # reused pages enter this slot's block-table row with the request's first step
            r.table_pending = [v for j, pg in enumerate(prefix_pages) for v in (r.slot, j, pg)]
            r.prefix_len = prefix_len
            r.kv_len = prefix_len
            r.prefill_target = len(ids)
            self.stats["cache_hit_tokens"] += prefix_len
            self.stats["prompt_tokens"] += len(ids)
            self.running.append(r)

    def _retract_one(self, exclude: Req) -> bool:
        """Out of pages: drain the in-flight steps, then send the request with the most outstanding work
        back to the queue (its KV is recomputed when it is re-admitted)."""
        cands = [r for r in self.running if r is not exclude and not r.finished]
        if not cands:
            return False
        self.drain()
        victim = max(cands, key=lambda r: r.params.max_new_tokens - len(r.output_ids))
        self.running.remove(victim)
        victim._retracted = True
        self._release(victim)
        victim._retracted = False
        victim.kv_len = 0
        victim.scheduled_outputs = len(victim.output_ids)
        self.waiting.appendleft(victim)
        self.stats["retractions"] += 1
        return True

    def schedule(self) -> Optional[StepInput]:
        self._admit()
        prefill = [r for r in self.running if r.kv_len < r.prefill_target]
        decode = [r for r in self.running if r.kv_len >= r.prefill_target and not r.finished
                  and r.scheduled_outputs < r.params.max_new_tokens]
        if prefill:
            if not self.args.enable_mixed_chunk:
                decode = []
            return self._build_extend(prefill, decode)
        if decode:
            return self._build_decode(decode)
        return None

    def _build_decode(self, reqs: List[Req]) -> Optional[StepInput]:
        upd: List[int] = []
        ok_reqs = []
        for r in reqs:
            while not self._ensure_pages(r, r.kv_len + 1, upd):
                if not self._retract_one(r):
                    raise RuntimeError("KV pool exhausted by a single request")
                if r not in self.running:
                    break
            if r in self.running:
                ok_reqs.append(r)
        reqs = [r for r in ok_reqs if r.slot is not None]
        if not reqs:
            return None
        B = len(reqs)
        pos = np.fromiter((r.kv_len for r in reqs), dtype=np.int64, count=B)
        slots = np.fromiter((r.pages[r.kv_len // self.P] * self.P + r.kv_len % self.P for r in reqs),
                            dtype=np.int64, count=B)
        step = self._make_step(ForwardMode.DECODE, reqs, [True] * B, np.zeros(B, np.int64), pos, slots,
                               np.arange(B, dtype=np.int64), pos.astype(np.int32) + 1, np.zeros(1, np.int32),
                               upd, num_decode=B, max_extend=0)
        for r in reqs:
            r.kv_len += 1
            r.scheduled_outputs += 1
            r.last_step = step.epoch
        return step

    def _build_extend(self, prefill: List[Req], decode: List[Req]) -> Optional[StepInput]:
        budget = self.args.chunked_prefill_size
        upd: List[int] = []
        chunks: List[Tuple[Req, int]] = []
        for r in prefill:
            if budget <= 0:
                break
            n = min(r.prefill_target - r.kv_len, budget)
            G = self.args.prefill_chunk_grid
            if G:  # chunks end on the request's grid (a prefix hit then replays the same chunks)
                n = min(n, G - r.kv_len % G)
            if not self._ensure_pages(r, r.kv_len + n, upd):
                break
            chunks.append((r, n))
            budget -= n
        dec_ok = []
        for r in decode:
            if self._ensure_pages(r, r.kv_len + 1, upd):
                dec_ok.append(r)
        if not chunks and not dec_ok:
            return None
        if not chunks:
            return self._build_decode_from_upd(dec_ok, upd)
        D = len(dec_ok)
        reqs = dec_ok + [r for r, _ in chunks]
        T = D + sum(n for _, n in chunks)
        ids = np.zeros(T, np.int64)
        pos = np.empty(T, np.int64)
        slots = np.empty(T, np.int64)
        logits_idx = np.empty(len(reqs), np.int64)
        seq = np.empty(len(reqs), np.int32)
        qo = np.zeros(len(chunks) + 1, np.int32)
        sampled = []
        for i, r in enumerate(dec_ok):
            pos[i] = r.kv_len
            slots[i] = r.pages[r.kv_len // self.P] * self.P + r.kv_len % self.P
            logits_idx[i] = i
            seq[i] = r.kv_len + 1
            sampled.append(True)
        row = D
        max_ext = 0
        rt = __import__("sglang_neuron_b200._ext", fromlist=["_runtime"])._runtime
        for j, (r, n) in enumerate(chunks):
            all_ids = r.all_ids()
            ids[row:row + n] = all_ids[r.kv_len:r.kv_len + n]
            pos[row:row + n] = np.arange(r.kv_len, r.kv_len + n)
            if rt is not None:
                slots[row:row + n] = rt.slots_for_range(r.pages, self.P, r.kv_len, r.kv_len + n)
            else:
                p = np.arange(r.kv_len, r.kv_len + n)
                slots[row:row + n] = np.asarray(r.pages, np.int64)[p // self.P] * self.P + p % self.P
            logits_idx[D + j] = row + n - 1
            seq[D + j] = r.kv_len + n
            qo[j + 1] = qo[j] + n
            sampled.append(r.kv_len + n >= r.prefill_target)
            row += n
            max_ext = max(max_ext, n)
        step = self._make_step(ForwardMode.EXTEND, reqs, sampled, ids, pos, slots, logits_idx, seq, qo, upd,
                               num_decode=D, max_extend=max_ext)
        for r in dec_ok:
            r.kv_len += 1
            r.scheduled_outputs += 1
            r.last_step = step.epoch
        for (r, n), s in zip(chunks, sampled[D:]):
            r.kv_len += n
            if s:
                r.scheduled_outputs += 1
            r.last_step = step.epoch
        return step

    def _build_decode_from_upd(self, reqs, upd):
        B = len(reqs)
        pos = np.fromiter((r.kv_len for r in reqs), dtype=np.int64, count=B)
        slots = np.fromiter((r.pages[r.kv_len // self.P] * self.P + r.kv_len % self.P for r in reqs),
                            dtype=np.int64, count=B)
        step = self._make_step(ForwardMode.DECODE, reqs, [True] * B, np.zeros(B, np.int64), pos, slots,
                               np.arange(B, dtype=np.int64), pos.astype(np.int32) + 1, np.zeros(1, np.int32),
                               upd, num_decode=B, max_extend=0)
        for r in reqs:
            r.kv_len += 1
            r.scheduled_outputs += 1
            r.last_step = step.epoch
        return step

    def _make_step(self, mode, reqs, sampled, ids, pos, slots, logits_idx, seq, qo, upd, num_decode, max_extend):
        B = len(reqs)
        pending = [v for r in reqs for v in r.table_pending]
        if pending:
            upd = pending + list(upd)
            for r in reqs:
                r.table_pending = []
        temp = np.fromiter((r.params.temperature for r in reqs), dtype=np.float32, count=B)
        top_p = np.fromiter((r.params.top_p for r in reqs), dtype=np.float32, count=B)
        top_k = np.fromiter((r.params.top_k for r in reqs), dtype=np.int64, count=B)
        seeds = np.fromiter((r.seed for r in reqs), dtype=np.int64, count=B)
        slot_idx = np.fromiter((r.slot for r in reqs), dtype=np.int64, count=B)
        needs = any(r.params.needs_filter for r in reqs)
        lp = [r.params.top_logprobs_num for r in reqs if r.params.return_logprob]
        logprob_k = max(lp) if lp else -1
        step = StepInput(mode=mode, epoch=self.epoch, reqs=list(reqs), sampled=list(sampled), batch_size=B,
                         num_tokens=len(pos), num_decode=num_decode, input_ids=ids, positions=pos,
                         out_cache_loc=slots, logits_idx=logits_idx, req_idx=slot_idx, seeds=seeds, top_k=top_k,
                         seq_lens=seq, qo_indptr=qo, page_upd=np.asarray(upd, dtype=np.int32), temperature=temp,
                         top_p=top_p, max_extend=max_extend, max_seq_len=int(seq.max()) if B else 0,
                         needs_topk_topp=needs, logprob_k=logprob_k)
        self.epoch += 1
        return step

    # ------------------------------------------------------------------------------------------
    def _process(self, step: StepInput, ids_host, event) -> None:
        if event is not None:
            event.synchronize()
        ev = getattr(step, "device_events", None)
        if ev is not None:  # per-step device time (the readback event above completed after it)
            ev[1].synchronize()
            self.device_ms.append((int(step.mode != ForwardMode.DECODE), ev[0].elapsed_time(ev[1])))
        watch = getattr(self.runner, "status_watch", None)
        if watch is not None:
            watch.check()
        ids = ids_host.numpy() if hasattr(ids_host, "numpy") else np.asarray(ids_host)
        lpr = step.logprob_host.numpy() if step.logprob_host is not None else None
        now = time.perf_counter()
        for i, (r, s) in enumerate(zip(step.reqs, step.sampled)):
            if not s or r.finished:
                continue
            tok = int(ids[i])
            if not 0 <= tok < self.cfg.vocab_size:
                # a corrupted logits row (NaN / inf) must not reach the detokenizer or the relay: refuse the
                # id and end only this request. Parity: refuse_invalid_token_ids (async_execution.py:237).
                logger.error("request %s: sampled token id %d outside the vocabulary; request ended", r.rid, tok)
                self.stats["invalid_token_ids"] += 1
                self._finish(r, "error: invalid token id")
                if self.on_token is not None:
                    self.on_token(r)
                continue
            r.output_ids.append(tok)
            if lpr is not None and r.params.return_logprob:
                k = r.params.top_logprobs_num
                K = (lpr.shape[1] - 1) // 2
                r.output_logprobs.append(float(lpr[i, 0]))
                if k > 0:
                    r.output_top_logprobs.append([(float(lpr[i, 1 + j]), int(lpr[i, 1 + K + j])) for j in range(k)])
            if r.first_token_time is None:
                r.first_token_time = now
            r.token_times.append(now)
            self.stats["output_tokens"] += 1
            if (tok in r.eos_ids) or (r.params.stop_token_ids and tok in r.params.stop_token_ids):
                self._finish(r, "stop")
            elif len(r.output_ids) >= r.params.max_new_tokens:
                self._finish(r, "length")
            elif r.params.stop and self.stop_checker is not None and self.stop_checker(r):
                self._finish(r, "stop")
            if self.dp_groups > 1 and self.dp_leader:
                lp = None
                if lpr is not None and r.params.return_logprob:
                    lp = (r.output_logprobs[-1], r.output_top_logprobs[-1] if r.params.top_logprobs_num > 0 else None)
                self._outbox.append((r.rid, tok, r.finished, r.finish_reason, lp))
            if self.on_token is not None:
                self.on_token(r)
        self.alloc.retire(step.epoch)
        if self.swa is not None:
            self.swa.retire(step.epoch)

    def _finish(self, r: Req, reason: str) -> None:
        r.finished = True
        r.finish_reason = reason
        if r in self.running:
            self.running.remove(r)
        self._release(r)
        self.finished_reqs.append(r)
        self.finished_by_rid[r.rid] = r

    def drain(self) -> None:
        while self.inflight:
            self._process(*self.inflight.popleft())

    def step(self) -> None:
        """One scheduler iteration: admit, launch one forward, and process the previous step's tokens."""
        self._sync_arrivals()
        if self.dp_groups > 1:
            return self._step_dp()
        with self.trace.span("select", self.epoch):
            step = self.schedule()
        if self._fence is not None:
            key = (hash((int(step.mode), step.batch_size, step.num_tokens, step.max_extend)) & 0x3FFFFFFFFFFF
                   if step is not None else 0)
            got = self._fence.max([key, -key], timeout_s=1800.0)
            if got[0] != -got[1]:
                raise RuntimeError(f"ranks are about to launch different step programs (epoch {self.epoch})")
        if step is not None:
            t0 = time.perf_counter()
            if self.hicache is not None:
                self.hicache.wait_loads()
            with self.trace.span("launch", step.epoch, step.batch_size, step.num_tokens):
                ids_host, ev = self.runner.run_step(step)
            self.inflight.append((step, ids_host, ev))
            self.stats["steps"] += 1
            self.stats["decode_steps" if step.mode == ForwardMode.DECODE else "extend_steps"] += 1
            self.step_times.append((step.epoch, t0, step.batch_size, step.num_tokens))
        keep = self.inflight_depth - 1 if (self.overlap and step is not None) else 0
        while len(self.inflight) > keep:
            done = self.inflight[0][0]
            with self.trace.span("result", done.epoch, done.batch_size, done.num_tokens):
                self._process(*self.inflight.popleft())

    def _step_dp(self) -> None:
        """DP attention lockstep: every rank exchanges (rows it will run, busy, tokens published since the last
        exchange); the step's MoE exchange is sized by the largest group and groups without rows run an idle
        forward. Parity: the reference's DP-attention lockstep with idle dummies
        (sglang_neuron/model_executor/graph_runner.py:822-869 `plan_step`, :1639 `run_idle`)."""
        from ..parallel.collectives import dp_exchange
        step = self.schedule()
        n = step.num_tokens if step is not None else 0
        busy = bool(self.waiting or self.running or self.inflight)
        info = dp_exchange((n, busy, self._outbox))
        self._outbox = []
        for _, _, out in info:
            for rid, tok, fin, reason, lp in out:
                r = self._remote.get(rid)
                if r is None:
                    continue
                r.output_ids.append(tok)
                if lp is not None:
                    r.output_logprobs.append(lp[0])
                    if lp[1] is not None:
                        r.output_top_logprobs.append(lp[1])
                if r.first_token_time is None:
                    r.first_token_time = time.perf_counter()
                if fin:
                    r.finished, r.finish_reason = True, reason
                    self.finished_reqs.append(r)
                    self.finished_by_rid[rid] = r
                    del self._remote[rid]
                if self.on_token is not None:
                    self.on_token(r)
        rows = max(i[0] for i in info)
        self._global_busy = rows > 0 or any(i[1] for i in info)
        if rows == 0:
            return
        if step is None:
            self.runner.run_idle(rows)
            return
        step.dp_rows = rows
        t0 = time.perf_counter()
        ids_host, ev = self.runner.run_step(step)
        self.stats["steps"] += 1
        self.stats["decode_steps" if step.mode == ForwardMode.DECODE else "extend_steps"] += 1
        self.step_times.append((step.epoch, t0, step.batch_size, step.num_tokens))
        self._process(step, ids_host, ev)

    def run_until_idle(self, max_steps: int = 1 << 62) -> None:
        n = 0
        while self.has_work() and n < max_steps:
            self.step()
            n += 1
        self.drain()


_flag_seq = [0]


def _make_shm(st, width: int, tag: str):
    """Node shared-memory MIN/MAX over the replica's ranks (the native runtime's ShmReduce), or None when the
    runtime is not built or the replica spans one rank; gloo stays the fallback."""
    import os
    import torch.distributed as dist
    from .._ext import _runtime
    if st.replica_size == 1 or _runtime is None or not hasattr(_runtime, "ShmReduce") or not dist.is_initialized():
        return None
    _flag_seq[0] += 1  # every rank builds its schedulers in the same order, so the names match
    name = f"/snb_{os.environ.get('MASTER_PORT', '0')}_{st.replica_base}_{st.replica_size}_{_flag_seq[0]}_{tag}"
    # the replica's rank 0 creates (and zeroes) the segment before the others open it; every rank must end
    # up on the same path, so a rank that cannot map the segment sends all of them back to gloo
    import torch
    flag = None
    try:
        if st.replica_rank == 0:
            flag = _runtime.ShmReduce(name, st.replica_size, 0, width, True)
    except RuntimeError as e:
        logger.warning("shared-memory arrival flag unavailable (%s); using gloo", e)
    dist.barrier(group=st.replica_cpu_group)
    try:
        if st.replica_rank != 0:
            flag = _runtime.ShmReduce(name, st.replica_size, st.replica_rank, width, False)
    except RuntimeError as e:
        logger.warning("shared-memory arrival flag unavailable (%s); using gloo", e)
    ok = torch.tensor([1 if flag is not None else 0], dtype=torch.int32)
    dist.all_reduce(ok, op=dist.ReduceOp.MIN, group=st.replica_cpu_group)
    return flag if int(ok) == 1 else None


def _retracted_flag(self) -> bool:
    return getattr(self, "_retracted", False)


Req.retracted_flag = _retracted_flag
