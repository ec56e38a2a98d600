"""Background serving loop: a thread owns the Engine and runs scheduler steps while requests are in flight;
asyncio callers submit requests and receive token deltas through per-request queues.

Parity: SGLang's TokenizerManager <-> Scheduler split as the reference serves it (request intake on one
side, the scheduler's overlap loop on the other, streaming results back). Here both live in one process
and talk through a lock-protected inbox and thread-safe event-loop callbacks.
"""
from __future__ import annotations

import asyncio
import itertools
import logging
import threading
import time
from typing import Dict, List, Optional

from ..managers.schedule_batch import SamplingParams
from ..parallel.state import get_state

logger = logging.getLogger(__name__)


class _Stream:
    def __init__(self, loop: asyncio.AbstractEventLoop):
        self.loop = loop
        self.queue: asyncio.Queue = asyncio.Queue()


class EngineLoop:
    def __init__(self, engine):
        self.engine = engine
        self.inbox: List = []
        self.lock = threading.Lock()
        self.wake = threading.Event()
        self.streams: Dict[str, _Stream] = {}
        self.stop_flag = False
        self.ids = itertools.count()
        self.started = time.time()
        self.thread = threading.Thread(target=self._run, name="snb-scheduler", daemon=True)
        engine.scheduler.on_token = self._on_token
        self.thread.start()

    # -- called from asyncio handlers ------------------------------------------------------------
    def submit(self, input_ids: List[int], params: SamplingParams, rid: Optional[str] = None) -> (str, _Stream):
        rid = rid or f"http-{next(self.ids)}"
        st = _Stream(asyncio.get_running_loop())
        with self.lock:
            self.streams[rid] = st
            self.inbox.append((rid, input_ids, params))
        self.wake.set()
        return rid, st

    def abort(self, rid: str) -> None:
        with self.lock:
            self.engine.scheduler.abort(rid)
        self.wake.set()

    def shutdown(self) -> None:
        self.stop_flag = True
        self.wake.set()
        self.thread.join(timeout=10)

    # -- scheduler thread --------------------------------------------------------------------------
    def _on_token(self, req) -> None:
        st = self.streams.get(req.rid)
        if st is None:
            return
        off = req.stream_offset
        new = req.output_ids[off:]
        req.stream_offset = len(req.output_ids)
        item = {"rid": req.rid, "new_ids": list(new), "finished": req.finished,
                "finish_reason": req.finish_reason, "prompt_tokens": req.prompt_len,
                "completion_tokens": len(req.output_ids), "cached_tokens": req.prefix_len}
        if req.params.return_logprob:
            item["new_logprobs"] = list(req.output_logprobs[off:])
            item["new_top_logprobs"] = list(req.output_top_logprobs[off:])
        st.loop.call_soon_threadsafe(st.queue.put_nowait, item)
        if req.finished:
            self.streams.pop(req.rid, None)

    def _run(self) -> None:
        sched = self.engine.scheduler
        while not self.stop_flag:
            with self.lock:
                batch, self.inbox = self.inbox, []
            for rid, ids, params in batch:
                try:
                    sched.add_request(rid, ids, params)
                except Exception as e:  # reject the request, keep serving
                    st = self.streams.pop(rid, None)
                    if st is not None:
                        st.loop.call_soon_threadsafe(st.queue.put_nowait, {"rid": rid, "error": str(e),
                                                                           "finished": True})
            if sched.has_work():
                sched.step()
            else:
                self.wake.wait(timeout=0.05)
                self.wake.clear()
                if get_state().replica_size > 1:
                    # heartbeat: follower ranks wait inside the step's arrival sync; an idle step every
                    # 50 ms keeps them from running into the process group's timeout
                    sched.step()
