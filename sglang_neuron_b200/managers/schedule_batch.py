"""Requests, sampling parameters and the host-side description of one step (StepInput).

Parity: SGLang's Req / ScheduleBatch as the reference drives them, plus the reference's fixed decode token
I/O (FixedDecodeTokenIO, sglang_neuron/model_executor/token_io.py:9): a decode step carries no token ids
from the host; the device relay supplies them.
"""
from __future__ import annotations

import dataclasses
import time
from typing import List, Optional, Tuple

import numpy as np

from ..model_executor.forward_batch import ForwardMode


@dataclasses.dataclass
class SamplingParams:
    max_new_tokens: int = 128
    temperature: float = 0.0
    top_k: int = 0
    top_p: float = 1.0
    seed: Optional[int] = None
    stop_token_ids: Optional[List[int]] = None
    ignore_eos: bool = False
    stop: Optional[List[str]] = None   # text stop sequences (need a tokenizer)
    n: int = 1                         # samples per prompt (expanded by the API layer)
    return_logprob: bool = False       # log-probability of every generated token (raw distribution)
    top_logprobs_num: int = 0          # plus the k most likely tokens at every position

    @property
    def needs_filter(self) -> bool:
        return self.temperature > 0 and (self.top_k > 0 or self.top_p < 1.0)

    @classmethod
    def from_dict(cls, d: Optional[dict]) -> "SamplingParams":
        if not d:
            return cls()
        known = {f.name for f in dataclasses.fields(cls)}
        sp = cls(**{k: v for k, v in d.items() if k in known})
        if isinstance(sp.stop, str):
            sp.stop = [sp.stop]
        return sp


class Req:
    def __init__(self, rid: str, input_ids: List[int], params: SamplingParams, eos_ids=None):
        self.rid = rid
        self.origin_input_ids = list(input_ids)
        self.params = params
        self.eos_ids = set(eos_ids or [])
        self.output_ids: List[int] = []
        self.slot: Optional[int] = None          # row of the device block table / token relay
        self.pages: List[int] = []                # page ids holding this request's KV, in order
        self.owned_from = 0                       # pages[owned_from:] belong to the request (not the radix tree)
        self.prefix_node = None                   # radix node pinned while running
        self.prefix_len = 0                       # tokens reused from the prefix cache
        self.table_pending: List[int] = []        # (slot, index, page) triples of reused pages not yet in the table
        self.swa_pages: List[int] = []            # window-pool page per logical page (0 once released)
        self.swa_freed = 0                        # swa_pages[:swa_freed] are released
        self.output_logprobs: List[float] = []    # per generated token (when params.return_logprob)
        self.output_top_logprobs: List[List[Tuple[float, int]]] = []
        self.kv_len = 0                           # tokens whose KV is written (or being written by launched steps)
        self.scheduled_outputs = 0                # outputs that launched steps will have produced
        self.finished = False
        self.finish_reason: Optional[str] = None
        self.seed = params.seed if params.seed is not None else (hash(rid) & 0x7FFFFFFF)
        self.arrival = time.perf_counter()
        self.first_token_time: Optional[float] = None
        self.token_times: List[float] = []
        self.last_step = -1                       # epoch of the last launched step that touched this request
        self.stream_offset = 0

    @property
    def prompt_len(self) -> int:
        return len(self.origin_input_ids)

    def all_ids(self) -> List[int]:
        return self.origin_input_ids + self.output_ids

    @property
    def fill_target(self) -> int:
        """Tokens that must be in the KV before the next sample (prompt + outputs known on the host)."""
        return self.prompt_len + max(0, len(self.output_ids) - 0)

    @property
    def in_prefill(self) -> bool:
        return self.scheduled_outputs == 0

    def remaining_outputs(self) -> int:
        return self.params.max_new_tokens - self.scheduled_outputs


@dataclasses.dataclass
class StepInput:
    """Host arrays of one step. Rows [0, num_decode) are decode rows (one token each), rows after that are
    extend rows grouped by request (qo_indptr is relative to the first extend row)."""
    mode: ForwardMode
    epoch: int
    reqs: List[Req]
    sampled: List[bool]              # per request: does this step produce an output token for it
    batch_size: int
    num_tokens: int
    num_decode: int
    input_ids: np.ndarray
    positions: np.ndarray
    out_cache_loc: np.ndarray
    logits_idx: np.ndarray
    req_idx: np.ndarray
    seeds: np.ndarray
    top_k: np.ndarray
    seq_lens: np.ndarray
    qo_indptr: np.ndarray
    page_upd: np.ndarray
    temperature: np.ndarray
    top_p: np.ndarray
    max_extend: int = 0
    max_seq_len: int = 0
    needs_topk_topp: bool = False
    relay_first_token: Optional[np.ndarray] = None
    logprob_k: int = -1                 # >= 0: compute token logprobs (+ top-k) for this step
    logprob_host: Optional[object] = None  # host view [B, 1 + 2k] filled by the runner
    device_events: Optional[tuple] = None  # (start, end) CUDA timing events of the step's device work

    def arrays(self):
        return {
            "input_ids": self.input_ids, "positions": self.positions, "out_cache_loc": self.out_cache_loc,
            "logits_idx": self.logits_idx, "req_idx": self.req_idx, "seeds": self.seeds, "top_k": self.top_k,
            "seq_lens": self.seq_lens, "qo_indptr": self.qo_indptr, "page_upd": self.page_upd,
            "temperature": self.temperature, "top_p": self.top_p,
        }

    def decode_arrays(self, bs: int, dummy_slot: int, upd_per_row: int = 1):
        """Arrays padded to a captured bucket of `bs` rows (padding rows point at the dummy slot); the page
        update area holds `upd_per_row` triples per row."""
        B = self.batch_size
        pad = bs - B

        def padded(a, fill, dt):
            if pad == 0:
                return a.astype(dt, copy=False)
            return np.concatenate([a.astype(dt, copy=False), np.full(pad, fill, dtype=dt)])

        pu = np.zeros((bs * upd_per_row, 3), dtype=np.int32)
        pu[:, 0] = dummy_slot
        upd = self.page_upd.reshape(-1, 3)
        # at most one new page (+ its window-pool page) per decode row
        pu[: len(upd)] = upd
        return {
            "req_idx": padded(self.req_idx, dummy_slot, np.int64),
            "positions": padded(self.positions, 0, np.int64),
            "out_cache_loc": padded(self.out_cache_loc, -1, np.int64),
            "seeds": padded(self.seeds, 0, np.int64),
            "seq_lens": padded(self.seq_lens, 0, np.int32),
            "page_upd": pu.reshape(-1),
            "temperature": padded(self.temperature, 0.0, np.float32),
            "top_k": padded(self.top_k, 0, np.int64),
            "top_p": padded(self.top_p, 1.0, np.float32),
        }
