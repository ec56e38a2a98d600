"""CUDA-graph capture of decode steps for every batch-size bucket at startup, with the plain (greedy /
temperature) sampler and with the filtered (top-k / top-p) sampler.

Parity: the reference compiles every prefill and decode shape at warm-up (NeuronModelRuntime.warmup_all,
sglang_neuron/model_executor/graph_runner.py:692-757; BucketConfig decode batch buckets :149-253) and its
`NeuronGraphRunner.can_run_graph` (:1692-1768) serves decode/idle batches up to the largest bucket. Here each
bucket is a torch.cuda.CUDAGraph whose inputs live in one static device buffer with a fixed layout; a step
packs its host arrays in the same layout, one cudaMemcpyAsync lands them in that buffer, and replay() runs
embedding -> layers -> LM head -> sampler -> token relay with no host work in between.
"""
from __future__ import annotations

import bisect
import gc
import logging
from typing import Dict

import numpy as np
import torch

from .. import _ext
from .forward_batch import ForwardBatch, ForwardMode

logger = logging.getLogger(__name__)


class CudaGraphRunner:
    def __init__(self, runner):
        self.r = runner
        self.args = runner.args
        self.bs_list = self.args.graph_batch_sizes()
        self.max_bs = self.bs_list[-1]
        from .model_runner import Layout
        mb = self.max_bs
        # page-update triples per row: a new page, plus its window-pool page under the hybrid SWA layout
        self.upr = 2 if getattr(runner.kv_pool, "swa", None) is not None else 1
        self.layout = Layout([
            ("req_idx", torch.int64, mb), ("positions", torch.int64, mb), ("out_cache_loc", torch.int64, mb),
            ("seeds", torch.int64, mb), ("seq_lens", torch.int32, mb), ("page_upd", torch.int32, 3 * self.upr * mb),
            ("temperature", torch.float32, mb), ("top_k", torch.int64, mb), ("top_p", torch.float32, mb),
        ])
        self.static = torch.zeros(self.layout.nbytes, dtype=torch.uint8, device=runner.device)
        self.views = self.layout.views(self.static)
        self.out_ids = torch.zeros(mb, dtype=torch.int64, device=runner.device)
        self.graphs: Dict[int, torch.cuda.CUDAGraph] = {}
        self.launches: Dict[int, int] = {}
        # the same buckets with the filtered (top-k / top-p) sampler: radix-select candidate pools per vocab
        # shard, one gather, filters and Gumbel-max on the pool, all on the device
        self.graphs_f: Dict[int, torch.cuda.CUDAGraph] = {}
        self.launches_f: Dict[int, int] = {}
        self.pool = None
        self.capture_all()

    def can_run(self, step) -> bool:
        return step.batch_size <= self.max_bs and len(step.page_upd) <= 3 * self.upr * step.batch_size

    def _fb(self, bs: int) -> ForwardBatch:
        v = self.views
        r = self.r
        req_idx = v["req_idx"][:bs]
        block_table = r.req_to_page.table.index_select(0, req_idx)
        input_ids = r.relay.index_select(0, req_idx)
        splits = r.backend.splits_for(bs, r.model.attention_layers()[0].num_kv_heads, self.args.context_length)
        return ForwardBatch(mode=ForwardMode.DECODE, batch_size=bs, num_tokens=bs, input_ids=input_ids,
                            positions=v["positions"][:bs], out_cache_loc=v["out_cache_loc"][:bs],
                            seq_lens=v["seq_lens"][:bs], block_table=block_table,
                            logits_idx=torch.arange(bs, device=r.device), temperature=v["temperature"][:bs],
                            seeds=v["seeds"][:bs], decode_splits=splits, max_seq_len=self.args.context_length)

    def _body(self, bs: int, filtered: bool = False) -> None:
        r = self.r
        r.apply_page_updates(self.views["page_upd"][: 3 * self.upr * bs])
        fb = self._fb(bs)
        if filtered:
            fb.top_k = self.views["top_k"][:bs]
            fb.top_p = self.views["top_p"][:bs]
            fb.needs_topk_topp = True
        h = r.model(fb)
        r.sample(h, fb, self.views["req_idx"][:bs], out=self.out_ids[:bs])

    def capture_all(self) -> None:
        r = self.r
        # padding state: every row points at the dummy request, writes nothing, attends to nothing
        self._fill_padding(0, self.max_bs)
        stream = torch.cuda.Stream(device=r.device)
        stream.wait_stream(torch.cuda.current_stream(r.device))
        with torch.cuda.stream(stream):
            for bs in reversed(self.bs_list):
                for filtered, graphs, launches in ((False, self.graphs, self.launches),
                                                   (True, self.graphs_f, self.launches_f)):
                    for _ in range(2):  # warm-up (allocator, lazy init) outside the graph
                        self._body(bs, filtered)
                    g = torch.cuda.CUDAGraph()
                    n0 = _ext.launch_count()
                    # no garbage collection inside the capture: collecting an unreachable object that owns a
                    # CUDA graph (an earlier engine's runner, say) destroys that graph, a call the capture
                    # forbids, and the capture is invalidated
                    gc.collect()
                    gc_was_on = gc.isenabled()
                    gc.disable()
                    try:
                        with torch.cuda.graph(g, pool=self.pool, stream=stream):
                            self._body(bs, filtered)
                    finally:
                        if gc_was_on:
                            gc.enable()
                    launches[bs] = _ext.launch_count() - n0
                    if self.pool is None:
                        self.pool = g.pool()
                    graphs[bs] = g
        torch.cuda.current_stream(r.device).wait_stream(stream)
        torch.cuda.synchronize(r.device)
        from ..parallel.contract import assert_graphs_consistent
        kvh = r.model.attention_layers()[0].num_kv_heads
        self.digest = assert_graphs_consistent({
            "bs": self.bs_list, "launches": [self.launches[b] for b in self.bs_list],
            "launches_filtered": [self.launches_f[b] for b in self.bs_list],
            "splits": [r.backend.splits_for(b, kvh, self.args.context_length) for b in self.bs_list]})
        logger.info("captured %d decode graphs (bs %s, digest %s)", len(self.graphs), self.bs_list, self.digest)

    def _fill_padding(self, start: int, end: int) -> None:
        v = self.views
        v["req_idx"][start:end] = self.r.dummy_req
        v["positions"][start:end] = 0
        v["out_cache_loc"][start:end] = -1
        v["seeds"][start:end] = 0
        v["seq_lens"][start:end] = 0
        v["temperature"][start:end] = 0
        v["top_k"][start:end] = 0
        v["top_p"][start:end] = 1.0
        pu = v["page_upd"].view(-1, 3)
        pu[start * self.upr:end * self.upr, 0] = self.r.dummy_req
        pu[start * self.upr:end * self.upr, 1] = 0
        pu[start * self.upr:end * self.upr, 2] = 0

    def replay(self, step) -> torch.Tensor:
        B = step.batch_size
        bs = self.bs_list[bisect.bisect_left(self.bs_list, B)]
        arrays = step.decode_arrays(bs, self.r.dummy_req, self.upr)
        self.r.io.upload(self.layout, arrays, dst=self.static)
        if step.needs_topk_topp:
            self.graphs_f[bs].replay()
            _ext.add_launches(self.launches_f[bs])
        else:
            self.graphs[bs].replay()
            _ext.add_launches(self.launches[bs])
        return self.out_ids[:B]
