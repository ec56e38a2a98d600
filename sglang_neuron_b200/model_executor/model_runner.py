"""Model runner: owns the model, the KV pool, the block tables, the token relay and the step I/O, and runs
one forward (eager for prefill/mixed steps, CUDA-graph replay for decode steps).

Parity: NeuronModelRuntime (sglang_neuron/model_executor/graph_runner.py:273-1654): `build_model_inputs`
pads to a bucket and stages uploads (:990-1197), `_run` launches and records a pending sample (:1233),
`run_decode`/`run_prefill` (:1359, :1577). The reference's device_io (backend/device_io.py:150-413) keeps a
pinned upload ring and one readback per step; here `StepIO` is that ring: each step's inputs are packed
into one pinned buffer and land on the device with a single cudaMemcpyAsync, and the sampled tokens come
back with one async device->host copy into a pinned slot guarded by a CUDA event.

Token relay (parity: async_execution.TokenRelay, async_execution.py:508): the sampler writes every
request's next token into `relay[req_slot]` on the device, and the next decode step gathers its input ids
from there, so the host never waits for a token before launching the next step.
"""
from __future__ import annotations

import logging
import math
import os
from typing import Dict, List, Optional, Tuple

import numpy as np
import torch

from ..attention.backend import AttentionBackend
from ..configs.model_config import ModelConfig
from ..mem_cache.memory_pool import MHATokenToKVPool, MLATokenToKVPool, ReqToPagePool
from ..models.families import get_model_class
from ..models.weights import RandomSource, SafetensorsSource, load_model_weights
from ..ops.sampling import sample_tokens
from ..parallel.collectives import tp_all_gather_into
from ..parallel.state import get_state
from ..server_args import ServerArgs
from .forward_batch import ForwardBatch, ForwardMode

logger = logging.getLogger(__name__)

_ALIGN = 16
_STEP_TIMER = os.environ.get("SGLANG_B200_STEP_TIMER", "1") != "0"


class PinnedRing:
    """A ring of pinned host buffers; a slot is reused only after the event recorded on it completed."""

    def __init__(self, nbytes: int, slots: int, pin: bool):
        self.bufs = [torch.empty(nbytes, dtype=torch.uint8, pin_memory=pin) for _ in range(slots)]
        self.events: List[Optional[torch.cuda.Event]] = [None] * slots
        self.i = 0

    def acquire(self) -> Tuple[int, torch.Tensor]:
        i = self.i
        self.i = (self.i + 1) % len(self.bufs)
        ev = self.events[i]
        if ev is not None:
            ev.synchronize()
        return i, self.bufs[i]

    def mark(self, i: int, ev) -> None:
        self.events[i] = ev


class Layout:
    """Byte layout of one packed step: named sections (dtype, count) at 16-byte aligned offsets."""

    def __init__(self, sections: List[Tuple[str, torch.dtype, int]]):
        self.slots: Dict[str, Tuple[int, torch.dtype, int]] = {}
        off = 0
        for name, dt, n in sections:
            sz = torch.empty(0, dtype=dt).element_size() * n
            self.slots[name] = (off, dt, n)
            off += (sz + _ALIGN - 1) // _ALIGN * _ALIGN
        self.nbytes = max(off, _ALIGN)

    def views(self, buf: torch.Tensor) -> Dict[str, torch.Tensor]:
        out = {}
        for name, (off, dt, n) in self.slots.items():
            el = torch.empty(0, dtype=dt).element_size()
            out[name] = buf[off:off + n * el].view(dt)
        return out


_NP = {torch.int64: np.int64, torch.int32: np.int32, torch.float32: np.float32}


class StepIO:
    """Packs host arrays into one pinned buffer and uploads them with one copy; reads sampled ids back.

    Two streams: the host->device copy of a step's inputs runs on a copy stream into a device staging slot
    (so its PCIe latency overlaps the step still running on the compute stream), and the compute stream takes
    the bytes from there with one device-to-device copy after waiting on the copy's event. Parity: the
    reference's device_io copy queue and pinned upload ring (sglang_neuron/backend/device_io.py:150-413)."""

    def __init__(self, device, max_bytes: int, max_batch: int):
        self.device = torch.device(device)
        self.cuda = self.device.type == "cuda"
        self.up = PinnedRing(max_bytes, 4, self.cuda)
        self.down = PinnedRing(max_batch * 8, 8, self.cuda)
        self.h2d_bytes = 0
        self.d2h_bytes = 0
        self.copy_stream = torch.cuda.Stream(device=self.device) if self.cuda else None
        self.stage = ([torch.empty(max_bytes, dtype=torch.uint8, device=self.device) for _ in range(4)]
                      if self.cuda else None)

    def upload(self, layout: Layout, arrays: Dict[str, np.ndarray], dst: Optional[torch.Tensor] = None):
        slot, host = self.up.acquire()
        hv = layout.views(host[:layout.nbytes])
        for name, arr in arrays.items():
            v = hv[name]
            n = len(arr)
            v.numpy()[:n] = arr
        if dst is None:
            dst = torch.empty(layout.nbytes, dtype=torch.uint8, device=self.device)
        if self.cuda:
            cur = torch.cuda.current_stream(self.device)
            stage = self.stage[slot]
            with torch.cuda.stream(self.copy_stream):
                stage[:layout.nbytes].copy_(host[:layout.nbytes], non_blocking=True)
                arrived = torch.cuda.Event()
                arrived.record(self.copy_stream)
            cur.wait_event(arrived)
            dst[:layout.nbytes].copy_(stage[:layout.nbytes], non_blocking=True)
            ev = torch.cuda.Event()
            ev.record(cur)
            self.up.mark(slot, ev)  # host slot and staging slot are free once the device copy ran
        else:
            dst[:layout.nbytes].copy_(host[:layout.nbytes])
        self.h2d_bytes += layout.nbytes
        return layout.views(dst[:layout.nbytes])

    def readback(self, ids: torch.Tensor):
        """Async copy of [B] int64 ids into a pinned slot; returns (host view, event). It stays on the compute
        stream: the ids of a replayed graph live in the graph's static output, which the next replay rewrites."""
        slot, host = self.down.acquire()
        n = ids.numel()
        hv = host[: n * 8].view(torch.int64)
        hv.copy_(ids, non_blocking=self.cuda)
        self.d2h_bytes += n * 8
        ev = None
        if self.cuda:
            ev = torch.cuda.Event()
            ev.record()
            self.down.mark(slot, ev)
        return hv, ev


class KernelStatusWatch:
    """The kernels' bounded-wait status words, copied to pinned memory after every step (stream-ordered,
    a few bytes) and checked once the step's event has completed: a kernel that gave up on a wait makes the
    engine raise at the next step boundary instead of letting every later wait run into its time limit."""

    def __init__(self, sources: List[torch.Tensor]):
        self.sources = sources
        self.host = torch.zeros(4 * len(sources), dtype=torch.int32, pin_memory=True)

    def snapshot(self, io: "StepIO") -> None:
        for i, s in enumerate(self.sources):
            self.host[4 * i:4 * i + 4].copy_(s[:4], non_blocking=True)
        io.d2h_bytes += 16 * len(self.sources)

    def check(self) -> None:
        if bool(self.host.any()):
            codes = self.host.view(-1, 4)[:, 0].tolist()
            raise RuntimeError(f"an sm_100a kernel reported an error status {codes} (1-4: a bounded wait ran out, "
                               "5: an index past its buffer was skipped, 6: a static capacity was exceeded)")


class ModelRunner:
    def __init__(self, args: ServerArgs, cfg: ModelConfig, device=None):
        self.args = args
        self.cfg = cfg
        st = get_state()
        self.device = torch.device(device if device is not None else st.device)
        self.cuda = self.device.type == "cuda"
        self.dtype = args.torch_dtype() if self.cuda else torch.float32
        cls = get_model_class(cfg.architecture)
        self.model = cls(cfg, self.dtype, self.device, max_pos=args.context_length + 128)
        self.model.sp_min_tokens = args.sp_min_tokens
        self.draft = None
        if args.speculative_algorithm == "MTP":
            from ..speculative.mtp import MTPDraftHead
            self.draft = MTPDraftHead(self.model, self.dtype, self.device)
        self.load_weights()
        from ..parallel.contract import assert_fleet_consistent
        self.fleet_digest = assert_fleet_consistent({
            "arch": cfg.architecture, "layers": cfg.num_layers, "hidden": cfg.hidden_size,
            "windows": [cfg.layer_window(i) for i in range(cfg.num_layers)],
            "tp": list(st.replica_tp) if st.replica_tp else st.tp_size, "pp": st.pp_size,
            "dp": st.dp_size, "page": args.page_size, "kv": str(args.kv_cache_dtype), "dtype": str(self.dtype),
            "spec": args.speculative_algorithm or ""})
        self.page_size = args.page_size
        self.max_pages_per_req = (args.context_length + self.page_size - 1) // self.page_size + 1
        self.max_reqs = args.max_running_requests
        self.kv_dtype = args.resolved_kv_dtype(cfg.architecture) if self.cuda else torch.float32
        self.init_kv_pool()
        # one extra request slot: padding rows of a captured batch point at it
        self.dummy_req = self.max_reqs
        self.req_to_page = ReqToPagePool(self.max_reqs + 1, self.max_pages_per_req, self.device)
        a0 = self.model.attention_layers()[0]
        num_sms = torch.cuda.get_device_properties(self.device).multi_processor_count if self.cuda else 148
        self.backend = AttentionBackend(max(self.max_reqs, 1) + 1, a0.num_heads, getattr(a0, "head_dim", 128),
                                        self.device, num_sms=num_sms)
        self.model.bind_kv_cache(self.kv_pool, self.backend)
        if self.draft is not None:
            self.draft.block.self_attn.kv_pool = self.kv_pool
            self.draft.block.self_attn.backend = self.backend
        self.relay = torch.zeros(self.max_reqs + 1, dtype=torch.int64, device=self.device)
        head = self.model.lm_head  # None on pipeline stages before the last
        self.vocab_start = head.start if head is not None else 0
        self.vocab_valid = head.end - head.start if head is not None else 0
        max_tokens = max(args.chunked_prefill_size, args.max_prefill_tokens) + self.max_reqs
        self.max_step_tokens = max_tokens
        self.io = StepIO(self.device, self._extend_layout(max_tokens, self.max_reqs + 1,
                                                          self.max_reqs * self.max_pages_per_req).nbytes,
                         self.max_reqs + 1)
        self.graph_runner = None
        self.logits_hook = None  # test seam: called with (ForwardBatch, local logits) of eager steps
        self._logprobs = None
        self.status_watch = None
        from .. import env_registry
        if self.cuda and env_registry.get_bool("SGLANG_B200_KERNEL_STATUS_CHECK", True):
            from ..ops import gemm as gemm_ops, moe as moe_ops
            from ..parallel import collectives
            srcs = [gemm_ops._status_buf(self.device), moe_ops._status(self.device)]
            if collectives._custom_allreduce is not None:
                srcs.append(collectives._custom_allreduce.status)
            self.status_watch = KernelStatusWatch(srcs)
        if (self.cuda and not args.disable_cuda_graph and self.model.graph_capturable
                and self.draft is None and st.pp_size == 1):
            from .graph_runner import CudaGraphRunner
            self.graph_runner = CudaGraphRunner(self)

    # ------------------------------------------------------------------------------------------
    def load_weights(self) -> None:
        fmt = self.args.load_format
        if fmt == "auto":
            import os
            fmt = "safetensors" if os.path.isdir(self.args.model) else "random"
        if fmt == "random":
            src = RandomSource(self.cfg, self.device, seed=self.args.seed, std=self.args.random_weight_std,
                               gen_device=self.args.random_gen_device)
        else:
            src = SafetensorsSource(self.args.model, self.device)
        load_model_weights(self.model, src)
        if self.draft is not None:
            self.draft.load(src.get)
        if self.cuda:
            # GEMM weights as contiguous 128 x 64 tiles (one DRAM stream per TMA box)
            from ..layers.linear import pack_linear_weights
            pack_linear_weights(self.model)
            if self.draft is not None:
                pack_linear_weights(self.draft)
            torch.cuda.synchronize(self.device)
            torch.cuda.empty_cache()

    def init_kv_pool(self) -> None:
        cfg, args = self.cfg, self.args
        attn = self.model.attention_layers()
        P = self.page_size
        # this pipeline stage's layers (+ the MTP block's one extra layer)
        layer_ids = [a.layer_id for a in attn] + ([cfg.num_layers] if self.draft is not None else [])
        n_layers = len(layer_ids)
        # the stage's KV layout, declared before any pool is built and checked to match on every rank
        from ..mem_cache.kv_spec import declare
        from ..parallel.contract import assert_fleet_consistent
        self.kv_spec = declare(cfg, attn, P, self.kv_dtype, args.enable_hybrid_swa, get_state().dcp_size,
                               extra_layer_ids=[cfg.num_layers] if self.draft is not None else [])
        if get_state().cpu_group is not None:  # the stage's TP ranks (stages of a pipeline differ by design)
            assert_fleet_consistent({"kv_spec": self.kv_spec.digest()}, group=get_state().cpu_group)
        # hybrid sliding-window layout: sliding layers in a window pool sized by the scheduling bound
        swa_layers = self.kv_spec.pool_layers("window")
        swa_pages, swa_bytes = 0, 0
        if swa_layers:
            from ..mem_cache.hybrid_swa import check_window_pool, window_pool_pages
            win = max(a.window for a in attn if a.layer_id in swa_layers)
            need = window_pool_pages(self.max_reqs, win, P, args.chunked_prefill_size)
            swa_pages = args.swa_pool_pages or need
            check_window_pool(swa_pages, self.max_reqs, win, P, args.chunked_prefill_size)
            swa_bytes = swa_pages * MHATokenToKVPool.bytes_per_page(len(swa_layers), P, attn[0].num_kv_heads,
                                                                    cfg.head_dim, self.kv_dtype)
            n_layers -= len(swa_layers)
            self.swa_window = win
        if cfg.is_mla:
            per_page = MLATokenToKVPool.bytes_per_page(n_layers, P, cfg.kv_lora_rank, cfg.qk_rope_head_dim,
                                                       self.kv_dtype)
        else:
            per_page = MHATokenToKVPool.bytes_per_page(n_layers, P, attn[0].num_kv_heads, cfg.head_dim,
                                                       self.kv_dtype)
        if args.max_total_tokens:
            num_pages = args.max_total_tokens // P + 1
        elif self.cuda:
            free, total = torch.cuda.mem_get_info(self.device)
            reserve = 6 * (1 << 30) + int(0.04 * total)
            budget = max(0, int(free * args.mem_fraction_static) - reserve - swa_bytes)
            num_pages = max(2, budget // per_page)
            cap = (self.max_reqs * self.max_pages_per_req) // get_state().dcp_size + self.max_reqs + 2
            num_pages = min(num_pages, max(cap, 2))
        else:
            # decode context parallelism: each rank holds 1/dcp of every context (+ a partial page each)
            D = get_state().dcp_size
            num_pages = (self.max_reqs * self.max_pages_per_req) // D + (self.max_reqs + 2 if D > 1 else 1)
        self.num_pages = int(num_pages)
        if cfg.is_mla:
            self.kv_pool = MLATokenToKVPool(n_layers, self.num_pages, P, cfg.kv_lora_rank,
                                            cfg.qk_rope_head_dim, self.kv_dtype, self.device, layer_ids=layer_ids)
            if get_state().dcp_size > 1:
                from ..parallel.dcp import DcpView
                self.kv_pool.dcp = DcpView(P)
        else:
            self.kv_pool = MHATokenToKVPool(len(layer_ids), self.num_pages, P, attn[0].num_kv_heads, cfg.head_dim,
                                            self.kv_dtype, self.device, layer_ids=layer_ids,
                                            layer_pages={l: swa_pages for l in swa_layers} if swa_layers else None)
        logger.info("KV pool: %d pages x %d tokens (%.2f GB, %s)", self.num_pages, P,
                    self.num_pages * per_page / 1e9, self.kv_dtype)
        self.swa_num_pages = swa_pages
        if swa_layers:
            from ..mem_cache.hybrid_swa import SwaTranslate
            self.kv_pool.swa = SwaTranslate(self.num_pages, P, self.device)
            logger.info("window pool for %d sliding layers: %d pages (%.2f GB, window %d)", len(swa_layers),
                        swa_pages, swa_bytes / 1e9, self.swa_window)

    # ------------------------------------------------------------------------------------------
    @staticmethod
    def _extend_layout(T: int, B: int, U: int) -> Layout:
        return Layout([
            ("input_ids", torch.int64, T), ("positions", torch.int64, T), ("out_cache_loc", torch.int64, T),
            ("logits_idx", torch.int64, B), ("req_idx", torch.int64, B), ("seeds", torch.int64, B),
            ("top_k", torch.int64, B), ("seq_lens", torch.int32, B), ("qo_indptr", torch.int32, B + 1),
            ("page_upd", torch.int32, 3 * U), ("temperature", torch.float32, B), ("top_p", torch.float32, B),
        ])

    def apply_page_updates(self, upd: torch.Tensor) -> None:
        """upd: [U*3] int32 (req_slot, page_index, page_id) triples."""
        if upd.numel() == 0:
            return
        u = upd.view(-1, 3).long()
        swa = getattr(self.kv_pool, "swa", None)
        if swa is not None:
            # (-1, main page, window page) triples go to the window-page map, the rest to the block table
            # (map triples are redirected to the dummy row's first entry, which nothing reads)
            m = swa.apply(u)
            row = torch.where(m, torch.full_like(u[:, 0], self.dummy_req), u[:, 0])
            col = torch.where(m, torch.zeros_like(u[:, 1]), u[:, 1])
            val = torch.where(m, torch.zeros_like(u[:, 2]), u[:, 2])
            self.req_to_page.table[row, col] = val.to(torch.int32)
            return
        self.req_to_page.table[u[:, 0], u[:, 1]] = u[:, 2].to(torch.int32)

    def run_step(self, step) -> Tuple[torch.Tensor, Optional[torch.cuda.Event]]:
        """Launch one forward for a host-built StepInput; returns (pinned host ids view, event). With the step
        timer on (default on GPUs, SGLANG_B200_STEP_TIMER=0 turns it off) the step carries a pair of timing
        events around its device work; the scheduler reads the elapsed time once the step's results arrive."""
        t0 = None
        if self.cuda and _STEP_TIMER:
            t0 = torch.cuda.Event(enable_timing=True)
            t0.record()
        out = self._run_step(step)
        if t0 is not None:
            t1 = torch.cuda.Event(enable_timing=True)
            t1.record()
            step.device_events = (t0, t1)
        return out

    def _run_step(self, step) -> Tuple[torch.Tensor, Optional[torch.cuda.Event]]:
        if (step.mode == ForwardMode.DECODE and step.logprob_k < 0 and self.graph_runner is not None
                and not getattr(step, "dp_rows", 0) and self.graph_runner.can_run(step)):
            ids = self.graph_runner.replay(step)
        else:
            ids = self.forward_eager(step)
        if self.status_watch is not None:
            self.status_watch.snapshot(self.io)
        if step.logprob_k >= 0 and self._logprobs is not None:
            info = self._logprobs
            host = torch.empty(info.shape, dtype=torch.float32, pin_memory=self.cuda)
            host.copy_(info, non_blocking=self.cuda)  # ordered before the readback event
            self.io.d2h_bytes += info.numel() * 4
            step.logprob_host = host
        self._logprobs = None
        return self.io.readback(ids)

    def run_idle(self, rows: int) -> None:
        """DP attention: this attention group has no rows this step; join the other groups' MoE exchanges."""
        self.model.forward_idle(rows)

    def forward_eager(self, step) -> torch.Tensor:
        B, T = step.batch_size, step.num_tokens
        U = len(step.page_upd) // 3
        layout = self._extend_layout(T, B, U)
        arrays = step.arrays()
        v = self.io.upload(layout, arrays)
        self.apply_page_updates(v["page_upd"])
        req_idx = v["req_idx"]
        input_ids = v["input_ids"]
        D = step.num_decode
        if D > 0:
            # decode rows take their token from the device relay (the host may not know it yet)
            input_ids[:D] = self.relay.index_select(0, req_idx[:D])
        if step.mode == ForwardMode.EXTEND and step.relay_first_token is not None:
            pass
        block_table = self.req_to_page.table.index_select(0, req_idx.view(-1))
        fb = ForwardBatch(
            mode=step.mode, batch_size=B, num_tokens=T, input_ids=input_ids, positions=v["positions"],
            out_cache_loc=v["out_cache_loc"], seq_lens=v["seq_lens"], block_table=block_table,
            logits_idx=v["logits_idx"], qo_indptr=v["qo_indptr"], max_extend=step.max_extend,
            max_seq_len=step.max_seq_len, temperature=v["temperature"], seeds=v["seeds"], top_k=v["top_k"],
            top_p=v["top_p"], needs_topk_topp=step.needs_topk_topp)
        fb.extra["num_decode"] = D
        fb.extra["logprob_k"] = getattr(step, "logprob_k", -1)
        fb.extra["dp_rows"] = getattr(step, "dp_rows", 0)  # DP attention: rows per group in the MoE exchange
        # split count depends only on (rows, kv heads, context length) so eager and captured decode
        # reduce in the same order and produce identical tokens
        kvh = self.model.attention_layers()[0].num_kv_heads
        fb.decode_splits = self.backend.splits_for(B if step.mode == ForwardMode.DECODE else max(D, 1), kvh,
                                                   self.args.context_length)
        h = self.forward_model(fb)
        if get_state().pp_size > 1:
            return self._pp_sample(h, fb, req_idx)
        return self.sample(h, fb, req_idx)

    def _pp_sample(self, h, fb: ForwardBatch, req_idx: torch.Tensor) -> torch.Tensor:
        """Pipeline parallelism: the last stage samples; its ids reach every rank of the replica (scheduler
        and token relay), so the first stage can feed them back as the next decode input."""
        from ..parallel.collectives import pp_broadcast_ids
        B = int(fb.logits_idx.numel())
        if h is not None:
            ids = self.sample(h, fb, req_idx)
        else:
            ids = torch.empty(B, dtype=torch.int64, device=self.device)
        ids = pp_broadcast_ids(ids.contiguous())
        self.relay.index_copy_(0, req_idx.view(-1), ids.view(-1))
        k = fb.extra.get("logprob_k", -1)
        if k >= 0:  # the last stage's logprobs go to every rank of the replica too
            info = self._logprobs if self._logprobs is not None else torch.empty(
                B, 1 + 2 * k, dtype=torch.float32, device=self.device)
            self._logprobs = pp_broadcast_ids(info.contiguous())
        return ids

    def forward_model(self, fb: ForwardBatch) -> torch.Tensor:
        if fb.mode == ForwardMode.EXTEND and fb.extra.get("num_decode", 0) > 0:
            return self._forward_mixed(fb)
        return self.model(fb)

    def _forward_mixed(self, fb: ForwardBatch) -> torch.Tensor:
        """Decode rows [0, D) and extend rows [D, T) share every GEMM; attention splits per part."""
        D = fb.extra["num_decode"]
        dec = ForwardBatch(mode=ForwardMode.DECODE, batch_size=D, num_tokens=D, input_ids=fb.input_ids[:D],
                           positions=fb.positions[:D], out_cache_loc=fb.out_cache_loc[:D],
                           seq_lens=fb.seq_lens[:D], block_table=fb.block_table[:D], logits_idx=fb.logits_idx[:D],
                           decode_splits=fb.decode_splits)
        ext = ForwardBatch(mode=ForwardMode.EXTEND, batch_size=fb.batch_size - D, num_tokens=fb.num_tokens - D,
                           input_ids=fb.input_ids[D:], positions=fb.positions[D:], out_cache_loc=fb.out_cache_loc[D:],
                           seq_lens=fb.seq_lens[D:], block_table=fb.block_table[D:], logits_idx=fb.logits_idx[D:],
                           qo_indptr=fb.qo_indptr, max_extend=fb.max_extend)
        fb.extra["parts"] = (D, dec, ext)
        return self.model(fb)

    def sample(self, h_last: torch.Tensor, fb: ForwardBatch, req_idx: torch.Tensor,
               out: Optional[torch.Tensor] = None) -> torch.Tensor:
        st = get_state()
        logits = self.model.compute_logits(h_last)
        if self.logits_hook is not None:
            self.logits_hook(fb, logits)
        B = h_last.shape[0]
        positions = fb.positions.index_select(0, fb.logits_idx) + 1
        if fb.needs_topk_topp:
            # per-shard top-256 candidate pools, one gather, filters + Gumbel-max on the merged pool
            from ..ops.sampling import sample_filtered
            merge = None
            if st.tp_size > 1:
                def merge(vals, ids):
                    from ..parallel.collectives import tp_all_gather_into
                    n = vals.shape[1]
                    pack = torch.cat([vals, ids.float()], dim=1).contiguous()
                    g = torch.empty(st.tp_size * pack.shape[0], pack.shape[1], dtype=torch.float32,
                                    device=vals.device)
                    tp_all_gather_into(g, pack)
                    g = g.view(st.tp_size, pack.shape[0], -1)
                    av = g[:, :, :n].permute(1, 0, 2).reshape(pack.shape[0], -1)
                    ai = g[:, :, n:].permute(1, 0, 2).reshape(pack.shape[0], -1)
                    mv, sel = av.topk(n, dim=-1)
                    return mv, ai.gather(1, sel).long()
            ids = sample_filtered(logits, fb.temperature, fb.top_k, fb.top_p, fb.seeds, positions,
                                  self.vocab_start, self.vocab_valid, merge)
            if out is not None:
                out.copy_(ids)
                ids = out
        elif st.tp_size == 1:
            ids = sample_tokens(logits, fb.temperature, fb.seeds, positions, out=out,
                                valid_vocab=self.vocab_valid)
        else:
            vals = torch.empty(B, dtype=torch.float32, device=logits.device)
            local = sample_tokens(logits, fb.temperature, fb.seeds, positions, out_vals=vals,
                                  vocab_offset=self.vocab_start, valid_vocab=self.vocab_valid)
            pair = torch.stack([vals, local.float()], dim=1).contiguous()
            gathered = torch.empty(st.tp_size * B, 2, dtype=torch.float32, device=logits.device)
            tp_all_gather_into(gathered, pair)
            g = gathered.view(st.tp_size, B, 2)
            best = g[:, :, 0].argmax(dim=0)  # first max = lowest rank = lowest token id on ties
            ids_f = g[:, :, 1].gather(0, best[None, :])[0]
            ids = ids_f.long()
            if out is not None:
                out.copy_(ids)
                ids = out
        self.relay.index_copy_(0, req_idx.view(-1), ids.view(-1))
        k = fb.extra.get("logprob_k", -1) if fb.extra else -1
        if k >= 0:
            self._logprobs = self._logprob_info(logits, ids, k)
        return ids

    def _logprob_info(self, logits: torch.Tensor, ids: torch.Tensor, k: int) -> torch.Tensor:
        """[B, 1 + 2k] fp32: log-probability of each chosen id under the raw (temperature 1) distribution, then
        the top-k log-probabilities and their ids (as fp32). Vocabulary-sharded logits are merged with one
        gather of per-shard (max, sum of exp) and of per-shard top-k, and a max-reduce of the chosen logit.
        Parity: the reference sampler's per-shard logsumexp and exact top-logprobs
        (sglang_neuron/sampling.py:212-470)."""
        st = get_state()
        lg = logits[:, : self.vocab_valid].float()
        B = lg.shape[0]
        m = lg.max(dim=-1).values
        se = torch.exp(lg - m[:, None]).sum(dim=-1)
        local = ids.view(-1).long() - self.vocab_start
        own = (local >= 0) & (local < self.vocab_valid)
        chosen = torch.where(own, lg.gather(1, local.clamp(0, max(self.vocab_valid - 1, 0))[:, None])[:, 0],
                             torch.full_like(m, float("-inf")))
        kk = min(k, self.vocab_valid)
        tv, ti = (lg.topk(kk, dim=-1) if kk > 0 else (lg[:, :0], torch.zeros(B, 0, dtype=torch.long,
                                                                                  device=lg.device)))
        ti = ti + self.vocab_start
        if st.tp_size > 1:
            import torch.distributed as dist
            from ..parallel.collectives import tp_all_gather_into
            pack = torch.cat([m[:, None], se[:, None], chosen[:, None], tv, ti.float()], dim=1).contiguous()
            g = torch.empty(st.tp_size * B, pack.shape[1], dtype=torch.float32, device=lg.device)
            tp_all_gather_into(g, pack)
            g = g.view(st.tp_size, B, -1)
            M = g[:, :, 0].max(dim=0).values
            se = (g[:, :, 1] * torch.exp(g[:, :, 0] - M[None])).sum(dim=0)
            m = M
            chosen = g[:, :, 2].max(dim=0).values
            if kk > 0:
                allv = g[:, :, 3:3 + kk].permute(1, 0, 2).reshape(B, -1)
                alli = g[:, :, 3 + kk:3 + 2 * kk].permute(1, 0, 2).reshape(B, -1)
                tv, sel = allv.topk(kk, dim=-1)
                ti = alli.gather(1, sel)
            del dist
        lse = m + torch.log(se)
        out = torch.zeros(B, 1 + 2 * k, dtype=torch.float32, device=lg.device)
        out[:, 0] = chosen - lse
        if kk > 0:
            out[:, 1:1 + kk] = tv - lse[:, None]
            out[:, 1 + k:1 + k + kk] = ti.float()
        return out
