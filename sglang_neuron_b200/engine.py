"""Public offline API: `Engine(...).generate(...)`.

Parity: sglang.Engine as served by the reference (SGLang's engine + the plugin's runtime). One Engine per
process group: with tp_size > 1 the caller launches one process per GPU (torchrun or
`Engine.launch_spmd`), every rank constructs the Engine, and rank 0 owns request intake; the other ranks
follow the broadcast request stream in lockstep.
"""
from __future__ import annotations

import itertools
import logging
import os
import time
from typing import Dict, List, Optional, Sequence, Union

import torch

from .configs.model_config import ModelConfig, resolve_model_config
from .managers.schedule_batch import SamplingParams
from .managers.scheduler import Scheduler
from .model_executor.model_runner import ModelRunner
from .parallel.state import get_state, init_process_group_from_env, initialize_parallel
from .server_args import ServerArgs

logger = logging.getLogger(__name__)


def trim_at_stop(text: str, stops) -> str:
    """The text up to the first occurrence of any stop sequence (OpenAI semantics: the stop is not returned)."""
    if not stops:
        return text
    cut = min((i for i in (text.find(s) for s in stops) if i >= 0), default=-1)
    return text if cut < 0 else text[:cut]


class Engine:
    def __init__(self, args: Optional[ServerArgs] = None, **kwargs):
        args = args or ServerArgs(**kwargs)
        from . import env_registry, general_plugin, serving_policy
        from .platform import check_hybrid_swa
        check_hybrid_swa(args)
        if args.device == "cuda" and (not torch.cuda.is_available()
                                      or env_registry.get_bool("SGLANG_B200_CPU_MODE", False)):
            args.device = "cpu"
        # this launch's serving policy: resolved once, exported, and read back by every part of the rank
        # (scheduler overlap depth, graph capture, the plugin's runtime hooks)
        serving_policy.export(serving_policy.resolve(args))
        general_plugin.register()
        self.policy = serving_policy.current()
        if not self.policy.cuda_graph:
            args.disable_cuda_graph = True
        self.args = args
        overrides = {}
        self.cfg: ModelConfig = resolve_model_config(args.model, **overrides)
        if int(os.environ.get("WORLD_SIZE", "1")) > 1:
            init_process_group_from_env()
        if args.device == "cuda":
            local = int(os.environ.get("LOCAL_RANK", "0"))
            torch.cuda.set_device(local)
            device = torch.device("cuda", local)
        else:
            device = torch.device("cpu")
        if args.dcp_size > 1 and not self.cfg.is_mla:
            raise ValueError("decode context parallelism splits the latent (MLA) KV pool; "
                             f"{self.cfg.architecture} has none")
        st = initialize_parallel(args.tp_size, args.ep_size, args.dp_size, device, pp_size=args.pp_size,
                                 dp_attention=args.enable_dp_attention, dcp_size=args.dcp_size,
                                 replica_tp=args.replica_tp_sizes)
        self.rank = st.rank
        self.custom_ar = None
        if st.tp_size > 1 and device.type == "cuda":
            from . import env_registry
            from .ops.gemm import cublas_baseline
            if not env_registry.get_bool("SGLANG_B200_DISABLE_FUSED_COLLECTIVES", False) and not cublas_baseline():
                from .parallel.collectives import set_custom_allreduce
                from .parallel.symm_mem import make_tp_allreduce
                self.custom_ar = make_tp_allreduce()
                set_custom_allreduce(self.custom_ar)
        self.runner = ModelRunner(args, self.cfg, device)
        self.scheduler = Scheduler(args, self.cfg, self.runner)
        self.tokenizer = None
        tok_path = args.tokenizer or (args.model if os.path.isdir(args.model) else None)
        if tok_path:
            try:
                from transformers import AutoTokenizer
                self.tokenizer = AutoTokenizer.from_pretrained(tok_path)
            except Exception as e:  # no tokenizer files: token-id mode
                logger.info("tokenizer unavailable (%s); serving token ids", e)
        self._ids = itertools.count()
        if self.tokenizer is not None:
            self.scheduler.stop_checker = self._stop_hit

    def _stop_hit(self, r) -> bool:
        """A text stop sequence appears in the decoded tail of the output (the tail covers the longest stop
        sequence: every token decodes to at least one character or none)."""
        longest = max(len(s) for s in r.params.stop)
        tail = self.tokenizer.decode(r.output_ids[-(longest + 4):])
        return any(s in tail for s in r.params.stop)

    def abort(self, rid: str) -> None:
        self.scheduler.abort(rid)

    # ------------------------------------------------------------------------------------------
    def _to_ids(self, prompt) -> List[int]:
        if isinstance(prompt, str):
            if self.tokenizer is None:
                raise ValueError("text prompts need a tokenizer; pass token ids instead")
            return self.tokenizer.encode(prompt)
        return [int(t) for t in prompt]

    def submit(self, prompt, sampling_params: Optional[Union[dict, SamplingParams]] = None, rid: Optional[str] = None):
        """Queue one request. On a follower rank (replica rank > 0) nothing is queued locally: requests arrive
        through rank 0's broadcast, and the returned rid is the one rank 0 assigns to the same call."""
        sp = sampling_params if isinstance(sampling_params, SamplingParams) else SamplingParams.from_dict(sampling_params)
        if sp.stop and self.tokenizer is None:
            raise ValueError("text stop sequences need a tokenizer; use stop_token_ids")
        rid = rid or f"req-{next(self._ids)}"
        if get_state().replica_rank != 0:
            return rid
        return self.scheduler.add_request(rid, self._to_ids(prompt), sp)

    def step(self) -> None:
        self.scheduler.step()

    def generate(self, prompts: Sequence, sampling_params=None) -> List[Dict]:
        """Blocking generation for a list of prompts (token-id lists or strings)."""
        if isinstance(sampling_params, list):
            sps = sampling_params
        else:
            sps = [sampling_params] * len(prompts)
        if self.args.speculative_algorithm == "MTP":
            return self._generate_spec(prompts, sps)
        handles = [self.submit(p, sp) for p, sp in zip(prompts, sps)]
        if get_state().attn_dp_size > 1:
            # DP attention: every rank steps until the exchanged state says no group has work left
            self.scheduler.step()
            while self.scheduler.has_work():
                self.scheduler.step()
            reqs = [self.scheduler.reqs_by_rid[h if isinstance(h, str) else h.rid] for h in handles]
        elif get_state().replica_rank != 0:
            # follower: step in lockstep until rank 0's matching requests have finished here too
            want = set(handles)
            while not want.issubset(self.scheduler.finished_by_rid):
                self.scheduler.step()
            self.scheduler.drain()
            reqs = [self.scheduler.finished_by_rid[r] for r in handles]
        else:
            reqs = handles
            self.scheduler.run_until_idle()
        out = []
        for r in reqs:
            d = {"rid": r.rid, "output_ids": list(r.output_ids), "finish_reason": r.finish_reason,
                 "prompt_tokens": r.prompt_len, "completion_tokens": len(r.output_ids),
                 "cached_tokens": r.prefix_len}
            if r.first_token_time is not None:
                d["ttft_s"] = r.first_token_time - r.arrival
            if self.tokenizer is not None:
                d["text"] = trim_at_stop(self.tokenizer.decode(r.output_ids), r.params.stop)
            if r.params.return_logprob:
                d["output_token_logprobs"] = [[lp, t] for lp, t in zip(r.output_logprobs, r.output_ids)]
                if r.params.top_logprobs_num > 0:
                    d["output_top_logprobs"] = [[[lp, t] for lp, t in row] for row in r.output_top_logprobs]
            out.append(d)
        return out

    def _generate_spec(self, prompts, sps) -> List[Dict]:
        """Speculative (MTP) generation: greedy, host-synchronous verify/accept steps."""
        from .managers.schedule_batch import Req
        from .speculative.mtp import MTPWorker
        if not hasattr(self, "_mtp"):
            self._mtp = MTPWorker(self, self.args.speculative_num_draft_tokens)
        sched = self.scheduler
        reqs = []
        for p, sp in zip(prompts, sps):
            sp = sp if isinstance(sp, SamplingParams) else SamplingParams.from_dict(sp)
            if sp.temperature > 0:
                raise ValueError("MTP speculative decoding serves greedy sampling only")
            r = Req(f"req-{next(self._ids)}", self._to_ids(p), sp)
            if not sched.free_slots:
                raise RuntimeError("no free request slot")
            r.slot = sched.free_slots.pop()
            reqs.append(r)
        self._mtp.generate(reqs)
        out = []
        for r in reqs:
            out.append({"rid": r.rid, "output_ids": list(r.output_ids), "finish_reason": r.finish_reason,
                        "prompt_tokens": r.prompt_len, "completion_tokens": len(r.output_ids)})
            sched.alloc.free(list(r.pages))
            r.pages = []
            sched.free_slots.append(r.slot)
        return out

    def flush_cache(self) -> None:
        self.scheduler.drain()
        if self.scheduler.radix is not None and not self.scheduler.running:
            if self.scheduler.hicache is not None:
                self.scheduler.hicache.reset()
            freed = self.scheduler.radix.reset()
            if freed:
                self.scheduler.alloc.free(list(freed))

    def shutdown(self) -> None:
        self.scheduler.drain()
        if self.runner.graph_runner is not None:
            # every captured graph (the filtered-sampler ones hold NCCL calls under TP) goes before the process
            # group, or its destruction waits on them
            self.runner.graph_runner.graphs.clear()
            self.runner.graph_runner.graphs_f.clear()
        if self.custom_ar is not None:
            from .parallel.collectives import set_custom_allreduce
            torch.cuda.synchronize()
            set_custom_allreduce(None)
            self.custom_ar.close()
            self.custom_ar = None
