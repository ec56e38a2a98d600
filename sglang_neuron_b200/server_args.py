"""Launch arguments of the engine and the HTTP server.

Parity: the reference resolves SGLang's ServerArgs in `NeuronSRTPlatform.apply_server_args_defaults`
(sglang_neuron/platform.py:585-663): page size, KV dtype, chunked prefill, decode batch buckets, graph
capture and memory fraction. Here the same knobs are one dataclass with B200 defaults.
"""
from __future__ import annotations

import argparse
import dataclasses
from typing import List, Optional


@dataclasses.dataclass
class ServerArgs:
    model: str = "qwen3-0.6b"                # preset name or checkpoint directory
    tokenizer: Optional[str] = None          # tokenizer directory (defaults to `model` when it is a path)
    load_format: str = "auto"                # auto | random | safetensors
    seed: int = 0
    dtype: str = "bfloat16"                  # activation/weight dtype (float32 for the CPU oracle)
    device: str = "cuda"
    tp_size: int = 1
    ep_size: Optional[int] = None
    dp_size: int = 1                         # DP replicas, or attention groups inside TP with enable_dp_attention
    enable_dp_attention: bool = False        # dp_size attention groups split the tp_size ranks; experts span all
    pp_size: int = 1
    dcp_size: int = 1                        # decode context parallelism (MLA models): TP ranks splitting each context's pages
    sp_min_tokens: int = 512                 # TP > 1: prefill steps of >= this many tokens run sequence-parallel between layers (0: off)
    page_size: int = 16
    kv_cache_dtype: str = "auto"             # auto | bf16 | fp8_e4m3
    context_length: int = 8192
    max_running_requests: int = 256
    max_total_tokens: Optional[int] = None   # KV capacity in tokens (default: from free memory)
    mem_fraction_static: float = 0.85
    chunked_prefill_size: int = 8192
    max_prefill_tokens: int = 16384
    enable_mixed_chunk: bool = True          # decode rows ride along with prefill chunks
    disable_radix_cache: bool = False
    prefill_chunk_grid: int = 0               # >0: prefill chunks end on multiples of this (per request) and prefix
                                              # hits are rounded down to it, so a hit replays the uncached chunking
    enable_hybrid_swa: bool = False           # sliding-window layers keep their K/V in a small window pool
    swa_pool_pages: int = 0                   # window pool pages (0: the sizing bound for max_running_requests)
    enable_hierarchical_cache: bool = False   # host (pinned memory) tier below the device prefix cache
    hicache_ratio: float = 2.0                # host pages = ratio x device KV pages (when hicache_host_pages is 0)
    hicache_host_pages: int = 0
    disable_cuda_graph: bool = False
    cuda_graph_max_bs: int = 256
    cuda_graph_bs: Optional[List[int]] = None
    disable_overlap_schedule: bool = False
    schedule_policy: str = "fcfs"            # fcfs | lpm (longest prefix match)
    speculative_algorithm: Optional[str] = None   # None | "MTP"
    speculative_num_draft_tokens: int = 3
    disaggregation_mode: str = "null"        # null | prefill | decode
    replica_tp_sizes: Optional[List[int]] = None  # DP replicas of different TP sizes, in rank order (PD on one box:
                                                  # [prefill TP, decode TP]); tp_size is this rank's own replica's
    host: str = "127.0.0.1"
    port: int = 30000
    log_level: str = "info"
    enable_metrics: bool = False
    host_trace_dir: Optional[str] = None
    random_weight_std: float = 0.02
    random_gen_device: Optional[str] = None   # device whose RNG draws random-init weights (default: `device`)

    def resolved_kv_dtype(self, arch: str):
        import torch
        if self.kv_cache_dtype in ("fp8", "fp8_e4m3"):
            return torch.float8_e4m3fn
        if self.kv_cache_dtype in ("bf16", "bfloat16"):
            return torch.bfloat16
        if self.device == "cpu" or self.dtype == "float32":
            return torch.float32
        # GPT-OSS serves an FP8 KV cache; others default to bf16
        return torch.float8_e4m3fn if arch == "GptOssForCausalLM" else torch.bfloat16

    def torch_dtype(self):
        import torch
        return {"bfloat16": torch.bfloat16, "bf16": torch.bfloat16, "float32": torch.float32,
                "fp32": torch.float32, "float16": torch.float16}[self.dtype]

    def graph_batch_sizes(self) -> List[int]:
        if self.cuda_graph_bs:
            return sorted(set(self.cuda_graph_bs))
        ladder = [1, 2, 4, 8, 12, 16, 24, 32, 40, 48, 56, 64, 80, 96, 112, 128, 160, 192, 224, 256, 320, 384, 448, 512]
        cap = min(self.cuda_graph_max_bs, self.max_running_requests)
        out = [b for b in ladder if b <= cap]
        if not out or out[-1] != cap:
            out.append(cap)
        return out

    @staticmethod
    def add_cli_args(p: argparse.ArgumentParser) -> None:
        for f in dataclasses.fields(ServerArgs):
            name = "--" + f.name.replace("_", "-")
            if f.type in ("bool", bool):
                p.add_argument(name, action="store_true", default=f.default)
            elif f.name in ("cuda_graph_bs", "replica_tp_sizes"):
                p.add_argument(name, type=int, nargs="+", default=None)
            else:
                typ = {"int": int, "float": float, "str": str}.get(str(f.type).replace("Optional[", "").rstrip("]"), str)
                p.add_argument(name, type=typ, default=f.default)

    @classmethod
    def from_cli(cls, ns: argparse.Namespace) -> "ServerArgs":
        return cls(**{f.name: getattr(ns, f.name) for f in dataclasses.fields(cls)})
