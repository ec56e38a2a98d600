"""The B200 platform object: resolves launch arguments (catalog lookup, refusals, serving policy) and hands out
this build's classes (graph runner, KV pools, paged allocator, speculative worker, quantisation configs).

Parity: `NeuronSRTPlatform` (sglang_neuron/platform.py:569-796) and its device mixin (device.py:23-83):
`apply_server_args_defaults` (:585), `get_graph_runner_cls` (:690), `get_kv_pool_cls` (:695),
`get_paged_allocator_cls` (:757), `get_quantization_config` (:772), `get_speculative_worker_cls` (:683),
`refuse_unserved` (:110), `check_kv_cache` (:223), `default_decode_batch_sizes` (:445) and the megakernel
seams (:716-755). Device memory comes from cudaMemGetInfo instead of neuron-ls; the group-coordinator device
is the GPU; the communication backend is NCCL for device groups and gloo for host groups.
"""
from __future__ import annotations

import logging
import os
from typing import List, Optional

import torch

from . import env_registry, serving_policy
from .models.catalog import model_spec

logger = logging.getLogger(__name__)


def refuse_unserved(args, spec) -> None:
    if args.speculative_algorithm and args.speculative_algorithm not in spec.spec_algorithms:
        raise ValueError(f"{spec.architecture} does not serve speculative algorithm {args.speculative_algorithm!r}")
    if args.tp_size > spec.max_tp:
        raise ValueError(f"tp_size {args.tp_size} exceeds {spec.max_tp} for {spec.architecture}")
    if args.dp_size < 1 or args.tp_size < 1 or args.pp_size < 1:
        raise ValueError("tp_size, pp_size and dp_size must be >= 1")
    if args.pp_size > 1 and args.speculative_algorithm:
        raise ValueError("speculative decoding is not served with pipeline parallelism")
    check_hybrid_swa(args)


def check_hybrid_swa(args) -> None:
    if args.prefill_chunk_grid and (args.prefill_chunk_grid % args.page_size
                                    or args.prefill_chunk_grid > args.chunked_prefill_size):
        raise ValueError("prefill_chunk_grid must be a multiple of page_size and at most chunked_prefill_size")
    if args.dcp_size > 1:
        if (args.tp_size % args.dcp_size or args.enable_hierarchical_cache or args.disaggregation_mode != "null"
                or args.speculative_algorithm or args.pp_size > 1 or args.enable_dp_attention):
            raise ValueError("dcp_size must divide tp_size, and DCP is not served with the host KV tier, PD "
                             "disaggregation, speculative decoding, pipeline parallelism or DP attention")
    if args.enable_dp_attention and args.dp_size > 1:
        if args.speculative_algorithm or args.disaggregation_mode != "null" or args.pp_size > 1:
            raise ValueError("DP attention is not served with speculative decoding, PD disaggregation or "
                             "pipeline parallelism")
        if args.tp_size % args.dp_size:
            raise ValueError(f"dp_size {args.dp_size} must divide tp_size {args.tp_size} under DP attention")
    if args.enable_hybrid_swa:
        # the window pool keeps only the pages inside the window: prefix reuse, host tiers and KV hand-off,
        # which all need a prefix's whole KV, are not served with it
        if args.enable_hierarchical_cache or args.disaggregation_mode != "null" or args.speculative_algorithm:
            raise ValueError("the hybrid sliding-window pool is not served with the host KV tier, PD "
                             "disaggregation or speculative decoding")
        if not args.disable_radix_cache:
            logger.info("hybrid sliding-window pool: prefix cache disabled")
            args.disable_radix_cache = True


def check_kv_cache(args, spec) -> None:
    kv = args.kv_cache_dtype
    if kv != "auto" and kv not in spec.kv_dtypes and not (kv == "fp8" and "fp8_e4m3" in spec.kv_dtypes):
        raise ValueError(f"{spec.architecture} serves KV dtypes {spec.kv_dtypes}, not {kv!r}")
    if args.page_size not in (1, 4, 8, 16, 32, 64, 128):
        raise ValueError(f"page_size {args.page_size} is not supported")


def default_decode_batch_sizes(args) -> List[int]:
    return args.graph_batch_sizes()


class DeviceMixin:
    """Device queries of the platform (parity: NeuronDeviceMixin, sglang_neuron/device.py:23-83)."""

    device_name = "cuda"
    device_type = "cuda"
    dispatch_key = "CUDA"

    def get_device_total_memory(self, device_id: int = 0) -> int:
        return torch.cuda.get_device_properties(device_id).total_memory

    def get_available_memory(self, device_id: int = 0) -> int:
        free, _ = torch.cuda.mem_get_info(device_id)
        return free

    def get_device_capability(self, device_id: int = 0):
        return torch.cuda.get_device_capability(device_id)

    def synchronize(self) -> None:
        torch.cuda.synchronize()

    def get_torch_distributed_backend(self) -> str:
        return "nccl"

    def get_group_coordinator_device(self, local_rank: int) -> torch.device:
        return torch.device("cuda", local_rank)


class B200SRTPlatform(DeviceMixin):
    """Selected by `SGLANG_PLATFORM=b200` (see general_plugin.register) or by `activate()`."""

    name = "b200"
    capabilities = ("cuda_graph", "tcgen05", "tma", "nvlink_p2p")

    def apply_server_args_defaults(self, args):
        env_registry.refuse_unknown()
        from .configs.model_config import resolve_model_config
        cfg = resolve_model_config(args.model)
        spec = model_spec(cfg.architecture)
        refuse_unserved(args, spec)
        check_kv_cache(args, spec)
        if not spec.cuda_graph:
            args.disable_cuda_graph = True
        if args.device == "cuda" and not torch.cuda.is_available():
            args.device = "cpu"
        policy = serving_policy.resolve(args)
        serving_policy.export(policy)
        return args

    def supports_decode_context_parallel(self) -> bool:
        return False

    def get_default_attention_backend(self) -> str:
        return "b200"

    def supports_speculative_algorithm(self, algorithm: str) -> bool:
        return algorithm in ("MTP",)

    def get_speculative_worker_cls(self, algorithm: str):
        from .speculative.mtp import MTPWorker
        if algorithm != "MTP":
            raise ValueError(f"speculative algorithm {algorithm!r} is not served")
        return MTPWorker

    def get_graph_runner_cls(self):
        from .model_executor.graph_runner import CudaGraphRunner
        return CudaGraphRunner

    def get_kv_pool_cls(self, *, kind: str):
        from .mem_cache import memory_pool
        return {"mha": memory_pool.MHATokenToKVPool, "mla": memory_pool.MLATokenToKVPool}[kind]

    def get_paged_allocator_cls(self):
        from ._ext import _runtime
        if _runtime is not None:
            return _runtime.PageAllocator
        from .mem_cache.allocator import PyPageAllocator
        return PyPageAllocator

    def get_quantization_config(self, quantization: str):
        from .quant import get_quant_config
        return get_quant_config(quantization)

    def get_compile_backend(self, mode: Optional[str] = None) -> str:
        return "cuda_graph"

    def get_dispatch_key_name(self) -> str:
        return self.dispatch_key

    def init_backend(self) -> None:
        from .process_init import init_process
        init_process()

    # -- megakernel seams (per-layer decode giga-kernel registration) ------------------------------
    def get_megakernel_target(self) -> str:
        return "sm_100a"

    def install_megakernel_dispatch(self, *, model, built, binding):
        model.megakernel = (built, binding)
        return model
