"""Serving policy: resolved once in the launching process, exported as JSON in SGLANG_B200_SERVING_POLICY,
and read (never re-derived) by every rank.

Parity: sglang_neuron/serving_policy.py (`ServingPolicy` :32, `resolve` :426, `export` :551, `current` :559,
`set_launch_setting` :534): role, async execution, overlap depth, giga decode, decode result lag, prefix
cache backend and parallel sizes travel in one frozen object so policy stays out of user flags.

Readers: `Engine` resolves and exports the policy of its launch, then the scheduler takes its overlap depth,
the model runner its graph capture and the plugin's runtime hooks their sampler from `current()`.
"""
from __future__ import annotations

import dataclasses
import json
import os
from typing import Dict, Optional

ENV = "SGLANG_B200_SERVING_POLICY"


@dataclasses.dataclass(frozen=True)
class ServingPolicy:
    role: str = "aggregated"              # aggregated | prefill | decode
    async_execution: bool = True          # overlap scheduling: launch step N+1 before reading step N
    max_inflight_launches: int = 2
    cuda_graph: bool = True
    mixed_chunk: bool = True
    prefix_cache: str = "radix-page"      # radix-page | none
    tp_size: int = 1
    ep_size: int = 1
    dp_size: int = 1
    fused_collectives: bool = True        # NVLink fused GEMM+collective kernels when available
    kv_cache_dtype: str = "auto"
    page_size: int = 16
    speculative: Optional[str] = None
    sampler: str = "device"               # device | host (SGLANG_B200_SAMPLER)
    launch_settings: Dict[str, str] = dataclasses.field(default_factory=dict)


def resolve(args, environ=os.environ) -> ServingPolicy:
    """The launch's policy from its arguments and the registered environment switches. A host sampler runs
    outside CUDA graphs, so it turns graph capture off (recorded as a launch setting)."""
    from . import env_registry
    role = {"null": "aggregated"}.get(args.disaggregation_mode, args.disaggregation_mode)
    sampler = (env_registry.get("SGLANG_B200_SAMPLER", "device", environ) or "device").strip().lower()
    if sampler not in ("device", "host"):
        raise ValueError(f"SGLANG_B200_SAMPLER={sampler!r}: expected 'device' or 'host'")
    depth = int(env_registry.get("SGLANG_B200_MAX_INFLIGHT_LAUNCHES", "2", environ))
    if depth < 1:
        raise ValueError("SGLANG_B200_MAX_INFLIGHT_LAUNCHES must be >= 1")
    async_exec = not args.disable_overlap_schedule and depth > 1
    pol = ServingPolicy(
        role=role, async_execution=async_exec, max_inflight_launches=depth if async_exec else 1,
        cuda_graph=not args.disable_cuda_graph and sampler == "device",
        mixed_chunk=args.enable_mixed_chunk, prefix_cache="none" if args.disable_radix_cache else "radix-page",
        tp_size=args.tp_size, ep_size=args.ep_size or args.tp_size, dp_size=args.dp_size,
        fused_collectives=not env_registry.get_bool("SGLANG_B200_DISABLE_FUSED_COLLECTIVES", False, environ),
        kv_cache_dtype=args.kv_cache_dtype, page_size=args.page_size, speculative=args.speculative_algorithm,
        sampler=sampler)
    if sampler == "host" and not args.disable_cuda_graph:
        pol = set_launch_setting(pol, "cuda_graph", "off", "the host sampler reads logits on the host each step")
    return pol


def export(policy: ServingPolicy, environ=os.environ) -> str:
    s = json.dumps(dataclasses.asdict(policy), sort_keys=True)
    environ[ENV] = s
    return s


def current(environ=os.environ) -> Optional[ServingPolicy]:
    s = environ.get(ENV)
    if not s:
        return None
    return ServingPolicy(**json.loads(s))


def set_launch_setting(policy: ServingPolicy, key: str, value: str, reason: str) -> ServingPolicy:
    """Record a launch setting fixed by the platform, with the reason it is fixed."""
    ls = dict(policy.launch_settings)
    ls[key] = f"{value}  # {reason}"
    return dataclasses.replace(policy, launch_settings=ls)
