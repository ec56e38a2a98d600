"""Registry of every `SGLANG_B200_*` environment variable, by class; unknown names are refused.

Parity: sglang_neuron/env_registry.py (`refuse_unknown`, :125) keeps one table of the plugin's environment
names so a typo cannot silently disable a setting. Same rule here for the `SGLANG_B200_` prefix.
"""
from __future__ import annotations

import os
from typing import Dict, Mapping

PREFIX = "SGLANG_B200_"

# name -> (class, description)
REGISTRY: Dict[str, tuple] = {
    "SGLANG_B200_SERVING_POLICY": ("policy", "JSON serving policy exported by the launching process"),
    "SGLANG_B200_HOST_TRACE": ("trace", "directory for per-rank host-trace TSV files"),
    "SGLANG_B200_HOST_TRACE_SPANS": ("trace", "comma-separated extra host-trace spans"),
    "SGLANG_B200_PROFILE_RANKS": ("profile", "ranks that profile from process start"),
    "SGLANG_B200_PROFILE_SERVE_START": ("profile", "first decode step of a bounded profile window"),
    "SGLANG_B200_PROFILE_SERVE_STEPS": ("profile", "length of the bounded profile window in steps"),
    "SGLANG_B200_PROFILE_DIR": ("profile", "output directory of profile windows"),
    "SGLANG_B200_MAX_INFLIGHT_LAUNCHES": ("runtime", "steps launched ahead of result processing (overlap depth)"),
    "SGLANG_B200_SAMPLER": ("runtime", "'device' (default) or 'host' sampling"),
    "SGLANG_B200_DISABLE_FUSED_COLLECTIVES": ("parallel", "use NCCL instead of the NVLink fused kernels"),
    "SGLANG_B200_MOE_FUSED_ACT_QUANT": ("kernels", "1: gate/up GEMM epilogue writes MXFP8 directly (default: separate quantise)"),
    "SGLANG_B200_PDL": ("kernels", "programmatic dependent launch of the sm_100a kernels (0 turns it off)"),
    "SGLANG_B200_STEP_FENCE": ("debug", "1: ranks check through shared memory that each step launches the same program"),
    "SGLANG_B200_FUSED_AR_NORM": ("collectives", "residual add + RMSNorm inside the NVLink all-reduce kernels (0 turns it off)"),
    "SGLANG_B200_NVLS": ("parallel", "allow NVLS multimem (0/1)"),
    "SGLANG_B200_PD_TRANSFER": ("disagg", "KV transfer backend for PD: 'p2p' (default) or 'fake'"),
    "SGLANG_B200_PD_BOOTSTRAP_PORT": ("disagg", "bootstrap port of a prefill server"),
    "SGLANG_B200_KERNEL_STATUS_CHECK": ("debug", "read kernel status words after every step (0/1)"),
    "SGLANG_B200_BUILD_CACHE": ("build", "directory of the digest-keyed kernel build cache"),
    "SGLANG_B200_CPU_MODE": ("debug", "force the CPU oracle path (torch reference ops)"),
    "SGLANG_B200_NUMA_BIND": ("placement", "bind each rank's threads to its GPU's NUMA node (0/1)"),
    "SGLANG_B200_PROGRAM_FENCE_CHECK": ("debug", "all-gather the captured-graph id each step and compare"),
}


class UnknownEnvError(ValueError):
    pass


def refuse_unknown(environ: Mapping[str, str] = os.environ) -> None:
    unknown = sorted(k for k in environ if k.startswith(PREFIX) and k not in REGISTRY)
    if unknown:
        raise UnknownEnvError(f"unknown {PREFIX}* variables (typo?): {', '.join(unknown)}")


def get(name: str, default=None, environ: Mapping[str, str] = os.environ):
    if name not in REGISTRY:
        raise UnknownEnvError(f"{name} is not a registered variable")
    return environ.get(name, default)


def get_bool(name: str, default: bool = False, environ: Mapping[str, str] = os.environ) -> bool:
    v = get(name, None, environ)
    if v is None:
        return default
    return v.strip().lower() in ("1", "true", "yes", "on")
