"""Registry of every `SGLANG_B200_*` environment variable, by class; unknown names are refused.

Parity: sglang_neuron/env_registry.py (`refuse_unknown`, :125) keeps one table of the plugin's environment
names so a typo cannot silently disable a setting. Same rule here for the `SGLANG_B200_` prefix, and every
registered name has a reader (tests/test_runtime_cpu.py checks that each name appears in the package or the
native sources besides this table).
"""
from __future__ import annotations

import os
from typing import Dict, Mapping

PREFIX = "SGLANG_B200_"

# name -> (class, description)
REGISTRY: Dict[str, tuple] = {
    "SGLANG_B200_SERVING_POLICY": ("policy", "JSON serving policy exported by the launching process"),
    "SGLANG_B200_HOST_TRACE": ("trace", "directory for per-rank host-trace TSV files"),
    "SGLANG_B200_PROFILE_RANKS": ("profile", "comma-separated ranks that take the serve profile window (default: all)"),
    "SGLANG_B200_PROFILE_SERVE_START": ("profile", "first scheduler step of the bounded serve profile window"),
    "SGLANG_B200_PROFILE_SERVE_STEPS": ("profile", "length of the bounded profile window in steps"),
    "SGLANG_B200_PROFILE_DIR": ("profile", "output directory of the serve profile window (default profile_out)"),
    "SGLANG_B200_MAX_INFLIGHT_LAUNCHES": ("runtime", "steps launched ahead of result processing (overlap depth)"),
    "SGLANG_B200_SAMPLER": ("runtime", "'device' (default) or 'host' sampling"),
    "SGLANG_B200_DISABLE_FUSED_COLLECTIVES": ("parallel", "use NCCL instead of the NVLink fused kernels"),
    "SGLANG_B200_MOE_FUSED_ACT_QUANT": ("kernels", "1: gate/up GEMM epilogue writes MXFP8 directly (default: separate quantise)"),
    "SGLANG_B200_FUSED_ROUTE": ("kernels", "decode-sized MoE routing (router GEMM, top-k, align, quantise) in one launch (0 turns it off)"),
    "SGLANG_B200_BASELINE": ("bench", "'nccl': comparison build with cuBLAS dense GEMMs and NCCL collectives (no fused kernels)"),
    "SGLANG_B200_GEMM_2CTA": ("kernels", "decode-sized bf16 GEMMs may run two CTAs per SM to split K over more SMs (0 turns it off)"),
    "SGLANG_B200_SP_NVLINK": ("collectives", "1: sequence-parallel all-gather / reduce-scatter through the NVLink kernels instead of NCCL"),
    "SGLANG_B200_DENSE_GEMM": ("kernels", "plain dense GEMMs: 'cublas' (default, measured faster) or 'tcgen05' (this package's kernel)"),
    "SGLANG_B200_STEP_TIMER": ("profile", "per-step device time from CUDA events around each step (default 1; /metrics p50 by step kind)"),
    "SGLANG_B200_PDL": ("kernels", "programmatic dependent launch of the sm_100a kernels (0 turns it off)"),
    "SGLANG_B200_STEP_FENCE": ("debug", "1: ranks check through shared memory that each step launches the same program"),
    "SGLANG_B200_FUSED_AR_NORM": ("collectives", "residual add + RMSNorm inside the NVLink all-reduce kernels (0 turns it off)"),
    "SGLANG_B200_NVLS": ("parallel", "allow NVLS multimem (0/1)"),
    "SGLANG_B200_KERNEL_STATUS_CHECK": ("debug", "copy and check the kernels' bounded-wait status words after every step (default 1)"),
    "SGLANG_B200_CPU_MODE": ("debug", "1: serve on the CPU oracle path (torch reference ops) even with a GPU"),
    "SGLANG_B200_NUMA_BIND": ("placement", "bind each rank's threads to its GPU's NUMA node (0/1)"),
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
