"""Model catalog: one ModelSpec per served Hugging Face architecture.

Parity: sglang_neuron/models/catalog.py:41-144 (`ModelSpec`: package, KV dtypes, quantisations, decode
layouts, spec algorithms, ...) and `MODELS` (:188-300). The B200 catalog lists what this build serves and
what it refuses, so the platform can refuse an unserved launch before any weight is read.
"""
from __future__ import annotations

import dataclasses
from typing import Dict, Optional, Tuple


@dataclasses.dataclass(frozen=True)
class ModelSpec:
    architecture: str
    family: str                                   # module under sglang_neuron_b200.models
    kv_dtypes: Tuple[str, ...] = ("bf16", "fp8_e4m3")
    quantizations: Tuple[Optional[str], ...] = (None,)
    expert_format: Optional[str] = None           # "mxfp4" | "mxfp8" for MoE families
    attention: str = "gqa"                        # "gqa" | "mla"
    sliding_window: bool = False
    sinks: bool = False
    spec_algorithms: Tuple[str, ...] = ()
    cuda_graph: bool = True
    max_tp: int = 8
    notes: str = ""


MODELS: Dict[str, ModelSpec] = {
    "Qwen3ForCausalLM": ModelSpec("Qwen3ForCausalLM", "families"),
    "LlamaForCausalLM": ModelSpec("LlamaForCausalLM", "families", notes="served by the Qwen3 dense graph"),
    "Glm4ForCausalLM": ModelSpec("Glm4ForCausalLM", "families", notes="partial interleaved rotary, QKV bias"),
    "Qwen3MoeForCausalLM": ModelSpec("Qwen3MoeForCausalLM", "families", expert_format="mxfp8",
                                     quantizations=(None, "fp8")),
    "GptOssForCausalLM": ModelSpec("GptOssForCausalLM", "families", kv_dtypes=("fp8_e4m3", "bf16"),
                                   quantizations=("mxfp4",), expert_format="mxfp4", sliding_window=True,
                                   sinks=True),
    "DeepseekV2ForCausalLM": ModelSpec("DeepseekV2ForCausalLM", "deepseek_v2", kv_dtypes=("bf16",),
                                       expert_format="mxfp8", attention="mla", spec_algorithms=("MTP",),
                                       cuda_graph=True, notes="absorbed MLA on sm_100a kernels; decode CUDA-graph "
                                       "captured with the bf16 latent pool"),
}

REFUSED: Dict[str, str] = {
    "Qwen3_5MoeForCausalLM": "GDN hybrid (Qwen3.5) is not built on B200",
    "GlmMoeDsaForCausalLM": "GLM-5.2 (MLA + DeepSeek sparse attention) is not built on B200",
    "KimiK3ForCausalLM": "Kimi-K3 (KDA + MLA) is not built on B200",
}


def model_spec(architecture: str) -> ModelSpec:
    if architecture in MODELS:
        return MODELS[architecture]
    if architecture in REFUSED:
        raise ValueError(REFUSED[architecture])
    raise ValueError(f"architecture {architecture!r} is not served; served: {sorted(MODELS)}")
