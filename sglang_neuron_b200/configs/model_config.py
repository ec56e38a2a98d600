"""Model configuration: one normalised view over the Hugging Face config.json of every served family.

Parity: the reference keeps per-family config classes (sglang_neuron/models/transformer/config.py:13
`TransformerConfig`, models/deepseek_v2/config.py, models/gpt_oss/config.py:29-72) and a catalog of
ModelSpecs (models/catalog.py:41-144). Here a single dataclass covers the four benchmarked families and the
named presets give the exact shapes of the benchmark configurations (Qwen3-0.6B/8B, Qwen3-30B-A3B,
DeepSeek-V2-Lite, GPT-OSS-120B) for random-init runs where no checkpoint is at hand.
"""
from __future__ import annotations

import dataclasses
import json
import os
from typing import Any, Dict, List, Optional


@dataclasses.dataclass
class ModelConfig:
    architecture: str
    hidden_size: int
    num_layers: int
    num_heads: int
    num_kv_heads: int
    head_dim: int
    intermediate_size: int
    vocab_size: int
    rms_norm_eps: float = 1e-6
    rope_theta: float = 10000.0
    rope_scaling: Optional[Dict[str, Any]] = None
    rotary_dim: Optional[int] = None          # partial rotary (GLM-4); None = head_dim
    rope_neox: bool = True                    # halves (NeoX) vs interleaved pairs
    max_position_embeddings: int = 32768
    qk_norm: bool = False
    attention_bias: bool = False
    o_proj_bias: bool = False
    tie_word_embeddings: bool = False
    # sliding window / sinks (GPT-OSS)
    sliding_window: int = 0
    layer_types: Optional[List[str]] = None   # "full_attention" / "sliding_attention" per layer
    attention_sinks: bool = False
    # MoE
    num_experts: int = 0
    num_experts_per_tok: int = 0
    moe_intermediate_size: int = 0
    norm_topk_prob: bool = True
    routed_scaling_factor: float = 1.0
    n_shared_experts: int = 0
    first_k_dense_replace: int = 0
    moe_layer_freq: int = 1
    router_bias: bool = False
    expert_bias: bool = False
    swiglu_limit: float = 0.0                 # >0: clamped SwiGLU (GPT-OSS)
    swiglu_alpha: float = 1.702
    # MLA (DeepSeek-V2)
    kv_lora_rank: int = 0
    q_lora_rank: int = 0
    qk_nope_head_dim: int = 0
    qk_rope_head_dim: int = 0
    v_head_dim: int = 0
    # quantisation of the expert weights ("mxfp4" for GPT-OSS checkpoints, "fp8" block-scaled)
    quantization: Optional[str] = None
    torch_dtype: str = "bfloat16"
    # speculative decoding (MTP) draft layers
    num_nextn_predict_layers: int = 0
    eos_token_id: Optional[List[int]] = None

    # ------------------------------------------------------------------
    @property
    def is_moe(self) -> bool:
        return self.num_experts > 0

    @property
    def is_mla(self) -> bool:
        return self.kv_lora_rank > 0

    @property
    def rot_dim(self) -> int:
        if self.is_mla:
            return self.qk_rope_head_dim
        return self.rotary_dim or self.head_dim

    def layer_window(self, i: int) -> int:
        if self.sliding_window <= 0:
            return 0
        if self.layer_types is None:
            return self.sliding_window
        return self.sliding_window if self.layer_types[i] == "sliding_attention" else 0

    def is_moe_layer(self, i: int) -> bool:
        if not self.is_moe:
            return False
        if i < self.first_k_dense_replace:
            return False
        return (i % max(1, self.moe_layer_freq)) == 0 if self.moe_layer_freq > 1 else True

    @property
    def kv_cache_dim(self) -> int:
        """Values stored per token per layer per KV head (MLA: one latent row of kv_lora + rope)."""
        if self.is_mla:
            return self.kv_lora_rank + self.qk_rope_head_dim
        return self.head_dim

    def to_dict(self) -> Dict[str, Any]:
        return dataclasses.asdict(self)

    # ------------------------------------------------------------------
    @classmethod
    def from_hf(cls, hf: Dict[str, Any]) -> "ModelConfig":
        arch = (hf.get("architectures") or ["?"])[0]
        H = hf["hidden_size"]
        nh = hf["num_attention_heads"]
        kw: Dict[str, Any] = dict(
            architecture=arch,
            hidden_size=H,
            num_layers=hf["num_hidden_layers"],
            num_heads=nh,
            num_kv_heads=hf.get("num_key_value_heads", nh),
            head_dim=hf.get("head_dim") or H // nh,
            intermediate_size=hf.get("intermediate_size", 0),
            vocab_size=hf["vocab_size"],
            rms_norm_eps=hf.get("rms_norm_eps", 1e-6),
            rope_theta=float(hf.get("rope_theta", 10000.0)),
            rope_scaling=hf.get("rope_scaling"),
            max_position_embeddings=hf.get("max_position_embeddings", 32768),
            tie_word_embeddings=bool(hf.get("tie_word_embeddings", False)),
            torch_dtype=str(hf.get("torch_dtype", "bfloat16")),
        )
        eos = hf.get("eos_token_id")
        kw["eos_token_id"] = [eos] if isinstance(eos, int) else eos
        if arch in ("Qwen3ForCausalLM", "Qwen3MoeForCausalLM"):
            kw["qk_norm"] = True
            kw["attention_bias"] = bool(hf.get("attention_bias", False))
        if arch in ("Glm4ForCausalLM", "GlmForCausalLM"):
            kw["attention_bias"] = True
            kw["rotary_dim"] = int(kw["head_dim"] * hf.get("partial_rotary_factor", 0.5))
            kw["rope_neox"] = False
        if arch == "Qwen3MoeForCausalLM":
            kw.update(num_experts=hf["num_experts"], num_experts_per_tok=hf["num_experts_per_tok"],
                      moe_intermediate_size=hf["moe_intermediate_size"],
                      norm_topk_prob=bool(hf.get("norm_topk_prob", True)))
        if arch in ("DeepseekV2ForCausalLM", "DeepseekV3ForCausalLM"):
            kw.update(num_experts=hf.get("n_routed_experts", 0), num_experts_per_tok=hf.get("num_experts_per_tok", 0),
                      moe_intermediate_size=hf.get("moe_intermediate_size", 0),
                      norm_topk_prob=bool(hf.get("norm_topk_prob", False)),
                      routed_scaling_factor=float(hf.get("routed_scaling_factor", 1.0)),
                      n_shared_experts=hf.get("n_shared_experts", 0) or 0,
                      first_k_dense_replace=hf.get("first_k_dense_replace", 0),
                      moe_layer_freq=hf.get("moe_layer_freq", 1),
                      kv_lora_rank=hf["kv_lora_rank"], q_lora_rank=hf.get("q_lora_rank") or 0,
                      qk_nope_head_dim=hf["qk_nope_head_dim"], qk_rope_head_dim=hf["qk_rope_head_dim"],
                      v_head_dim=hf["v_head_dim"], rope_neox=False,
                      num_nextn_predict_layers=hf.get("num_nextn_predict_layers", 0) or 0)
            kw["head_dim"] = hf["qk_nope_head_dim"] + hf["qk_rope_head_dim"]
            kw["num_kv_heads"] = 1
        if arch == "GptOssForCausalLM":
            kw.update(num_experts=hf["num_local_experts"], num_experts_per_tok=hf["num_experts_per_tok"],
                      moe_intermediate_size=hf["intermediate_size"], norm_topk_prob=True,
                      attention_bias=True, o_proj_bias=True, sliding_window=hf.get("sliding_window", 128),
                      layer_types=hf.get("layer_types"), attention_sinks=True, router_bias=True, expert_bias=True,
                      swiglu_limit=float(hf.get("swiglu_limit", 7.0)),
                      quantization=(hf.get("quantization_config") or {}).get("quant_method", "mxfp4"))
            if kw["layer_types"] is None:
                kw["layer_types"] = ["sliding_attention" if i % 2 == 0 else "full_attention"
                                     for i in range(kw["num_layers"])]
        return cls(**kw)

    @classmethod
    def from_path(cls, path: str) -> "ModelConfig":
        with open(os.path.join(path, "config.json")) as f:
            return cls.from_hf(json.load(f))


def _gpt_oss(layers: int, experts: int) -> Dict[str, Any]:
    return {
        "architectures": ["GptOssForCausalLM"], "hidden_size": 2880, "num_hidden_layers": layers,
        "num_attention_heads": 64, "num_key_value_heads": 8, "head_dim": 64, "intermediate_size": 2880,
        "vocab_size": 201088, "rms_norm_eps": 1e-5, "rope_theta": 150000.0,
        "rope_scaling": {"rope_type": "yarn", "factor": 32.0, "beta_fast": 32.0, "beta_slow": 1.0,
                         "truncate": False, "original_max_position_embeddings": 4096},
        "max_position_embeddings": 131072, "num_local_experts": experts, "num_experts_per_tok": 4,
        "sliding_window": 128, "swiglu_limit": 7.0, "tie_word_embeddings": False,
        "quantization_config": {"quant_method": "mxfp4"}, "eos_token_id": [200002, 199999],
    }


# The benchmark configurations' model shapes (random-init runs).
PRESETS: Dict[str, Dict[str, Any]] = {
    "qwen3-0.6b": {
        "architectures": ["Qwen3ForCausalLM"], "hidden_size": 1024, "num_hidden_layers": 28,
        "num_attention_heads": 16, "num_key_value_heads": 8, "head_dim": 128, "intermediate_size": 3072,
        "vocab_size": 151936, "rms_norm_eps": 1e-6, "rope_theta": 1000000.0, "tie_word_embeddings": True,
        "max_position_embeddings": 40960, "eos_token_id": 151645,
    },
    "qwen3-8b": {
        "architectures": ["Qwen3ForCausalLM"], "hidden_size": 4096, "num_hidden_layers": 36,
        "num_attention_heads": 32, "num_key_value_heads": 8, "head_dim": 128, "intermediate_size": 12288,
        "vocab_size": 151936, "rms_norm_eps": 1e-6, "rope_theta": 1000000.0, "tie_word_embeddings": False,
        "max_position_embeddings": 40960, "eos_token_id": 151645,
    },
    "qwen3-30b-a3b": {
        "architectures": ["Qwen3MoeForCausalLM"], "hidden_size": 2048, "num_hidden_layers": 48,
        "num_attention_heads": 32, "num_key_value_heads": 4, "head_dim": 128, "intermediate_size": 6144,
        "moe_intermediate_size": 768, "num_experts": 128, "num_experts_per_tok": 8, "norm_topk_prob": True,
        "vocab_size": 151936, "rms_norm_eps": 1e-6, "rope_theta": 1000000.0, "tie_word_embeddings": False,
        "max_position_embeddings": 40960, "eos_token_id": 151645,
    },
    "deepseek-v2-lite": {
        "architectures": ["DeepseekV2ForCausalLM"], "hidden_size": 2048, "num_hidden_layers": 27,
        "num_attention_heads": 16, "num_key_value_heads": 16, "intermediate_size": 10944,
        "moe_intermediate_size": 1408, "n_routed_experts": 64, "num_experts_per_tok": 6, "n_shared_experts": 2,
        "first_k_dense_replace": 1, "moe_layer_freq": 1, "norm_topk_prob": False, "routed_scaling_factor": 1.0,
        "kv_lora_rank": 512, "q_lora_rank": None, "qk_nope_head_dim": 128, "qk_rope_head_dim": 64,
        "v_head_dim": 128, "vocab_size": 102400, "rms_norm_eps": 1e-6, "rope_theta": 10000.0,
        "rope_scaling": {"type": "yarn", "factor": 40, "original_max_position_embeddings": 4096,
                         "beta_fast": 32, "beta_slow": 1, "mscale": 0.707, "mscale_all_dim": 0.707},
        "max_position_embeddings": 163840, "tie_word_embeddings": False, "eos_token_id": 100001,
        "num_nextn_predict_layers": 1,
    },
    "gpt-oss-120b": _gpt_oss(36, 128),
    "gpt-oss-20b": _gpt_oss(24, 32),
}


def get_preset(name: str, **overrides) -> ModelConfig:
    hf = dict(PRESETS[name])
    hf.update(overrides)
    return ModelConfig.from_hf(hf)


def resolve_model_config(model: str, **overrides) -> ModelConfig:
    """`model` is a preset name or a directory holding config.json."""
    if model in PRESETS:
        return get_preset(model, **overrides)
    cfg = ModelConfig.from_path(model)
    for k, v in overrides.items():
        setattr(cfg, k, v)
    return cfg
