"""Decoder families: Qwen3 (dense; GLM-4 shares the shell), Qwen3-MoE, GPT-OSS and DeepSeek-V2 (MLA).

Each class maps the Hugging Face checkpoint names of its family onto the shared blocks of models/common.py.
Parity: the reference's per-family packages models/qwen3 (sglang_model.py:13-54), models/glm4,
models/qwen3_moe (sglang_model.py, moe.py), models/gpt_oss (config.py, mxfp4/*) and models/deepseek_v2
(model.py, weights.py) with their `EntryClass` registrations.
"""
from __future__ import annotations

import torch
from torch import nn

from ..configs.model_config import ModelConfig
from .common import CausalLM, DecoderLayer, DenseMLP, GQAAttention, MoEBlock


class Qwen3ForCausalLM(CausalLM):
    """Dense transformer with QK-norm (Qwen3); also serves Llama-style dense checkpoints."""

    def make_layer(self, i: int) -> DecoderLayer:
        cfg = self.cfg
        mlp = DenseMLP(cfg.hidden_size, cfg.intermediate_size, self.dtype, self.device)
        return DecoderLayer(cfg, i, self.dtype, self.device, self.max_pos, mlp=mlp)

    def load_layers(self, get) -> None:
        for l in self.layers:
            l.self_attn.load(get)
            l.mlp.load(get, f"model.layers.{l.layer_id}.mlp.")


class Glm4ForCausalLM(Qwen3ForCausalLM):
    """GLM-4: QKV bias, partial interleaved rotary; the gate/up projection ships fused."""

    def load_layers(self, get) -> None:
        for l in self.layers:
            l.self_attn.load(get)
            p = f"model.layers.{l.layer_id}.mlp."
            gu = get(p + "gate_up_proj.weight")
            I = gu.shape[0] // 2
            l.mlp.gate_up.load_part(0, gu[:I])
            l.mlp.gate_up.load_part(1, gu[I:])
            l.mlp.down.load(get(p + "down_proj.weight"))


class Qwen3MoeForCausalLM(CausalLM):
    def make_layer(self, i: int) -> DecoderLayer:
        cfg = self.cfg
        mlp = (MoEBlock(cfg, i, self.dtype, self.device) if cfg.is_moe_layer(i)
               else DenseMLP(cfg.hidden_size, cfg.intermediate_size, self.dtype, self.device))
        return DecoderLayer(cfg, i, self.dtype, self.device, self.max_pos, mlp=mlp)

    def load_layers(self, get) -> None:
        for l in self.layers:
            l.self_attn.load(get)
            p = f"model.layers.{l.layer_id}.mlp."
            if isinstance(l.mlp, MoEBlock):
                m = l.mlp
                m.router.load(get(p + "gate.weight"))
                rng = range(m.e_lo, m.e_lo + m.e_local)
                w13 = torch.stack([torch.cat([get(f"{p}experts.{e}.gate_proj.weight"),
                                              get(f"{p}experts.{e}.up_proj.weight")], 0) for e in rng])
                w2 = torch.stack([get(f"{p}experts.{e}.down_proj.weight") for e in rng])
                m.set_experts_from_dense(w13.float(), w2.float())
            else:
                l.mlp.load(get, p)


class GptOssForCausalLM(CausalLM):
    """GPT-OSS: attention with QKV/O bias, learned sinks, alternating sliding (128) / full layers, YaRN;
    128 MXFP4 experts (top-4) with clamped SwiGLU."""

    def make_layer(self, i: int) -> DecoderLayer:
        mlp = MoEBlock(self.cfg, i, self.dtype, self.device)
        return DecoderLayer(self.cfg, i, self.dtype, self.device, self.max_pos, mlp=mlp)

    def load_layers(self, get) -> None:
        cfg = self.cfg
        H, I, E = cfg.hidden_size, cfg.moe_intermediate_size, cfg.num_experts
        for l in self.layers:
            l.self_attn.load(get)
            p = f"model.layers.{l.layer_id}.mlp."
            m = l.mlp
            m.router.load(get(p + "router.weight"), get(p + "router.bias"))
            sl = slice(m.e_lo, m.e_lo + m.e_local)
            b13 = get(p + "experts.gate_up_proj_blocks")[sl].reshape(m.e_local, 2 * I, H // 2)
            s13 = get(p + "experts.gate_up_proj_scales")[sl]
            bias13 = get(p + "experts.gate_up_proj_bias")[sl]
            b2 = get(p + "experts.down_proj_blocks")[sl].reshape(m.e_local, H, I // 2)
            s2 = get(p + "experts.down_proj_scales")[sl]
            bias2 = get(p + "experts.down_proj_bias")[sl]
            m.set_experts_mxfp4(b13.contiguous(), s13.contiguous(), bias13, b2.contiguous(), s2.contiguous(), bias2,
                                interleaved=True)


ENTRY_CLASSES = {
    "Qwen3ForCausalLM": Qwen3ForCausalLM,
    "LlamaForCausalLM": Qwen3ForCausalLM,
    "Glm4ForCausalLM": Glm4ForCausalLM,
    "Qwen3MoeForCausalLM": Qwen3MoeForCausalLM,
    "GptOssForCausalLM": GptOssForCausalLM,
}


def get_model_class(arch: str):
    if arch in ("DeepseekV2ForCausalLM", "DeepseekV3ForCausalLM"):
        from .deepseek_v2 import DeepseekV2ForCausalLM
        return DeepseekV2ForCausalLM
    if arch not in ENTRY_CLASSES:
        raise ValueError(f"architecture {arch!r} is not served (served: {sorted(ENTRY_CLASSES)} + DeepseekV2)")
    return ENTRY_CLASSES[arch]
