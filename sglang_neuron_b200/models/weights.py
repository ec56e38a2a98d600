"""Weight sources: safetensors checkpoints (lazy, mmap'd, per-tensor) and deterministic random init keyed by
the Hugging Face tensor name, so both go through the same per-family loading code.

Parity: SafetensorsCheckpoint / SafetensorsWeightLoader (sglang_neuron/utils/checkpoints.py:54,
utils/weight_loader.py:24) read each rank's shard lazily; random init is this build's stand-in for
checkpoints that cannot be downloaded here (BASELINE runs use random-init weights of the named shapes).
"""
from __future__ import annotations

import glob
import hashlib
import json
import os
from typing import Dict, Optional, Tuple

import torch

from ..configs.model_config import ModelConfig


class SafetensorsSource:
    def __init__(self, path: str, device):
        from safetensors import safe_open
        self.device = device
        self.files: Dict[str, str] = {}
        idx = os.path.join(path, "model.safetensors.index.json")
        if os.path.exists(idx):
            with open(idx) as f:
                wm = json.load(f)["weight_map"]
            for name, fn in wm.items():
                self.files[name] = os.path.join(path, fn)
        else:
            for fn in glob.glob(os.path.join(path, "*.safetensors")):
                with safe_open(fn, "pt") as f:
                    for name in f.keys():
                        self.files[name] = fn
        self._open = {}

    def __contains__(self, name: str) -> bool:
        return name in self.files

    def get(self, name: str) -> torch.Tensor:
        from safetensors import safe_open
        fn = self.files.get(name)
        if fn is None:
            raise KeyError(f"checkpoint tensor {name!r} missing")
        h = self._open.get(fn)
        if h is None:
            h = safe_open(fn, "pt")
            self._open[fn] = h
        return h.get_tensor(name).to(self.device)


class DictSource:
    def __init__(self, table: Dict[str, torch.Tensor], device):
        self.table, self.device = table, device

    def __contains__(self, name):
        return name in self.table

    def get(self, name: str) -> torch.Tensor:
        if name not in self.table:
            raise KeyError(f"checkpoint tensor {name!r} missing")
        return self.table[name].to(self.device)


def _seed_of(seed: int, name: str) -> int:
    return int.from_bytes(hashlib.sha256(f"{seed}:{name}".encode()).digest()[:8], "little") & ((1 << 63) - 1)


def hf_shape(cfg: ModelConfig, name: str) -> Tuple[Tuple[int, ...], torch.dtype]:
    """Shape/dtype of a Hugging Face tensor of this architecture (used by random init)."""
    H, Hq, Hkv, D = cfg.hidden_size, cfg.num_heads, cfg.num_kv_heads, cfg.head_dim
    bf = torch.bfloat16
    leaf = name.split(".")
    if name in ("model.embed_tokens.weight", "lm_head.weight"):
        return (cfg.vocab_size, H), bf
    if name.endswith("eh_proj.weight"):
        return (H, 2 * H), bf
    if name.endswith("norm.weight"):
        if "q_norm" in name or "k_norm" in name:
            return (D,), bf
        if "kv_a_layernorm" in name:
            return (cfg.kv_lora_rank,), bf
        if "q_a_layernorm" in name:
            return (cfg.q_lora_rank,), bf
        return (H,), bf
    if ".self_attn." in name:
        kind = leaf[-2]
        is_bias = leaf[-1] == "bias"
        if cfg.is_mla:
            nope, rope, vd, r = cfg.qk_nope_head_dim, cfg.qk_rope_head_dim, cfg.v_head_dim, cfg.kv_lora_rank
            shapes = {"q_proj": (Hq * (nope + rope), H), "kv_a_proj_with_mqa": (r + rope, H),
                      "kv_b_proj": (Hq * (nope + vd), r), "o_proj": (H, Hq * vd)}
            return shapes[kind], bf
        if leaf[-1] == "sinks":
            return (Hq,), bf
        shapes = {"q_proj": (Hq * D, H), "k_proj": (Hkv * D, H), "v_proj": (Hkv * D, H), "o_proj": (H, Hq * D)}
        s = shapes[kind]
        return ((s[0],) if is_bias else s), bf
    if ".mlp." in name:
        if cfg.architecture == "GptOssForCausalLM":
            E, I = cfg.num_experts, cfg.moe_intermediate_size
            table = {
                "router.weight": ((E, H), bf), "router.bias": ((E,), bf),
                "experts.gate_up_proj_blocks": ((E, 2 * I, H // 32, 16), torch.uint8),
                "experts.gate_up_proj_scales": ((E, 2 * I, H // 32), torch.uint8),
                "experts.gate_up_proj_bias": ((E, 2 * I), bf),
                "experts.down_proj_blocks": ((E, H, I // 32, 16), torch.uint8),
                "experts.down_proj_scales": ((E, H, I // 32), torch.uint8),
                "experts.down_proj_bias": ((E, H), bf),
            }
            key = ".".join(name.split(".mlp.")[1].split(".")[-2:])
            return table[key]
        tail = name.split(".mlp.")[1]
        if tail == "gate.weight":
            return (cfg.num_experts, H), bf
        inter = cfg.intermediate_size
        if "experts." in tail and "shared_experts" not in tail:
            inter = cfg.moe_intermediate_size
        elif "shared_experts" in tail:
            inter = cfg.moe_intermediate_size * max(1, cfg.n_shared_experts)
        if tail.endswith("gate_up_proj.weight"):
            return (2 * inter, H), bf
        if tail.endswith("gate_proj.weight") or tail.endswith("up_proj.weight"):
            return (inter, H), bf
        if tail.endswith("down_proj.weight"):
            return (H, inter), bf
    raise KeyError(f"no shape rule for {name!r}")


class RandomSource:
    """Deterministic random weights: each tensor is a pure function of (seed, name), so every TP rank
    builds identical replicated tensors and consistent shards."""

    def __init__(self, cfg: ModelConfig, device, seed: int = 0, std: float = 0.02, mx_scale_exp: int = -7,
                 gen_device=None):
        self.cfg, self.device, self.seed, self.std = cfg, torch.device(device), seed, std
        self.mx_scale = 127 + mx_scale_exp
        # CPU and CUDA generators give different streams for one seed: generate on `gen_device` (default:
        # the target device) when two devices must see identical weights.
        self.gen_device = torch.device(gen_device) if gen_device is not None else self.device

    def __contains__(self, name):
        return True

    def get(self, name: str) -> torch.Tensor:
        shape, dtype = hf_shape(self.cfg, name)
        gd = self.gen_device
        g = torch.Generator(device=gd)
        g.manual_seed(_seed_of(self.seed, name))
        if name.endswith("norm.weight"):
            t = torch.ones(shape, dtype=dtype, device=gd)
        elif name.endswith("_blocks"):
            t = torch.randint(0, 256, shape, generator=g, device=gd, dtype=torch.uint8)
        elif name.endswith("_scales"):
            t = torch.randint(self.mx_scale - 1, self.mx_scale + 2, shape, generator=g, device=gd, dtype=torch.uint8)
        elif name.endswith("sinks"):
            t = torch.randn(shape, generator=g, device=gd).to(dtype)
        else:
            t = (torch.randn(shape, generator=g, device=gd) * self.std).to(dtype)
        return t.to(self.device)


def load_model_weights(model, source) -> None:
    """Run a family's loader against a source with `.get(name)`."""
    model.load_common(source.get)
    model.load_layers(source.get)
