"""DeepSeek-V2 (MLA absorbed attention over the paged latent pool, MoE with shared experts, dense first
layer, YaRN with mscale) on the CPU tier against Hugging Face transformers' DeepseekV2ForCausalLM."""
import pytest
import torch

from sglang_neuron_b200.configs import model_config as mc
from sglang_neuron_b200.engine import Engine
from sglang_neuron_b200.models.weights import RandomSource
from sglang_neuron_b200.parallel.state import destroy_parallel
from sglang_neuron_b200.server_args import ServerArgs

TINY = dict(num_hidden_layers=2, vocab_size=1000, hidden_size=256, intermediate_size=512, moe_intermediate_size=64,
            n_routed_experts=8, num_experts_per_tok=2, n_shared_experts=1, num_attention_heads=4,
            num_key_value_heads=4, kv_lora_rank=64, qk_nope_head_dim=32, qk_rope_head_dim=16, v_head_dim=32)


def test_tiny_deepseek_v2_matches_reference():
    transformers = pytest.importorskip("transformers")
    destroy_parallel()
    mc.PRESETS["dsv2-tiny"] = dict(mc.PRESETS["deepseek-v2-lite"], **TINY)
    args = ServerArgs(model="dsv2-tiny", device="cpu", dtype="float32", page_size=8, context_length=256,
                      max_running_requests=4, chunked_prefill_size=24, random_weight_std=0.05)
    eng = Engine(args)
    g = torch.Generator().manual_seed(2)
    prompts = [torch.randint(0, 1000, (n,), generator=g).tolist() for n in (29, 9)]
    outs = eng.generate(prompts, {"max_new_tokens": 8})
    cfg = eng.cfg
    hf = dict(mc.PRESETS["dsv2-tiny"])
    hf.pop("architectures")
    hf_cfg = transformers.DeepseekV2Config(**{k: v for k, v in hf.items() if k not in ("eos_token_id",)})
    hf_cfg._attn_implementation = "eager"
    ref = transformers.DeepseekV2ForCausalLM(hf_cfg).float().eval()
    src = RandomSource(cfg, "cpu", seed=0, std=0.05)
    sd = {}
    for name in ref.state_dict():
        if name.endswith("mlp.experts.gate_up_proj"):
            pre = name[: -len("gate_up_proj")]
            sd[name] = torch.stack([torch.cat([src.get(f"{pre}{e}.gate_proj.weight"), src.get(f"{pre}{e}.up_proj.weight")])
                                    for e in range(cfg.num_experts)]).float()
        elif name.endswith("mlp.experts.down_proj"):
            pre = name[: -len("down_proj")]
            sd[name] = torch.stack([src.get(f"{pre}{e}.down_proj.weight") for e in range(cfg.num_experts)]).float()
        else:
            sd[name] = src.get(name).float()
    ref.load_state_dict(sd, strict=False)
    # DeepSeek-V2 scales the softmax by mscale(factor, mscale_all_dim)^2 under YaRN (the original model code,
    # SGLang and the reference do); transformers' port omits it, so align the reference to the model.
    for layer, mine in zip(ref.model.layers, eng.runner.model.layers):
        layer.self_attn.scaling = mine.self_attn.scaling
    for p, o in zip(prompts, outs):
        full = torch.tensor([p + o["output_ids"]])
        with torch.no_grad():
            logits = ref(full).logits[0]
        assert o["output_ids"] == logits[len(p) - 1:-1].argmax(-1).tolist()
