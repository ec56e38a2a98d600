"""GPT-OSS graph on the CPU tier against Hugging Face transformers' GptOssForCausalLM built from the same
(dequantised MXFP4) weights: sinks, alternating sliding/full attention, YaRN, clamped SwiGLU, top-4 routing."""
import pytest
import torch

from sglang_neuron_b200.configs import model_config as mc
from sglang_neuron_b200.engine import Engine
from sglang_neuron_b200.models.weights import RandomSource
from sglang_neuron_b200.ops.moe import dequant_mxfp4
from sglang_neuron_b200.parallel.state import destroy_parallel
from sglang_neuron_b200.server_args import ServerArgs

TINY = dict(num_hidden_layers=2, vocab_size=1000, hidden_size=256, intermediate_size=128, num_local_experts=8,
            num_attention_heads=4, num_key_value_heads=2, head_dim=64, sliding_window=8)


def _hf_gpt_oss(cfg, src):
    transformers = pytest.importorskip("transformers")
    hf_cfg = transformers.GptOssConfig(
        num_hidden_layers=cfg.num_layers, num_local_experts=cfg.num_experts, vocab_size=cfg.vocab_size,
        hidden_size=cfg.hidden_size, intermediate_size=cfg.moe_intermediate_size, head_dim=cfg.head_dim,
        num_attention_heads=cfg.num_heads, num_key_value_heads=cfg.num_kv_heads, sliding_window=cfg.sliding_window,
        rope_theta=cfg.rope_theta, rope_scaling=dict(cfg.rope_scaling), num_experts_per_tok=cfg.num_experts_per_tok,
        layer_types=cfg.layer_types, rms_norm_eps=cfg.rms_norm_eps, tie_word_embeddings=False,
        max_position_embeddings=cfg.max_position_embeddings, swiglu_limit=cfg.swiglu_limit)
    hf_cfg._attn_implementation = "eager"
    model = transformers.GptOssForCausalLM(hf_cfg).float().eval()
    sd = model.state_dict()
    new = {}
    H, I = cfg.hidden_size, cfg.moe_intermediate_size
    for name in sd:
        if ".mlp.experts." in name:
            p = name.split(".mlp.experts.")[0] + ".mlp.experts."
            if name.endswith("gate_up_proj"):
                blocks = src.get(p + "gate_up_proj_blocks").reshape(cfg.num_experts, 2 * I, H // 2)
                w = dequant_mxfp4(blocks, src.get(p + "gate_up_proj_scales"))  # [E, 2I, H]
                new[name] = w.transpose(1, 2).contiguous()
            elif name.endswith("down_proj"):
                blocks = src.get(p + "down_proj_blocks").reshape(cfg.num_experts, H, I // 2)
                w = dequant_mxfp4(blocks, src.get(p + "down_proj_scales"))  # [E, H, I]
                new[name] = w.transpose(1, 2).contiguous()
            else:
                new[name] = src.get(name).float()
        else:
            new[name] = src.get(name).float()
    model.load_state_dict(new)
    return model


def test_tiny_gpt_oss_matches_reference():
    destroy_parallel()
    mc.PRESETS["gpt-oss-tiny"] = dict(mc.PRESETS["gpt-oss-120b"], **TINY)
    args = ServerArgs(model="gpt-oss-tiny", device="cpu", dtype="float32", page_size=4, context_length=256,
                      max_running_requests=4, chunked_prefill_size=16, disable_cuda_graph=True,
                      random_weight_std=0.05)
    eng = Engine(args)
    g = torch.Generator().manual_seed(1)
    prompts = [torch.randint(0, 1000, (n,), generator=g).tolist() for n in (30, 11)]
    outs = eng.generate(prompts, {"max_new_tokens": 10})
    ref = _hf_gpt_oss(eng.cfg, RandomSource(eng.cfg, "cpu", seed=0, std=0.05))
    for p, o in zip(prompts, outs):
        full = torch.tensor([p + o["output_ids"]])
        with torch.no_grad():
            logits = ref(full).logits[0]
        ref_tokens = logits[len(p) - 1:-1].argmax(-1).tolist()
        assert o["output_ids"] == ref_tokens
