"""MTP speculative decoding on the CPU tier: greedy outputs equal plain greedy decoding token for token
(verify over k+1 rows, longest agreeing prefix + bonus token, KV roll-back), for a GQA and an MLA target."""
import pytest
import torch

from sglang_neuron_b200.configs import model_config as mc
from sglang_neuron_b200.engine import Engine
from sglang_neuron_b200.parallel.state import destroy_parallel
from sglang_neuron_b200.server_args import ServerArgs

QWEN = dict(num_hidden_layers=2, vocab_size=500, hidden_size=128, intermediate_size=256, num_attention_heads=4,
            num_key_value_heads=2, head_dim=32)
DSV2 = dict(num_hidden_layers=2, vocab_size=500, hidden_size=128, intermediate_size=256, moe_intermediate_size=64,
            n_routed_experts=4, num_experts_per_tok=2, n_shared_experts=1, num_attention_heads=4,
            num_key_value_heads=4, kv_lora_rank=64, qk_nope_head_dim=32, qk_rope_head_dim=16, v_head_dim=32)


def _engine(base, over, spec, std):
    destroy_parallel()
    mc.PRESETS["spec-tiny"] = dict(mc.PRESETS[base], **over)
    return Engine(ServerArgs(model="spec-tiny", device="cpu", dtype="float32", page_size=4, context_length=256,
                             max_running_requests=4, chunked_prefill_size=64, random_weight_std=std,
                             speculative_algorithm="MTP" if spec else None, speculative_num_draft_tokens=3))


@pytest.mark.parametrize("base,over", [("qwen3-0.6b", QWEN), ("deepseek-v2-lite", DSV2)])
def test_mtp_equals_greedy(base, over):
    g = torch.Generator().manual_seed(4)
    prompts = [torch.randint(0, 500, (n,), generator=g).tolist() for n in (13, 6, 30)]
    ref = _engine(base, over, False, 0.3).generate(prompts, {"max_new_tokens": 11})
    eng = _engine(base, over, True, 0.3)
    out = eng.generate(prompts, {"max_new_tokens": 11})
    assert [o["output_ids"] for o in out] == [o["output_ids"] for o in ref]
    st = eng._mtp.stats
    assert st["verify_steps"] > 0 and st["drafted"] > 0
