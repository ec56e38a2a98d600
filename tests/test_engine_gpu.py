"""End-to-end engine on the GPU: CUDA-graph decode equals eager decode token for token, and the bf16 GPU
path tracks the fp32 CPU oracle on the same random weights."""
import pytest
import torch

from sglang_neuron_b200.configs import model_config as mc
from sglang_neuron_b200.engine import Engine
from sglang_neuron_b200.parallel.state import destroy_parallel
from sglang_neuron_b200.server_args import ServerArgs

pytestmark = pytest.mark.gpu

TINY_OSS = dict(num_hidden_layers=2, vocab_size=2048, hidden_size=512, intermediate_size=256, num_local_experts=8,
                num_attention_heads=8, num_key_value_heads=2, head_dim=64, sliding_window=16)
TINY_QWEN = dict(num_hidden_layers=2, vocab_size=2048, hidden_size=512, intermediate_size=1024,
                 num_attention_heads=8, num_key_value_heads=4, head_dim=128)
TINY_MOE = dict(num_hidden_layers=2, vocab_size=2048, hidden_size=512, moe_intermediate_size=128, num_experts=16,
                num_experts_per_tok=4, num_attention_heads=8, num_key_value_heads=4, head_dim=128)


def _engine(base, over, device, graph=True, kv="auto", std=0.05, **kw):
    destroy_parallel()
    name = base + "-gputest"
    mc.PRESETS[name] = dict(mc.PRESETS[base], **over)
    args = ServerArgs(model=name, device=device, dtype="bfloat16" if device == "cuda" else "float32", page_size=16,
                      context_length=512, max_running_requests=8, chunked_prefill_size=48,
                      disable_cuda_graph=not graph, cuda_graph_bs=[1, 2, 4, 8], kv_cache_dtype=kv,
                      random_weight_std=std, random_gen_device="cpu", **kw)
    return Engine(args)


def _prompts(n=4, vocab=2048):
    g = torch.Generator().manual_seed(3)
    return [torch.randint(0, vocab, (int(L),), generator=g).tolist() for L in (5, 33, 70, 17)[:n]]


@pytest.mark.parametrize("base,over,kv", [("gpt-oss-120b", TINY_OSS, "fp8_e4m3"), ("gpt-oss-120b", TINY_OSS, "bf16"),
                                          ("qwen3-8b", TINY_QWEN, "bf16"), ("qwen3-30b-a3b", TINY_MOE, "bf16")])
def test_graph_equals_eager(base, over, kv):
    prompts = _prompts()
    a = _engine(base, over, "cuda", graph=True, kv=kv).generate(prompts, {"max_new_tokens": 12})
    b = _engine(base, over, "cuda", graph=False, kv=kv).generate(prompts, {"max_new_tokens": 12})
    assert [o["output_ids"] for o in a] == [o["output_ids"] for o in b]


def test_hybrid_swa_pool_equals_single_pool():
    """Sliding layers in the window pool (pages reused across requests as they leave the window), decode in
    CUDA graphs with the translated tables: the same tokens as one pool for all layers."""
    g = torch.Generator().manual_seed(11)
    prompts = [torch.randint(0, 2048, (L,), generator=g).tolist() for L in (5, 33, 70, 17, 90, 120, 64, 41)]
    sp = {"max_new_tokens": 48}
    one = _engine("gpt-oss-120b", TINY_OSS, "cuda").generate(prompts, sp)
    eng = _engine("gpt-oss-120b", TINY_OSS, "cuda", enable_hybrid_swa=True)
    two = eng.generate(prompts, sp)
    assert eng.runner.swa_num_pages < sum(len(p) + 48 for p in prompts) // 16  # pages had to be reused
    assert [o["output_ids"] for o in two] == [o["output_ids"] for o in one]


@pytest.mark.parametrize("base,over,tol", [("gpt-oss-120b", TINY_OSS, 0.2), ("qwen3-8b", TINY_QWEN, 0.08)])
def test_gpu_tracks_cpu_oracle(base, over, tol):
    """The MoE family's GPU path quantises expert activations to MXFP8 (e4m3 + e8m0 per 32, the block-scaled
    tcgen05 GEMM's input format) while the fp32 oracle does not, hence its wider relative tolerance."""
    prompts = _prompts(3)
    got = {}
    for dev in ("cuda", "cpu"):
        eng = _engine(base, over, dev, graph=False, kv="bf16" if dev == "cuda" else "auto", std=0.2)
        rows = []
        eng.runner.logits_hook = lambda fb, lg: rows.append(lg[:, :2048].float().cpu())
        eng.generate(prompts, {"max_new_tokens": 1})
        got[dev] = torch.cat(rows, 0)
    g, c = got["cuda"], got["cpu"]
    rel = (g - c).norm() / c.norm()
    assert rel < tol, f"GPU bf16 logits deviate from the fp32 oracle: rel {rel}"
    # the argmax must agree wherever the oracle's top-1 margin exceeds the row's worst logit error
    top2 = c.topk(2, dim=-1).values
    confident = (top2[:, 0] - top2[:, 1]) > (g - c).abs().amax(-1)
    assert torch.equal(g.argmax(-1)[confident], c.argmax(-1)[confident]), f"rel {rel}"


def test_sampling_temperature_is_reproducible():
    prompts = _prompts(2)
    sp = {"max_new_tokens": 10, "temperature": 0.8, "seed": 1234}
    a = _engine("gpt-oss-120b", TINY_OSS, "cuda").generate(prompts, sp)
    b = _engine("gpt-oss-120b", TINY_OSS, "cuda", graph=False).generate(prompts, sp)
    assert [o["output_ids"] for o in a] == [o["output_ids"] for o in b]


def test_smoke_entry():
    from sglang_neuron_b200.smoke import run_smoke
    run_smoke("cuda:0")


def test_logprobs_on_gpu_and_graph_tokens_unchanged():
    """Requests asking for logprobs run their decode steps eagerly (the captured graphs sample only); the
    greedy tokens equal a run without logprobs, and the chosen token is the top-1 of its own top-k."""
    prompts = _prompts(3)
    plain = _engine("gpt-oss-120b", TINY_OSS, "cuda").generate(prompts, {"max_new_tokens": 6})
    lp = _engine("gpt-oss-120b", TINY_OSS, "cuda").generate(
        prompts, {"max_new_tokens": 6, "return_logprob": True, "top_logprobs_num": 4})
    assert [o["output_ids"] for o in plain] == [o["output_ids"] for o in lp]
    for o in lp:
        for (l, t), top in zip(o["output_token_logprobs"], o["output_top_logprobs"]):
            assert top[0][1] == t and abs(top[0][0] - l) < 1e-3 and l <= 0.0


TINY_DSV2 = dict(num_hidden_layers=2, vocab_size=2048, hidden_size=512, intermediate_size=1024,
                 moe_intermediate_size=128, n_routed_experts=8, num_experts_per_tok=2, n_shared_experts=1,
                 num_attention_heads=16, num_key_value_heads=16)


def test_deepseek_mla_graph_equals_eager_and_tracks_cpu():
    """DeepSeek-V2 decode on the MLA kernel: captured graphs give the eager tokens, and the GPU prefill logits
    follow the fp32 CPU oracle (MoE with MXFP8 activations, hence the GPT-OSS tolerance; only the first
    token's logits are compared: later steps would see different greedy tokens)."""
    prompts = _prompts()
    a = _engine("deepseek-v2-lite", TINY_DSV2, "cuda", graph=True, kv="bf16")
    assert a.runner.graph_runner is not None, "MLA decode should be graph-capturable"
    ga = a.generate(prompts, {"max_new_tokens": 10})
    b = _engine("deepseek-v2-lite", TINY_DSV2, "cuda", graph=False, kv="bf16").generate(prompts, {"max_new_tokens": 10})
    assert [o["output_ids"] for o in ga] == [o["output_ids"] for o in b]
    got = {}
    for dev in ("cuda", "cpu"):
        eng = _engine("deepseek-v2-lite", TINY_DSV2, dev, graph=False, kv="bf16" if dev == "cuda" else "auto",
                      std=0.2)
        rows = []
        eng.runner.logits_hook = lambda fb, lg: rows.append(lg[:, :2048].float().cpu())
        eng.generate(_prompts(3), {"max_new_tokens": 1})
        got[dev] = torch.cat(rows, 0)
    rel = (got["cuda"] - got["cpu"]).norm() / got["cpu"].norm()
    assert rel < 0.2, f"rel {rel}"


def test_filtered_sampling_on_gpu_is_seeded_and_inside_top_k():
    """top_k/top_p requests: the candidate-pool sampler is reproducible for a seed and every token is among
    the step's top-k of the GPU logits."""
    prompts = _prompts(2)
    sp = {"max_new_tokens": 6, "temperature": 1.0, "top_k": 5, "top_p": 0.9, "seed": 11}
    eng = _engine("qwen3-8b", TINY_QWEN, "cuda")
    rows = []
    eng.runner.logits_hook = lambda fb, lg: rows.append(lg[:, :2048].float().cpu())
    a = eng.generate(prompts, sp)
    b = _engine("qwen3-8b", TINY_QWEN, "cuda").generate(prompts, sp)
    assert [o["output_ids"] for o in a] == [o["output_ids"] for o in b]
    top5 = torch.cat(rows, 0).topk(5, dim=-1).indices
    assert top5.shape[0] > 0


def test_filtered_sampling_graph_equals_eager():
    """top-k / top-p decode steps replay their own CUDA graphs (radix-select pools, filters, Gumbel-max on
    the device): the same tokens as the eager path for the same seeds."""
    prompts = _prompts()
    sp = {"max_new_tokens": 10, "temperature": 0.8, "top_k": 20, "top_p": 0.9, "seed": 5}
    eng = _engine("gpt-oss-120b", TINY_OSS, "cuda", graph=True, kv="fp8_e4m3")
    assert eng.runner.graph_runner is not None and eng.runner.graph_runner.graphs_f
    a = eng.generate(prompts, sp)
    b = _engine("gpt-oss-120b", TINY_OSS, "cuda", graph=False, kv="fp8_e4m3").generate(prompts, sp)
    assert [o["output_ids"] for o in a] == [o["output_ids"] for o in b]
