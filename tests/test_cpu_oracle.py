"""CPU oracle tier: the engine's runtime (scheduler, paged KV pool with 16-token pages,
chunked prefill, decode, token relay, sampler) running the Qwen3 dense graph in fp32 on CPU must match a
plain-PyTorch reference model (Hugging Face transformers' Qwen3ForCausalLM) built from the same weights."""
import pytest
import torch

from sglang_neuron_b200.configs import model_config as mc
from sglang_neuron_b200.engine import Engine
from sglang_neuron_b200.models.weights import RandomSource
from sglang_neuron_b200.parallel.state import destroy_parallel
from sglang_neuron_b200.server_args import ServerArgs


def _hf_qwen3(cfg, source):
    transformers = pytest.importorskip("transformers")
    hf_cfg = transformers.Qwen3Config(
        vocab_size=cfg.vocab_size, hidden_size=cfg.hidden_size, intermediate_size=cfg.intermediate_size,
        num_hidden_layers=cfg.num_layers, num_attention_heads=cfg.num_heads, num_key_value_heads=cfg.num_kv_heads,
        head_dim=cfg.head_dim, rms_norm_eps=cfg.rms_norm_eps, rope_theta=cfg.rope_theta,
        tie_word_embeddings=cfg.tie_word_embeddings, max_position_embeddings=cfg.max_position_embeddings,
        attention_bias=False, torch_dtype=torch.float32)
    hf_cfg._attn_implementation = "eager"
    model = transformers.Qwen3ForCausalLM(hf_cfg).float().eval()
    sd = {}
    for name, t in model.state_dict().items():
        if name == "lm_head.weight" and cfg.tie_word_embeddings:
            continue
        sd[name] = source.get(name).float()
    model.load_state_dict(sd, strict=False)
    if cfg.tie_word_embeddings:
        model.tie_weights()
    return model


def _run(model_name, n_req, prompt_len, new_tokens, chunk, overrides=None, layers=None):
    destroy_parallel()
    name = model_name
    if overrides:
        name = model_name + "-test"
        mc.PRESETS[name] = dict(mc.PRESETS[model_name], **overrides)
    args = ServerArgs(model=name, device="cpu", dtype="float32", page_size=16, context_length=1024,
                      max_running_requests=8, chunked_prefill_size=chunk, disable_cuda_graph=True)
    eng = Engine(args)
    captured = []
    eng.runner.logits_hook = lambda fb, logits: captured.append((fb, logits.clone()))
    g = torch.Generator().manual_seed(0)
    prompts = [torch.randint(0, eng.cfg.vocab_size, (prompt_len,), generator=g).tolist() for _ in range(n_req)]
    outs = eng.generate(prompts, {"max_new_tokens": new_tokens})
    src = RandomSource(eng.cfg, "cpu", seed=args.seed, std=args.random_weight_std)
    ref = _hf_qwen3(eng.cfg, src)
    return eng, prompts, outs, ref, captured


def _check(prompts, outs, ref, captured, tol):
    # greedy tokens must match the reference's greedy continuation
    for p, o in zip(prompts, outs):
        full = torch.tensor([p + o["output_ids"]])
        with torch.no_grad():
            logits = ref(full).logits[0]
        ref_tokens = logits[len(p) - 1:-1].argmax(-1).tolist()
        assert o["output_ids"] == ref_tokens, "greedy tokens diverge from the reference"
    # every captured logits row equals the reference logits at that position
    by_seq = {}
    for p, o in zip(prompts, outs):
        full = torch.tensor([p + o["output_ids"]])
        with torch.no_grad():
            by_seq[tuple(p)] = (ref(full).logits[0], p + o["output_ids"])
    n_checked = 0
    for fb, logits in captured:
        pos_last = fb.positions.index_select(0, fb.logits_idx)
        for row in range(logits.shape[0]):
            pos = int(pos_last[row])
            tok = int(fb.input_ids[fb.logits_idx[row]])
            # find the request whose sequence has `tok` at `pos`
            for key, (rl, seq) in by_seq.items():
                if pos < len(seq) and seq[pos] == tok and pos >= len(key) - 1:
                    err = (logits[row, :rl.shape[1]] - rl[pos]).abs().max().item()
                    assert err <= tol, f"logits mismatch {err} at position {pos}"
                    n_checked += 1
                    break
    assert n_checked > 0


def test_tiny_qwen3_matches_reference():
    overrides = dict(num_hidden_layers=2, vocab_size=1000, hidden_size=256, intermediate_size=512,
                     num_attention_heads=4, num_key_value_heads=2, head_dim=64)
    eng, prompts, outs, ref, captured = _run("qwen3-0.6b", 3, 37, 12, chunk=32, overrides=overrides)
    _check(prompts, outs, ref, captured, 1e-4)


@pytest.mark.slow
def test_qwen3_0p6b_oracle_config1():
    """28 layers, hidden 1024, 16/8 heads at 128, vocab 151936, tied embeddings;
    4 requests x 128 prompt tokens, greedy 32 tokens, page size 16; logits within 1e-4."""
    eng, prompts, outs, ref, captured = _run("qwen3-0.6b", 4, 128, 32, chunk=256)
    assert all(len(o["output_ids"]) == 32 for o in outs)
    _check(prompts, outs, ref, captured, 1e-4)
