"""Token log-probabilities on the CPU tier: the engine's logprob of each greedy token and its top-k equal
log_softmax of the oracle logits; the vocabulary-sharded merge (TP=2, gloo) gives the same numbers; the
HTTP /generate and /v1/completions routes return them in SGLang / OpenAI shapes."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from sglang_neuron_b200.configs import model_config as mc
from sglang_neuron_b200.engine import Engine
from sglang_neuron_b200.parallel.state import destroy_parallel
from sglang_neuron_b200.server_args import ServerArgs

TINY = dict(num_hidden_layers=2, vocab_size=1000, hidden_size=128, intermediate_size=256,
            num_attention_heads=4, num_key_value_heads=2, head_dim=32)


def _args(**kw):
    mc.PRESETS["lp-tiny"] = dict(mc.PRESETS["qwen3-0.6b"], **TINY)
    base = dict(model="lp-tiny", device="cpu", dtype="float32", context_length=256, max_running_requests=4,
                chunked_prefill_size=64, random_weight_std=0.05)
    base.update(kw)
    return ServerArgs(**base)


def _prompts():
    g = torch.Generator().manual_seed(4)
    return [torch.randint(1, 1000, (n,), generator=g).tolist() for n in (9, 30)]


def test_logprobs_match_log_softmax():
    destroy_parallel()
    eng = Engine(_args())
    rows = []
    eng.runner.logits_hook = lambda fb, lg: rows.append(lg[:, :1000].float().clone())
    outs = eng.generate(_prompts(), {"max_new_tokens": 4, "return_logprob": True, "top_logprobs_num": 3})
    # rebuild per-request logits in output order from the hooked steps
    lps = torch.log_softmax(torch.cat(rows, 0), dim=-1)
    for o in outs:
        assert len(o["output_token_logprobs"]) == 4 and len(o["output_top_logprobs"]) == 4
        for (lp, tok), top in zip(o["output_token_logprobs"], o["output_top_logprobs"]):
            # greedy: the chosen token is the top-1 and its logprob the largest of the row it came from
            assert top[0][1] == tok and abs(top[0][0] - lp) < 1e-5
            match = (lps.max(dim=-1).values - lp).abs().min().item()
            assert match < 1e-4
            assert top[0][0] >= top[1][0] >= top[2][0]


def _tp_run(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), WORLD_SIZE=str(world), RANK=str(rank),
                      LOCAL_RANK=str(rank))
    destroy_parallel()
    eng = Engine(_args(tp_size=world))
    outs = eng.generate(_prompts(), {"max_new_tokens": 4, "return_logprob": True, "top_logprobs_num": 2})
    q.put((rank, [(o["output_token_logprobs"], o["output_top_logprobs"]) for o in outs]))
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()


def _launch(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    ps = [ctx.Process(target=_tp_run, args=(r, world, port, q)) for r in range(world)]
    for p in ps:
        p.start()
    res = dict(q.get(timeout=300) for _ in ps)
    for p in ps:
        p.join(timeout=60)
    return res


def test_sharded_logprobs_equal_tp1():
    one = _launch(1)[0]
    two = _launch(2)
    for (lp1, top1), (lp2, top2) in zip(one, two[0]):
        assert [t for _, t in lp1] == [t for _, t in lp2]
        assert max(abs(a[0] - b[0]) for a, b in zip(lp1, lp2)) < 1e-4
        assert [[t for _, t in row] for row in top1] == [[t for _, t in row] for row in top2]
    assert two[0] == two[1]


def test_http_logprob_shapes():
    pytest.importorskip("fastapi")
    from fastapi.testclient import TestClient
    from sglang_neuron_b200.entrypoints.http_server import build_app
    destroy_parallel()
    eng = Engine(_args())
    holder = {}
    with TestClient(build_app(eng, holder)) as c:
        r = c.post("/generate", json={"input_ids": [1, 2, 3], "sampling_params": {"max_new_tokens": 3},
                                      "return_logprob": True, "top_logprobs_num": 2}).json()
        m = r["meta_info"]
        assert len(m["output_token_logprobs"]) == 3 and m["output_token_logprobs"][0][1] == r["output_ids"][0]
        assert len(m["output_top_logprobs"][0]) == 2
        r2 = c.post("/v1/completions", json={"prompt": [1, 2, 3], "max_tokens": 3, "temperature": 0,
                                             "logprobs": 2}).json()
        lp = r2["choices"][0]["logprobs"]
        assert len(lp["token_logprobs"]) == 3 and len(lp["top_logprobs"][0]) == 2
        assert abs(lp["token_logprobs"][0] - m["output_token_logprobs"][0][0]) < 1e-5
    if "loop" in holder:
        holder["loop"].shutdown()
