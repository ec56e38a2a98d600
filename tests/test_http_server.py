"""HTTP server on the CPU tier: /generate (blocking and streaming), /v1/completions, info routes, /metrics."""
import json

import pytest

from sglang_neuron_b200.configs import model_config as mc
from sglang_neuron_b200.engine import Engine
from sglang_neuron_b200.parallel.state import destroy_parallel
from sglang_neuron_b200.server_args import ServerArgs


@pytest.fixture(scope="module")
def client():
    fastapi = pytest.importorskip("fastapi")
    from fastapi.testclient import TestClient
    from sglang_neuron_b200.entrypoints.http_server import build_app
    destroy_parallel()
    mc.PRESETS["http-tiny"] = dict(mc.PRESETS["qwen3-0.6b"], num_hidden_layers=2, vocab_size=512, hidden_size=128,
                                   intermediate_size=256, num_attention_heads=4, num_key_value_heads=2, head_dim=32)
    eng = Engine(ServerArgs(model="http-tiny", device="cpu", dtype="float32", context_length=256,
                            max_running_requests=8, chunked_prefill_size=64))
    holder = {}
    with TestClient(build_app(eng, holder)) as c:
        yield c, eng
    if "loop" in holder:
        holder["loop"].shutdown()


def test_generate_and_openai(client):
    c, eng = client
    assert c.get("/health").text == "ok"
    r = c.post("/generate", json={"input_ids": [1, 2, 3, 4, 5], "sampling_params": {"max_new_tokens": 6}})
    assert r.status_code == 200, r.text
    out = r.json()
    assert len(out["output_ids"]) == 6 and out["meta_info"]["finish_reason"] == "length"
    # identical greedy request through the offline engine API gives the same tokens
    r2 = c.post("/v1/completions", json={"prompt": [1, 2, 3, 4, 5], "max_tokens": 6, "temperature": 0})
    assert r2.status_code == 200, r2.text
    assert r2.json()["choices"][0]["token_ids"] == out["output_ids"]
    assert r2.json()["usage"]["completion_tokens"] == 6


def test_streaming_and_info(client):
    c, eng = client
    with c.stream("POST", "/generate", json={"input_ids": [7, 8, 9], "sampling_params": {"max_new_tokens": 4},
                                             "stream": True}) as r:
        chunks = [l for l in r.iter_lines() if l.startswith("data: ")]
    assert chunks[-1] == "data: [DONE]"
    last = json.loads(chunks[-2][6:])
    assert len(last["output_ids"]) == 4
    info = c.get("/get_model_info").json()
    assert info["architecture"] == "Qwen3ForCausalLM"
    m = c.get("/metrics").text
    assert "snb_generated_tokens_total" in m
    assert c.post("/generate", json={"text": "hello"}).status_code == 400  # no tokenizer: ids only
