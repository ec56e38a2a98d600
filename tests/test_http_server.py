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


def test_abort_n_and_stop_rules(client):
    """/abort_request ends a running request with finish_reason 'abort'; OpenAI n>1 returns n choices with
    distinct seeds; text stop sequences need a tokenizer (400 without one)."""
    import threading
    c, eng = client
    res = {}

    def long_req():
        res["r"] = c.post("/generate", json={"input_ids": [3, 4, 5], "rid": "abort-me",
                                             "sampling_params": {"max_new_tokens": 200, "ignore_eos": True}}).json()
    th = threading.Thread(target=long_req)
    th.start()
    import time
    time.sleep(0.3)
    assert c.post("/abort_request", json={"rid": "abort-me"}).json()["success"]
    th.join(timeout=60)
    assert res["r"]["meta_info"]["finish_reason"] == "abort"
    assert len(res["r"]["output_ids"]) < 200
    r = c.post("/v1/completions", json={"prompt": [1, 2, 3], "max_tokens": 4, "temperature": 1.0, "seed": 5,
                                        "n": 3}).json()
    assert [ch["index"] for ch in r["choices"]] == [0, 1, 2]
    assert r["usage"]["completion_tokens"] == 12
    assert c.post("/generate", json={"input_ids": [1, 2], "sampling_params": {"stop": ["x"]}}).status_code == 400


def test_trim_at_stop():
    from sglang_neuron_b200.engine import trim_at_stop
    assert trim_at_stop("hello world. bye", ["."]) == "hello world"
    assert trim_at_stop("abc", ["z", "bc"]) == "a"
    assert trim_at_stop("abc", None) == "abc"


def test_text_stop_sequences_with_a_tokenizer():
    """Generation stops at the first step whose decoded tail contains a stop sequence; the text is cut before
    it (a character-per-token stand-in tokenizer)."""
    from sglang_neuron_b200.parallel.state import destroy_parallel as _dp

    class CharTok:
        def decode(self, ids):
            return "".join(chr(97 + int(t) % 26) for t in ids)

        def encode(self, text):
            return [ord(ch) - 97 for ch in text]

    _dp()
    eng = Engine(ServerArgs(model="http-tiny", device="cpu", dtype="float32", context_length=256,
                            max_running_requests=4, chunked_prefill_size=64))
    free = eng.generate([[1, 2, 3, 4]], {"max_new_tokens": 12, "ignore_eos": True})[0]["output_ids"]
    eng.tokenizer = CharTok()
    eng.scheduler.stop_checker = eng._stop_hit
    stop = CharTok().decode(free[4:6])  # a sequence the greedy run produces at tokens 4-5
    out = eng.generate([[1, 2, 3, 4]], {"max_new_tokens": 12, "ignore_eos": True, "stop": [stop]})[0]
    assert out["finish_reason"] == "stop"
    assert out["output_ids"] == free[:len(out["output_ids"])] and len(out["output_ids"]) <= 6
    assert stop not in out["text"] and out["text"] == CharTok().decode(free)[: CharTok().decode(free).find(stop)]
