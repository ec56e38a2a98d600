"""Request balancer on loopback: two CPU engine servers and one dead address behind one endpoint; requests
spread over the live replicas, a connection failure moves a request to the next replica, streaming passes
through, and greedy outputs equal the replicas' own."""
import asyncio
import socket
import threading
import time

import pytest

from sglang_neuron_b200.configs import model_config as mc
from sglang_neuron_b200.engine import Engine
from sglang_neuron_b200.parallel.state import destroy_parallel
from sglang_neuron_b200.server_args import ServerArgs


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _serve(app, port):
    import uvicorn
    srv = uvicorn.Server(uvicorn.Config(app, host="127.0.0.1", port=port, log_level="error"))
    th = threading.Thread(target=srv.run, daemon=True)
    th.start()
    for _ in range(200):
        if srv.started:
            break
        time.sleep(0.05)
    return srv, th


@pytest.fixture(scope="module")
def cluster():
    pytest.importorskip("aiohttp")
    pytest.importorskip("uvicorn")
    from sglang_neuron_b200.disaggregation.balancer import build_app as build_balancer
    from sglang_neuron_b200.entrypoints.http_server import build_app
    mc.PRESETS["lb-tiny"] = dict(mc.PRESETS["qwen3-0.6b"], num_hidden_layers=2, vocab_size=512, hidden_size=128,
                                 intermediate_size=256, num_attention_heads=4, num_key_value_heads=2, head_dim=32)
    servers, holders, urls = [], [], []
    for _ in range(2):
        destroy_parallel()
        eng = Engine(ServerArgs(model="lb-tiny", device="cpu", dtype="float32", context_length=256,
                                max_running_requests=8, chunked_prefill_size=64))
        h = {}
        port = _port()
        servers.append(_serve(build_app(eng, h), port))
        holders.append(h)
        urls.append(f"http://127.0.0.1:{port}")
    dead = f"http://127.0.0.1:{_port()}"  # nothing listens here
    lb_port = _port()
    app = build_balancer([dead] + urls, retries=2)
    servers.append(_serve(app, lb_port))
    yield f"http://127.0.0.1:{lb_port}", urls, app
    for srv, th in servers:
        srv.should_exit = True
        th.join(timeout=10)
    for h in holders:
        if "loop" in h:
            h["loop"].shutdown()


def test_balancer_spreads_retries_and_streams(cluster):
    from sglang_neuron_b200.benchmarks import bench_serving
    lb, urls, app = cluster
    prompts = bench_serving.make_prompts(8, 10, 4, vocab=512, ratio=1.0, seed=2)
    res = asyncio.run(bench_serving.run_benchmark(lb, prompts, concurrency=4))  # streaming requests
    assert res["completed"] == 8 and res["failed"] == 0, res.get("first_error")
    info = app.state.backends.info()
    live = [info[u]["served"] for u in urls]
    assert sum(live) == 8 and min(live) > 0, info
    assert sum(v["failed"] for v in info.values()) >= 1, info  # the dead address was tried and skipped
    assert all(v["outstanding"] == 0 for v in info.values())


def test_balancer_blocking_generate_matches_backend(cluster):
    import aiohttp
    lb, urls, _ = cluster

    async def go():
        body = {"input_ids": [5, 6, 7, 8], "sampling_params": {"max_new_tokens": 5}}
        async with aiohttp.ClientSession() as s:
            async with s.post(lb + "/generate", json=body) as r:
                a = (await r.json())["output_ids"]
            async with s.post(urls[0] + "/generate", json=body) as r:
                b = (await r.json())["output_ids"]
        return a, b
    a, b = asyncio.run(go())
    assert a == b and len(a) == 5
