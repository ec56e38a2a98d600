"""Serving benchmark client and report against a real HTTP server (uvicorn on a loopback port, CPU engine)."""
import asyncio
import socket
import threading
import time

import pytest

from sglang_neuron_b200.benchmarks import bench_report, bench_serving
from sglang_neuron_b200.configs import model_config as mc
from sglang_neuron_b200.engine import Engine
from sglang_neuron_b200.parallel.state import destroy_parallel
from sglang_neuron_b200.server_args import ServerArgs


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


@pytest.fixture(scope="module")
def server():
    pytest.importorskip("aiohttp")
    uvicorn = pytest.importorskip("uvicorn")
    from sglang_neuron_b200.entrypoints.http_server import build_app
    destroy_parallel()
    mc.PRESETS["bs-tiny"] = dict(mc.PRESETS["qwen3-0.6b"], num_hidden_layers=2, vocab_size=512, hidden_size=128,
                                 intermediate_size=256, num_attention_heads=4, num_key_value_heads=2, head_dim=32)
    eng = Engine(ServerArgs(model="bs-tiny", device="cpu", dtype="float32", context_length=256,
                            max_running_requests=8, chunked_prefill_size=64))
    holder = {}
    port = _free_port()
    srv = uvicorn.Server(uvicorn.Config(build_app(eng, holder), host="127.0.0.1", port=port, log_level="error"))
    th = threading.Thread(target=srv.run, daemon=True)
    th.start()
    for _ in range(200):
        if srv.started:
            break
        time.sleep(0.05)
    yield f"http://127.0.0.1:{port}"
    srv.should_exit = True
    th.join(timeout=10)
    if "loop" in holder:
        holder["loop"].shutdown()


def test_bench_serving_end_to_end(server, tmp_path):
    prompts = bench_serving.make_prompts(6, 12, 5, vocab=512, ratio=1.0, seed=3)
    res = asyncio.run(bench_serving.run_benchmark(server, prompts, concurrency=3))
    assert res["completed"] == 6 and res["failed"] == 0, res
    assert res["total_output_tokens"] == 30
    assert res["ttft_ms_p50"] is not None and res["output_tok_s"] > 0
    assert res["tpot_ms_p50"] is not None and res["itl_ms_p50"] is not None
    f = tmp_path / "runs.jsonl"
    out = bench_serving.main(["--base-url", server, "--num-prompts", "4", "--concurrency", "2", "--input-len", "8",
                              "--output-len", "3", "--vocab", "512", "--tag", "ours", "--output-file", str(f)])
    assert out["completed"] == 4
    table = bench_report.render(bench_report.load(str(f)), baseline=bench_report.load(str(f)))
    assert "| ours | 2 | 4 |" in table and "1.0" in table


def test_summary_statistics():
    R = bench_serving.RequestResult
    rs = [R(prompt_len=4, output_len=3, ttft=0.1, latency=0.3, itls=[0.1, 0.1]),
          R(prompt_len=4, output_len=5, ttft=0.2, latency=0.6, itls=[0.1] * 4),
          R(prompt_len=4, ok=False, error="x")]
    s = bench_serving.summarize(rs, duration=2.0, concurrency=2)
    assert s["completed"] == 2 and s["failed"] == 1 and s["total_output_tokens"] == 8
    assert s["output_tok_s"] == 4.0 and s["ttft_ms_p50"] == pytest.approx(150.0)
    assert s["tpot_ms_p50"] == pytest.approx(100.0) and s["itl_ms_p50"] == pytest.approx(100.0)


def test_parity_solo_vs_waves(server):
    from sglang_neuron_b200.benchmarks import parity
    res = parity.run(server, server, num=6, input_len=16, output_len=6, wave=3, vocab=512)
    assert res["a_solo_vs_a_wave"]["mismatched"] == 0, res
    assert res["a_wave_vs_b_wave"]["mismatched"] == 0, res
