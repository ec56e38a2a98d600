"""One tiny decode of the flagship family (GPT-OSS shape, scaled down) on a CUDA device through the public
Engine API: random-init MXFP4 experts, FP8 KV, CUDA-graph decode."""
import torch

from .configs import model_config as mc
from .engine import Engine
from .parallel.state import destroy_parallel
from .server_args import ServerArgs

SMOKE = dict(num_hidden_layers=2, vocab_size=4096, hidden_size=512, intermediate_size=256, num_local_experts=8,
             num_attention_heads=8, num_key_value_heads=2, head_dim=64, sliding_window=16)


def run_smoke(device: str = "cuda:0") -> dict:
    destroy_parallel()
    mc.PRESETS["gpt-oss-smoke"] = dict(mc.PRESETS["gpt-oss-120b"], **SMOKE)
    if device.startswith("cuda"):
        torch.cuda.set_device(torch.device(device))
    args = ServerArgs(model="gpt-oss-smoke", device="cuda" if device.startswith("cuda") else "cpu",
                      page_size=16, context_length=256, max_running_requests=4, chunked_prefill_size=64,
                      cuda_graph_bs=[1, 2, 4], kv_cache_dtype="fp8_e4m3")
    eng = Engine(args)
    out = eng.generate([[1, 2, 3, 4, 5, 6, 7], list(range(100, 140))], {"max_new_tokens": 6})
    assert all(len(o["output_ids"]) == 6 for o in out), out
    eng.shutdown()
    return {"outputs": [o["output_ids"] for o in out]}


if __name__ == "__main__":
    print(run_smoke())
