"""sglang_neuron_b200: a Blackwell-native (sm_100a) LLM serving framework with the capabilities of
sglang-neuron: paged KV pools, CUDA-graph model runtime, Qwen3 / Qwen3-MoE / DeepSeek-V2 / GPT-OSS model
families, MXFP4/FP8 quantisation, speculative decoding, tensor/expert parallelism over NVLink and
disaggregated prefill/decode.

`activate()` mirrors the reference's platform entry point (sglang_neuron/__init__.py:4-12): it returns the
platform class path when an sm_100 GPU is visible, else None so another platform can claim the process.
"""

__version__ = "0.1.0"


def activate():
    try:
        import torch
    except ImportError:  # pragma: no cover
        return None
    if not torch.cuda.is_available():
        return None
    major, _minor = torch.cuda.get_device_capability(0)
    if major != 10:
        return None
    return "sglang_neuron_b200.platform.B200SRTPlatform"
