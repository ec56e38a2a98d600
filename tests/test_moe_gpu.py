"""Block-scaled grouped expert GEMM (tcgen05 kind::mxf8f6f4) against fp32 PyTorch references."""
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _rand_experts(E, H, I, fp4, bias, seed=0, interleaved=True):
    from sglang_neuron_b200.ops.moe import quant_mxfp4, quant_mxfp8_ref, ExpertWeights
    g = torch.Generator().manual_seed(seed)
    w13 = torch.randn(E, 2 * I, H, generator=g) * 0.05
    w2 = torch.randn(E, H, I, generator=g) * 0.05
    if fp4:
        b13, s13 = quant_mxfp4(w13)
        b2, s2 = quant_mxfp4(w2)
    else:
        b13, s13 = quant_mxfp8_ref(w13)
        b2, s2 = quant_mxfp8_ref(w2)
    bb13 = torch.randn(E, 2 * I, generator=g) * 0.1 if bias else None
    bb2 = torch.randn(E, H, generator=g) * 0.1 if bias else None
    to = lambda t: t.to(DEV) if t is not None else None  # noqa: E731
    return ExpertWeights(to(b13), to(s13), to(bb13), to(b2), to(s2), to(bb2), H, I, interleaved)


@pytest.mark.parametrize("T,E,H,I,fp4,act,bias", [
    (1, 16, 2880, 2880, True, "swiglu_clamp", True),
    (8, 16, 2880, 2880, True, "swiglu_clamp", True),
    (64, 32, 2880, 2880, True, "swiglu_clamp", True),
    (300, 8, 2880, 2880, True, "swiglu_clamp", True),
    (40, 16, 2048, 768, False, "silu", False),
    (500, 16, 2048, 768, False, "silu", False),
    (63, 32, 2880, 2880, True, "swiglu_clamp", True),
    (41, 16, 2048, 768, False, "silu", False),
    (301, 8, 2880, 2880, True, "swiglu_clamp", True),
])
def test_fused_moe(T, E, H, I, fp4, act, bias, monkeypatch):
    from sglang_neuron_b200.ops.moe import fused_moe, fused_moe_ref, topk_route
    # odd T: the gate/up epilogue writes MXFP8 directly (opt-in path); even T: separate quantise launch
    monkeypatch.setenv("SGLANG_B200_MOE_FUSED_ACT_QUANT", "1" if T % 2 else "0")
    from sglang_neuron_b200.ops.gemm import check_status
    torch.manual_seed(T)
    ew = _rand_experts(E, H, I, fp4, bias, seed=T, interleaved=fp4)
    x = (torch.randn(T, H, device=DEV) * 2).to(torch.bfloat16)
    logits = torch.randn(T, E, device=DEV)
    K = 4
    w, ids = topk_route(logits, K, 0)
    out = fused_moe(x, w, ids, ew, act)
    torch.cuda.synchronize()
    from sglang_neuron_b200.ops.moe import _status
    assert int(_status(x.device)[0]) == 0, "moe kernel reported a bounded-wait timeout"
    ref_q = fused_moe_ref(x, w, ids, ew, act, quant_act=True).float()
    ref = fused_moe_ref(x, w, ids, ew, act, quant_act=False).float()
    o = out.float()
    err_q = (o - ref_q).abs().max().item()
    scale = ref.abs().max().item()
    assert err_q <= 2e-2 * scale + 1e-2, f"vs activation-quantised reference: {err_q} (scale {scale})"
    rel = (o - ref).norm() / ref.norm()
    assert rel < 0.08, f"relative error vs unquantised fp32 reference {rel}"
