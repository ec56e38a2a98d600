"""The allocation-free decode-attention entry point, called through its exported C symbol.

Callers of this symbol are the ones that cannot allocate device memory while they run (allocator callbacks,
fully pre-reserved runtimes, plain C/FFI hosts without a caching allocator). The test checks that it
matches the regular `decode_attention` op, which takes caller-provided scratch, on two calls in a row (the
second call reuses the library-resident scratch the first call left behind).

This file is named so that pytest collects it last.
"""
import ctypes
import os
import re

import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "sglang_neuron_b200")
HEADER = os.path.join(ROOT, "csrc", "snb_noalloc.h")

# C parameter type in the header -> ctypes type used for the call
_CTYPES = {"void*": ctypes.c_void_p, "const void*": ctypes.c_void_p, "const int32_t*": ctypes.c_void_p,
           "const float*": ctypes.c_void_p, "cudaStream_t": ctypes.c_void_p, "int": ctypes.c_int,
           "float": ctypes.c_float}


def _header_argtypes():
    """ctypes argument types read from the prototype in csrc/snb_noalloc.h, so the call below cannot drift
    from the declared signature."""
    text = open(HEADER).read()
    m = re.search(r"int snb_decode_attention_noalloc\(([^)]*)\);", text)
    assert m, "prototype not found in the header"
    types = []
    for p in m.group(1).split(","):
        p = " ".join(p.split())
        t = p.rsplit(" ", 1)[0].replace(" *", "*")
        types.append(_CTYPES[t])
    return types


def _lib():
    import sglang_neuron_b200._C as ext  # loads the library (and its device array) into this process
    lib = ctypes.CDLL(ext.__file__)
    fn = lib.snb_decode_attention_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = _header_argtypes()
    cap = lib.snb_decode_attention_noalloc_scratch_capacity
    cap.restype = ctypes.c_longlong
    return fn, cap()


def _case(seed, B, Hq, Hkv, D, P, fp8, window, with_sinks, short=False):
    g = torch.Generator().manual_seed(seed)
    ctx = torch.randint(1, 700, (B,), generator=g)
    if short:  # empty contexts and contexts shorter than the split count: splits with no keys (lse = -inf)
        ctx[0] = 0
        ctx[1:3] = torch.tensor([1, 3])
    max_pages = int((ctx.max() + P - 1) // P) + 1
    n_pages = B * max_pages + 2
    perm = torch.randperm(n_pages, generator=g)
    bt = perm[: B * max_pages].view(B, max_pages).to(torch.int32)
    dt = torch.float8_e4m3fn if fp8 else torch.bfloat16
    kc = (torch.randn(n_pages, Hkv, P, D, generator=g) * 0.7).to(dt)
    vc = torch.randn(n_pages, Hkv, P, D, generator=g).to(dt)
    q = torch.randn(B, Hq * D, generator=g).to(torch.bfloat16)
    sinks = torch.randn(Hq, generator=g) if with_sinks else None
    dev = "cuda"
    return (q.to(dev), kc.to(dev), vc.to(dev), bt.to(dev), ctx.to(torch.int32).to(dev),
            sinks.to(dev) if sinks is not None else None)


@pytest.mark.parametrize("fp8,window,with_sinks,D,Hq,Hkv", [(True, 0, True, 64, 64, 8), (False, 128, True, 64, 64, 8),
                                                           (False, 0, False, 128, 32, 8)])
def test_noalloc_matches_decode_attention_two_calls(fp8, window, with_sinks, D, Hq, Hkv):
    from sglang_neuron_b200.ops.attention import decode_attention
    fn, capacity = _lib()
    P, S = 16, 4
    ks, vs = (0.9, 1.1) if fp8 else (1.0, 1.0)
    scale = D ** -0.5
    from sglang_neuron_b200.ops.attention import decode_attention_ref
    for call in range(2):
        B = 6 if call == 0 else 9
        q, kc, vc, bt, seq, sinks = _case(100 + call, B, Hq, Hkv, D, P, fp8, window, with_sinks, short=call == 1)
        assert B * Hq * S * (D + 1) <= capacity
        ref = decode_attention(q, kc, vc, bt, seq, Hq, Hkv, D, P, window, scale, ks, vs, sinks, num_splits=S)
        out = torch.full_like(ref, float("nan"))
        stream = torch.cuda.current_stream().cuda_stream
        rc = fn(out.data_ptr(), out.stride(0), q.data_ptr(), q.stride(0), kc.data_ptr(), vc.data_ptr(), int(fp8),
                bt.data_ptr(), bt.stride(0), seq.data_ptr(), B, Hq, Hkv, D, P, window, scale, ks, vs,
                sinks.data_ptr() if sinks is not None else None, S, stream)
        torch.cuda.synchronize()
        assert rc == 0, f"entry point returned {rc}"
        err = (out.float() - ref.float()).abs().max().item()
        tol = 2e-2 + 2e-2 * ref.float().abs().max().item()
        assert err <= tol, f"call {call}: max err {err} > {tol}"
        # the fp32 PyTorch reference on CPU copies, so a fault shared by both kernels cannot pass
        cpu = decode_attention_ref(q.cpu(), kc.cpu(), vc.cpu(), bt.cpu(), seq.cpu(), Hq, Hkv, D, P, window, scale,
                                   ks, vs, sinks.cpu() if sinks is not None else None)
        err = (out.float().cpu() - cpu).abs().max().item()
        tol = 2e-2 + 2e-2 * cpu.abs().max().item()
        assert err <= tol, f"call {call}: max err vs fp32 reference {err} > {tol}"


def test_noalloc_rejects_oversized_request():
    fn, capacity = _lib()
    q, kc, vc, bt, seq, _ = _case(7, 2, 8, 1, 64, 16, False, 0, False)
    out = torch.empty_like(q)
    huge_splits = capacity // (2 * 8 * 65) + 1
    rc = fn(out.data_ptr(), out.stride(0), q.data_ptr(), q.stride(0), kc.data_ptr(), vc.data_ptr(), 0, bt.data_ptr(),
            bt.stride(0), seq.data_ptr(), 2, 8, 1, 64, 16, 0, 0.125, 1.0, 1.0, None, huge_splits,
            torch.cuda.current_stream().cuda_stream)
    assert rc == -2
