"""Kernel microbenchmarks with roofline fractions (CUDA-event timed, warm, L2 flushed between iterations).

    python -m sglang_neuron_b200.benchmarks.kernels moe --tokens 64        # one GPT-OSS-120B MoE layer
    python -m sglang_neuron_b200.benchmarks.kernels moe_stages --tokens 1087 --ep 8   # per-stage, one EP rank
    python -m sglang_neuron_b200.benchmarks.kernels gemm --tokens 64 --n 5120 --k 2880
    python -m sglang_neuron_b200.benchmarks.kernels attn --batch 64 --ctx 1536
    python -m sglang_neuron_b200.benchmarks.kernels mla --batch 32 --ctx 4096       # DeepSeek-V2-Lite MLA

Peaks come from MEASURED_PEAKS.json at the repository root when present (hbm_gbs, bf16_tflops), else the
pool's fallback figures (6650 GB/s, 1590 TFLOP/s). Pass --iters 1 --warmup 1 for a profiler capture.
"""
from __future__ import annotations

import argparse
import json
import os

import torch

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, "fallback"


_flush = None


def flush_l2():
    global _flush
    if _flush is None:
        _flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    _flush.zero_()


def timeit(fn, iters: int, warmup: int) -> float:
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    tot = 0.0
    for _ in range(iters):
        flush_l2()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        fn()
        e.record()
        torch.cuda.synchronize()
        tot += s.elapsed_time(e)
    return tot / iters * 1e3  # us


def graph_time(fns, reps: int = 5) -> float:
    """Per-launch device time (us) of the callables `fns` run back to back inside one CUDA graph: no host
    launch overhead between kernels, programmatic dependent launch overlap included, as in the engine's
    decode graphs. Callers cycle over buffers larger than L2 so every launch reads from DRAM."""
    for f in fns:  # warm-up (lazy init, tensor maps)
        f()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for f in fns:
            f()
    g.replay()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(reps):
        g.replay()
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e) * 1e3 / (reps * len(fns))


def bench_moe(a):
    from ..ops import moe
    E, H, I, K = a.experts, 2880, 2880, 4
    g = torch.Generator(device="cuda").manual_seed(0)
    w13 = torch.randint(0, 256, (E, 2 * I, H // 2), device="cuda", dtype=torch.uint8, generator=g)
    s13 = torch.randint(119, 122, (E, 2 * I, H // 32), device="cuda", dtype=torch.uint8, generator=g)
    w2 = torch.randint(0, 256, (E, H, I // 2), device="cuda", dtype=torch.uint8, generator=g)
    s2 = torch.randint(119, 122, (E, H, I // 32), device="cuda", dtype=torch.uint8, generator=g)
    b13 = torch.zeros(E, 2 * I, device="cuda", dtype=torch.bfloat16)
    b2 = torch.zeros(E, H, device="cuda", dtype=torch.bfloat16)
    ew = moe.ExpertWeights(w13, s13, b13, w2, s2, b2, H, I, True)
    T = a.tokens
    x = torch.randn(T, H, device="cuda").to(torch.bfloat16)
    w, ids = moe.topk_route(torch.randn(T, E, device="cuda"), K)
    n_active = int(torch.unique(ids).numel())
    fn = lambda: moe.fused_moe(x, w, ids, ew)  # noqa: E731
    us = timeit(fn, a.iters, a.warmup)
    if a.iters > 1:  # in a CUDA graph, back to back (each call streams > L2 of expert weights)
        us = graph_time([fn] * 4)
    bytes_w = n_active * (ew.w13[0].numel() + ew.w2[0].numel() + ew.sfa13[0].numel() + ew.sfa2[0].numel())
    flops = 2 * T * K * (2 * I * H + H * I)
    hbm, tf, src = peaks()
    ach = bytes_w / (us * 1e-6) / 1e9
    print(json.dumps({"kernel": "fused_moe (route+align+quant+2x tcgen05 mxf8f6f4 grouped GEMM+combine)",
                      "tokens": T, "experts": E, "active_experts": n_active, "us": round(us, 2),
                      "weight_GBps": round(ach, 1), f"hbm_frac_of_{src}": round(ach / hbm, 3),
                      "tflops": round(flops / (us * 1e-6) / 1e12, 2)}))


def bench_moe_stages(a):
    """Per-stage device time of one MoE layer (routing, alignment, MXFP8 quantise, gate/up GEMM, activation
    quantise, down GEMM, combine), each timed alone (PDL off, L2 flushed). --ep N keeps 1/N of the experts
    local, as one rank of EP N sees them."""
    from .._ext import kernels
    from ..ops import moe
    kernels().set_pdl(False)
    E, H, I, K = a.experts, 2880, 2880, 4
    El = E // a.ep
    g = torch.Generator(device="cuda").manual_seed(0)
    w13 = torch.randint(0, 256, (El, 2 * I, H // 2), device="cuda", dtype=torch.uint8, generator=g)
    s13 = torch.randint(119, 122, (El, 2 * I, H // 32), device="cuda", dtype=torch.uint8, generator=g)
    w2 = torch.randint(0, 256, (El, H, I // 2), device="cuda", dtype=torch.uint8, generator=g)
    s2 = torch.randint(119, 122, (El, H, I // 32), device="cuda", dtype=torch.uint8, generator=g)
    ew = moe.ExpertWeights(w13, s13, torch.zeros(El, 2 * I, device="cuda", dtype=torch.bfloat16), w2, s2,
                           torch.zeros(El, H, device="cuda", dtype=torch.bfloat16), H, I, True)
    T = a.tokens
    x = torch.randn(T, H, device="cuda").to(torch.bfloat16)
    logits = torch.randn(T, E, device="cuda")
    w, ids = moe.topk_route(logits, K)
    bn = a.bn or moe.pick_bn(T, K, El)
    al = moe.MoEAlignment(T * K, El, bn, "cuda")
    moe.moe_align(ids, 0, El, al)
    R = al.r_max
    used = al.seg_offsets[El:El + 1]
    xq, sfb = moe.gather_quant_mxfp8(x, al.sorted_src, R, bn, used=used)
    act = torch.empty(R, I, dtype=torch.bfloat16, device="cuda")
    y = torch.empty(R, H, dtype=torch.bfloat16, device="cuda")
    out = torch.empty(T, H, dtype=torch.bfloat16, device="cuda")
    st = {
        "route": lambda: moe.topk_route(logits, K),
        "align": lambda: moe.moe_align(ids, 0, El, al),
        "quant_x_all_rows": lambda: moe.gather_quant_mxfp8(x, al.sorted_src, R, bn),
        "quant_x": lambda: moe.gather_quant_mxfp8(x, al.sorted_src, R, bn, used=used),
        "gate_up": lambda: moe.moe_gemm(act, xq, sfb, ew.w13, ew.sfa13, ew.b13, al, moe.EPI_SWIGLU_CLAMP, 2 * I),
        "quant_act": lambda: moe.gather_quant_mxfp8(act, None, R, bn, used=used),
        "down": lambda: moe.moe_gemm(y, xq[:, :I] if I == H else xq, sfb, ew.w2, ew.sfa2, ew.b2, al, moe.EPI_BIAS, H),
        "combine": lambda: moe.moe_combine(out, y, al.inv_map, w),
    }
    res = {"tokens": T, "experts_local": El, "bn": bn, "rows_capacity": R, "rows_used": int(used.item())}
    only = set(a.only.split(",")) if a.only else None
    for k, f in st.items():
        if only is None or k in only:
            res[k + "_us"] = round(timeit(f, a.iters, a.warmup), 2)
    if only is not None:
        kernels().set_pdl(True)
        print(json.dumps(res))
        return
    res["fused_moe_us"] = round(timeit(lambda: moe.fused_moe(x, w, ids, ew, al=al, bn=bn), a.iters, a.warmup), 2)
    kernels().set_pdl(True)
    print(json.dumps(res))


def bench_route(a):
    """The one-launch MoE routing kernel against router GEMM + top-k + align + quantise (four launches)."""
    from ..ops import moe
    from ..ops.gemm import TiledWeight, linear
    T, E, H, K = a.tokens, a.experts, 2880, 4
    El = E // a.ep
    x = torch.randn(T, H, device="cuda").to(torch.bfloat16)
    wr = TiledWeight((torch.randn(E, H, device="cuda") * 0.02).to(torch.bfloat16))
    bias = torch.zeros(E, device="cuda", dtype=torch.bfloat16)
    bn = moe.pick_bn(T, K, El)
    al = moe.MoEAlignment(T * K, El, bn, "cuda")

    def sep():
        w, ids = moe.topk_route(linear(x, wr, bias), K)
        moe.moe_align(ids, 0, El, al)
        moe.gather_quant_mxfp8(x, al.sorted_src, al.r_max, bn, used=al.seg_offsets[El:El + 1])

    fused = lambda: moe.fused_route_quant(x, wr, E, bias, K, 0, 1.0, 0, El, bn)  # noqa: E731
    res = {"tokens": T, "experts": E, "experts_local": El,
           "fused_us": round(timeit(fused, a.iters, a.warmup), 2), "separate_us": round(timeit(sep, a.iters, a.warmup), 2)}
    if a.iters > 1:
        res["fused_in_graph_us"] = round(graph_time([fused] * 8), 2)
        res["separate_in_graph_us"] = round(graph_time([sep] * 8), 2)
    print(json.dumps(res))


def bench_gemm(a):
    from ..ops.gemm import linear
    T, N, K = a.tokens, a.n, a.k
    x = torch.randn(T, K, device="cuda").to(torch.bfloat16)
    w = (torch.randn(N, K, device="cuda") * 0.02).to(torch.bfloat16)
    from ..ops.gemm import TiledWeight, pick_splits
    wt = TiledWeight(w)  # the engine's layout: contiguous 128 x 64 weight tiles
    us = timeit(lambda: linear(x, wt), a.iters, a.warmup)
    res = {"kernel": "gemm_bf16 (tcgen05 kind::f16, tiled weights; K split across a cluster, DSMEM reduce)",
           "T": T, "N": N, "K": K, "us_single_cold": round(us, 2)}
    if a.iters > 1:
        res["us_row_major_weights"] = round(timeit(lambda: linear(x, w), a.iters, a.warmup), 2)
        # back-to-back launches in a CUDA graph over distinct weight copies (> 512 MB in total, > L2)
        n = max(2, min(64, (512 << 20) // (N * K * 2) + 1))
        ws = [TiledWeight((torch.randn(N, K, device="cuda") * 0.02).to(torch.bfloat16)) for _ in range(n)]
        outs = [torch.empty(T, N, device="cuda", dtype=torch.bfloat16) for _ in range(2)]
        us = graph_time([lambda i=i: linear(x, ws[i], out=outs[i % 2]) for i in range(n)])
        res["us_in_graph"] = round(us, 2)
        res["copies"] = n
        # cuBLAS on the same shapes (row-major weights, the plain library GEMM), for comparison
        wr = [w.untiled().contiguous() for w in ws]
        res["us_cublas_in_graph"] = round(graph_time([lambda i=i: torch.matmul(x, wr[i].t(), out=outs[i % 2])
                                                      for i in range(n)]), 2)
        del wr
    if a.iters > 1:  # grid-per-tile kernel with split-K partials + reduce launch, for comparison
        sp = pick_splits(T, N, K, torch.cuda.get_device_properties(0).multi_processor_count)
        res["us_grid_splitk"] = round(timeit(lambda: linear(x, w, splits=sp), a.iters, a.warmup), 2)
        res["splits"] = sp
    hbm, tf, src = peaks()
    byt = (N * K + T * K + T * N) * 2
    fl = 2 * T * N * K
    res[f"hbm_frac_of_{src}"] = round(byt / (us * 1e-6) / 1e9 / hbm, 3)
    res[f"tensor_frac_of_{src}"] = round(fl / (us * 1e-6) / 1e12 / tf, 3)
    print(json.dumps(res))


def bench_attn(a):
    from ..ops.attention import DecodeScratch, decode_attention, default_num_splits
    B, L, P, Hq, Hkv, D = a.batch, a.ctx, a.page, a.hq, a.hkv, a.head_dim
    kv_dt = torch.bfloat16 if a.kv == "bf16" else torch.float8_e4m3fn
    pages_per = (L + P - 1) // P
    n_pages = B * pages_per + 1
    kc = torch.randn(n_pages, Hkv, P, D, device="cuda").to(kv_dt)
    vc = torch.randn(n_pages, Hkv, P, D, device="cuda").to(kv_dt)
    bt = (torch.arange(B * pages_per, device="cuda", dtype=torch.int32) + 1).view(B, pages_per)
    seq = torch.full((B,), L, device="cuda", dtype=torch.int32)
    q = torch.randn(B, Hq * D, device="cuda").to(torch.bfloat16)
    sinks = torch.randn(Hq, device="cuda")
    S = a.splits or default_num_splits(B, Hkv, L)
    sc = DecodeScratch(B, Hq, D, S, "cuda")
    from .._ext import kernels
    kernels().set_decode_fp8_variant(a.variant)
    us = timeit(lambda: decode_attention(q, kc, vc, bt, seq, Hq, Hkv, D, P, 0, None, 1.0, 1.0, sinks, S, sc),
                a.iters, a.warmup)
    res = {"kernel": f"decode_attention (paged GQA, {a.kv} KV, sinks)", "batch": B, "ctx": L, "splits": S,
           "head_dim": D,
           "heads": f"{Hq}/{Hkv}", "page": P,
           "variant": ["head-major", "token-major bulk", "token-major cp.async"][a.variant],
           "us_single_cold": round(us, 2)}
    if a.iters > 1:  # back to back in a CUDA graph over KV copies that together exceed L2
        n = max(2, (512 << 20) // (2 * kc.numel()) + 1)
        kvs = [(torch.randn_like(kc, dtype=torch.float32).to(kc.dtype), torch.randn_like(vc, dtype=torch.float32)
                .to(vc.dtype)) for _ in range(n)]
        us = graph_time([lambda i=i: decode_attention(q, kvs[i][0], kvs[i][1], bt, seq, Hq, Hkv, D, P, 0, None, 1.0,
                                                      1.0, sinks, S, sc) for i in range(n)])
        res["us_in_graph"] = round(us, 2)
    hbm, tf, src = peaks()
    byt = B * L * Hkv * D * 2 * kc.element_size()
    res[f"hbm_frac_of_{src}"] = round(byt / (us * 1e-6) / 1e9 / hbm, 3)
    print(json.dumps(res))


def bench_mla(a):
    """Absorbed-MLA kernels at DeepSeek-V2-Lite shape (16 heads, 576-wide latent rows, 16-token pages): one
    prompt of --ctx tokens prefilled (extend), and a decode batch of --batch requests at --ctx tokens."""
    from ..ops.mla import mla_decode, mla_extend
    H, P, L = a.mla_heads, a.page, a.ctx
    scale = 1.0 / (192 ** 0.5)
    pages = (L + P - 1) // P
    res = {"kernel": "mla (absorbed, bf16 latent pool)", "heads": H, "ctx": L, "page": P}
    # extend: one request, the whole prompt in one chunk
    cache = (torch.randn(pages + 1, 1, P, 576, device="cuda") * 0.5).to(torch.bfloat16)
    bt = torch.arange(1, pages + 1, device="cuda", dtype=torch.int32).view(1, pages)
    q = (torch.randn(L, H, 576, device="cuda") * 0.5).to(torch.bfloat16)
    lens = torch.tensor([L], dtype=torch.int32, device="cuda")
    qo = torch.tensor([0, L], dtype=torch.int32, device="cuda")
    us = timeit(lambda: mla_extend(q, cache, bt, lens, qo, L, P, scale), a.iters, a.warmup)
    flops = 2.0 * H * (576 + 512) * L * (L + 1) / 2
    _, tf, src = peaks()
    res.update({"extend_us": round(us, 1), "extend_tflops": round(flops / us / 1e6, 1),
                f"extend_frac_of_{src}_bf16": round(flops / us / 1e6 / tf, 3)})
    # decode: batch B at context L
    B = a.batch
    cache = (torch.randn(B * pages + 1, 1, P, 576, device="cuda") * 0.5).to(torch.bfloat16)
    bt = (torch.arange(B * pages, device="cuda", dtype=torch.int32) + 1).view(B, pages)
    q = (torch.randn(B, H, 576, device="cuda") * 0.5).to(torch.bfloat16)
    seq = torch.full((B,), L, dtype=torch.int32, device="cuda")
    S = a.splits or max(1, min(16, 4 * 148 // max(1, B)))
    us = timeit(lambda: mla_decode(q, cache, bt, seq, P, scale, S), a.iters, a.warmup)
    hbm, _, src = peaks()
    byt = B * L * 576 * 2
    res.update({"decode_batch": B, "decode_splits": S, "decode_us": round(us, 1),
                f"decode_hbm_frac_of_{src}": round(byt / (us * 1e-6) / 1e9 / hbm, 3)})
    print(json.dumps(res))


def main():
    p = argparse.ArgumentParser()
    p.add_argument("which", choices=["moe", "moe_stages", "route", "gemm", "attn", "mla"])
    p.add_argument("--ep", type=int, default=1)
    p.add_argument("--bn", type=int, default=0, help="moe_stages: force the token tile (16/32/64/128)")
    p.add_argument("--only", default="", help="moe_stages: comma-separated stages to time")
    p.add_argument("--tokens", type=int, default=64)
    p.add_argument("--experts", type=int, default=128)
    p.add_argument("--n", type=int, default=5120)
    p.add_argument("--k", type=int, default=2880)
    p.add_argument("--batch", type=int, default=64)
    p.add_argument("--ctx", type=int, default=1536)
    p.add_argument("--splits", type=int, default=0)
    p.add_argument("--hq", type=int, default=64)
    p.add_argument("--hkv", type=int, default=8)
    p.add_argument("--page", type=int, default=16)
    p.add_argument("--mla-heads", type=int, default=16)
    p.add_argument("--head-dim", type=int, default=64)
    p.add_argument("--kv", default="fp8", choices=["fp8", "bf16"])
    p.add_argument("--variant", type=int, default=1, help="attn: FP8 kernel, 0 head-major, 1 token-major (bulk copies), 2 token-major (cp.async)")
    p.add_argument("--iters", type=int, default=20)
    p.add_argument("--warmup", type=int, default=3)
    a = p.parse_args()
    {"moe": bench_moe, "moe_stages": bench_moe_stages, "route": bench_route, "gemm": bench_gemm,
     "attn": bench_attn, "mla": bench_mla}[a.which](a)


if __name__ == "__main__":
    main()
