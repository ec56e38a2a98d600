"""Numerics of the sm_100a kernels against plain PyTorch fp32 references."""
import math

import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _close(a, b, atol, rtol, what=""):
    a = a.float().cpu()
    b = b.float().cpu()
    err = (a - b).abs().max().item()
    tol = atol + rtol * b.abs().max().item()
    assert err <= tol, f"{what}: max err {err} > {tol}"


def test_extension_loaded():
    from sglang_neuron_b200._ext import kernels
    assert kernels() is not None


@pytest.mark.parametrize("H", [1024, 2880, 4096])
def test_rmsnorm(H):
    from sglang_neuron_b200.ops.norm import rmsnorm, rmsnorm_ref, fused_add_rmsnorm
    torch.manual_seed(0)
    x = torch.randn(37, H, device=DEV, dtype=torch.bfloat16)
    w = torch.randn(H, device=DEV, dtype=torch.bfloat16)
    _close(rmsnorm(x, w, 1e-6), rmsnorm_ref(x.float(), w.float(), 1e-6), 2e-2, 1e-2, "rmsnorm")
    r = torch.randn_like(x)
    ref_sum = x.float() + r.float()
    ref = rmsnorm_ref(ref_sum, w.float(), 1e-6)
    xx, rr = fused_add_rmsnorm(x.clone(), r.clone(), w, 1e-6)
    _close(rr, ref_sum, 2e-2, 1e-2, "residual")
    _close(xx, ref, 3e-2, 2e-2, "fused norm")


@pytest.mark.parametrize("D,neox,norm,fp8,rot", [(64, True, False, True, 64), (128, True, True, False, 128),
                                                  (64, False, False, False, 64), (128, True, False, True, 64),
                                                  (256, False, True, False, 256), (128, False, True, True, 96)])
def test_rope_kv_write(D, neox, norm, fp8, rot):
    from sglang_neuron_b200.ops.rope import build_cos_sin_cache, rope_qk_norm_kv_write
    torch.manual_seed(1)
    T, Hq, Hkv, P = 21, 8, 2, 16
    cs = build_cos_sin_cache(rot, 4096, 150000.0, {"rope_type": "yarn", "factor": 32.0,
                                                 "original_max_position_embeddings": 4096,
                                                 "beta_fast": 32.0, "beta_slow": 1.0, "truncate": False}, DEV)
    qkv = torch.randn(T, (Hq + 2 * Hkv) * D, device=DEV, dtype=torch.bfloat16)
    q, k, v = qkv.split([Hq * D, Hkv * D, Hkv * D], dim=1)
    pos = torch.randint(0, 4000, (T,), device=DEV)
    slots = torch.randperm(64, device=DEV)[:T]
    slots[3] = -1
    cdt = torch.float8_e4m3fn if fp8 else torch.bfloat16
    kc = torch.zeros(4, Hkv, P, D, device=DEV, dtype=cdt)
    vc = torch.zeros_like(kc)
    qn = torch.rand(D, device=DEV, dtype=torch.bfloat16) + 0.5 if norm else None
    kn = torch.rand(D, device=DEV, dtype=torch.bfloat16) + 0.5 if norm else None
    # CPU reference on copies
    qkv_c = qkv.cpu().float()
    qc, kc_ref_in, vc_in = qkv_c.split([Hq * D, Hkv * D, Hkv * D], dim=1)
    qc, kc_ref_in = qc.clone(), kc_ref_in.clone()
    kcache_ref = torch.zeros(4, Hkv, P, D, dtype=torch.float32)
    vcache_ref = torch.zeros_like(kcache_ref)
    rope_qk_norm_kv_write(qc, kc_ref_in, vc_in, pos.cpu(), cs.cpu(), Hq, Hkv, D, rot, neox,
                          qn.cpu().float() if norm else None, kn.cpu().float() if norm else None, 1e-6,
                          kcache_ref, vcache_ref, slots.cpu(), P, 0.5 if fp8 else 1.0, 0.25 if fp8 else 1.0)
    rope_qk_norm_kv_write(q, k, v, pos, cs, Hq, Hkv, D, rot, neox, qn, kn, 1e-6, kc, vc, slots, P,
                          0.5 if fp8 else 1.0, 0.25 if fp8 else 1.0)
    _close(q, qc, 3e-2, 2e-2, "q")
    _close(k, kc_ref_in, 3e-2, 2e-2, "k")
    # fp8 caches hold x / scale; compare dequantised values against the fp32 reference cache
    ks, vs = (0.5, 0.25) if fp8 else (1.0, 1.0)
    tol = 0.15 if fp8 else 3e-2
    _close(kc.float() * ks, kcache_ref, tol, 6e-2, "k cache")
    _close(vc.float() * vs, vcache_ref, tol, 6e-2, "v cache")


def _make_paged(B, ctx_lens, Hkv, D, P, dtype, seed=0):
    g = torch.Generator().manual_seed(seed)
    max_pages = max((c + P - 1) // P for c in ctx_lens) + 1
    n_pages = B * max_pages + 3
    perm = torch.randperm(n_pages, generator=g)
    bt = torch.zeros(B, max_pages, dtype=torch.int32)
    for b in range(B):
        bt[b] = perm[b * max_pages:(b + 1) * max_pages]
    kc = (torch.randn(n_pages, Hkv, P, D, generator=g) * 0.7)
    vc = torch.randn(n_pages, Hkv, P, D, generator=g)
    return kc.to(dtype), vc.to(dtype), bt


@pytest.mark.parametrize("D,Hq,Hkv,window,sinks,fp8,splits,P", [
    (64, 64, 8, 0, True, True, 1, 16), (64, 64, 8, 128, True, True, 4, 16), (128, 32, 8, 0, False, False, 3, 16),
    (128, 16, 8, 0, False, False, 1, 16), (64, 8, 1, 0, True, False, 8, 16), (64, 64, 8, 100, True, True, 2, 16),
    (128, 32, 8, 0, True, True, 3, 16), (128, 64, 8, 77, False, True, 1, 16), (64, 32, 8, 0, True, True, 2, 64),
    (64, 64, 8, 0, False, True, 3, 128), (64, 16, 2, 0, True, True, 1, 32)])
def test_decode_attention(D, Hq, Hkv, window, sinks, fp8, splits, P):
    from sglang_neuron_b200.ops.attention import decode_attention, decode_attention_ref
    torch.manual_seed(2)
    ctx = [1, 17, 300, 1000, 64, 129]
    B = len(ctx)
    dt = torch.float8_e4m3fn if fp8 else torch.bfloat16
    kc, vc, bt = _make_paged(B, ctx, Hkv, D, P, dt)
    if fp8:  # stale bytes past each request's end (NaN patterns included) must not leak into the output
        for b, c in enumerate(ctx):
            for t in range(c, ((c + P - 1) // P + 1) * P):
                pg = int(bt[b, t // P])
                kc[pg, :, t % P] = float("nan")
                vc[pg, :, t % P] = float("nan")
    q = torch.randn(B, Hq * D, dtype=torch.bfloat16)
    sk = torch.randn(Hq) if sinks else None
    seq = torch.tensor(ctx, dtype=torch.int32)
    ks, vs = (0.8, 1.3) if fp8 else (1.0, 1.0)
    ref = decode_attention_ref(q.float(), kc, vc, bt, seq, Hq, Hkv, D, P, window, None, ks, vs, sk)
    out = decode_attention(q.to(DEV), kc.to(DEV), vc.to(DEV), bt.to(DEV), seq.to(DEV), Hq, Hkv, D, P, window,
                           None, ks, vs, sk.to(DEV) if sinks else None, num_splits=splits)
    _close(out, ref, 2e-2, 2e-2, "decode")


@pytest.mark.parametrize("D,Hq,Hkv,window,sinks,fp8", [(64, 64, 8, 0, True, True), (64, 64, 8, 128, True, False),
                                                       (128, 32, 8, 0, False, False), (128, 16, 8, 0, False, True)])
def test_extend_attention(D, Hq, Hkv, window, sinks, fp8):
    from sglang_neuron_b200.ops.attention import extend_attention, extend_attention_ref
    torch.manual_seed(3)
    P = 16
    prefix = [0, 40, 0, 300]
    ext = [5, 70, 200, 33]
    kv = [p + e for p, e in zip(prefix, ext)]
    B = len(kv)
    dt = torch.float8_e4m3fn if fp8 else torch.bfloat16
    kc, vc, bt = _make_paged(B, kv, Hkv, D, P, dt, seed=4)
    qo = torch.tensor([0] + list(torch.tensor(ext).cumsum(0)), dtype=torch.int32)
    q = torch.randn(int(qo[-1]), Hq * D, dtype=torch.bfloat16)
    sk = torch.randn(Hq) if sinks else None
    kvl = torch.tensor(kv, dtype=torch.int32)
    ref = extend_attention_ref(q.float(), kc, vc, bt, qo, kvl, Hq, Hkv, D, P, window, None, 1.0, 1.0, sk)
    out = extend_attention(q.to(DEV), kc.to(DEV), vc.to(DEV), bt.to(DEV), qo.to(DEV), kvl.to(DEV), max(ext), Hq,
                           Hkv, D, P, window, None, 1.0, 1.0, sk.to(DEV) if sinks else None)
    _close(out, ref, 2e-2, 2e-2, "extend")


def test_sampling_greedy_and_gumbel():
    from sglang_neuron_b200.ops.sampling import sample_tokens, gumbel_noise_ref
    torch.manual_seed(5)
    V = 201088
    logits = torch.randn(6, V, device=DEV)
    logits[0, 77] = 50.0
    logits[1, 5] = logits[1, 9] = 60.0  # tie -> smallest id
    ids = sample_tokens(logits)
    assert ids[0].item() == 77 and ids[1].item() == 5
    assert torch.equal(ids.cpu(), logits.argmax(-1).cpu()) or ids[1].item() == 5
    temp = torch.tensor([0.0, 0.7, 1.0, 1.3, 0.0, 2.0], device=DEV)
    seeds = torch.arange(6, device=DEV) * 1000 + 7
    pos = torch.arange(6, device=DEV) + 11
    ids = sample_tokens(logits, temp, seeds, pos).cpu()
    for b in range(6):
        t = float(temp[b])
        row = logits[b].float().cpu()
        if t > 0:
            row = row / t + gumbel_noise_ref(int(seeds[b]), int(pos[b]), V)
        best = row.max().item()
        assert row[ids[b]].item() >= best - 1e-3


def test_topk_route_and_align_combine():
    from sglang_neuron_b200.ops.moe import (topk_route, topk_route_ref, MoEAlignment, moe_align, moe_combine)
    torch.manual_seed(6)
    T, E, K = 77, 128, 4
    logits = torch.randn(T, E, device=DEV)
    for mode in (0, 1):
        w, ids = topk_route(logits, K, mode)
        wr, idr = topk_route_ref(logits.cpu(), K, mode)
        assert torch.equal(ids.cpu().long(), idr.long())
        _close(w, wr, 1e-5, 1e-4, "route w")
    w, ids = topk_route(logits, K, 0)
    bn = 16
    al = MoEAlignment(T * K, E, bn, DEV)
    moe_align(ids, 0, E, al)
    seg = al.seg_offsets.cpu()
    src = al.sorted_src.cpu()
    inv = al.inv_map.cpu()
    idc = ids.cpu().reshape(-1)
    for i in range(T * K):
        r = int(inv[i])
        e = int(idc[i])
        assert seg[e] <= r < seg[e + 1]
        assert int(src[r]) == i // K
    assert int(al.tile_offsets[-1]) * bn == int(seg[-1])
    # combine
    H = 256
    y = torch.randn(al.r_max, H, device=DEV, dtype=torch.bfloat16)
    out = torch.empty(T, H, device=DEV, dtype=torch.bfloat16)
    moe_combine(out, y, al.inv_map, w)
    ref = torch.zeros(T, H)
    for t in range(T):
        for j in range(K):
            ref[t] += float(w[t, j]) * y[int(inv[t * K + j])].float().cpu()
    _close(out, ref, 2e-2, 1e-2, "combine")


@pytest.mark.parametrize("H,K,accumulate", [(2880, 4, True), (2048, 6, False), (256, 16, True)])
def test_moe_combine_rows_missing_and_accumulate(H, K, accumulate):
    """Combine against fp32: tokens whose experts live on another EP rank (inv_map -1), accumulation into the
    residual, K from 4 to 16."""
    from sglang_neuron_b200.ops.moe import moe_combine
    torch.manual_seed(8)
    T, R = 37, 300
    y = torch.randn(R, H, device=DEV, dtype=torch.bfloat16)
    inv = torch.randint(0, R, (T * K,), dtype=torch.int32)
    inv[torch.rand(T * K) < 0.3] = -1
    w = torch.rand(T, K, device=DEV)
    base = torch.randn(T, H, device=DEV, dtype=torch.bfloat16)
    out = base.clone()
    moe_combine(out, y, inv.to(DEV), w, accumulate)
    ref = base.float().cpu() if accumulate else torch.zeros(T, H)
    for t in range(T):
        for j in range(K):
            r = int(inv[t * K + j])
            if r >= 0:
                ref[t] += float(w[t, j]) * y[r].float().cpu()
    _close(out, ref, 2e-2, 2e-2, "combine")


@pytest.mark.parametrize("bn", [16, 64, 128])
def test_gather_quant_mxfp8(bn):
    from sglang_neuron_b200.ops.moe import gather_quant_mxfp8
    torch.manual_seed(7)
    T, H = 50, 2880
    x = torch.randn(T, H, dtype=torch.bfloat16) * 3
    rows = 4 * bn
    src = torch.randint(-1, T, (rows,), dtype=torch.int32)
    q_ref, sf_ref = gather_quant_mxfp8(x, src, rows, bn)
    q, sf = gather_quant_mxfp8(x.to(DEV), src.to(DEV), rows, bn)
    # compare the scale bytes the MMA reads: (row i of each BN tile, 32-block kk) of every K block
    from sglang_neuron_b200.ops.moe import sf_atom_offset, sf_chunk_bytes
    KB = (H + 127) // 128
    i = torch.arange(bn).repeat_interleave(4)
    kk = torch.arange(4).repeat(bn)
    offs = sf_atom_offset(i, kk)
    # rows with a source (padding rows, src < 0, are left untouched: no GEMM output of theirs is read)
    ok_rows = torch.nonzero(src >= 0).flatten()
    tile, ii = ok_rows // bn, ok_rows % bn
    sel = torch.cat([(((tile * KB + kb) * sf_chunk_bytes(bn)) + sf_atom_offset(ii, torch.tensor(kk)))
                     for kb in range(KB) for kk in range(4)])
    assert torch.equal(sf.cpu()[sel], sf_ref[sel])
    assert (q.cpu()[ok_rows].float() - q_ref[ok_rows].float()).abs().max().item() <= 32.0 * 0.07


@pytest.mark.parametrize("T,F,K,bias,splits", [(1, 2880, 2880, True, None), (16, 5120, 2880, False, None),
                                               (77, 4096, 4096, True, None), (300, 1024, 3072, False, None),
                                               (1000, 384, 512, True, None), (64, 2880, 4096, True, 5),
                                               (5, 128, 2880, True, 3), (64, 5120, 2880, False, 1)])
def test_gemm_bf16_tcgen05(T, F, K, bias, splits):
    from sglang_neuron_b200.ops.gemm import linear, check_status
    torch.manual_seed(8)
    x = torch.randn(T, K, device=DEV, dtype=torch.bfloat16)
    w = torch.randn(F, K, device=DEV, dtype=torch.bfloat16) * 0.05
    b = torch.randn(F, device=DEV, dtype=torch.bfloat16) if bias else None
    y = linear(x, w, b, splits=splits)
    torch.cuda.synchronize()
    check_status(x.device)
    ref = x.float() @ w.float().t() + (b.float() if bias else 0)
    _close(y, ref, 3e-2, 1e-2, "gemm")


@pytest.mark.parametrize("T,F,K,bias", [(1, 2880, 2880, True), (64, 5120, 2880, False), (64, 2880, 4096, True),
                                        (64, 128, 2880, True), (33, 201088 // 16, 2880, False),
                                        (130, 2880, 4096, True), (600, 5120, 2880, True), (7, 1000, 520, True),
                                        (2048, 1536, 1024, False)])
def test_gemm_default_path(T, F, K, bias):
    _gemm_default_path(T, F, K, bias, tiled=False)


@pytest.mark.parametrize("T,F,K,bias", [(1, 2880, 2880, True), (64, 5120, 2880, False), (64, 2880, 4096, True),
                                        (64, 128, 2880, True), (7, 1000, 520, True), (130, 2880, 4096, True),
                                        (600, 5120, 2880, True)])
def test_gemm_tiled_weight(T, F, K, bias):
    """Pre-tiled weights (contiguous 128 x 64 tiles) through the same kernel."""
    _gemm_default_path(T, F, K, bias, tiled=True)


def _gemm_default_path(T, F, K, bias, tiled):
    """Default GEMM path (K split across a thread-block cluster, partials summed through distributed shared
    memory, for decode shapes): repeated calls give bit-identical results (fixed summation order)."""
    from sglang_neuron_b200.ops.gemm import TiledWeight, linear, linear_partials, check_status
    torch.manual_seed(9)
    x = torch.randn(T, K, device=DEV, dtype=torch.bfloat16)
    w = torch.randn(F, K, device=DEV, dtype=torch.bfloat16) * 0.05
    b = torch.randn(F, device=DEV, dtype=torch.bfloat16) if bias else None
    wg = TiledWeight(w) if tiled else w
    y1 = linear(x, wg, b)
    y2 = linear(x, wg, b)
    if tiled:
        assert torch.equal(wg.untiled(), w)
        ys = linear(x, wg, b, splits=3)
        part = linear_partials(x, wg, 2).view(2, T, F).sum(0)
        torch.cuda.synchronize()
        _close(ys, x.float() @ w.float().t() + (b.float() if bias else 0), 3e-2, 1e-2, "gemm_tiled_splitk")
        _close(part, x.float() @ w.float().t(), 3e-2, 1e-2, "gemm_tiled_partials")
    out = torch.empty(T, F + 8, device=DEV, dtype=torch.bfloat16)[:, :F]  # strided output rows
    linear(x, wg, b, out=out)
    torch.cuda.synchronize()
    check_status(x.device)
    ref = x.float() @ w.float().t() + (b.float() if bias else 0)
    _close(y1, ref, 3e-2, 1e-2, "gemm_default")
    assert torch.equal(y1, y2)
    assert torch.equal(out, y1)


def test_kv_page_copy_device_host_round_trip():
    """HiCache page copies: device pages -> pinned host slots -> other device pages, every layer buffer in
    one launch per direction (the kernel addresses pinned host memory directly)."""
    from sglang_neuron_b200.mem_cache.hicache import HiCache
    from sglang_neuron_b200.mem_cache.memory_pool import MHATokenToKVPool
    torch.manual_seed(12)
    pool = MHATokenToKVPool(3, 40, 16, 2, 64, torch.float8_e4m3fn, DEV)
    for b in pool.k_buffers + pool.v_buffers:
        b.copy_(torch.randn(b.shape, device=DEV).to(b.dtype))
    hc = HiCache(pool, 16, 10, torch.device(DEV))
    toks = list(range(16 * 5))
    src = [3, 9, 17, 4, 30]
    assert hc.write_through(toks, src) == 5
    hc.sync_writes()
    slots = hc.match(toks, 1, 4)
    assert len(slots) == 4
    dst = [35, 36, 37, 38]
    hc.load(slots, dst)
    hc.wait_loads()
    torch.cuda.synchronize()
    for b in pool.k_buffers + pool.v_buffers:
        assert torch.equal(b[dst].view(torch.uint8), b[src[1:]].view(torch.uint8))


@pytest.mark.parametrize("H,ctx,splits,P", [(16, [1, 17, 300, 1000], 1, 16), (16, [64, 129, 5], 4, 16),
                                            (20, [33, 700], 3, 64), (8, [1000, 2], 2, 16)])
def test_mla_decode_kernel(H, ctx, splits, P):
    """Tensor-core absorbed-MLA decode vs the fp32 PyTorch reference (stale/NaN bytes past each request's
    end are never read)."""
    from sglang_neuron_b200.ops.mla import _one, mla_decode
    torch.manual_seed(13)
    B = len(ctx)
    max_pages = max((c + P - 1) // P for c in ctx) + 1
    n_pages = B * max_pages + 2
    perm = torch.randperm(n_pages - 1)[: B * max_pages] + 1
    bt = perm.view(B, max_pages).to(torch.int32)
    cache = (torch.randn(n_pages, 1, P, 576) * 0.5).to(torch.bfloat16)
    for b, c in enumerate(ctx):  # poison the tail of each request's last page
        for t in range(c, ((c + P - 1) // P) * P):
            cache[int(bt[b, t // P]), 0, t % P] = float("nan")
    q = (torch.randn(B, H, 576) * 0.5).to(torch.bfloat16)
    scale = 0.0625
    ref = torch.stack([_one(q[b:b + 1].float(), cache.float(), bt[b], ctx[b], torch.tensor([ctx[b] - 1]), 512,
                            scale, P)[0] for b in range(B)])
    out = mla_decode(q.to(DEV), cache.to(DEV), bt.to(DEV), torch.tensor(ctx, dtype=torch.int32, device=DEV), P,
                     scale, splits)
    torch.cuda.synchronize()
    _close(out, ref, 2e-2, 2e-2, "mla_decode")


@pytest.mark.parametrize("H,chunks,P", [(16, [(0, 37), (100, 5), (16, 64)], 16), (2, [(0, 130), (33, 1), (7, 40)], 16),
                                        (4, [(250, 90)], 64)])
def test_mla_extend_kernel(H, chunks, P):
    """Absorbed-MLA prefill on tensor cores (rows = (token, head) pairs, per-row causal limits) vs the fp32
    PyTorch reference, for chunks with and without a cached prefix; NaN poison past each request's end."""
    from sglang_neuron_b200.ops.mla import _one, mla_extend
    torch.manual_seed(17)
    B = len(chunks)
    lens = [p + n for p, n in chunks]
    max_pages = max((L + P - 1) // P for L in lens) + 1
    n_pages = B * max_pages + 2
    perm = torch.randperm(n_pages - 1)[: B * max_pages] + 1
    bt = perm.view(B, max_pages).to(torch.int32)
    cache = (torch.randn(n_pages, 1, P, 576) * 0.5).to(torch.bfloat16)
    for b, L in enumerate(lens):
        for t in range(L, ((L + P - 1) // P) * P):
            cache[int(bt[b, t // P]), 0, t % P] = float("nan")
    T = sum(n for _, n in chunks)
    q = (torch.randn(T, H, 576) * 0.5).to(torch.bfloat16)
    qo = [0]
    for _, n in chunks:
        qo.append(qo[-1] + n)
    scale = 0.0625
    ref = torch.cat([_one(q[qo[b]:qo[b + 1]].float(), cache.float(), bt[b], lens[b],
                          torch.arange(chunks[b][0], lens[b]), 512, scale, P) for b in range(B)])
    out = mla_extend(q.to(DEV), cache.to(DEV), bt.to(DEV), torch.tensor(lens, dtype=torch.int32, device=DEV),
                     torch.tensor(qo, dtype=torch.int32, device=DEV), max(n for _, n in chunks), P, scale)
    torch.cuda.synchronize()
    _close(out, ref, 2e-2, 2e-2, "mla_extend")


@pytest.mark.parametrize("D,H,chunks,P", [(2, 8, [(0, 37), (100, 1), (16, 64)], 16), (4, 4, [(250, 90), (3, 1)], 16)])
def test_mla_extend_kernel_dcp_partials_merge(D, H, chunks, P):
    """Decode context parallelism on one GPU: the D ranks' local page sets (logical page j on rank j % D)
    are attended separately by the kernel with log2-sum-exp outputs; merging the partials gives attention
    over the whole context (fp32 reference)."""
    from sglang_neuron_b200.ops.mla import _one, mla_extend
    from sglang_neuron_b200.parallel.dcp import merge_partials
    torch.manual_seed(23)
    B = len(chunks)
    lens = [p + n for p, n in chunks]
    n_log = max((L + P - 1) // P for L in lens) + 1
    full = (torch.randn(B, n_log * P, 576) * 0.5).to(torch.bfloat16)
    nxt = [1] * D
    gbt = torch.zeros(B, n_log, dtype=torch.int32)
    for b in range(B):
        for j in range(n_log):
            gbt[b, j] = nxt[j % D] * D + j % D
            nxt[j % D] += 1
    n_local = max(nxt) + 1
    caches = [torch.zeros(n_local, 1, P, 576, dtype=torch.bfloat16) for _ in range(D)]
    for b in range(B):
        for t in range(n_log * P):
            g = int(gbt[b, t // P])
            caches[g % D][g // D, 0, t % P] = full[b, t] if t < lens[b] else float("nan")
    T = sum(n for _, n in chunks)
    q = (torch.randn(T, H, 576) * 0.5).to(torch.bfloat16)
    qo = [0]
    for _, n in chunks:
        qo.append(qo[-1] + n)
    scale = 0.0625
    seq = torch.tensor(lens, dtype=torch.int32, device=DEV)
    qo_t = torch.tensor(qo, dtype=torch.int32, device=DEV)
    os_, ls_ = [], []
    for d in range(D):
        lbt = torch.div(gbt[:, d::D], D, rounding_mode="floor").contiguous().to(DEV)
        lse = torch.empty(T, H, dtype=torch.float32, device=DEV)
        os_.append(mla_extend(q.to(DEV), caches[d].to(DEV), lbt, seq, qo_t, max(n for _, n in chunks), P, scale,
                              dcp=(D, d), lse_out=lse))
        ls_.append(lse)
    got = merge_partials(torch.stack(os_), torch.stack(ls_))
    torch.cuda.synchronize()
    ref_cache = full.view(B, n_log, 1, P, 576).float()
    ref = torch.cat([_one(q[qo[b]:qo[b + 1]].float(), ref_cache[b], torch.arange(n_log, dtype=torch.int32), lens[b],
                          torch.arange(chunks[b][0], lens[b]), 512, scale, P) for b in range(B)])
    _close(got, ref, 2e-2, 2e-2, "mla_extend dcp")


@pytest.mark.parametrize("T,E,K,mode,El,e_lo", [(64, 128, 4, 0, 128, 0), (37, 128, 4, 0, 16, 32),
                                                 (96, 64, 6, 1, 64, 0), (5, 128, 4, 0, 128, 0),
                                                 (128, 128, 4, 0, 16, 112)])
def test_fused_route_matches_separate_launches(T, E, K, mode, El, e_lo):
    """The one-launch routing kernel against the fp32 router logits and the separate align/quantise ops."""
    from sglang_neuron_b200.ops import moe
    from sglang_neuron_b200.ops.gemm import TiledWeight
    torch.manual_seed(T + E)
    H = 2880
    x = torch.randn(T, H, device=DEV).to(torch.bfloat16)
    wr = (torch.randn(E, H, device=DEV) * 0.02).to(torch.bfloat16)
    bias = (torch.randn(E, device=DEV) * 0.1).to(torch.bfloat16)
    scale = 1.0 if mode == 0 else 2.5
    bn = moe.pick_bn(T, K, El)
    w, ids, al, xq, sfb = moe.fused_route_quant(x, TiledWeight(wr), E, bias, K, mode, scale, e_lo, El, bn)
    torch.cuda.synchronize()
    assert int(moe._status(x.device)[0]) == 0
    # selection: the fp32 logits of the chosen experts are the top-k (up to bf16 rounding of near ties)
    lf = (x.float() @ wr.float().t() + bias.float()).cpu()
    top = lf.topk(K, dim=-1).values
    got = lf.gather(1, ids.long().cpu())
    assert (got.sort(dim=-1, descending=True).values - top).abs().max().item() <= 0.02
    lb = lf.to(torch.bfloat16).float()  # the kernel rounds its logits to bf16 like the router GEMM's output
    if mode == 0:
        w_ref = torch.softmax(lb.gather(1, ids.long().cpu()), dim=-1) * scale
    else:
        w_ref = torch.softmax(lb, dim=-1).gather(1, ids.long().cpu()) * scale
    _close(w.cpu(), w_ref, 2e-2, 2e-2, "routing weights")
    # alignment: segments as moe_align lays them out for the same ids, every entry mapped back to its token
    al2 = moe.MoEAlignment(T * K, El, bn, DEV)
    moe.moe_align(ids, e_lo, El, al2)
    assert torch.equal(al.seg_offsets, al2.seg_offsets) and torch.equal(al.tile_offsets, al2.tile_offsets)
    used = int(al.seg_offsets[El])
    inv = al.inv_map[: T * K].cpu()
    src = al.sorted_src.cpu()
    for i in range(T * K):
        e = int(ids.view(-1)[i]) - e_lo
        if 0 <= e < El:
            assert int(src[int(inv[i])]) == i // K
        else:
            assert int(inv[i]) == -1
    assert int((src[:used] >= 0).sum()) == int((inv >= 0).sum())
    # quantised rows: byte-identical to the separate quantise kernel over the same permutation
    q2, sf2 = moe.gather_quant_mxfp8(x, al.sorted_src, al.r_max, bn, used=al.seg_offsets[El:El + 1])
    torch.cuda.synchronize()
    ok_rows = torch.nonzero(src[:used] >= 0).flatten()  # padding rows are left untouched by both kernels
    assert torch.equal(xq[:used].view(torch.uint8)[ok_rows.to(DEV)], q2[:used].view(torch.uint8)[ok_rows.to(DEV)])
    # scale bytes the MMA reads for those rows: (row i of its BN tile, 32-block kk) of every K block
    KB = (H + 127) // 128
    tile, ii = ok_rows // bn, ok_rows % bn
    idx = torch.cat([(((tile * KB + kb) * moe.sf_chunk_bytes(bn)) + moe.sf_atom_offset(ii, torch.tensor(kk)))
                     for kb in range(KB) for kk in range(4)]).to(DEV)
    assert torch.equal(sfb[idx], sf2[idx])


@pytest.mark.parametrize("kv", ["fp8", "bf16"])
@pytest.mark.parametrize("variant", [0, 1, 2])
@pytest.mark.parametrize("D,Hq,Hkv,window,sinks,splits,P", [
    (64, 32, 2, 0, True, 2, 16), (128, 32, 2, 50, False, 1, 32), (64, 64, 8, 200, True, 1, 64),
    (128, 64, 8, 0, True, 2, 128), (64, 32, 8, 0, False, 1, 16), (128, 32, 8, 0, False, 3, 16)])
def test_decode_attention_pipelined_variants(kv, variant, D, Hq, Hkv, window, sinks, splits, P):
    """The decode kernels behind one switch against the fp32 reference: for e4m3 caches the head-major kernel
    (query heads as MMA rows) and the token-major kernel (S^T = K Q^T) fed by bulk copies or cp.async; for bf16
    caches the register-prefetch kernel and the same token-major kernel. GQA groups of 4, 8 and 16 heads; stale
    NaN bytes past each request's end (except for the register-prefetch kernel, which the engine feeds zeroed
    pools)."""
    from sglang_neuron_b200._ext import kernels
    from sglang_neuron_b200.ops.attention import decode_attention, decode_attention_ref
    torch.manual_seed(5)
    ctx = [1, 17, 300, 1000, 64, 129, 128, 33]
    B = len(ctx)
    fp8 = kv == "fp8"
    kc, vc, bt = _make_paged(B, ctx, Hkv, D, P, torch.float8_e4m3fn if fp8 else torch.bfloat16)
    if fp8 or variant != 0:
        for b, c in enumerate(ctx):
            for t in range(c, ((c + P - 1) // P + 1) * P):
                pg = int(bt[b, t // P])
                kc[pg, :, t % P] = float("nan")
                vc[pg, :, t % P] = float("nan")
    q = torch.randn(B, Hq * D, dtype=torch.bfloat16)
    sk = torch.randn(Hq) if sinks else None
    seq = torch.tensor(ctx, dtype=torch.int32)
    ks, vs = (0.8, 1.3) if fp8 else (1.0, 1.0)
    ref = decode_attention_ref(q.float(), kc, vc, bt, seq, Hq, Hkv, D, P, window, None, ks, vs, sk)
    kernels().set_decode_fp8_variant(variant)
    try:
        out = decode_attention(q.to(DEV), kc.to(DEV), vc.to(DEV), bt.to(DEV), seq.to(DEV), Hq, Hkv, D, P, window,
                               None, ks, vs, sk.to(DEV) if sinks else None, num_splits=splits)
    finally:
        kernels().set_decode_fp8_variant(1)
    _close(out, ref, 2e-2, 2e-2, f"decode {kv} variant {variant}")


def test_decode_attention_merge_counters_rearm():
    """FP8 split-K decode with the in-kernel merge: one scratch (counters included) over several calls and
    batch sizes, each output against the fp32 reference."""
    from sglang_neuron_b200.ops.attention import DecodeScratch, decode_attention, decode_attention_ref
    torch.manual_seed(21)
    D, Hq, Hkv, P, S = 64, 64, 8, 16, 4
    sc = DecodeScratch(8, Hq, D, S, DEV)
    for call, ctx in enumerate([[5, 700, 64], [1000, 3, 77, 129, 512, 2, 16, 300], [40]]):
        B = len(ctx)
        kc, vc, bt = _make_paged(B, ctx, Hkv, D, P, torch.float8_e4m3fn)
        q = torch.randn(B, Hq * D, dtype=torch.bfloat16)
        sk = torch.randn(Hq)
        seq = torch.tensor(ctx, dtype=torch.int32)
        ref = decode_attention_ref(q.float(), kc, vc, bt, seq, Hq, Hkv, D, P, 0, None, 0.9, 1.2, sk)
        out = decode_attention(q.to(DEV), kc.to(DEV), vc.to(DEV), bt.to(DEV), seq.to(DEV), Hq, Hkv, D, P, 0, None,
                               0.9, 1.2, sk.to(DEV), num_splits=S, scratch=sc)
        _close(out, ref, 2e-2, 2e-2, f"decode call {call}")
        assert int(sc.merge_cnt.abs().sum()) == 0, "merge counters must be re-armed"


def test_allreduce_peer_wait_runs_out_with_status():
    """A world-of-2 all-reduce whose second rank never publishes (its slot is a buffer of this GPU that nobody
    writes a flag into): the bounded peer wait runs out after its short budget, the kernel records
    SNB_ERR_TIMEOUT_PEER and returns, and the context stays usable. No GPU fault is involved."""
    import time
    from sglang_neuron_b200._ext import kernels
    from sglang_neuron_b200.parallel.symm_mem import IpcAllReduce
    k = kernels()
    cap = 1 << 20
    p0, _ = k.symm_alloc(cap, 2)
    p1, _ = k.symm_alloc(cap, 2)
    ar = IpcAllReduce(cap, ptrs=[p0, p1], wait_ns=50_000_000)  # 50 ms instead of the 2 s default
    try:
        x = torch.randn(64 * 2880, device=DEV).to(torch.bfloat16)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        ar.all_reduce(x)
        torch.cuda.synchronize()
        dt = time.perf_counter() - t0
        assert int(ar.status[0]) == 4, "expected SNB_ERR_TIMEOUT_PEER"
        assert dt < 1.0, f"the wait took {dt:.3f} s, not its 50 ms budget"
        # the context is still usable
        assert torch.isfinite((x.float() * 2).sum()).item()
    finally:
        torch.cuda.synchronize()
        ar.close()


@pytest.mark.parametrize("B,V,K,dt,ties", [(64, 201088, 256, torch.bfloat16, False), (3, 25136, 256, torch.bfloat16, True),
                                            (5, 1000, 40, torch.float32, False), (2, 100, 256, torch.float32, False),
                                            (7, 151936, 1, torch.bfloat16, True)])
def test_topk_pool_radix_select(B, V, K, dt, ties):
    """The radix-select candidate pool against a stable descending sort (value desc, index asc), including
    heavy ties and rows shorter than the pool."""
    from sglang_neuron_b200._ext import kernels
    torch.manual_seed(V + K)
    x = torch.randn(B, V + 3) * 4
    if ties:
        x = x.round()  # few distinct values: the K-th value is shared by many entries
    x = x.to(dt)
    kk = min(K, V)
    vals = torch.empty(B, kk, dtype=torch.float32, device=DEV)
    ids = torch.empty(B, kk, dtype=torch.int64, device=DEV)
    kernels().topk_pool(x.to(DEV), V, kk, 7, vals, ids)
    torch.cuda.synchronize()
    ref_v, ref_i = x[:, :V].float().sort(dim=-1, descending=True, stable=True)
    assert torch.equal(vals.cpu(), ref_v[:, :kk])
    assert torch.equal(ids.cpu(), ref_i[:, :kk] + 7)


def test_rope_kv_write_skips_slot_past_pool_with_bounds_status():
    """A KV slot whose page lies past the pool is not written: the kernel records SNB_ERR_BOUNDS (5) with the
    slot, the other rows land normally. The check is always compiled in, so no fault is involved."""
    from sglang_neuron_b200.ops.gemm import _status_buf
    from sglang_neuron_b200.ops.rope import build_cos_sin_cache, rope_qk_norm_kv_write
    T, Hq, Hkv, D, P, pages = 3, 4, 2, 64, 16, 4
    q = torch.randn(T, Hq * D, device=DEV).to(torch.bfloat16)
    k = torch.randn(T, Hkv * D, device=DEV).to(torch.bfloat16)
    v = torch.randn(T, Hkv * D, device=DEV).to(torch.bfloat16)
    kc = torch.zeros(pages + 1, Hkv, P, D, device=DEV, dtype=torch.bfloat16)  # one guard page past the pool
    vc = torch.zeros_like(kc)
    pos = torch.tensor([0, 1, 2], device=DEV)
    cs = build_cos_sin_cache(D, 64, 10000.0, None, DEV)
    slots = torch.tensor([5, pages * P + 3, 17], device=DEV)  # the middle slot is in the guard page
    st = _status_buf(q.device)
    st.zero_()
    rope_qk_norm_kv_write(q, k, v, pos, cs, Hq, Hkv, D, D, True, k_cache=kc[:pages], v_cache=vc[:pages],
                          slots=slots, page_size=P)
    torch.cuda.synchronize()
    code, where = int(st[0]), int(st[1])
    st.zero_()
    assert code == 5 and where == pages * P + 3
    assert kc[pages].abs().sum().item() == 0 and vc[pages].abs().sum().item() == 0  # guard page untouched
    assert vc[0, :, 5].abs().sum().item() > 0 and vc[1, :, 1].abs().sum().item() > 0  # the others landed
