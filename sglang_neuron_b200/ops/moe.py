"""MoE ops: top-k routing, device counting-sort permutation, MXFP8 gather-quantisation, the block-scaled
grouped expert GEMM and the weighted combine. MX formats follow the OCP Microscaling spec: blocks of 32
values share one e8m0 scale; MXFP4 values are e2m1 (two per byte, low nibble first), MXFP8 values e4m3.
"""
import math
from typing import Optional

import torch

from .._ext import kernels

E2M1_VALUES = torch.tensor([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0,
                            -0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0], dtype=torch.float32)


# ----------------------------------------------------------------------------------------------
# routing
# ----------------------------------------------------------------------------------------------
def topk_route_ref(logits: torch.Tensor, k: int, mode: int = 0, scale: float = 1.0):
    lf = logits.float()
    if mode == 0:
        vals, ids = torch.topk(lf, k, dim=-1)
        w = torch.softmax(vals, dim=-1) * scale
    else:
        probs = torch.softmax(lf, dim=-1)
        w, ids = torch.topk(probs, k, dim=-1)
        w = w * scale
    return w, ids.to(torch.int32)


def topk_route(logits: torch.Tensor, k: int, mode: int = 0, scale: float = 1.0):
    """mode 0: softmax over the top-k logits (GPT-OSS, Qwen3-MoE with norm_topk_prob);
    mode 1: softmax over all experts, then the top-k probabilities (DeepSeek-V2)."""
    if not logits.is_cuda:
        return topk_route_ref(logits, k, mode, scale)
    T = logits.shape[0]
    w = torch.empty(T, k, dtype=torch.float32, device=logits.device)
    ids = torch.empty(T, k, dtype=torch.int32, device=logits.device)
    kernels().topk_route(w, ids, logits.contiguous(), k, mode, scale)
    return w, ids


def max_sorted_rows(num_entries: int, num_experts: int, bn: int) -> int:
    r = num_entries + num_experts * (bn - 1)
    return ((r + bn - 1) // bn) * bn


class MoEAlignment:
    """Device buffers of one expert permutation (static capacity, reusable across CUDA-graph replays)."""

    def __init__(self, max_entries: int, num_local_experts: int, bn: int, device):
        self.bn = bn
        self.num_local_experts = num_local_experts
        self.r_max = max_sorted_rows(max_entries, num_local_experts, bn)
        # every element is written by moe_align before any reader runs, so no fill kernels are needed
        alloc = torch.empty if torch.device(device).type == "cuda" else torch.zeros
        self.seg_offsets = alloc(num_local_experts + 1, dtype=torch.int32, device=device)
        self.tile_offsets = alloc(num_local_experts + 1, dtype=torch.int32, device=device)
        self.sorted_src = torch.full((self.r_max,), -1, dtype=torch.int32, device=device) if alloc is torch.zeros \
            else torch.empty(self.r_max, dtype=torch.int32, device=device)
        self.inv_map = torch.full((max_entries,), -1, dtype=torch.int32, device=device) if alloc is torch.zeros \
            else torch.empty(max_entries, dtype=torch.int32, device=device)


def moe_align_ref(ids: torch.Tensor, e_lo: int, e_local: int, bn: int, al: MoEAlignment):
    flat = ids.reshape(-1).long()
    K = ids.shape[1] if ids.dim() == 2 else 1
    al.sorted_src.fill_(-1)
    al.inv_map[: flat.numel()].fill_(-1)
    off = 0
    tiles = 0
    for e in range(e_local):
        sel = torch.nonzero(flat == e + e_lo).flatten()
        al.seg_offsets[e] = off
        al.tile_offsets[e] = tiles
        n = sel.numel()
        if n:
            al.sorted_src[off:off + n] = (sel // K).to(torch.int32)
            al.inv_map[sel] = torch.arange(off, off + n, dtype=torch.int32)
        padded = ((n + bn - 1) // bn) * bn
        off += padded
        tiles += padded // bn
    al.seg_offsets[e_local] = off
    al.tile_offsets[e_local] = tiles


def moe_align(ids: torch.Tensor, e_lo: int, e_local: int, al: MoEAlignment):
    if not ids.is_cuda:
        return moe_align_ref(ids, e_lo, e_local, al.bn, al)
    kernels().moe_align(ids, e_lo, e_local, al.bn, al.seg_offsets, al.tile_offsets, al.sorted_src,
                        al.inv_map[: ids.numel()])


def moe_combine(out: torch.Tensor, y: torch.Tensor, inv_map: torch.Tensor, w: torch.Tensor,
                accumulate: bool = False):
    if not out.is_cuda:
        T, K = w.shape
        idx = inv_map[: T * K].long().view(T, K)
        valid = (idx >= 0).float()
        g = y[idx.clamp(min=0)].float() * (w.float() * valid)[..., None]
        r = g.sum(1)
        if accumulate:
            r = r + out.float()
        out.copy_(r.to(out.dtype))
        return out
    kernels().moe_combine(out, y, inv_map, w, accumulate)
    return out


# ----------------------------------------------------------------------------------------------
# MX formats
# ----------------------------------------------------------------------------------------------
def dequant_mxfp4(blocks: torch.Tensor, scales: torch.Tensor) -> torch.Tensor:
    """blocks: [..., K/2] uint8 (low nibble first), scales: [..., K/32] uint8 e8m0 -> [..., K] fp32."""
    lut = E2M1_VALUES.to(blocks.device)
    lo = (blocks & 0x0F).long()
    hi = (blocks >> 4).long()
    vals = torch.stack([lut[lo], lut[hi]], dim=-1).reshape(*blocks.shape[:-1], blocks.shape[-1] * 2)
    s = torch.exp2(scales.float() - 127.0)
    return (vals.view(*vals.shape[:-1], -1, 32) * s[..., None]).reshape(vals.shape)


def quant_mxfp4(x: torch.Tensor):
    """fp32/bf16 [..., K] -> (blocks uint8 [..., K/2], scales uint8 [..., K/32]); round to nearest e2m1."""
    xf = x.float().reshape(*x.shape[:-1], -1, 32)
    amax = xf.abs().amax(-1, keepdim=True)
    X = torch.where(amax > 0, torch.ceil(torch.log2(amax / 6.0)), torch.zeros_like(amax)).clamp(-127, 127)
    y = xf / torch.exp2(X)
    lut = E2M1_VALUES[:8].to(x.device)
    mag = y.abs().unsqueeze(-1)
    code = (mag - lut).abs().argmin(-1)
    code = code + (y < 0).long() * 8
    code = code.reshape(*x.shape[:-1], -1)
    blocks = (code[..., 0::2] | (code[..., 1::2] << 4)).to(torch.uint8)
    return blocks, (X.squeeze(-1) + 127).to(torch.uint8)


def quant_mxfp8_ref(x: torch.Tensor):
    """[..., K] -> (e4m3 values as float8 tensor, e8m0 scales uint8 [..., K/32])."""
    xf = x.float().reshape(*x.shape[:-1], -1, 32)
    amax = xf.abs().amax(-1, keepdim=True)
    X = torch.where(amax > 0, torch.ceil(torch.log2(amax / 448.0)), torch.zeros_like(amax)).clamp(-127, 127)
    q = (xf / torch.exp2(X)).clamp(-448, 448).to(torch.float8_e4m3fn)
    return q.reshape(x.shape), (X.squeeze(-1) + 127).to(torch.uint8)


def dequant_mxfp8(q: torch.Tensor, scales: torch.Tensor) -> torch.Tensor:
    qf = q.float().reshape(*q.shape[:-1], -1, 32)
    return (qf * torch.exp2(scales.float() - 127.0)[..., None]).reshape(q.shape)


def sf_chunk_bytes(bn: int) -> int:
    return min(bn, 32) * 16


def sf_atom_offset(row_in_tile: torch.Tensor, kk: torch.Tensor) -> torch.Tensor:
    """Byte offset of (row, 32-block kk) inside one scale-factor chunk (tcgen05.cp 32x128b.warpx4 order)."""
    return (row_in_tile % 32) * 16 + (row_in_tile // 32) * 4 + kk


def gather_quant_mxfp8(x: torch.Tensor, src: Optional[torch.Tensor], rows: int, bn: int, kp: int = None,
                       used: Optional[torch.Tensor] = None, skip: Optional[torch.Tensor] = None):
    """Permute rows of x by `src` (-1 = zero row) and quantise to MXFP8 with scales in chunk-atom order.
    `used` ([1] int32 on the device, the routed row count) lets the kernel skip rows no GEMM tile reads.
    Padding rows (src < 0, or skip[r] < 0 when rows are already in permuted order) are left untouched on the
    GPU: their GEMM output rows are never read. Returns (q [rows, kp] float8_e4m3fn, sf uint8 flat)."""
    H = x.shape[1]
    kp = H if kp is None else kp
    KB = (kp + 127) // 128
    nsf = (rows // bn) * KB * sf_chunk_bytes(bn)
    q = torch.empty(rows, kp, dtype=torch.float8_e4m3fn, device=x.device)
    if x.is_cuda:
        # the kernel writes every scale byte the MMA reads (rows < BN of each chunk, all K blocks); the
        # remaining bytes of a chunk belong to rows the MMA never reads, so no fill is needed
        sf = torch.empty(nsf, dtype=torch.uint8, device=x.device)
        kernels().gather_quant_mxfp8(q, sf, x, src, bn, used, skip)
        return q, sf
    sf = torch.full((nsf,), 127, dtype=torch.uint8, device=x.device)
    s = src.long() if src is not None else torch.arange(rows)
    xs = torch.zeros(rows, kp, dtype=torch.float32)
    valid = s >= 0
    xs[valid, :H] = x[s[valid]].float()
    qv, sc = quant_mxfp8_ref(xs[:, :KB * 128] if kp >= KB * 128 else torch.nn.functional.pad(xs, (0, KB * 128 - kp)))
    q.copy_(qv[:, :kp])
    sc = sc.clone()
    nblk_valid = (H + 31) // 32
    sc[:, nblk_valid:] = 127
    sc[~valid] = 127
    r = torch.arange(rows)
    tile = r // bn
    i = r % bn
    for blk in range(KB * 4):
        kb, kk = blk // 4, blk % 4
        off = (tile * KB + kb) * sf_chunk_bytes(bn) + sf_atom_offset(i, torch.tensor(kk))
        sf[off] = sc[:, blk]
    return q, sf


# ----------------------------------------------------------------------------------------------
# grouped expert GEMM (tcgen05 block-scaled) and the fused MoE forward
# ----------------------------------------------------------------------------------------------
SF_ATOM = 512
EPI_SWIGLU_CLAMP, EPI_SILU, EPI_BIAS = 0, 1, 2


def gated_row_order(inter: int, interleaved: bool) -> torch.Tensor:
    """Source row for each arranged row of a gate/up weight [2*inter, K]: each 128-row tile holds 64 gate
    rows then the 64 matching up rows. interleaved=True: source rows alternate gate/up (GPT-OSS
    checkpoints); False: source is [gate (inter rows); up (inter rows)] (Qwen3-MoE, DeepSeek-V2)."""
    assert inter % 64 == 0, "gated expert intermediate size must be a multiple of 64"
    n_tiles = inter // 64
    mt = torch.arange(n_tiles).repeat_interleave(128)
    i = torch.arange(128).repeat(n_tiles)
    j = mt * 64 + (i % 64)
    is_up = i >= 64
    if interleaved:
        return torch.where(is_up, 2 * j + 1, 2 * j)
    return torch.where(is_up, inter + j, j)


def arrange_sf_atoms(scales: torch.Tensor, F: int, K: int) -> torch.Tensor:
    """scales: [E, F, K/32] uint8 (row-major e8m0) -> [E, MT, KB, 512] atoms (pad rows/blocks with 2^0)."""
    E = scales.shape[0]
    MT, KB = (F + 127) // 128, (K + 127) // 128
    padded = torch.full((E, MT * 128, KB * 4), 127, dtype=torch.uint8, device=scales.device)
    padded[:, :F, : scales.shape[2]] = scales
    # [E, MT, m1(4), m0(32), KB, kk(4)] -> [E, MT, KB, m0, m1, kk]
    v = padded.view(E, MT, 4, 32, KB, 4).permute(0, 1, 4, 3, 2, 5).contiguous()
    return v.view(E, MT, KB, SF_ATOM)


def tile_weights(w: torch.Tensor, fp4: bool) -> torch.Tensor:
    """[E, F, row_bytes] packed MXFP4 (two values per byte) or MXFP8 rows -> [E, MT, KB, 128, bpr]: every
    (expert, 128-row tile, 128-value K block) becomes one contiguous block (8 KB for fp4, 16 KB for fp8), so
    each pipeline stage of the grouped GEMM reads a single sequential run of HBM. Rows past F and values past
    K are zero (they contribute nothing: the matching scales are 2^0 and the activations are zero there)."""
    E, F, rb = w.shape
    bpr = 64 if fp4 else 128
    MT, KB = (F + 127) // 128, (rb + bpr - 1) // bpr
    src = w if w.dtype == torch.uint8 else w.view(torch.uint8)
    out = torch.zeros(E, MT * 128, KB * bpr, dtype=torch.uint8, device=w.device)
    out[:, :F, :rb] = src
    out = out.view(E, MT, 128, KB, bpr).permute(0, 1, 3, 2, 4).contiguous()
    return out if w.dtype == torch.uint8 else out.view(w.dtype)


def untile_weights(t: torch.Tensor, F: int, row_bytes: int) -> torch.Tensor:
    E, MT, KB, _, bpr = t.shape
    u = t.view(torch.uint8) if t.dtype != torch.uint8 else t
    u = u.permute(0, 1, 3, 2, 4).reshape(E, MT * 128, KB * bpr)[:, :F, :row_bytes]
    return u if t.dtype == torch.uint8 else u.contiguous().view(t.dtype)


class ExpertWeights:
    """Device layout of one MoE layer's local experts for the grouped GEMM.

    w13: gate/up weights with rows arranged per gated_row_order, MXFP4 packed ([E, 2I, H/2] uint8) or
    MXFP8 ([E, 2I, H] float8_e4m3fn); sfa13: [E, MT, KB, 512] scale atoms; b13: arranged bias [E, 2I] or None.
    w2/sfa2/b2: the down projection [E, H, I(/2)].
    """

    def __init__(self, w13, s13, b13, w2, s2, b2, hidden: int, inter: int, interleaved: bool):
        self.hidden, self.inter = hidden, inter
        order = gated_row_order(inter, interleaved).to(w13.device)
        self.fp4 = w13.dtype == torch.uint8
        self.w13 = tile_weights(w13.index_select(1, order), self.fp4)
        self.sfa13 = arrange_sf_atoms(s13.index_select(1, order), 2 * inter, hidden)
        self.b13 = b13.index_select(1, order).to(torch.bfloat16).contiguous() if b13 is not None else None
        self.w2 = tile_weights(w2, self.fp4)
        self.sfa2 = arrange_sf_atoms(s2, hidden, inter)
        self.b2 = b2.to(torch.bfloat16).contiguous() if b2 is not None else None
        self.num_experts = w13.shape[0]


_status_bufs = {}


def _status(device):
    key = (device.type, device.index)
    if key not in _status_bufs:
        _status_bufs[key] = torch.zeros(4, dtype=torch.int32, device=device)
    return _status_bufs[key]


_sms = {}


def moe_gemm(out, xq, sfb, w, sfa, bias, al: MoEAlignment, epi: int, F: int, alpha=1.702, limit=7.0,
             qout=None, sfout=None):
    """qout/sfout (gated epilogues): write the activation as MXFP8 e4m3 [R, F/2] + atom-order e8m0 scales
    (the down projection's B operand) instead of bf16 to `out`."""
    key = out.device.index
    if key not in _sms:
        _sms[key] = torch.cuda.get_device_properties(out.device).multi_processor_count
    kernels().moe_gemm(out, xq, sfb, w, sfa, bias, al.seg_offsets, al.tile_offsets, al.bn, epi, alpha, limit,
                       _sms[key], _status(out.device), F, qout, sfout)
    return out


def _fused_act_quant() -> bool:
    """Off by default: measured on the GPT-OSS decode bench the fused epilogue (per-token warp max + scale
    per 32 columns) matched the separate quantise launch at 64 tokens (284.7 vs 280.8 us per MoE layer) and
    cost ~2.3 ms per step in mixed prefill steps (4223 -> 3666 tok/s)."""
    from .. import env_registry
    return env_registry.get_bool("SGLANG_B200_MOE_FUSED_ACT_QUANT", False)


def pick_bn(num_tokens: int, top_k: int, num_experts: int) -> int:
    """Token tile of the grouped GEMM. Tiles of up to 32 tokens run two CTAs per SM and keep the weight stream
    near the HBM roofline; 64- and 128-token tiles run one CTA per SM whose epilogue (128 x BN accumulators
    through named barriers) cannot keep up (ncu on the 1087-token GPT-OSS layer: 27 % of DRAM bandwidth,
    barrier stalls first). Measured per layer at 1087 tokens: gate/up 333 us with 32-token tiles against 532
    (64) and 991 (128); at 16 local experts 65 us against 84 and 141. Larger token counts re-read each weight
    tile once per 32-token tile, from L2 (neighbouring CTAs take neighbouring tiles of the same expert)."""
    per_expert = num_tokens * top_k / max(1, num_experts)
    return 16 if per_expert <= 12 else 32


ROUTE_FUSED_MAX_LOGITS = 16384  # T * E the one-launch routing kernel stages in shared memory
_route_sync = {}


def fused_route_quant(x: torch.Tensor, router_w, num_experts: int, bias: Optional[torch.Tensor], k: int,
                      mode: int, scale: float, e_lo: int, e_local: int, bn: int):
    """Router GEMM + top-k + expert alignment + MXFP8 gather-quantise in one launch (decode-sized T).
    router_w: the router weight as ops.gemm.TiledWeight. Returns (topk_w, topk_ids, MoEAlignment, xq, sfb),
    the values topk_route(linear(x, router_w, bias)), moe_align and gather_quant_mxfp8 produce."""
    T, H = x.shape
    dev = x.device
    w = torch.empty(T, k, dtype=torch.float32, device=dev)
    ids = torch.empty(T, k, dtype=torch.int32, device=dev)
    al = MoEAlignment(T * k, e_local, bn, dev)
    R = al.r_max
    xq = torch.empty(R, H, dtype=torch.float8_e4m3fn, device=dev)
    sfb = torch.empty((R // bn) * ((H + 127) // 128) * sf_chunk_bytes(bn), dtype=torch.uint8, device=dev)
    kc = max(1, (H + 319) // 320)  # ~320-wide K chunks: E/16 x kc CTAs
    partial = torch.empty(kc * T * num_experts, dtype=torch.float32, device=dev)
    key = (dev.type, dev.index)
    if key not in _route_sync:
        _route_sync[key] = torch.zeros(2, dtype=torch.int32, device=dev)
    kernels().moe_route_fused(x, router_w.data, num_experts, bias, k, mode, scale, e_lo, e_local, bn, partial, w,
                              ids, al.seg_offsets, al.tile_offsets, al.sorted_src, al.inv_map, xq, sfb,
                              _route_sync[key], _status(dev), kc)
    return w, ids, al, xq, sfb


def fused_moe(x: torch.Tensor, topk_w: torch.Tensor, topk_ids: torch.Tensor, ew: ExpertWeights,
              activation: str = "swiglu_clamp", alpha: float = 1.702, limit: float = 7.0,
              e_lo: int = 0, bn: int = 0, al: Optional[MoEAlignment] = None, out=None,
              combine_fn=None, routed=None) -> torch.Tensor:
    """sum_j w[t,j] * expert_{id[t,j]}(x[t]) over the experts owned here ([e_lo, e_lo + E_local)).
    `combine_fn(out, y, inv_map, w) -> bool` may replace the final combine (e.g. with the combine fused into
    the expert-parallel all-reduce); it returns False to fall back to the local combine.
    `routed` = (MoEAlignment, xq, sfb) from fused_route_quant: alignment and quantisation are done."""
    T, H = x.shape
    K = topk_ids.shape[1]
    if not x.is_cuda:
        return fused_moe_ref(x, topk_w, topk_ids, ew, activation, alpha, limit, e_lo, out=out)
    E = ew.num_experts
    if routed is not None:
        al, xq, sfb = routed
        bn = al.bn
        R = al.r_max
        used = al.seg_offsets[E:E + 1]
    else:
        if bn <= 0:
            bn = pick_bn(T, K, E)
        if al is None or al.bn != bn:
            al = MoEAlignment(T * K, E, bn, x.device)
        moe_align(topk_ids, e_lo, E, al)
        R = al.r_max
        used = al.seg_offsets[E:E + 1]  # rows the local experts' segments occupy (<= R)
        xq, sfb = gather_quant_mxfp8(x, al.sorted_src, R, bn, used=used)
    epi = EPI_SWIGLU_CLAMP if activation == "swiglu_clamp" else EPI_SILU
    if _fused_act_quant():
        # the gate/up epilogue quantises its activation to MXFP8 in place of a separate gather-quantise launch
        aq = torch.empty(R, ew.inter, dtype=torch.float8_e4m3fn, device=x.device)
        sfb2 = torch.empty((R // bn) * ((ew.inter + 127) // 128) * sf_chunk_bytes(bn), dtype=torch.uint8,
                           device=x.device)
        no_bf16 = torch.empty(0, 1, dtype=torch.bfloat16, device=x.device)
        moe_gemm(no_bf16, xq, sfb, ew.w13, ew.sfa13, ew.b13, al, epi, 2 * ew.inter, alpha, limit, qout=aq,
                 sfout=sfb2)
    else:
        act = torch.empty(R, ew.inter, dtype=torch.bfloat16, device=x.device)
        moe_gemm(act, xq, sfb, ew.w13, ew.sfa13, ew.b13, al, epi, 2 * ew.inter, alpha, limit)
        aq, sfb2 = gather_quant_mxfp8(act, None, R, bn, used=used, skip=al.sorted_src)
    y = torch.empty(R, H, dtype=torch.bfloat16, device=x.device)
    moe_gemm(y, aq, sfb2, ew.w2, ew.sfa2, ew.b2, al, EPI_BIAS, H)
    if out is None:
        out = torch.empty(T, H, dtype=torch.bfloat16, device=x.device)
    if combine_fn is not None and combine_fn(out, y, al.inv_map[: T * K], topk_w):
        return out
    moe_combine(out, y, al.inv_map, topk_w)
    return out


def _unarrange_rows(w: torch.Tensor, inter: int, interleaved: bool) -> torch.Tensor:
    order = gated_row_order(inter, interleaved).to(w.device)
    out = torch.empty_like(w)
    out[:, order] = w
    return out


def expert_dense_weights(ew: ExpertWeights, e: int):
    """fp32 (w13 [2I, H] arranged order, w2 [H, I]) of one expert."""
    MT13 = (2 * ew.inter + 127) // 128
    KB13 = (ew.hidden + 127) // 128
    s13 = ew.sfa13[e].view(MT13, KB13, 32, 4, 4).permute(0, 3, 2, 1, 4).reshape(MT13 * 128, KB13 * 4)
    s13 = s13[: 2 * ew.inter, : ew.hidden // 32]
    MT2 = (ew.hidden + 127) // 128
    KB2 = (ew.inter + 127) // 128
    s2 = ew.sfa2[e].view(MT2, KB2, 32, 4, 4).permute(0, 3, 2, 1, 4).reshape(MT2 * 128, KB2 * 4)
    s2 = s2[: ew.hidden, : ew.inter // 32]
    if ew.fp4:
        w13 = dequant_mxfp4(untile_weights(ew.w13[e:e + 1], 2 * ew.inter, ew.hidden // 2)[0], s13)
        w2 = dequant_mxfp4(untile_weights(ew.w2[e:e + 1], ew.hidden, ew.inter // 2)[0], s2)
    else:
        w13 = dequant_mxfp8(untile_weights(ew.w13[e:e + 1], 2 * ew.inter, ew.hidden)[0], s13)
        w2 = dequant_mxfp8(untile_weights(ew.w2[e:e + 1], ew.hidden, ew.inter)[0], s2)
    return w13, w2


def fused_moe_ref(x, topk_w, topk_ids, ew: ExpertWeights, activation="swiglu_clamp", alpha=1.702, limit=7.0,
                  e_lo=0, quant_act=False, out=None):
    """fp32 reference of fused_moe. quant_act=True applies the kernel's MXFP8 activation rounding."""
    T, H = x.shape
    res = torch.zeros(T, H, dtype=torch.float32, device=x.device)
    xf = x.float()
    if quant_act:
        xf = dequant_mxfp8(*quant_mxfp8_ref(xf))
    ids = topk_ids.long()
    for e in range(ew.num_experts):
        tok, slot = torch.nonzero(ids == e + e_lo, as_tuple=True)
        if tok.numel() == 0:
            continue
        w13, w2 = expert_dense_weights(ew, e)
        h = xf[tok] @ w13.t()
        if ew.b13 is not None:
            h = h + ew.b13[e].float()
        h = h.view(-1, ew.inter // 64, 2, 64)
        g, u = h[:, :, 0, :].reshape(-1, ew.inter), h[:, :, 1, :].reshape(-1, ew.inter)
        if activation == "swiglu_clamp":
            g = g.clamp(max=limit)
            u = u.clamp(-limit, limit)
            a = (u + 1) * (g * torch.sigmoid(g * alpha))
        else:
            a = torch.nn.functional.silu(g) * u
        a = a.to(torch.bfloat16).float()
        if quant_act:
            a = dequant_mxfp8(*quant_mxfp8_ref(a))
        y = a @ w2.t()
        if ew.b2 is not None:
            y = y + ew.b2[e].float()
        y = y.to(torch.bfloat16).float()
        res.index_add_(0, tok, y * topk_w[tok, slot].float()[:, None])
    r = res.to(x.dtype)
    if out is not None:
        out.copy_(r)
        return out
    return r
