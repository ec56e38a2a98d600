"""Rotary embedding tables (default, YaRN) and the fused QK-norm + RoPE + paged K/V write op."""
import math
from typing import Optional

import torch

from .._ext import kernels
from .gemm import _status_buf


def _yarn_find_correction_dim(num_rotations, dim, base, max_pos):
    return (dim * math.log(max_pos / (num_rotations * 2 * math.pi))) / (2 * math.log(base))


def yarn_get_mscale(scale: float = 1.0, mscale: float = 1.0) -> float:
    if scale <= 1.0:
        return 1.0
    return 0.1 * mscale * math.log(scale) + 1.0


def rope_inv_freq(rot_dim: int, base: float, scaling: Optional[dict]):
    """Return (inv_freq [rot_dim/2] fp64 tensor, attention_factor applied to cos/sin)."""
    idx = torch.arange(0, rot_dim, 2, dtype=torch.float64) / rot_dim
    pos_freqs = base ** idx
    inv = 1.0 / pos_freqs
    if not scaling:
        return inv, 1.0
    kind = scaling.get("rope_type", scaling.get("type", "default"))
    if kind in ("default", None):
        return inv, 1.0
    if kind == "linear":
        return inv / float(scaling["factor"]), 1.0
    if kind == "yarn":
        factor = float(scaling["factor"])
        orig = int(scaling.get("original_max_position_embeddings", 4096))
        beta_fast = float(scaling.get("beta_fast", 32.0))
        beta_slow = float(scaling.get("beta_slow", 1.0))
        truncate = bool(scaling.get("truncate", True))
        low = _yarn_find_correction_dim(beta_fast, rot_dim, base, orig)
        high = _yarn_find_correction_dim(beta_slow, rot_dim, base, orig)
        if truncate:
            low, high = math.floor(low), math.ceil(high)
        low, high = max(low, 0), min(high, rot_dim - 1)
        if low == high:
            high += 0.001
        ramp = ((torch.arange(rot_dim // 2, dtype=torch.float64) - low) / (high - low)).clamp(0, 1)
        extrap = 1.0 - ramp
        inv = (inv / factor) * (1 - extrap) + inv * extrap
        if "attention_factor" in scaling and scaling["attention_factor"] is not None:
            att = float(scaling["attention_factor"])
        elif "mscale" in scaling and "mscale_all_dim" in scaling:
            att = yarn_get_mscale(factor, float(scaling["mscale"])) / yarn_get_mscale(
                factor, float(scaling["mscale_all_dim"]))
        else:
            att = yarn_get_mscale(factor)
        return inv, att
    if kind == "llama3":
        factor = float(scaling["factor"])
        lf = float(scaling.get("low_freq_factor", 1.0))
        hf = float(scaling.get("high_freq_factor", 4.0))
        orig = int(scaling.get("original_max_position_embeddings", 8192))
        low_wl, high_wl = orig / lf, orig / hf
        wl = 2 * math.pi / inv
        out = torch.where(wl > low_wl, inv / factor, inv)
        smooth = (orig / wl - lf) / (hf - lf)
        mid = (1 - smooth) * out / factor + smooth * out
        is_mid = (wl <= low_wl) & (wl >= high_wl)
        return torch.where(is_mid, mid, out), 1.0
    raise ValueError(f"unsupported rope scaling type {kind!r}")


def build_cos_sin_cache(rot_dim: int, max_pos: int, base: float, scaling: Optional[dict] = None,
                        device="cpu") -> torch.Tensor:
    """[max_pos, rot_dim] fp32: cos in the first rot_dim/2 columns, sin in the rest."""
    inv, att = rope_inv_freq(rot_dim, base, scaling)
    t = torch.arange(max_pos, dtype=torch.float64)
    freqs = torch.outer(t, inv)
    cache = torch.cat([freqs.cos() * att, freqs.sin() * att], dim=-1).float()
    return cache.to(device)


def apply_rope_ref(x: torch.Tensor, positions: torch.Tensor, cos_sin: torch.Tensor, rot_dim: int,
                   neox: bool) -> torch.Tensor:
    """x: [T, H, D] (any float dtype); returns fp32 result."""
    xf = x.float()
    half = rot_dim // 2
    cs = cos_sin[positions.long()]  # [T, rot_dim]
    cos = cs[:, None, :half]
    sin = cs[:, None, half:]
    out = xf.clone()
    if neox:
        x1 = xf[..., :half]
        x2 = xf[..., half:rot_dim]
        out[..., :half] = x1 * cos - x2 * sin
        out[..., half:rot_dim] = x2 * cos + x1 * sin
    else:
        x1 = xf[..., 0:rot_dim:2]
        x2 = xf[..., 1:rot_dim:2]
        out[..., 0:rot_dim:2] = x1 * cos - x2 * sin
        out[..., 1:rot_dim:2] = x2 * cos + x1 * sin
    return out


def _write_cache_ref(cache: torch.Tensor, vals: torch.Tensor, slots: torch.Tensor, page_size: int,
                     scale: float):
    # cache: [pages, Hkv, page, D]; vals: [T, Hkv, D]
    keep = slots >= 0
    if not bool(keep.any()):
        return
    s = slots[keep].long()
    v = vals[keep].float()
    if cache.dtype == torch.float8_e4m3fn:
        v = (v / scale).clamp(-448.0, 448.0)
    page = s // page_size
    off = s % page_size
    cache[page, :, off, :] = v.to(cache.dtype)


def rope_qk_norm_kv_write(q, k, v, positions, cos_sin, num_q_heads, num_kv_heads, head_dim, rot_dim,
                          neox=True, q_norm_w=None, k_norm_w=None, norm_eps=1e-6, k_cache=None,
                          v_cache=None, slots=None, page_size=1, k_scale=1.0, v_scale=1.0):
    """In place on q [T, Hq*D] and k [T, Hkv*D] views; writes k (post-RoPE) and v into the paged cache."""
    T = q.shape[0]
    if T == 0:
        return
    if q.is_cuda:
        empty = torch.empty(0, device=q.device, dtype=q.dtype)
        kernels().rope_qk_norm_kv_write(
            q, k, v, positions, cos_sin, num_q_heads, num_kv_heads, head_dim, rot_dim, neox, q_norm_w, k_norm_w,
            norm_eps, k_cache if k_cache is not None else empty, v_cache if v_cache is not None else empty,
            slots if slots is not None else torch.full((T,), -1, dtype=torch.long, device=q.device),
            page_size, k_scale, v_scale, status=_status_buf(q.device))
        return
    from .norm import rmsnorm_ref
    qv = q.reshape(T, num_q_heads, head_dim)
    kv = k.reshape(T, num_kv_heads, head_dim)
    qf = qv.float()
    kf = kv.float()
    if q_norm_w is not None:
        qf = rmsnorm_ref(qf, q_norm_w.float(), norm_eps)
    if k_norm_w is not None:
        kf = rmsnorm_ref(kf, k_norm_w.float(), norm_eps)
    qf = apply_rope_ref(qf, positions, cos_sin, rot_dim, neox)
    kf = apply_rope_ref(kf, positions, cos_sin, rot_dim, neox)
    q.copy_(qf.to(q.dtype).view(T, -1))
    k.copy_(kf.to(k.dtype).view(T, -1))
    if k_cache is not None and k_cache.numel() > 0 and slots is not None:
        _write_cache_ref(k_cache, k.reshape(T, num_kv_heads, head_dim), slots, page_size, k_scale)
        _write_cache_ref(v_cache, v.reshape(T, num_kv_heads, head_dim), slots, page_size, v_scale)
