"""Token sampling: greedy argmax (ties to the smallest id) and temperature sampling by Gumbel-max with
noise that is a pure function of (seed, position, token id)."""
from typing import Optional

import numpy as np
import torch

from .._ext import kernels

_M64 = (1 << 64) - 1


def _mix64(z: np.ndarray) -> np.ndarray:
    z = (z + np.uint64(0x9E3779B97F4A7C15)) & np.uint64(_M64)
    z = ((z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)) & np.uint64(_M64)
    z = ((z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)) & np.uint64(_M64)
    return z ^ (z >> np.uint64(31))


def gumbel_noise_ref(seed: int, pos: int, vocab: int) -> torch.Tensor:
    """Same construction as the kernel: u from the top 24 bits of a 64-bit mix, g = -log(-log(u))."""
    with np.errstate(over="ignore"):
        tok = np.arange(vocab, dtype=np.uint64)
        inner = _mix64(np.uint64(pos % (1 << 64)) * np.uint64(0x100000001B3) ^ _mix64(tok))
        h = _mix64(np.uint64(seed % (1 << 64)) ^ inner)
    u = ((h >> np.uint64(40)).astype(np.float64) + 0.5) / 16777216.0
    return torch.from_numpy(-np.log(-np.log(u))).float()


def sample_ref(logits: torch.Tensor, temperature: Optional[torch.Tensor] = None,
               seeds: Optional[torch.Tensor] = None, positions: Optional[torch.Tensor] = None,
               vocab_offset: int = 0, valid_vocab: int = 0, return_vals: bool = False):
    B = logits.shape[0]
    V = valid_vocab if valid_vocab > 0 else logits.shape[1]
    out = torch.empty(B, dtype=torch.long)
    vals = torch.empty(B, dtype=torch.float32)
    lf = logits[:, :V].float().cpu()
    for b in range(B):
        t = float(temperature[b]) if temperature is not None else 0.0
        row = lf[b]
        if t > 0:
            s = int(seeds[b]) if seeds is not None else 0
            p = int(positions[b]) if positions is not None else 0
            row = row / t + gumbel_noise_ref(s, p, V + vocab_offset)[vocab_offset:]
        m = row.max()
        out[b] = int(torch.nonzero(row == m)[0, 0]) + vocab_offset
        vals[b] = m
    if return_vals:
        return out.to(logits.device), vals.to(logits.device)
    return out.to(logits.device)


def sample_tokens(logits: torch.Tensor, temperature: Optional[torch.Tensor] = None,
                  seeds: Optional[torch.Tensor] = None, positions: Optional[torch.Tensor] = None,
                  out: Optional[torch.Tensor] = None, out_vals: Optional[torch.Tensor] = None,
                  vocab_offset: int = 0, valid_vocab: int = 0) -> torch.Tensor:
    if not logits.is_cuda:
        r, v = sample_ref(logits, temperature, seeds, positions, vocab_offset, valid_vocab, return_vals=True)
        if out_vals is not None:
            out_vals.copy_(v)
        if out is not None:
            out.copy_(r)
            return out
        return r
    if out is None:
        out = torch.empty(logits.shape[0], dtype=torch.long, device=logits.device)
    kernels().sample_tokens(out, logits, temperature, seeds, positions, out_vals, vocab_offset, valid_vocab)
    return out


def apply_top_k_top_p(logits: torch.Tensor, top_k: torch.Tensor, top_p: torch.Tensor) -> torch.Tensor:
    """Mask logits outside each row's top-k / nucleus top-p set to -inf (rows with k<=0 and p>=1 untouched)."""
    sorted_l, idx = logits.float().sort(dim=-1, descending=True)
    V = logits.shape[-1]
    ar = torch.arange(V, device=logits.device)[None, :]
    k = torch.where(top_k > 0, top_k, torch.full_like(top_k, V))
    mask = ar >= k[:, None]
    probs = sorted_l.softmax(-1)
    cum = probs.cumsum(-1) - probs
    mask |= cum > top_p[:, None].float()
    sorted_l = sorted_l.masked_fill(mask, float("-inf"))
    out = torch.empty_like(sorted_l).scatter_(-1, idx, sorted_l)
    return out.to(logits.dtype)


# ---- filtered sampling over a candidate pool ---------------------------------------------------------------
# Parity: the reference's topk_topp mode (sglang_neuron/sampling.py:337 sample_filtered_sharded_logits,
# sampling_topk.py): every vocabulary shard proposes its top-256 logits, one gather merges them, the filters
# and the Gumbel-max draw run on the 256-candidate pool. Top-k is exact for k <= 256; top-p is exact whenever
# the nucleus lies inside the pool.

POOL = 256
_C1 = 0x9E3779B97F4A7C15
_C2 = 0xBF58476D1CE4E5B9
_C3 = 0x94D049BB133111EB
_C4 = 0x100000001B3


def _i64(c: int) -> int:
    return c - (1 << 64) if c >= (1 << 63) else c


def _shr(z: torch.Tensor, s: int) -> torch.Tensor:
    """Logical right shift of int64 bit patterns."""
    return (z >> s) & ((1 << (64 - s)) - 1)


def _mix64_t(z: torch.Tensor) -> torch.Tensor:
    z = z + _i64(_C1)
    z = (z ^ _shr(z, 30)) * _i64(_C2)
    z = (z ^ _shr(z, 27)) * _i64(_C3)
    return z ^ _shr(z, 31)


def gumbel_noise_ids(seeds: torch.Tensor, positions: torch.Tensor, ids: torch.Tensor) -> torch.Tensor:
    """Gumbel noise of the listed token ids: the same function of (seed, position, token id) as the device
    sampler and gumbel_noise_ref. seeds/positions: [B]; ids: [B, N] -> [B, N] fp32."""
    tok = ids.long()
    inner = _mix64_t((positions.long()[:, None] * _i64(_C4)) ^ _mix64_t(tok))
    h = _mix64_t(seeds.long()[:, None] ^ inner)
    u = (_shr(h, 40).double() + 0.5) / 16777216.0
    return (-torch.log(-torch.log(u))).float()


def sample_filtered(logits: torch.Tensor, temperature: torch.Tensor, top_k: torch.Tensor, top_p: torch.Tensor,
                    seeds: torch.Tensor, positions: torch.Tensor, vocab_offset: int = 0, valid_vocab: int = 0,
                    merge=None, pool: int = POOL) -> torch.Tensor:
    """Top-k / top-p / temperature sampling of (a shard of) logits [B, V_local]. `merge(vals, ids)` combines
    the per-shard candidate pools of a vocabulary-sharded head (returns the merged, descending pool).
    Temperature is applied first; top-k keeps the k best; top-p keeps the smallest prefix of the sorted
    candidates whose probability reaches p; greedy rows (temperature 0) take the best candidate."""
    V = valid_vocab if valid_vocab > 0 else logits.shape[1]
    kp = min(pool, V)
    if logits.is_cuda:
        # radix-select kernel: the row's top-kp (value descending, index ascending), no full-vocabulary sort
        vals = torch.empty(logits.shape[0], kp, dtype=torch.float32, device=logits.device)
        ids = torch.empty(logits.shape[0], kp, dtype=torch.int64, device=logits.device)
        kernels().topk_pool(logits, V, kp, vocab_offset, vals, ids)
    else:
        lf = logits[:, :V].float()
        vals, ids = lf.topk(kp, dim=-1)
        ids = ids + vocab_offset
    if merge is not None:
        vals, ids = merge(vals, ids)
    P = vals.shape[1]
    t = temperature.float()
    s = vals / t.clamp(min=1e-6)[:, None]
    ar = torch.arange(P, device=vals.device)[None, :]
    k = torch.where(top_k > 0, top_k.long(), torch.full_like(top_k.long(), P))
    mask = ar >= k[:, None]
    probs = torch.softmax(s.masked_fill(mask, float("-inf")), dim=-1)
    cum = probs.cumsum(-1) - probs
    mask = mask | (cum >= top_p.float()[:, None])
    mask[:, 0] = False  # the best candidate always survives
    s = s.masked_fill(mask, float("-inf"))
    noisy = s + gumbel_noise_ids(seeds, positions, ids)
    pick = noisy.argmax(dim=-1)
    chosen = ids.gather(1, pick[:, None])[:, 0]
    return torch.where(t > 0, chosen, ids[:, 0]).long()
