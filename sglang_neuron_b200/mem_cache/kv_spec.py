"""The model's KV layout, declared before any pool is built.

Every attention layer of the running stage gets a `LayerSpec`: its kind (full attention, sliding window,
latent MLA row), window, KV heads and head width, and the pool that holds it (`main`, or `window` for the
sliding layers of a hybrid sliding-window layout). `KVSpec` adds the page size, the KV dtype and the
decode-context-parallel split; the model runner sizes and builds its pools from it, and every rank checks
that its declaration matches the others' before allocating (a rank with a different layout would exchange
pages or run collectives with mismatched shapes).

Parity: the reference's `KVLayout` / `declare` (sglang_neuron/model_executor/kv_layout.py:12,45: paired
layers, token CP size, zero-fresh pages, allocator class declared before pools) and `LayerSpec` / `KVSpec`
(sglang_neuron/mem_cache/kv_cache.py:11,16).
"""
from __future__ import annotations

import dataclasses
import hashlib
import json
from typing import List, Tuple


@dataclasses.dataclass(frozen=True)
class LayerSpec:
    layer_id: int
    kind: str          # "full" | "sliding" | "latent"
    window: int        # tokens attended (0: whole context)
    kv_heads: int      # KV heads held by this rank (1 for a latent row)
    head_dim: int      # K/V head width, or the latent row width (kv_lora + rope)
    pool: str          # "main" | "window"


@dataclasses.dataclass(frozen=True)
class KVSpec:
    page_size: int
    dtype: str
    dcp_size: int
    layers: Tuple[LayerSpec, ...]

    def pool_layers(self, pool: str) -> List[int]:
        return [l.layer_id for l in self.layers if l.pool == pool]

    @property
    def is_latent(self) -> bool:
        return any(l.kind == "latent" for l in self.layers)

    @property
    def max_window(self) -> int:
        return max((l.window for l in self.layers if l.pool == "window"), default=0)

    def digest(self) -> str:
        blob = json.dumps(dataclasses.asdict(self), sort_keys=True).encode()
        return hashlib.sha256(blob).hexdigest()[:16]


def declare(cfg, attn_layers, page_size: int, kv_dtype, hybrid_swa: bool, dcp_size: int = 1,
            extra_layer_ids=()) -> KVSpec:
    """The stage's KV layout from its attention layers (`extra_layer_ids`: layers outside the model list
    that share the pool, e.g. the MTP draft block, declared as full layers)."""
    specs = []
    for a in attn_layers:
        if cfg.is_mla:
            specs.append(LayerSpec(a.layer_id, "latent", 0, 1, cfg.kv_lora_rank + cfg.qk_rope_head_dim, "main"))
            continue
        w = int(getattr(a, "window", 0) or 0)
        kind = "sliding" if w > 0 else "full"
        specs.append(LayerSpec(a.layer_id, kind, w, a.num_kv_heads, cfg.head_dim,
                               "window" if (hybrid_swa and w > 0) else "main"))
    for lid in extra_layer_ids:
        ref = specs[0]
        specs.append(LayerSpec(lid, ref.kind if ref.kind == "latent" else "full", 0, ref.kv_heads, ref.head_dim,
                               "main"))
    return KVSpec(page_size, str(kv_dtype).replace("torch.", ""), dcp_size, tuple(specs))


def phase(role: str) -> str:
    """Graph family a serving role runs: aggregated servers run both phases. Parity: the reference's
    models/phase.py:5."""
    return {"aggregated": "all", "null": "all", "prefill": "prefill", "decode": "decode"}[role]
