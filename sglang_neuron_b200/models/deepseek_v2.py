"""DeepSeek-V2 / V2-Lite: multi-head latent attention (absorbed form) over a paged latent KV pool, MoE with
shared experts and a dense first layer.

Parity: sglang_neuron/models/deepseek_v2/model.py. `_project` (:101) builds q, the compact latent row
[kv_a_layernorm(c) || rope(k_pe)] (576 wide for V2-Lite) and q_nope . W_UK (the absorption); `_output` (:113)
multiplies the attended latent by W_UV, then o_proj and one all-reduce. On the GPU the latent row and the
query rope are one kernel (csrc/kernels/mla_rope.cu) and both absorptions are grouped tcgen05 GEMMs (every
head in one launch); the CPU tier keeps the PyTorch form as the oracle. The shared experts' TP partial is
summed with the routed partials in one all-reduce (:158-190). YaRN with mscale (config.py:56-80).
"""
from __future__ import annotations

import math

import torch
from torch import nn

from ..layers.linear import ColumnParallelLinear, ReplicatedLinear, RowParallelLinear
from ..model_executor.forward_batch import ForwardBatch
from ..ops.mla import mla_attention, mla_write_rows
from ..ops.rope import apply_rope_ref, yarn_get_mscale
from ..parallel.state import get_state
from .common import CausalLM, DecoderLayer, DenseMLP, MoEBlock, RMSNorm, RotaryCache


class MLAAttention(nn.Module):
    def __init__(self, cfg, layer_id: int, dtype, device, max_pos: int):
        super().__init__()
        st = get_state()
        self.cfg = cfg
        self.layer_id = layer_id
        self.num_heads = cfg.num_heads // st.tp_size
        self.num_kv_heads = 1
        self.nope, self.rope, self.vd, self.r = (cfg.qk_nope_head_dim, cfg.qk_rope_head_dim, cfg.v_head_dim,
                                                 cfg.kv_lora_rank)
        self.head_dim = self.r + self.rope  # latent row width (the kernels' "head dim")
        self.q_proj = ColumnParallelLinear(cfg.hidden_size, cfg.num_heads * (self.nope + self.rope), dtype=dtype,
                                           device=device)
        self.kv_a_proj = ReplicatedLinear(cfg.hidden_size, self.r + self.rope, dtype=dtype, device=device)
        self.kv_a_layernorm = RMSNorm(self.r, cfg.rms_norm_eps, dtype, device)
        # absorbed projections, per local head: W_UK [H, nope, r], W_UV [H, vd, r]
        self.w_uk = nn.Parameter(torch.zeros(self.num_heads, self.nope, self.r, dtype=dtype, device=device),
                                 requires_grad=False)
        self.w_uv = nn.Parameter(torch.zeros(self.num_heads, self.vd, self.r, dtype=dtype, device=device),
                                 requires_grad=False)
        self.o_proj = RowParallelLinear(cfg.num_heads * self.vd, cfg.hidden_size, dtype=dtype, device=device)
        scaling = (self.nope + self.rope) ** -0.5
        rs = cfg.rope_scaling or {}
        if rs.get("mscale_all_dim"):
            m = yarn_get_mscale(float(rs["factor"]), float(rs["mscale_all_dim"]))
            scaling = scaling * m * m
        self.scaling = scaling
        self.window = 0
        self.cos_sin = RotaryCache.get(cfg, device, max_pos)
        self.kv_pool = None
        self.backend = None
        self._uk = self._uv = None  # tiled absorption weights (CUDA, set at load)

    def sinks_f32(self):
        return None

    def kv_cache(self):
        return self.kv_pool.kv(self.layer_id)

    def _native(self, h: torch.Tensor) -> bool:
        kc = self.kv_pool.kv(self.layer_id)[0] if self.kv_pool is not None else None
        return (h.is_cuda and h.dtype == torch.bfloat16 and self._uk is not None and kc is not None
                and kc.dtype == torch.bfloat16 and self.rope % 2 == 0 and self.cos_sin.shape[1] == self.rope)

    def _forward_native(self, h: torch.Tensor, fb: ForwardBatch, norm=None) -> torch.Tensor:
        """Every step of the absorbed attention on sm_100a kernels: the latent row (norm + rope) and rope(q_pe)
        in one kernel, q_nope . W_UK and o_latent . W_UV as grouped tcgen05 GEMMs (one launch each, all heads),
        written straight into the query rows / the o_proj input."""
        from .._ext import kernels
        from ..ops.gemm import _status_buf
        T, H = h.shape[0], self.num_heads
        q = self.q_proj(h)                     # [T, H * (nope + rope)]
        kv_a = self.kv_a_proj(h)               # [T, r + rope]
        kc, _ = self.kv_cache()
        dcp = getattr(self.kv_pool, "dcp", None)
        loc = dcp.local(fb)[1] if dcp is not None else fb.out_cache_loc
        qf = torch.empty(T, H * (self.r + self.rope), dtype=h.dtype, device=h.device)
        k = kernels()
        k.mla_rope_latent(kv_a, q, H, self.nope, self.r, self.rope, self.kv_a_layernorm.weight,
                          self.kv_a_layernorm.eps, fb.positions, self.cos_sin, bool(self.cfg.rope_neox), kc, loc,
                          self.kv_pool.page_size, qf)
        st = _status_buf(h.device)
        k.gemm_bf16_grouped(qf, q, self._uk.data, H * self.r, st, self.nope, self.r, self.nope + self.rope, self.r,
                            self.r + self.rope)
        qf = qf.view(T, H, self.r + self.rope)
        if dcp is not None:
            from ..parallel.dcp import dcp_mla_attention
            o_lat = dcp_mla_attention(qf, kc, fb, self.r, self.scaling, self.kv_pool.page_size, dcp)
        else:
            o_lat = mla_attention(qf, kc, fb, self.r, self.scaling, self.kv_pool.page_size)  # [T, H, r]
        o = torch.empty(T, H * self.vd, dtype=h.dtype, device=h.device)
        k.gemm_bf16_grouped(o, o_lat.reshape(T, H * self.r), self._uv.data, H * self.vd, st, self.r, self.vd, self.r,
                            0, 0)
        return self.o_proj(o, norm=norm)

    def forward(self, h: torch.Tensor, fb: ForwardBatch, norm=None) -> torch.Tensor:
        if self._native(h):
            return self._forward_native(h, fb, norm)
        T = h.shape[0]
        q = self.q_proj(h).view(T, self.num_heads, self.nope + self.rope)
        kv_a = self.kv_a_proj(h)
        c = self.kv_a_layernorm(kv_a[:, : self.r].contiguous())
        k_pe = kv_a[:, self.r:].reshape(T, 1, self.rope)
        q_pe = apply_rope_ref(q[:, :, self.nope:], fb.positions, self.cos_sin, self.rope, False).to(h.dtype)
        k_pe = apply_rope_ref(k_pe, fb.positions, self.cos_sin, self.rope, False).to(h.dtype)
        latent_row = torch.cat([c, k_pe.view(T, self.rope)], dim=-1)
        kc, _ = self.kv_cache()
        dcp = getattr(self.kv_pool, "dcp", None)
        # under decode context parallelism only the owner rank of a token's page stores its row
        loc = dcp.local(fb)[1] if dcp is not None else fb.out_cache_loc
        mla_write_rows(kc, latent_row, loc, self.kv_pool.page_size)
        # absorption: q_lat[t,h,:] = q_nope[t,h,:] @ W_UK[h]
        q_lat = torch.einsum("thn,hnr->thr", q[:, :, : self.nope].float(), self.w_uk.float()).to(h.dtype)
        qf = torch.cat([q_lat, q_pe], dim=-1)  # [T, H, r + rope]
        if dcp is not None:
            from ..parallel.dcp import dcp_mla_attention
            o_lat = dcp_mla_attention(qf, kc, fb, self.r, self.scaling, self.kv_pool.page_size, dcp)
        else:
            o_lat = mla_attention(qf, kc, fb, self.r, self.scaling, self.kv_pool.page_size)  # [T, H, r]
        o = torch.einsum("thr,hvr->thv", o_lat.float(), self.w_uv.float()).to(h.dtype)
        return self.o_proj(o.reshape(T, self.num_heads * self.vd), norm=norm)

    def load(self, get):
        st = get_state()
        p = f"model.layers.{self.layer_id}.self_attn."
        self.q_proj.load(get(p + "q_proj.weight"))
        self.kv_a_proj.load(get(p + "kv_a_proj_with_mqa.weight"))
        self.kv_a_layernorm.weight.data.copy_(get(p + "kv_a_layernorm.weight"))
        kv_b = get(p + "kv_b_proj.weight").view(self.cfg.num_heads, self.nope + self.vd, self.r)
        h0 = st.tp_rank * self.num_heads
        kv_b = kv_b[h0:h0 + self.num_heads]
        self.w_uk.data.copy_(kv_b[:, : self.nope])
        self.w_uv.data.copy_(kv_b[:, self.nope:])
        self.o_proj.load(get(p + "o_proj.weight"))
        if self.w_uk.is_cuda and self.w_uk.dtype == torch.bfloat16:
            # the grouped GEMMs' weights: W_UK^T rows (head, latent col) over nope, W_UV rows (head, v) over r
            from ..ops.gemm import TiledWeight
            H = self.num_heads
            self._uk = TiledWeight(self.w_uk.data.transpose(1, 2).reshape(H * self.r, self.nope).contiguous())
            self._uv = TiledWeight(self.w_uv.data.reshape(H * self.vd, self.r).contiguous())


class DeepseekV2ForCausalLM(CausalLM):
    @property
    def graph_capturable(self) -> bool:
        """Decode runs the tensor-core MLA kernel (no host work) when the latent pool is bf16 on a GPU."""
        a = self.attention_layers()[0]
        return (self.device.type == "cuda" and a.kv_pool is not None and a.kv_pool.dtype == torch.bfloat16
                and a.r == 512 and a.rope == 64)

    def make_layer(self, i: int) -> DecoderLayer:
        cfg = self.cfg
        attn = MLAAttention(cfg, i, self.dtype, self.device, self.max_pos)
        if cfg.is_moe_layer(i):
            shared = cfg.moe_intermediate_size * cfg.n_shared_experts
            mlp = MoEBlock(cfg, i, self.dtype, self.device, shared_inter=shared)
        else:
            mlp = DenseMLP(cfg.hidden_size, cfg.intermediate_size, self.dtype, self.device)
        return DecoderLayer(cfg, i, self.dtype, self.device, self.max_pos, attn=attn, mlp=mlp)

    def load_layers(self, get) -> None:
        for l in self.layers:
            l.self_attn.load(get)
            p = f"model.layers.{l.layer_id}.mlp."
            if isinstance(l.mlp, MoEBlock):
                m = l.mlp
                m.router.load(get(p + "gate.weight"))
                rng = range(m.e_lo, m.e_lo + m.e_local)
                w13 = torch.stack([torch.cat([get(f"{p}experts.{e}.gate_proj.weight"),
                                              get(f"{p}experts.{e}.up_proj.weight")], 0) for e in rng])
                w2 = torch.stack([get(f"{p}experts.{e}.down_proj.weight") for e in rng])
                m.set_experts_from_dense(w13.float(), w2.float())
                if m.shared is not None:
                    m.shared.load(get, p + "shared_experts.")
            else:
                l.mlp.load(get, p)
