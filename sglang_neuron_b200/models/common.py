"""Building blocks shared by the decoder families: RMSNorm, GQA attention over the paged pool, dense and
MoE MLPs, the decoder layer and the causal-LM shell.

Parity (reference layer by layer):
  * attention: sglang_neuron/models/transformer/model.py:95-153 (fused QKV + QK-norm + RoPE + paged write,
    paged attention, o_proj + all-reduce) and models/gpt_oss/mxfp4/common.py:123 (QKV bias, sinks,
    sliding window on alternating layers).
  * dense MLP: models/transformer/model.py:156-173 (gate_up, SiLU*up, down + all-reduce).
  * MoE: models/qwen3_moe/moe.py:20-77 and gpt_oss/mxfp4/common.py:186-363 (replicated router, experts split
    in contiguous blocks by EP rank, one all-reduce of the expert partials).
  * causal LM: models/transformer/model.py:236-252 (vocab-sharded embedding, layers, final norm of the
    sampled rows only, vocab-sharded LM head).
"""
from __future__ import annotations

from typing import Iterable, List, Optional, Tuple

import torch
from torch import nn

from ..configs.model_config import ModelConfig
from ..layers.embedding import ParallelLMHead, VocabParallelEmbedding
from ..layers.linear import (MergedColumnParallelLinear, QKVParallelLinear, ReplicatedLinear,
                             RowParallelLinear)
from ..model_executor.forward_batch import ForwardBatch, ForwardMode
from ..ops import activation as act_ops
from ..ops import moe as moe_ops
from ..ops.norm import fused_add_rmsnorm, rmsnorm
from ..ops.rope import build_cos_sin_cache, rope_qk_norm_kv_write
from ..parallel.collectives import (FusedNorm, deferred_reduction, dp_gather_rows, dp_scatter_rows,
                                    fused_combine_all_reduce, pp_isend_hidden, pp_recv_hidden, pp_send_hidden,
                                    sp_all_gather,
                                    sp_gather_rows, sp_reduce_scatter, tp_all_reduce)
from ..parallel.state import get_state, pp_layer_range
from .. import env_registry

# decode-sized MoE routing in one launch (SGLANG_B200_FUSED_ROUTE=1); off by default, where the router GEMM,
# top-k, align and quantise run as separate launches (faster on a B200: 20 us against 27 us per layer)
_FUSED_ROUTE = env_registry.get_bool("SGLANG_B200_FUSED_ROUTE", False)


class RMSNorm(nn.Module):
    def __init__(self, dim: int, eps: float, dtype=torch.bfloat16, device=None):
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(dim, dtype=dtype, device=device), requires_grad=False)

    def forward(self, x: torch.Tensor, residual: Optional[torch.Tensor] = None):
        if residual is None:
            return rmsnorm(x, self.weight, self.eps)
        return fused_add_rmsnorm(x, residual, self.weight, self.eps)


class RotaryCache:
    """cos/sin table shared by all layers of a model (one per device)."""

    _cache = {}

    @classmethod
    def get(cls, cfg: ModelConfig, device, max_pos: Optional[int] = None) -> torch.Tensor:
        max_pos = max_pos or cfg.max_position_embeddings
        key = (cfg.rot_dim, max_pos, cfg.rope_theta, str(cfg.rope_scaling), str(device))
        t = cls._cache.get(key)
        if t is None:
            t = build_cos_sin_cache(cfg.rot_dim, max_pos, cfg.rope_theta, cfg.rope_scaling, device)
            cls._cache[key] = t
        return t


class GQAAttention(nn.Module):
    def __init__(self, cfg: ModelConfig, layer_id: int, dtype, device, max_pos: int):
        super().__init__()
        self.cfg = cfg
        self.layer_id = layer_id
        self.head_dim = cfg.head_dim
        self.qkv_proj = QKVParallelLinear(cfg.hidden_size, cfg.head_dim, cfg.num_heads, cfg.num_kv_heads,
                                          bias=cfg.attention_bias, dtype=dtype, device=device)
        self.num_heads = self.qkv_proj.num_heads
        self.num_kv_heads = self.qkv_proj.num_kv_heads
        self.o_proj = RowParallelLinear(cfg.num_heads * cfg.head_dim, cfg.hidden_size, bias=cfg.o_proj_bias,
                                        reduce=True, dtype=dtype, device=device)
        self.q_norm = RMSNorm(cfg.head_dim, cfg.rms_norm_eps, dtype, device) if cfg.qk_norm else None
        self.k_norm = RMSNorm(cfg.head_dim, cfg.rms_norm_eps, dtype, device) if cfg.qk_norm else None
        self.window = cfg.layer_window(layer_id)
        self.scaling = cfg.head_dim ** -0.5
        self.sinks = (nn.Parameter(torch.zeros(self.num_heads, dtype=torch.float32, device=device),
                                   requires_grad=False) if cfg.attention_sinks else None)
        self.cos_sin = RotaryCache.get(cfg, device, max_pos)
        self.kv_pool = None
        self.backend = None

    def sinks_f32(self):
        return self.sinks

    def kv_cache(self):
        return self.kv_pool.kv(self.layer_id)

    def forward(self, h: torch.Tensor, fb: ForwardBatch, norm=None) -> torch.Tensor:
        qkv = self.qkv_proj(h)
        qs, kvs = self.qkv_proj.q_size, self.qkv_proj.kv_size
        q = qkv[:, :qs]
        k = qkv[:, qs:qs + kvs]
        v = qkv[:, qs + kvs:]
        kc, vc = self.kv_cache()
        if self.window > 0 and self.kv_pool.swa is not None:
            fb = self.kv_pool.swa.batch(fb)  # block table and write slots in window-pool pages
        rope_qk_norm_kv_write(q, k, v, fb.positions, self.cos_sin, self.num_heads, self.num_kv_heads,
                              self.head_dim, self.cfg.rot_dim, self.cfg.rope_neox,
                              self.q_norm.weight if self.q_norm is not None else None,
                              self.k_norm.weight if self.k_norm is not None else None, self.cfg.rms_norm_eps,
                              kc, vc, fb.out_cache_loc, self.kv_pool.page_size, self.kv_pool.k_scale,
                              self.kv_pool.v_scale)
        o = self.backend.attend(q, self, fb)
        return self.o_proj(o, norm=norm)

    def load(self, get):
        p = f"model.layers.{self.layer_id}.self_attn."
        b = self.cfg.attention_bias
        self.qkv_proj.load(get(p + "q_proj.weight"), get(p + "k_proj.weight"), get(p + "v_proj.weight"),
                           get(p + "q_proj.bias") if b else None, get(p + "k_proj.bias") if b else None,
                           get(p + "v_proj.bias") if b else None)
        self.o_proj.load(get(p + "o_proj.weight"), get(p + "o_proj.bias") if self.cfg.o_proj_bias else None)
        if self.q_norm is not None:
            self.q_norm.weight.data.copy_(get(p + "q_norm.weight"))
            self.k_norm.weight.data.copy_(get(p + "k_norm.weight"))
        if self.sinks is not None:
            st = get_state()
            s = get(p + "sinks").float()
            self.sinks.data.copy_(s.narrow(0, st.tp_rank * self.num_heads, self.num_heads))


class DenseMLP(nn.Module):
    def __init__(self, hidden: int, inter: int, dtype, device, reduce: bool = True):
        super().__init__()
        self.gate_up = MergedColumnParallelLinear(hidden, [inter, inter], dtype=dtype, device=device)
        self.down = RowParallelLinear(inter, hidden, reduce=reduce, dtype=dtype, device=device)

    def forward(self, x, norm=None):
        return self.down(act_ops.silu_and_mul(self.gate_up(x)), norm=norm)

    def load(self, get, prefix: str):
        self.gate_up.load_part(0, get(prefix + "gate_proj.weight"))
        self.gate_up.load_part(1, get(prefix + "up_proj.weight"))
        self.down.load(get(prefix + "down_proj.weight"))


class MoEBlock(nn.Module):
    """Router (replicated) + this rank's block of experts; partial outputs are all-reduced over EP (=TP).

    Expert weights are kept in the tcgen05 block-scaled layout (ops.moe.ExpertWeights): MXFP4 for
    checkpoints that ship MXFP4 (GPT-OSS), MXFP8 (e4m3 + e8m0 per 32) quantised at load for bf16
    checkpoints (Qwen3-MoE, DeepSeek-V2) - the "block-scaled FP8 expert GEMM" configuration.
    """

    def __init__(self, cfg: ModelConfig, layer_id: int, dtype, device, shared_inter: int = 0):
        super().__init__()
        st = get_state()
        self.cfg = cfg
        self.layer_id = layer_id
        E = cfg.num_experts
        assert E % st.ep_size == 0, "experts must divide over EP ranks"
        self.e_local = E // st.ep_size
        self.e_lo = st.ep_rank * self.e_local
        self.top_k = cfg.num_experts_per_tok
        self.router = ReplicatedLinear(cfg.hidden_size, E, bias=cfg.router_bias, dtype=dtype, device=device)
        self.route_mode = 0 if (cfg.norm_topk_prob or cfg.architecture == "GptOssForCausalLM") else 1
        self.activation = "swiglu_clamp" if cfg.swiglu_limit > 0 else "silu"
        self.experts: Optional[moe_ops.ExpertWeights] = None
        self.shared = DenseMLP(cfg.hidden_size, shared_inter, dtype, device, reduce=False) if shared_inter else None
        self.device = device
        self.alignment_cache = {}

    def route(self, x: torch.Tensor):
        """(topk_w, topk_ids, routed): decode-sized CUDA batches take the one-launch routing kernel (router
        GEMM, top-k, alignment and MXFP8 quantise), whose `routed` result fused_moe consumes directly."""
        E = self.cfg.num_experts
        if (x.is_cuda and _FUSED_ROUTE and self.router._packed is not None and 0 < x.shape[0]
                and x.shape[0] * E <= moe_ops.ROUTE_FUSED_MAX_LOGITS and x.shape[1] % 64 == 0
                and x.stride(1) == 1 and (x.stride(0) * 2) % 16 == 0 and x.data_ptr() % 16 == 0):
            bn = moe_ops.pick_bn(x.shape[0], self.top_k, self.e_local)
            w, ids, al, xq, sfb = moe_ops.fused_route_quant(
                x, self.router._packed, E, self.router.bias, self.top_k, self.route_mode,
                self.cfg.routed_scaling_factor, self.e_lo, self.e_local, bn)
            return w, ids, (al, xq, sfb)
        logits = self.router(x)
        w, ids = moe_ops.topk_route(logits, self.top_k, self.route_mode, self.cfg.routed_scaling_factor)
        return w, ids, None

    def forward(self, x: torch.Tensor, norm=None) -> torch.Tensor:
        w, ids, routed = self.route(x)
        if self.shared is None and x.is_cuda and get_state().tp_size > 1:
            # combine + expert-parallel all-reduce (+ the next residual add and norm) in one NVLink kernel
            reduced = [False]

            def combine(out, y, inv_map, topk_w):
                reduced[0] = fused_combine_all_reduce(out, y, inv_map, topk_w, norm=norm)
                return reduced[0]

            out = moe_ops.fused_moe(x, w, ids, self.experts, self.activation, self.cfg.swiglu_alpha,
                                    self.cfg.swiglu_limit, e_lo=self.e_lo, combine_fn=combine, routed=routed)
            return out if reduced[0] else tp_all_reduce(out, norm=norm)
        out = moe_ops.fused_moe(x, w, ids, self.experts, self.activation, self.cfg.swiglu_alpha,
                                self.cfg.swiglu_limit, e_lo=self.e_lo, routed=routed)
        if self.shared is not None:
            out = out + self.shared(x)
        return tp_all_reduce(out, norm=norm)

    def forward_dp(self, x: torch.Tensor, rows: int) -> torch.Tensor:
        """DP attention: route every group's rows (all-gathered, padded to `rows` per group) through this
        rank's experts, sum the partials over all ranks and keep this group's rows. Shared experts run on the
        group's own rows, reduced over the attention group."""
        n = x.shape[0]
        xa = dp_gather_rows(x, rows)
        logits = self.router(xa)
        w, ids = moe_ops.topk_route(logits, self.top_k, self.route_mode, self.cfg.routed_scaling_factor)
        part = moe_ops.fused_moe(xa, w, ids, self.experts, self.activation, self.cfg.swiglu_alpha,
                                 self.cfg.swiglu_limit, e_lo=self.e_lo)
        y = dp_scatter_rows(part, rows, n)
        if self.shared is not None and n > 0:
            y = y + tp_all_reduce(self.shared(x))
        return y

    # -- weights ------------------------------------------------------------------------------
    def set_experts_from_dense(self, w13: torch.Tensor, w2: torch.Tensor, b13=None, b2=None,
                               interleaved: bool = False):
        """w13: [E_local, 2I, H] (gate rows then up rows unless interleaved), w2: [E_local, H, I] bf16/fp32.
        Quantised here to MXFP8 for the block-scaled grouped GEMM."""
        q13, s13 = moe_ops.quant_mxfp8_ref(w13)
        q2, s2 = moe_ops.quant_mxfp8_ref(w2)
        I = w2.shape[2]
        self.experts = moe_ops.ExpertWeights(q13, s13, b13, q2, s2, b2, self.cfg.hidden_size, I, interleaved)

    def set_experts_mxfp4(self, blocks13, scales13, b13, blocks2, scales2, b2, interleaved: bool = True):
        I = self.cfg.moe_intermediate_size
        self.experts = moe_ops.ExpertWeights(blocks13, scales13, b13, blocks2, scales2, b2, self.cfg.hidden_size, I,
                                             interleaved)


class DecoderLayer(nn.Module):
    def __init__(self, cfg: ModelConfig, layer_id: int, dtype, device, max_pos: int, attn=None, mlp=None):
        super().__init__()
        self.layer_id = layer_id
        self.input_layernorm = RMSNorm(cfg.hidden_size, cfg.rms_norm_eps, dtype, device)
        self.post_attention_layernorm = RMSNorm(cfg.hidden_size, cfg.rms_norm_eps, dtype, device)
        self.self_attn = attn if attn is not None else GQAAttention(cfg, layer_id, dtype, device, max_pos)
        self.mlp = mlp

    def forward(self, h: torch.Tensor, residual: Optional[torch.Tensor], fb: ForwardBatch, sp_rows: int = 0,
                next_norm=None):
        """sp_rows > 0: sequence-parallel step; h and residual are this rank's [sp_rows, H] block of the
        token rows, and the layer returns its block of the next hidden state.

        Under TP the residual add + RMSNorm after each all-reduce is offered to the all-reduce kernel
        (FusedNorm): the attention output comes back already post-attention-normed, and with `next_norm`
        (the next layer's input norm) the MLP output comes back as the next layer's normed input, which
        fb.extra["h_normed"] tells the next layer."""
        if fb.extra.pop("h_normed", False):
            pass  # the previous layer's all-reduce applied this layer's input norm (residual already updated)
        elif residual is None:
            residual = h.clone()
            h = self.input_layernorm(h)
        else:
            h, residual = self.input_layernorm(h, residual)
        dp_rows = fb.extra.get("dp_rows", 0)
        if dp_rows and isinstance(self.mlp, MoEBlock):
            h = self.self_attn(h, fb)
            h, residual = self.post_attention_layernorm(h, residual)
            return self.mlp.forward_dp(h, dp_rows), residual
        if sp_rows:
            T = fb.num_tokens
            with deferred_reduction():
                part = self.self_attn(sp_all_gather(h)[:T], fb)
            h, residual = self.post_attention_layernorm(sp_reduce_scatter(part, sp_rows), residual)
            with deferred_reduction():
                part = self.mlp(sp_all_gather(h)[:T])
            return sp_reduce_scatter(part, sp_rows), residual
        fn = FusedNorm.offer(residual, self.post_attention_layernorm)
        if fn is None:
            h = self.self_attn(h, fb)
            h, residual = self.post_attention_layernorm(h, residual)
        else:
            h = self.self_attn(h, fb, norm=fn)
            if not fn.done:
                h, residual = self.post_attention_layernorm(h, residual)
        fn = FusedNorm.offer(residual, next_norm)
        if fn is None:
            return self.mlp(h), residual
        h = self.mlp(h, norm=fn)
        if fn.done:
            fb.extra["h_normed"] = True
        return h, residual


class CausalLM(nn.Module):
    """Shared shell: embedding -> decoder layers -> final norm on the sampled rows -> vocab-sharded head."""

    graph_capturable = True

    def __init__(self, cfg: ModelConfig, dtype=torch.bfloat16, device="cpu", max_pos: Optional[int] = None):
        super().__init__()
        # prefill steps of at least this many tokens run sequence-parallel between layers (0: never)
        self.sp_min_tokens = 0
        self.cfg = cfg
        self.dtype = dtype
        self.device = torch.device(device)
        self.max_pos = max_pos or min(cfg.max_position_embeddings, 131072)
        st = get_state()
        # pipeline stage: a contiguous block of layers; the embedding on the first stage, the final norm and
        # the LM head on the last
        self.layer_start, self.layer_end = pp_layer_range(cfg.num_layers, st.pp_size, st.pp_rank)
        self.first_stage, self.last_stage = st.is_first_stage, st.is_last_stage
        self.embed_tokens = (VocabParallelEmbedding(cfg.vocab_size, cfg.hidden_size, dtype, device)
                             if self.first_stage else None)
        self.layers = nn.ModuleList([self.make_layer(i) for i in range(self.layer_start, self.layer_end)])
        self.norm = RMSNorm(cfg.hidden_size, cfg.rms_norm_eps, dtype, device) if self.last_stage else None
        self.lm_head = ParallelLMHead(cfg.vocab_size, cfg.hidden_size, dtype, device) if self.last_stage else None

    def make_layer(self, i: int) -> DecoderLayer:  # overridden by families
        raise NotImplementedError

    def attention_layers(self) -> List[nn.Module]:
        return [l.self_attn for l in self.layers]

    def bind_kv_cache(self, pool, backend) -> None:
        """Parity: NeuronModel.bind_kv_cache (sglang_neuron/models/base.py:123) binds pool buffers by layer id."""
        for a in self.attention_layers():
            a.kv_pool = pool
            a.backend = backend

    def sp_rows(self, fb: ForwardBatch) -> int:
        """Rows per TP rank when this step runs sequence-parallel between layers, else 0."""
        st = get_state()
        tp = st.tp_size
        if (tp == 1 or st.attn_dp_size > 1 or self.sp_min_tokens <= 0 or fb.mode != ForwardMode.EXTEND or fb.num_tokens < self.sp_min_tokens
                or (self.device.type == "cuda" and torch.cuda.is_current_stream_capturing())):
            return 0
        return -(-fb.num_tokens // tp)

    def forward(self, fb: ForwardBatch) -> Optional[torch.Tensor]:
        """Sampled rows after the final norm (last pipeline stage), or None on earlier stages (their output
        went to the next stage)."""
        rows = self.sp_rows(fb)
        if rows:
            return self._forward_sp(fb, rows)
        if (get_state().pp_size > 1 and fb.is_decode and fb.spec_tokens == 1 and fb.batch_size > 1
                and fb.num_tokens == fb.batch_size):
            return self._forward_pp_microbatched(fb)
        if self.first_stage:
            h = self.embed_tokens(fb.input_ids)
            residual = None
        else:
            h, residual = pp_recv_hidden(fb.num_tokens, self.cfg.hidden_size, self.dtype, self.device)
        n = len(self.layers)
        for i, layer in enumerate(self.layers):
            # the next layer's input norm rides on this layer's last all-reduce when the kernel can take it
            nxt = self.layers[i + 1].input_layernorm if i + 1 < n else None
            h, residual = layer(h, residual, fb, next_norm=nxt)
        fb.extra.pop("h_normed", None)
        if not self.last_stage:
            if residual is None:
                residual = torch.zeros_like(h)
            pp_send_hidden(h, residual)
            return None
        # only the rows that are sampled go through the final norm and the LM head
        h_last = h.index_select(0, fb.logits_idx)
        r_last = residual.index_select(0, fb.logits_idx)
        h_last, pre = self.norm(h_last, r_last)
        self.last_prenorm = pre  # h + residual of the sampled rows (consumed by the MTP draft head)
        return h_last

    def _forward_pp_microbatched(self, fb: ForwardBatch) -> Optional[torch.Tensor]:
        """Pipeline-parallel decode in micro-batches: the step's requests split into as many micro-batches as
        there are stages; a stage sends micro-batch m to the next one without waiting and goes on with m + 1,
        so the stages work on different micro-batches at the same time (P stages over M micro-batches take
        about (M + P - 1) / M stage-times instead of P). Every row is computed as in the whole batch (same
        split count, row-independent ops), so the tokens are the same. Parity: the reference's overlapped
        PP seam (sglang_neuron/distributed/pp_seam.py:306)."""
        P = get_state().pp_size
        M = min(P, fb.batch_size)
        bounds = [fb.batch_size * m // M for m in range(M + 1)]
        sends, outs = [], []
        n = len(self.layers)
        for m in range(M):
            sub = fb.slice_decode(bounds[m], bounds[m + 1])
            if self.first_stage:
                h, residual = self.embed_tokens(sub.input_ids), None
            else:
                h, residual = pp_recv_hidden(sub.num_tokens, self.cfg.hidden_size, self.dtype, self.device)
            for i, layer in enumerate(self.layers):
                nxt = self.layers[i + 1].input_layernorm if i + 1 < n else None
                h, residual = layer(h, residual, sub, next_norm=nxt)
            if residual is None:
                residual = torch.zeros_like(h)
            if not self.last_stage:
                sends.append(pp_isend_hidden(h, residual))
            else:
                outs.append((h, residual))
        for work, _buf in sends:
            work.wait()
        if not self.last_stage:
            return None
        h = torch.cat([o[0] for o in outs])
        residual = torch.cat([o[1] for o in outs])
        h_last, pre = self.norm(h.index_select(0, fb.logits_idx), residual.index_select(0, fb.logits_idx))
        self.last_prenorm = pre
        return h_last

    def forward_idle(self, rows: int) -> None:
        """DP attention, no requests in this attention group this step: take part in every MoE block's token
        exchange with zero rows, so the groups that do have rows can run."""
        x = torch.zeros(0, self.cfg.hidden_size, dtype=self.dtype, device=self.device)
        for layer in self.layers:
            if isinstance(layer.mlp, MoEBlock):
                layer.mlp.forward_dp(x, rows)

    def _forward_sp(self, fb: ForwardBatch, rows: int) -> Optional[torch.Tensor]:
        """Sequence-parallel forward: the embedding's vocabulary-shard partials are reduce-scattered, every
        layer keeps this rank's block of rows, and the sampled rows are gathered before the final norm."""
        if self.first_stage:
            with deferred_reduction():
                e = self.embed_tokens(fb.input_ids)
            h, residual = sp_reduce_scatter(e, rows), None
        else:
            h, residual = pp_recv_hidden(rows, self.cfg.hidden_size, self.dtype, self.device)
        for layer in self.layers:
            h, residual = layer(h, residual, fb, sp_rows=rows)
        if not self.last_stage:
            pp_send_hidden(h, torch.zeros_like(h) if residual is None else residual)
            return None
        pre = sp_gather_rows(h if residual is None else h + residual, fb.logits_idx, rows)
        self.last_prenorm = pre
        return self.norm(pre)

    def compute_logits(self, h_last: torch.Tensor) -> torch.Tensor:
        return self.lm_head(h_last)

    # -- weights ------------------------------------------------------------------------------
    def load_common(self, get) -> None:
        if self.embed_tokens is not None:
            self.embed_tokens.load(get("model.embed_tokens.weight"))
        if self.last_stage:
            self.norm.weight.data.copy_(get("model.norm.weight"))
            if self.cfg.tie_word_embeddings:
                self.lm_head.load(get("model.embed_tokens.weight"))
            else:
                self.lm_head.load(get("lm_head.weight"))
        for l in self.layers:
            p = f"model.layers.{l.layer_id}."
            l.input_layernorm.weight.data.copy_(get(p + "input_layernorm.weight"))
            l.post_attention_layernorm.weight.data.copy_(get(p + "post_attention_layernorm.weight"))

    def load_weights(self, weights: Iterable[Tuple[str, torch.Tensor]]) -> None:
        table = dict(weights)

        def get(name):
            if name not in table:
                raise KeyError(f"checkpoint tensor {name!r} missing")
            return table[name].to(self.device)

        self.load_common(get)
        self.load_layers(get)

    def load_layers(self, get) -> None:
        raise NotImplementedError
