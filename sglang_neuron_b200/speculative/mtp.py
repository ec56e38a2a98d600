"""MTP speculative decoding: a one-layer multi-token-prediction draft head proposes k tokens, the target
model verifies them in one forward over k+1 rows per request, and the longest greedy-agreeing prefix plus
one bonus token is accepted.

Parity: the reference's `NEURON_MTP` algorithm (sglang_neuron/speculative/neuron_mtp.py: one device step
verifies the previous drafts, accepts, drafts the next ones) and GLM-5.2's MTP draft chain. The draft head
follows the DeepSeek MTP module: x = eh_proj([enorm(embed(token)) || hnorm(h_prev)]) -> one decoder block ->
shared LM head; `h_prev` is the target's (pre-final-norm) hidden state of the previous position, or the
draft's own for later draft steps. The draft block keeps its KV in one extra layer of the target's paged
pool (same page table, same slots), written at the position of its input token.

Greedy decoding only: the accepted tokens are exactly the target's greedy tokens, so outputs equal plain
decoding token for token (the tests check this).
"""
from __future__ import annotations

import dataclasses
import logging
from typing import Dict, List, Optional, Tuple

import numpy as np
import torch
from torch import nn

from ..layers.linear import ReplicatedLinear
from ..model_executor.forward_batch import ForwardBatch, ForwardMode
from ..models.common import RMSNorm

logger = logging.getLogger(__name__)


class MTPDraftHead(nn.Module):
    """DeepSeek-style MTP module; its decoder block is built by the target family (layer id = num_layers)."""

    def __init__(self, target, dtype, device):
        super().__init__()
        cfg = target.cfg
        H = cfg.hidden_size
        self.layer_id = cfg.num_layers
        self.enorm = RMSNorm(H, cfg.rms_norm_eps, dtype, device)
        self.hnorm = RMSNorm(H, cfg.rms_norm_eps, dtype, device)
        self.eh_proj = ReplicatedLinear(2 * H, H, dtype=dtype, device=device)
        self.block = target.make_layer(self.layer_id)
        self.head_norm = RMSNorm(H, cfg.rms_norm_eps, dtype, device)
        self.target = target

    def forward(self, tokens: torch.Tensor, h_prev: torch.Tensor, fb: ForwardBatch):
        """Returns (logits of all rows, pre-norm hidden of all rows)."""
        e = self.enorm(self.target.embed_tokens(tokens))
        h = self.hnorm(h_prev)
        x = self.eh_proj(torch.cat([e, h], dim=-1))
        out, residual = self.block(x, None, fb)
        pre = out + residual
        logits = self.target.lm_head(self.head_norm(pre.clone()))
        return logits, pre

    def load(self, get) -> None:
        p = f"model.layers.{self.layer_id}."
        self.enorm.weight.data.copy_(get(p + "enorm.weight"))
        self.hnorm.weight.data.copy_(get(p + "hnorm.weight"))
        self.eh_proj.load(get(p + "eh_proj.weight"))
        self.head_norm.weight.data.copy_(get(p + "shared_head.norm.weight"))
        self.block.input_layernorm.weight.data.copy_(get(p + "input_layernorm.weight"))
        self.block.post_attention_layernorm.weight.data.copy_(get(p + "post_attention_layernorm.weight"))
        self.block.self_attn.load(get)
        mlp = self.block.mlp
        if hasattr(mlp, "experts"):
            from ..models.common import MoEBlock
            assert isinstance(mlp, MoEBlock)
            # draft block MoE: reuse the family loader conventions
            pp = p + "mlp."
            mlp.router.load(get(pp + "gate.weight"))
            rng = range(mlp.e_lo, mlp.e_lo + mlp.e_local)
            w13 = torch.stack([torch.cat([get(f"{pp}experts.{i}.gate_proj.weight"),
                                          get(f"{pp}experts.{i}.up_proj.weight")], 0) for i in rng])
            w2 = torch.stack([get(f"{pp}experts.{i}.down_proj.weight") for i in rng])
            mlp.set_experts_from_dense(w13.float(), w2.float())
            if mlp.shared is not None:
                mlp.shared.load(get, pp + "shared_experts.")
        else:
            mlp.load(get, p + "mlp.")


def mtp_weight_shape(cfg, name: str):
    """Shapes of the draft-head-only tensors (the block itself uses the family's rules)."""
    H = cfg.hidden_size
    bf = torch.bfloat16
    if name.endswith("eh_proj.weight"):
        return (H, 2 * H), bf
    return (H,), bf  # enorm / hnorm / shared_head.norm


@dataclasses.dataclass
class SpecState:
    drafts: List[int]        # proposed tokens after the last accepted one
    h_last: torch.Tensor     # target pre-norm hidden at the last accepted position (for re-drafting)


class MTPWorker:
    """Drives prefill + speculative decode steps for a batch of requests through the model runner (eager;
    acceptance on the device, two host reads per verify step). Used by Engine when speculative_algorithm ==
    "MTP"."""

    def __init__(self, engine, num_draft: int = 3):
        self.eng = engine
        self.runner = engine.runner
        self.k = num_draft
        self.stats = {"verify_steps": 0, "drafted": 0, "accepted": 0}

    # -- forward helpers ---------------------------------------------------------------------------
    def _fb(self, ids, pos, slots, reqs_rows: List[Tuple[object, int]], mode=ForwardMode.EXTEND) -> ForwardBatch:
        """Extend-mode batch; reqs_rows: (request, number of rows) in row order."""
        r = self.runner
        dev = r.device
        B = len(reqs_rows)
        qo = np.zeros(B + 1, np.int32)
        seq = np.zeros(B, np.int32)
        for i, (req, n) in enumerate(reqs_rows):
            qo[i + 1] = qo[i] + n
            seq[i] = pos[qo[i + 1] - 1] + 1
        slot_idx = torch.tensor([req.slot for req, _ in reqs_rows], dtype=torch.long, device=dev)
        T = len(ids)
        return ForwardBatch(
            mode=mode, batch_size=B, num_tokens=T,
            input_ids=torch.tensor(ids, dtype=torch.long, device=dev),
            positions=torch.tensor(pos, dtype=torch.long, device=dev),
            out_cache_loc=torch.tensor(slots, dtype=torch.long, device=dev),
            seq_lens=torch.tensor(seq, dtype=torch.int32, device=dev),
            block_table=r.req_to_page.table.index_select(0, slot_idx),
            logits_idx=torch.arange(T, dtype=torch.long, device=dev),
            qo_indptr=torch.tensor(qo, dtype=torch.int32, device=dev),
            max_extend=int(max(n for _, n in reqs_rows)), max_seq_len=int(seq.max()))

    def _slots(self, req, positions) -> List[int]:
        P = self.runner.page_size
        return [req.pages[p // P] * P + p % P for p in positions]

    def _ensure_pages(self, req, upto: int) -> None:
        sched = self.eng.scheduler
        upd: List[int] = []
        if not sched._ensure_pages(req, upto, upd):
            raise RuntimeError("KV pool exhausted during speculative decoding")
        if upd:
            u = torch.tensor(upd, dtype=torch.int32, device=self.runner.device)
            self.runner.apply_page_updates(u)

    def _target(self, fb: ForwardBatch):
        model = self.runner.model
        h = model(fb)  # final-normed rows (logits_idx = all rows)
        logits = model.compute_logits(h)
        return logits, model.last_prenorm

    def _draft_chain(self, reqs, first_tok: torch.Tensor, first_h: torch.Tensor, start_pos: List[int],
                     steps: Optional[int] = None) -> torch.Tensor:
        """`steps` (default k) draft tokens per request, kept on the device: step 1 consumes (first_tok,
        first_h) at start_pos, later steps the draft's own outputs. Returns [B, steps] int64 on the device."""
        head = self.runner.draft
        steps = self.k if steps is None else steps
        out = []
        tok, h = first_tok, first_h
        pos = list(start_pos)
        for _ in range(steps):
            for i, req in enumerate(reqs):
                self._ensure_pages(req, pos[i] + 1)
            slots = [self._slots(req, [pos[i]])[0] for i, req in enumerate(reqs)]
            fb = self._fb([0] * len(reqs), pos, slots, [(req, 1) for req in reqs])
            logits, pre = head(tok, h, fb)
            tok = logits[:, : self.runner.vocab_valid].float().argmax(-1)
            out.append(tok)
            h = pre
            pos = [p + 1 for p in pos]
        if not out:
            return torch.zeros(len(reqs), 0, dtype=torch.long, device=self.runner.device)
        return torch.stack(out, dim=1)

    # -- public ------------------------------------------------------------------------------------
    def prefill(self, reqs) -> None:
        """Run prompts through the target, seed the draft block's KV over the prompt, sample the first
        token and draft k tokens."""
        rows = []
        ids, pos, slots = [], [], []
        for req in reqs:
            L = req.prompt_len
            self._ensure_pages(req, L + self.k + 2)
            ids += req.origin_input_ids
            pos += list(range(L))
            slots += self._slots(req, range(L))
            rows.append((req, L))
        fb = self._fb(ids, pos, slots, rows)
        logits, pre = self._target(fb)
        greedy = logits[:, : self.runner.vocab_valid].float().argmax(-1)
        # draft block over the prompt: position i takes (token_i, target hidden at i-1); position 0 uses zeros
        tok = fb.input_ids
        h_prev = torch.cat([torch.zeros_like(pre[:1]), pre[:-1]], 0)
        starts = np.cumsum([0] + [n for _, n in rows])
        for s in starts[:-1]:
            h_prev[int(s)] = 0
        self.runner.draft(tok, h_prev, fb)
        firsts, last_h = [], []
        for i, (req, L) in enumerate(rows):
            end = int(starts[i + 1]) - 1
            first = int(greedy[end])
            req.output_ids.append(first)
            req.kv_len = L
            firsts.append(first)
            last_h.append(pre[end])
        drafts = self._draft_chain([r for r, _ in rows],
                                   torch.tensor(firsts, device=self.runner.device), torch.stack(last_h),
                                   [r.prompt_len for r, _ in rows]).tolist()  # one read for every draft
        for (req, _), d in zip(rows, drafts):
            req.spec_drafts = d

    def step(self, reqs) -> None:
        """One verify + accept + re-draft step for requests in decode phase. Acceptance runs on the device (the
        drafts against the target's greedy tokens, the accepted length as a cumulative product of matches); the
        host reads the target's tokens and the accepted lengths once, and the new drafts once."""
        k = self.k
        dev = self.runner.device
        ids, pos, slots, rows = [], [], [], []
        for req in reqs:
            p = req.kv_len
            self._ensure_pages(req, p + k + 2)
            toks = [req.output_ids[-1]] + req.spec_drafts
            ids += toks
            pos += list(range(p, p + k + 1))
            slots += self._slots(req, range(p, p + k + 1))
            rows.append((req, k + 1))
        fb = self._fb(ids, pos, slots, rows)
        logits, pre = self._target(fb)
        B = len(reqs)
        greedy = logits[:, : self.runner.vocab_valid].float().argmax(-1).view(B, k + 1)
        drafts = fb.input_ids.view(B, k + 1)[:, 1:]
        n_acc = (drafts == greedy[:, :k]).long().cumprod(dim=1).sum(dim=1)  # accepted drafts per request
        host = torch.cat([greedy, n_acc[:, None]], dim=1).tolist()      # the one read of this verify step
        self.stats["verify_steps"] += 1
        # accept
        mtp_ids, mtp_rows_h, mtp_pos, mtp_slots, mtp_rows = [], [], [], [], []
        for i, req in enumerate(reqs):
            g, n = host[i][: k + 1], int(host[i][k + 1])
            self.stats["drafted"] += k
            self.stats["accepted"] += n
            new = g[: n + 1]
            room = req.params.max_new_tokens - len(req.output_ids)
            new = new[:room]
            req.output_ids += new
            p = req.kv_len
            req.kv_len = p + len(new)
            # draft block catches up over the accepted positions: input token at position p+1+j is new[j],
            # paired with the target hidden of row j (position p+j)
            for j in range(len(new)):
                mtp_ids.append(new[j])
                mtp_rows_h.append(i * (k + 1) + j)
                mtp_pos.append(p + 1 + j)
            mtp_slots += self._slots(req, range(p + 1, p + 1 + len(new)))
            mtp_rows.append((req, len(new)))
        keep = [(r, n) for r, n in mtp_rows if len(r.output_ids) < r.params.max_new_tokens]
        fb2 = self._fb(mtp_ids, mtp_pos, mtp_slots, mtp_rows)
        h_rows = pre.index_select(0, torch.tensor(mtp_rows_h, dtype=torch.long, device=dev))
        d_logits, d_pre = self.runner.draft(fb2.input_ids, h_rows, fb2)
        if not keep:
            return
        ends = np.cumsum([n for _, n in mtp_rows]) - 1
        live_idx, starts, live = [], [], []
        for (req, n), e in zip(mtp_rows, ends):
            if len(req.output_ids) >= req.params.max_new_tokens:
                continue
            live_idx.append(int(e))
            starts.append(req.kv_len + 1)
            live.append(req)
        sel = torch.tensor(live_idx, dtype=torch.long, device=dev)
        first = d_logits.index_select(0, sel)[:, : self.runner.vocab_valid].float().argmax(-1)
        # the first draft came from the catch-up pass; chain the remaining k-1 on the device
        rest = self._draft_chain(live, first, d_pre.index_select(0, sel), starts, steps=self.k - 1)
        new_drafts = torch.cat([first[:, None], rest], dim=1).tolist()  # the one read of the new drafts
        for req, d in zip(live, new_drafts):
            req.spec_drafts = d

    def generate(self, reqs) -> None:
        self.prefill(reqs)
        live = [r for r in reqs if len(r.output_ids) < r.params.max_new_tokens]
        while live:
            self.step(live)
            live = [r for r in live if len(r.output_ids) < r.params.max_new_tokens]
        for r in reqs:
            r.finished = True
            r.finish_reason = "length"

    def acceptance_length(self) -> float:
        v = self.stats["verify_steps"]
        return 1.0 + (self.stats["accepted"] / max(1, self.stats["drafted"])) * self.k if v else 0.0
