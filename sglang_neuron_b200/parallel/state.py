"""Parallel state: tensor-parallel (attention and dense MLP), expert-parallel (MoE), pipeline-parallel
(contiguous layer stages) and data-parallel groups over one process per GPU.

Parity: the reference builds its groups in `initialize_neuron_parallel_state`
(sglang_neuron/parallel/state.py:77-152) with attention-TP, EP-TP and EP groups and group getters
(parallel/groups.py:158-211). On B200 the device groups are NCCL communicators created through
torch.distributed (one process per GPU); host-side control collectives use a gloo group, as in the
reference (gloo on the host). EP here spans the same ranks as TP: experts are split in contiguous blocks
by rank (`ep_group_ranks` rows = EP) and tokens are replicated over the group after attention.

DP attention (`initialize_parallel(..., dp_attention=True)`): the world of T ranks splits into D attention
groups of T/D ranks; `tp_*` then describe the attention group (QKV/o_proj, dense MLP, vocabulary shards,
sampling), experts are split over all T ranks (`ep_*`), and tokens cross groups only around the MoE
(all-gather before, reduce-scatter after, on `moe_group`). Parity: the reference's DP-attention groups
(sglang_neuron/parallel/groups.py:72 `dp_column_ranks`, parallel/state.py:125-126).

Rank layout: rank = (dp_rank * pp_size + pp_rank) * tp_size + tp_rank. A DP replica (pp_size x tp_size
ranks) runs one scheduler in lockstep; its replica rank 0 owns request intake. Pipeline stages hold
contiguous layer blocks (distributed/pipeline.py `StageSpec` in the reference: sglang_neuron/distributed/
pipeline.py:29); stage s+1's tensor-parallel rank r receives stage s's rank r hidden state.
"""
from __future__ import annotations

import dataclasses
import os
from datetime import timedelta
from typing import Optional, Sequence

import torch
import torch.distributed as dist


@dataclasses.dataclass
class ParallelState:
    world_size: int = 1
    rank: int = 0
    tp_size: int = 1
    tp_rank: int = 0
    ep_size: int = 1
    ep_rank: int = 0
    dp_size: int = 1
    dp_rank: int = 0
    tp_group: Optional[object] = None      # device (NCCL or gloo on CPU) group
    cpu_group: Optional[object] = None     # gloo group for host control
    device: torch.device = torch.device("cpu")
    pp_size: int = 1
    pp_rank: int = 0
    replica_group: Optional[object] = None      # device group of the DP replica (pp_size x tp_size ranks)
    replica_cpu_group: Optional[object] = None  # gloo group of the DP replica
    attn_dp_size: int = 1                       # DP-attention groups inside the replica (1: off)
    attn_dp_rank: int = 0
    moe_group: Optional[object] = None          # device group of all ranks (DP attention: MoE token exchange)
    dp_cross_group: Optional[object] = None     # ranks with this tp_rank in every attention group
    dcp_size: int = 1                           # decode context parallelism: ranks sharing one latent KV
    dcp_rank: int = 0
    dcp_group: Optional[object] = None          # consecutive TP ranks tp_rank // dcp_size
    replica_base_rank: int = -1                 # set when replicas differ in size (see initialize_replicas)
    replica_tp: tuple = ()                      # every replica's TP size when they differ (rank order)

    @property
    def is_first_rank(self) -> bool:
        return self.replica_rank == 0

    @property
    def replica_size(self) -> int:
        return self.pp_size * self.tp_size * self.attn_dp_size

    @property
    def replica_rank(self) -> int:
        return (self.pp_rank * self.attn_dp_size + self.attn_dp_rank) * self.tp_size + self.tp_rank

    @property
    def replica_base(self) -> int:
        """Global rank of this replica's rank 0."""
        if self.replica_base_rank >= 0:
            return self.replica_base_rank
        return self.dp_rank * self.replica_size

    @property
    def is_first_stage(self) -> bool:
        return self.pp_rank == 0

    @property
    def is_last_stage(self) -> bool:
        return self.pp_rank == self.pp_size - 1

    def stage_rank(self, pp_rank: int) -> int:
        """Global rank of the same tensor-parallel rank in pipeline stage `pp_rank` of this replica."""
        return self.replica_base + pp_rank * self.tp_size + self.tp_rank


def pp_layer_range(num_layers: int, pp_size: int, pp_rank: int):
    """Contiguous layer block [start, end) of a pipeline stage; earlier stages take the remainder."""
    if pp_size > num_layers:
        raise ValueError(f"pp_size {pp_size} exceeds the {num_layers} layers")
    base, extra = divmod(num_layers, pp_size)
    start = pp_rank * base + min(pp_rank, extra)
    return start, start + base + (1 if pp_rank < extra else 0)


_STATE = ParallelState()


def get_state() -> ParallelState:
    return _STATE


def set_state(state: ParallelState) -> None:
    global _STATE
    _STATE = state


def init_process_group_from_env(backend: Optional[str] = None, timeout_s: int = 600) -> None:
    """Initialise torch.distributed from RANK/WORLD_SIZE/MASTER_ADDR/MASTER_PORT if not done yet."""
    if dist.is_initialized():
        return
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world <= 1:
        return
    if backend is None:
        backend = "nccl" if torch.cuda.is_available() else "gloo"
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    kwargs = dict(backend=backend, timeout=timedelta(seconds=timeout_s))
    if backend == "nccl":
        local = int(os.environ.get("LOCAL_RANK", "0"))
        torch.cuda.set_device(local)
        kwargs["device_id"] = torch.device("cuda", local)
    dist.init_process_group(**kwargs)


def initialize_parallel(tp_size: int = 1, ep_size: Optional[int] = None, dp_size: int = 1,
                        device: Optional[torch.device] = None, pp_size: int = 1,
                        dp_attention: bool = False, dcp_size: int = 1,
                        replica_tp: Optional[Sequence[int]] = None) -> ParallelState:
    """Build the groups. Ranks are laid out DP-major, then PP: rank = (dp_rank * pp_size + pp_rank) * tp_size
    + tp_rank. With dp_attention, dp_size attention groups split the tp_size ranks instead (one replica).
    With replica_tp, the DP replicas have the given tensor-parallel sizes (see initialize_replicas)."""
    if replica_tp:
        if pp_size != 1 or dp_attention or dcp_size != 1 or len(replica_tp) != dp_size:
            raise ValueError("replicas of different TP sizes take one pipeline stage, no DP attention or DCP, and "
                             "dp_size equal to the number of replicas")
        st = initialize_replicas(replica_tp, device)
        if st.tp_size != tp_size or (ep_size not in (None, tp_size)):
            raise ValueError(f"rank {st.rank} belongs to a TP{st.tp_size} replica but was launched with tp_size "
                             f"{tp_size}")
        return st
    if dp_attention and dp_size > 1:
        return _initialize_dp_attention(tp_size, ep_size, dp_size, device, pp_size)
    ep_size = tp_size if ep_size is None else ep_size
    if ep_size != tp_size:
        raise ValueError("expert parallelism spans the tensor-parallel group here (ep_size must equal tp_size)")
    if dist.is_initialized():
        world, rank = dist.get_world_size(), dist.get_rank()
    else:
        world, rank = 1, 0
    if tp_size * pp_size * dp_size != world:
        raise ValueError(f"tp_size {tp_size} x pp_size {pp_size} x dp_size {dp_size} != world size {world}")
    dp_rank, rest = divmod(rank, pp_size * tp_size)
    pp_rank, tp_rank = divmod(rest, tp_size)
    tp_group = cpu_group = replica_group = replica_cpu_group = None
    if world > 1:
        for d in range(dp_size):
            for p_ in range(pp_size):
                base = (d * pp_size + p_) * tp_size
                ranks = list(range(base, base + tp_size))
                g = dist.new_group(ranks)
                cg = dist.new_group(ranks, backend="gloo")
                if d == dp_rank and p_ == pp_rank:
                    tp_group, cpu_group = g, cg
            if pp_size > 1:
                ranks = list(range(d * pp_size * tp_size, (d + 1) * pp_size * tp_size))
                g = dist.new_group(ranks)
                cg = dist.new_group(ranks, backend="gloo")
                if d == dp_rank:
                    replica_group, replica_cpu_group = g, cg
    if pp_size == 1:
        replica_group, replica_cpu_group = tp_group, cpu_group
    if device is None:
        device = torch.device("cuda", torch.cuda.current_device()) if torch.cuda.is_available() else torch.device("cpu")
    dcp_group = None
    if dcp_size > 1:
        if tp_size % dcp_size:
            raise ValueError(f"dcp_size {dcp_size} must divide tp_size {tp_size}")
        for d in range(dp_size):
            for p_ in range(pp_size):
                base = (d * pp_size + p_) * tp_size
                for k in range(tp_size // dcp_size):
                    ranks = list(range(base + k * dcp_size, base + (k + 1) * dcp_size))
                    g = dist.new_group(ranks)
                    if rank in ranks:
                        dcp_group = g
    st = ParallelState(world_size=world, rank=rank, tp_size=tp_size, tp_rank=tp_rank, ep_size=ep_size,
                       ep_rank=tp_rank, dp_size=dp_size, dp_rank=dp_rank, tp_group=tp_group,
                       cpu_group=cpu_group, device=device, pp_size=pp_size, pp_rank=pp_rank,
                       replica_group=replica_group, replica_cpu_group=replica_cpu_group,
                       dcp_size=dcp_size, dcp_rank=tp_rank % dcp_size, dcp_group=dcp_group)
    set_state(st)
    return st


def initialize_replicas(replica_tp: Sequence[int], device: Optional[torch.device] = None) -> ParallelState:
    """DP replicas of different tensor-parallel sizes, laid out in order: replica r holds ranks
    [sum(replica_tp[:r]), sum(replica_tp[:r + 1])). Used by disaggregated prefill/decode on one box, where the
    prefill group and the decode group may shard attention differently (the KV hand-off slices pages by head).
    Experts span each replica's TP group, as in initialize_parallel."""
    sizes = [int(t) for t in replica_tp]
    if not sizes or min(sizes) < 1:
        raise ValueError(f"replica_tp {replica_tp}: every replica needs at least one rank")
    world, rank = (dist.get_world_size(), dist.get_rank()) if dist.is_initialized() else (1, 0)
    if sum(sizes) != world:
        raise ValueError(f"replica TP sizes {sizes} sum to {sum(sizes)}, not the world size {world}")
    bases = [sum(sizes[:r]) for r in range(len(sizes))]
    dp_rank = max(r for r in range(len(sizes)) if bases[r] <= rank)
    tp_size, tp_rank = sizes[dp_rank], rank - bases[dp_rank]
    tp_group = cpu_group = None
    if world > 1:
        for r, (b, t) in enumerate(zip(bases, sizes)):  # every rank creates every group, in the same order
            ranks = list(range(b, b + t))
            g = dist.new_group(ranks)
            cg = dist.new_group(ranks, backend="gloo")
            if r == dp_rank:
                tp_group, cpu_group = g, cg
    if device is None:
        device = torch.device("cuda", torch.cuda.current_device()) if torch.cuda.is_available() else torch.device("cpu")
    st = ParallelState(world_size=world, rank=rank, tp_size=tp_size, tp_rank=tp_rank, ep_size=tp_size,
                       ep_rank=tp_rank, dp_size=len(sizes), dp_rank=dp_rank, tp_group=tp_group, cpu_group=cpu_group,
                       device=device, replica_group=tp_group, replica_cpu_group=cpu_group,
                       replica_base_rank=bases[dp_rank], replica_tp=tuple(sizes))
    set_state(st)
    return st


def _initialize_dp_attention(tp_size, ep_size, dp_size, device, pp_size) -> ParallelState:
    if pp_size != 1:
        raise ValueError("DP attention is not served with pipeline parallelism")
    if tp_size % dp_size:
        raise ValueError(f"dp_size {dp_size} must divide tp_size {tp_size} under DP attention")
    if ep_size not in (None, tp_size):
        raise ValueError("under DP attention experts span all tp_size ranks (ep_size must equal tp_size)")
    world, rank = (dist.get_world_size(), dist.get_rank()) if dist.is_initialized() else (1, 0)
    if world != tp_size:
        raise ValueError(f"tp_size {tp_size} != world size {world}")
    a = tp_size // dp_size
    g_rank, tp_rank = divmod(rank, a)
    tp_group = cpu_group = cross = None
    for g in range(dp_size):
        ranks = list(range(g * a, (g + 1) * a))
        dg, cg = dist.new_group(ranks), dist.new_group(ranks, backend="gloo")
        if g == g_rank:
            tp_group, cpu_group = dg, cg
    for t in range(a):
        ranks = list(range(t, tp_size, a))
        xg = dist.new_group(ranks)
        if t == tp_rank:
            cross = xg
    world_group = dist.new_group(list(range(world)))
    world_cpu = dist.new_group(list(range(world)), backend="gloo")
    if device is None:
        device = torch.device("cuda", torch.cuda.current_device()) if torch.cuda.is_available() else torch.device("cpu")
    st = ParallelState(world_size=world, rank=rank, tp_size=a, tp_rank=tp_rank, ep_size=tp_size, ep_rank=rank,
                       dp_size=1, dp_rank=0, tp_group=tp_group, cpu_group=cpu_group, device=device,
                       replica_group=world_group, replica_cpu_group=world_cpu, attn_dp_size=dp_size,
                       attn_dp_rank=g_rank, moe_group=world_group, dp_cross_group=cross)
    set_state(st)
    return st


def destroy_parallel() -> None:
    """Reset to a single-rank state (used by tests to build several worlds in one process)."""
    set_state(ParallelState())
