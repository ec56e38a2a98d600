"""Cross-rank agreement checks run once at startup.

* `assert_fleet_consistent`: every rank of the world hashes what it is about to serve (architecture, layer
  kinds, parallel layout, KV format, page size) and the digests are all-gathered over the host group: ranks
  that would run different programs are refused before the first collective of a forward can hang.
* `assert_graphs_consistent`: after CUDA-graph capture, every rank of a replica all-gathers a digest of its
  captured buckets (batch sizes, launches per graph, decode split counts): the ranks of a tensor-parallel
  group must replay identical kernel/collective sequences.

Parity: the reference's model contract fleet digest (sglang_neuron/models/contract.py:184, all_gather) and
its SPMD compile check (backend/spmd_check.py:42-125, all-gather of per-shape cache keys).
"""
from __future__ import annotations

import hashlib
import json
from typing import Any, Dict, Optional

import torch.distributed as dist

from .state import get_state


def digest(obj: Any) -> str:
    return hashlib.sha256(json.dumps(obj, sort_keys=True, default=str).encode()).hexdigest()[:16]


def _gather(value: str, group) -> list:
    out = [None] * dist.get_world_size(group)
    dist.all_gather_object(out, value, group=group)
    return out


def assert_fleet_consistent(payload: Dict[str, Any], group: Optional[object] = None) -> str:
    d = digest(payload)
    if not dist.is_initialized() or dist.get_world_size() == 1:
        return d
    st = get_state()
    if group is None:
        group = st.replica_cpu_group if st.dp_size == 1 else None
    if group is None:  # several DP replicas: compare over the whole world through a gloo group
        group = dist.new_group(backend="gloo")
    got = _gather(d, group)
    if len(set(got)) != 1:
        raise RuntimeError(f"ranks disagree on the served model/layout (digests {got}): refusing to start")
    return d


def assert_graphs_consistent(payload: Dict[str, Any]) -> str:
    d = digest(payload)
    st = get_state()
    if st.replica_size == 1 or not dist.is_initialized():
        return d
    got = _gather(d, st.replica_cpu_group)
    if len(set(got)) != 1:
        raise RuntimeError(f"ranks captured different decode graphs (digests {got})")
    return d
