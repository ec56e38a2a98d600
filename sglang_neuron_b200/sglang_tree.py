"""The one reader of the runtime topology (parallel sizes, DP widths, scheduler batch, rank label), and the
seam tests patch.

Parity: sglang_neuron/sglang_tree.py:17-86 (`parallel_of`, `dp_widths`, `scheduler_batch`, `rank_label`).
Readers: the server's `/get_server_info` route (parallel layout, rank label) and the host trace (file name per
rank label).
"""
from __future__ import annotations

from typing import Dict, Tuple

from .parallel.state import get_state


def parallel_of() -> Dict[str, int]:
    st = get_state()
    return {"tp": st.tp_size, "ep": st.ep_size, "dp": st.dp_size, "pp": st.pp_size, "dcp": st.dcp_size,
            "attn_dp": st.attn_dp_size, "world": st.world_size}


def dp_widths() -> Tuple[int, int]:
    st = get_state()
    return st.dp_size, st.tp_size


def scheduler_batch(args) -> int:
    return args.max_running_requests


def rank_label() -> str:
    st = get_state()
    lab = f"dp{st.dp_rank}-tp{st.tp_rank}"
    return lab + (f"-pp{st.pp_rank}" if st.pp_size > 1 else "")
