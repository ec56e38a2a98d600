"""Tensor-parallel collective microbenchmarks on N GPUs (run under torchrun, one rank per GPU):
NCCL all-reduce vs the one-shot NVLink all-reduce, MoE combine + all-reduce fused vs separate, and the
row-parallel GEMM with the all-reduce in its epilogue vs split-K GEMM + NCCL. Device time per op is the
max over ranks of CUDA-event time over `iters` back-to-back launches.

    torchrun --nproc-per-node 2 -m sglang_neuron_b200.benchmarks.collectives --tokens 64
"""
from __future__ import annotations

import argparse
import json
import os

import torch
import torch.distributed as dist


def main():
    p = argparse.ArgumentParser()
    p.add_argument("--tokens", type=int, default=64)
    p.add_argument("--hidden", type=int, default=2880)
    p.add_argument("--k-local", type=int, default=0)
    p.add_argument("--iters", type=int, default=50)
    p.add_argument("--graph", action="store_true",
                   help="time the ops replayed from a CUDA graph (no host launch cost between calls)")
    p.add_argument("--cta-sweep", action="store_true", help="one-shot all-reduce at several CTA counts")
    a = p.parse_args()
    from ..parallel.state import init_process_group_from_env, initialize_parallel
    from ..parallel.symm_mem import IpcAllReduce
    from ..ops.gemm import linear
    from ..parallel.collectives import fused_gemm_all_reduce, set_custom_allreduce
    from ..ops.moe import MoEAlignment, moe_align, moe_combine, topk_route
    init_process_group_from_env(timeout_s=120)
    world, rank = dist.get_world_size(), dist.get_rank()
    st = initialize_parallel(world, device=torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0"))))
    dev = st.device
    ar = IpcAllReduce()
    set_custom_allreduce(ar)
    T, H = a.tokens, a.hidden
    K = a.k_local or (4096 // world)
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    x = torch.randn(T, H, device=dev).to(torch.bfloat16)
    xa = torch.randn(T, K, device=dev).to(torch.bfloat16)
    wt = (torch.randn(H, K, device=dev) * 0.05).to(torch.bfloat16)
    E = 128 // world
    w, ids = topk_route(torch.randn(T, 128, device=dev), 4)
    al = MoEAlignment(T * 4, E, 16, dev)
    moe_align(ids, rank * E, E, al)
    y = torch.randn(al.r_max, H, device=dev).to(torch.bfloat16)
    out = torch.empty(T, H, device=dev, dtype=torch.bfloat16)

    def t_op(fn):
        for _ in range(5):
            fn()
        torch.cuda.synchronize()
        g = None
        if a.graph:
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                for _ in range(a.iters):
                    fn()
            g.replay()
            torch.cuda.synchronize()
        dist.barrier()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        if g is not None:
            g.replay()
        else:
            for _ in range(a.iters):
                fn()
        e.record()
        torch.cuda.synchronize()
        v = torch.tensor([s.elapsed_time(e) / a.iters * 1e3], device=dev)
        dist.all_reduce(v, op=dist.ReduceOp.MAX)
        del g
        return round(float(v), 2)

    if a.cta_sweep:
        from ..parallel.collectives import FusedNorm
        sweep = {}
        resid = torch.randn(T, H, device=dev).to(torch.bfloat16)
        nw = torch.ones(H, device=dev, dtype=torch.bfloat16)

        class _N:  # stand-in norm module for FusedNorm
            weight, eps = nw, 1e-5

        for c in (8, 16, 32, 64, 128, 148):
            ar.max_ctas = c
            sweep[f"oneshot_ctas{c}_us"] = t_op(lambda: ar.all_reduce(x, out))
            sweep[f"oneshot_norm_ctas{c}_us"] = t_op(lambda: ar.all_reduce(x, out, norm=FusedNorm(resid, nw, 1e-5)))
        ar.max_ctas = 64
        if rank == 0:
            print(json.dumps({"world": world, "tokens": T, "graph": a.graph, **sweep}), flush=True)

    res = {"world": world, "tokens": T, "hidden": H, "k_local": K, "graph": a.graph,
           "nccl_allreduce_us": t_op(lambda: dist.all_reduce(x)),
           "oneshot_allreduce_us": t_op(lambda: ar.all_reduce(x, out)),
           "combine_then_nccl_us": t_op(lambda: (moe_combine(out, y, al.inv_map, w), dist.all_reduce(out))),
           "combine_allreduce_fused_us": t_op(lambda: ar.combine_all_reduce(out, y, al.inv_map[: T * 4], w)),
           "gemm_splitk_then_nccl_us": t_op(lambda: dist.all_reduce(linear(xa, wt))),
           "gemm_then_oneshot_us": t_op(lambda: ar.all_reduce(linear(xa, wt), out)),
           "gemm_allreduce_fused_us": t_op(lambda: ar.gemm_all_reduce(xa, wt, None, sms)),
           "gemm_splitk_allreduce_fused_us": t_op(lambda: fused_gemm_all_reduce(xa, wt, None)),
           "status": int(ar.status[0])}
    try:
        from ..parallel.symm_mem import NvlsAllReduce
        nv = NvlsAllReduce()
        set_custom_allreduce(nv)
        res.update({"nvls_allreduce_us": t_op(lambda: nv.all_reduce(x, out)),
                    "nvls_combine_allreduce_us": t_op(lambda: nv.combine_all_reduce(out, y, al.inv_map[: T * 4], w)),
                    "nvls_gemm_splitk_allreduce_us": t_op(lambda: fused_gemm_all_reduce(xa, wt, None)),
                    "nvls_status": int(nv.status[0])})
        set_custom_allreduce(None)
        nv.close()
    except RuntimeError as e:
        res["nvls"] = f"unavailable: {e}"
    if rank == 0:
        print(json.dumps(res), flush=True)
    ar.close()
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
