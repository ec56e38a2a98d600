"""Multi-GPU tier (needs >= 2 GPUs): the one-shot NVLink all-reduce against NCCL, and a TP=2 engine whose
ranks agree token for token. Each rank is its own process on its own GPU; the process group has a short
timeout so a lost peer ends the test with an error instead of a hang."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

needs2 = pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _init(rank, world, port):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), WORLD_SIZE=str(world), RANK=str(rank),
                      LOCAL_RANK=str(rank), NCCL_NVLS_ENABLE="0")
    from sglang_neuron_b200.parallel.state import init_process_group_from_env
    init_process_group_from_env(timeout_s=60)


def _ar_worker(rank, world, port, q):
    _init(rank, world, port)
    import torch.distributed as dist
    from sglang_neuron_b200.parallel.state import initialize_parallel
    from sglang_neuron_b200.parallel.symm_mem import IpcAllReduce
    initialize_parallel(world, device=torch.device("cuda", rank))
    ar = IpcAllReduce(capacity_bytes=4 << 20)
    errs = []
    for i, n in enumerate([8, 2880 * 64, 4096 * 3, 1 << 20, 2880 * 64]):
        g = torch.Generator(device="cuda").manual_seed(100 * i + rank)
        x = torch.randn(n, generator=g, device="cuda").to(torch.bfloat16)
        ref = x.float().clone()
        dist.all_reduce(ref)
        out = ar.all_reduce(x)
        torch.cuda.synchronize()
        errs.append(((out.float() - ref).abs().max() / ref.abs().max()).item())
    # MoE combine fused with the all-reduce vs combine + NCCL all-reduce
    from sglang_neuron_b200.ops.moe import MoEAlignment, moe_align, moe_combine, topk_route
    T, H, E = 64, 2880, 16
    g = torch.Generator(device="cuda").manual_seed(7 + rank)
    w, ids = topk_route(torch.randn(T, E, device="cuda", generator=g), 4)
    al = MoEAlignment(T * 4, E // world, 16, "cuda")
    moe_align(ids, rank * (E // world), E // world, al)
    y = torch.randn(al.r_max, H, device="cuda", generator=g).to(torch.bfloat16)
    ref = torch.empty(T, H, device="cuda", dtype=torch.bfloat16)
    moe_combine(ref, y, al.inv_map, w)
    ref = ref.float()
    dist.all_reduce(ref)
    out = torch.empty(T, H, device="cuda", dtype=torch.bfloat16)
    for _ in range(3):  # repeated calls cycle the epoch / buffer halves
        ar.combine_all_reduce(out, y, al.inv_map[: T * 4], w)
    torch.cuda.synchronize()
    errs.append(((out.float() - ref).abs().max() / ref.abs().max()).item())
    # row-parallel GEMM with the all-reduce in its epilogue vs GEMM + NCCL
    from sglang_neuron_b200.ops.gemm import linear
    for T, F, Kl in [(64, 2880, 512), (7, 2880, 4096 // world), (1, 1024, 256)]:
        g = torch.Generator(device="cuda").manual_seed(11 + rank + T)
        x = torch.randn(T, Kl, device="cuda", generator=g).to(torch.bfloat16)
        wt = (torch.randn(F, Kl, device="cuda", generator=g) * 0.05).to(torch.bfloat16)
        ref = (x.float() @ wt.float().t())
        dist.all_reduce(ref)
        for _ in range(2):
            out = ar.gemm_all_reduce(x, wt, None, torch.cuda.get_device_properties(0).multi_processor_count)
        torch.cuda.synchronize()
        errs.append(((out.float() - ref).abs().max() / ref.abs().max()).item())
    # split-K GEMM + (partial sum, bias, all-reduce) kernel: the row-parallel path the engine takes
    from sglang_neuron_b200.parallel.collectives import fused_gemm_all_reduce, set_custom_allreduce
    set_custom_allreduce(ar)
    for T, F, Kl in [(64, 2880, 2048), (3, 2880, 4096 // world), (200, 1024, 512)]:
        g = torch.Generator(device="cuda").manual_seed(23 + rank + T)
        x = torch.randn(T, Kl, device="cuda", generator=g).to(torch.bfloat16)
        wt = (torch.randn(F, Kl, device="cuda", generator=g) * 0.05).to(torch.bfloat16)
        b = (torch.randn(F, device="cuda", generator=g)).to(torch.bfloat16)
        ref = (x.float() @ wt.float().t()) + b.float()
        dist.all_reduce(ref)
        for _ in range(2):
            out = fused_gemm_all_reduce(x, wt, b)
        torch.cuda.synchronize()
        errs.append(((out.float() - ref).abs().max() / ref.abs().max()).item())
    set_custom_allreduce(None)
    status = int(ar.status[0])
    ar.close()
    q.put((rank, errs, status))
    dist.barrier()
    dist.destroy_process_group()


def _nvls_worker(rank, world, port, q):
    """NVLS (multicast) all-reduce vs NCCL: plain, fused MoE combine, fused split-K partial sum."""
    _init(rank, world, port)
    import torch.distributed as dist
    from sglang_neuron_b200.parallel.state import initialize_parallel
    from sglang_neuron_b200.parallel.symm_mem import NvlsAllReduce
    initialize_parallel(world, device=torch.device("cuda", rank))
    try:
        ar = NvlsAllReduce(capacity_bytes=4 << 20)
    except Exception as e:  # no multicast on this machine
        q.put((rank, None, repr(e)))
        dist.barrier()
        dist.destroy_process_group()
        return
    errs = []
    for i, n in enumerate([8, 2880 * 64, 4096 * 3, 1 << 20, 2880 * 7]):
        g = torch.Generator(device="cuda").manual_seed(100 * i + rank)
        x = torch.randn(n, generator=g, device="cuda").to(torch.bfloat16)
        ref = x.float().clone()
        dist.all_reduce(ref)
        for _ in range(3):  # repeated calls advance the epoch
            out = ar.all_reduce(x)
        torch.cuda.synchronize()
        errs.append(((out.float() - ref).abs().max() / ref.abs().max()).item())
    from sglang_neuron_b200.ops.moe import MoEAlignment, moe_align, moe_combine, topk_route
    T, H, E = 64, 2880, 16
    g = torch.Generator(device="cuda").manual_seed(7 + rank)
    w, ids = topk_route(torch.randn(T, E, device="cuda", generator=g), 4)
    al = MoEAlignment(T * 4, E // world, 16, "cuda")
    moe_align(ids, rank * (E // world), E // world, al)
    y = torch.randn(al.r_max, H, device="cuda", generator=g).to(torch.bfloat16)
    ref = torch.empty(T, H, device="cuda", dtype=torch.bfloat16)
    moe_combine(ref, y, al.inv_map, w)
    ref = ref.float()
    dist.all_reduce(ref)
    out = torch.empty(T, H, device="cuda", dtype=torch.bfloat16)
    ar.combine_all_reduce(out, y, al.inv_map[: T * 4], w)
    torch.cuda.synchronize()
    errs.append(((out.float() - ref).abs().max() / ref.abs().max()).item())
    from sglang_neuron_b200.ops.gemm import linear_partials
    T, F, Kl = 64, 2880, 512
    x = torch.randn(T, Kl, device="cuda", generator=g).to(torch.bfloat16)
    wt = (torch.randn(F, Kl, device="cuda", generator=g) * 0.05).to(torch.bfloat16)
    b = torch.randn(F, device="cuda", generator=g).to(torch.bfloat16)
    ref = x.float() @ wt.float().t() + b.float()
    dist.all_reduce(ref)
    part = linear_partials(x, wt, 4)
    out = torch.empty(T, F, device="cuda", dtype=torch.bfloat16)
    ar.splitk_all_reduce(part, 4, T, F, b, out)
    torch.cuda.synchronize()
    errs.append(((out.float() - ref).abs().max() / ref.abs().max()).item())
    status = int(ar.status[0])
    ar.close()
    q.put((rank, errs, status))
    dist.barrier()
    dist.destroy_process_group()


def _ar_norm_worker(rank, world, port, q):
    """All-reduce + residual add + RMSNorm in one launch (one-shot, split-K GEMM, MoE combine forms) against
    NCCL all-reduce + the fp32 add + norm."""
    _init(rank, world, port)
    import torch.distributed as dist
    from sglang_neuron_b200.parallel.collectives import FusedNorm, fused_gemm_all_reduce, set_custom_allreduce
    from sglang_neuron_b200.parallel.state import initialize_parallel
    from sglang_neuron_b200.parallel.symm_mem import IpcAllReduce
    initialize_parallel(world, device=torch.device("cuda", rank))
    ar = IpcAllReduce(capacity_bytes=4 << 20)
    set_custom_allreduce(ar)
    errs = []

    class Norm:
        def __init__(self, H, g):
            self.weight = (1 + 0.1 * torch.randn(H, device="cuda", generator=g)).to(torch.bfloat16)
            self.eps = 1e-5

    def ref_norm(s, res, nm):
        v = s + res.float()
        return v * torch.rsqrt(v.pow(2).mean(-1, keepdim=True) + nm.eps) * nm.weight.float(), v

    def check(out, res_after, s, res_before, nm):
        want, v = ref_norm(s, res_before, nm)
        errs.append(((out.float() - want).abs().max() / want.abs().max()).item())
        errs.append(((res_after.float() - v).abs().max() / v.abs().max()).item())

    for T, H in [(64, 2880), (1, 2880), (13, 4096), (200, 1024)]:
        g = torch.Generator(device="cuda").manual_seed(5 * T + rank)
        gw = torch.Generator(device="cuda").manual_seed(99 + T)  # same weight on every rank
        nm = Norm(H, gw)
        x = torch.randn(T, H, generator=g, device="cuda").to(torch.bfloat16)
        res = torch.randn(T, H, generator=gw, device="cuda").to(torch.bfloat16)
        s = x.float()
        dist.all_reduce(s)
        res0 = res.clone()
        fn = FusedNorm.offer(res, nm)
        out = ar.all_reduce(x, norm=fn)
        torch.cuda.synchronize()
        assert fn.done
        check(out, res, s, res0, nm)
        # split-K GEMM partials + bias + all-reduce + add + norm
        Kl = 512
        xa = torch.randn(T, Kl, device="cuda", generator=g).to(torch.bfloat16)
        wt = (torch.randn(H, Kl, device="cuda", generator=g) * 0.05).to(torch.bfloat16)
        s = xa.float() @ wt.float().t()
        dist.all_reduce(s)
        res0 = res.clone()
        fn = FusedNorm.offer(res, nm)
        out = fused_gemm_all_reduce(xa, wt, None, norm=fn)
        torch.cuda.synchronize()
        if out is not None and fn.done:
            check(out, res, s, res0, nm)
    # MoE combine + all-reduce + add + norm
    from sglang_neuron_b200.ops.moe import MoEAlignment, moe_align, moe_combine, topk_route
    T, H, E = 64, 2880, 16
    g = torch.Generator(device="cuda").manual_seed(7 + rank)
    gw = torch.Generator(device="cuda").manual_seed(1234)
    nm = Norm(H, gw)
    res = torch.randn(T, H, generator=gw, device="cuda").to(torch.bfloat16)
    w, ids = topk_route(torch.randn(T, E, device="cuda", generator=g), 4)
    al = MoEAlignment(T * 4, E // world, 16, "cuda")
    moe_align(ids, rank * (E // world), E // world, al)
    y = torch.randn(al.r_max, H, device="cuda", generator=g).to(torch.bfloat16)
    comb = torch.empty(T, H, device="cuda", dtype=torch.bfloat16)
    moe_combine(comb, y, al.inv_map, w)
    s = comb.float()
    dist.all_reduce(s)
    res0 = res.clone()
    fn = FusedNorm.offer(res, nm)
    out = torch.empty(T, H, device="cuda", dtype=torch.bfloat16)
    ar.combine_all_reduce(out, y, al.inv_map[: T * 4], w, norm=fn)
    torch.cuda.synchronize()
    check(out, res, s, res0, nm)
    set_custom_allreduce(None)
    status = int(ar.status[0])
    ar.close()
    q.put((rank, errs, status))
    dist.barrier()
    dist.destroy_process_group()


def _engine_worker(rank, world, port, q):
    _init(rank, world, port)
    import torch.distributed as dist
    from sglang_neuron_b200.configs import model_config as mc
    from sglang_neuron_b200.engine import Engine
    from sglang_neuron_b200.server_args import ServerArgs
    mc.PRESETS["mg-oss"] = dict(mc.PRESETS["gpt-oss-120b"], num_hidden_layers=2, vocab_size=2048, hidden_size=512,
                                intermediate_size=256, num_local_experts=8, num_attention_heads=8,
                                num_key_value_heads=2, head_dim=64, sliding_window=16)
    eng = Engine(ServerArgs(model="mg-oss", tp_size=world, page_size=16, context_length=256,
                            max_running_requests=4, chunked_prefill_size=64, cuda_graph_bs=[1, 2, 4],
                            random_weight_std=0.05))
    g = torch.Generator().manual_seed(3)
    prompts = [torch.randint(0, 2048, (n,), generator=g).tolist() for n in (9, 40)]
    out = eng.generate(prompts, {"max_new_tokens": 8})
    eng.shutdown()
    q.put((rank, [o["output_ids"] for o in out]))
    dist.barrier()
    dist.destroy_process_group()


def _logits_worker(rank, world, port, q, extra):
    """Prefill logits of one 40-token and one 9-token prompt (max_new_tokens=1) under a layout `extra`."""
    if world > 1:
        _init(rank, world, port)
    import torch.distributed as dist
    from sglang_neuron_b200.configs import model_config as mc
    from sglang_neuron_b200.engine import Engine
    from sglang_neuron_b200.server_args import ServerArgs
    mc.PRESETS["mg-oss"] = dict(mc.PRESETS["gpt-oss-120b"], num_hidden_layers=2, vocab_size=2048, hidden_size=512,
                                intermediate_size=256, num_local_experts=8, num_attention_heads=8,
                                num_key_value_heads=2, head_dim=64, sliding_window=16)
    eng = Engine(ServerArgs(model="mg-oss", tp_size=extra.pop("tp", world), page_size=16, context_length=256,
                            max_running_requests=4, chunked_prefill_size=64, disable_cuda_graph=True,
                            random_weight_std=0.05, random_gen_device="cpu", **extra))
    rows = []
    eng.runner.logits_hook = lambda fb, lg: rows.append(lg[:, :2048].float().cpu())
    g = torch.Generator().manual_seed(3)
    prompts = [torch.randint(0, 2048, (n,), generator=g).tolist() for n in (40, 9)]
    eng.generate(prompts, {"max_new_tokens": 1})
    eng.shutdown()
    # by value (numpy): a tensor would be shared through a file descriptor that dies with this process
    q.put((rank, torch.cat(rows, 0).numpy() if rows else None))
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def _spawn(fn, world, *args):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=fn, args=(r, world, port, q) + args) for r in range(world)]
    for p in ps:
        p.start()
    res = {}
    for _ in ps:
        item = q.get(timeout=240)
        res[item[0]] = item[1:]
    for p in ps:
        p.join(timeout=60)
    return res


@needs2
def test_one_shot_allreduce_matches_nccl():
    res = _spawn(_ar_worker, 2)
    for rank, (errs, status) in res.items():
        assert status == 0, f"rank {rank}: bounded wait expired"
        assert max(errs) < 1e-2, f"rank {rank}: {errs}"


@needs2
def test_allreduce_with_fused_residual_norm_matches_nccl():
    res = _spawn(_ar_norm_worker, 2)
    for rank, (errs, status) in res.items():
        assert status == 0, f"rank {rank}: bounded wait expired"
        assert len(errs) >= 12 and max(errs) < 2e-2, f"rank {rank}: {errs}"


@needs2
def test_nvls_allreduce_matches_nccl():
    res = _spawn(_nvls_worker, 2)
    for rank, (errs, status) in res.items():
        if errs is None:
            pytest.skip(f"no NVLink multicast: {status}")
        assert status == 0, f"rank {rank}: bounded wait expired"
        assert max(errs) < 2e-2, f"rank {rank}: {errs}"


@needs2
def test_tp2_engine_ranks_agree():
    res = _spawn(_engine_worker, 2)
    assert res[0][0] == res[1][0]
    assert all(len(o) == 8 for o in res[0][0])


def _rel(a, b):
    a, b = torch.as_tensor(a), torch.as_tensor(b)
    return ((a - b).norm() / b.norm()).item()


@needs2
def test_sequence_parallel_prefill_tracks_all_reduce_prefill():
    """TP=2 prefill with every step sequence-parallel (NCCL reduce-scatter / all-gather between layers)
    against the all-reduce layout: same logits up to bf16 summation order."""
    ar = _spawn(_logits_worker, 2, {"sp_min_tokens": 0})
    sp = _spawn(_logits_worker, 2, {"sp_min_tokens": 1})
    for r in (0, 1):
        assert _rel(sp[r][0], ar[r][0]) < 2e-2


@needs2
def test_dp_attention_prefill_tracks_single_gpu():
    """Two attention groups of one GPU each (request 0 on GPU 0, request 1 on GPU 1, experts split over
    both, token rows exchanged around each MoE block) against one GPU running both requests."""
    one = _spawn(_logits_worker, 1, {"tp": 1})[0][0]
    dp = _spawn(_logits_worker, 2, {"dp_size": 2, "enable_dp_attention": True})
    assert dp[0][0].shape[0] == 1 and dp[1][0].shape[0] == 1
    assert _rel(dp[0][0], one[0:1]) < 2e-2
    assert _rel(dp[1][0], one[1:2]) < 2e-2


PD_TINY = dict(num_hidden_layers=2, vocab_size=1000, hidden_size=256, intermediate_size=512,
               num_attention_heads=4, num_key_value_heads=2, head_dim=64)


def _pd_engine(dp_size):
    from sglang_neuron_b200.configs import model_config as mc
    from sglang_neuron_b200.engine import Engine
    from sglang_neuron_b200.server_args import ServerArgs
    mc.PRESETS["pd-gpu-tiny"] = dict(mc.PRESETS["qwen3-0.6b"], **PD_TINY)
    return Engine(ServerArgs(model="pd-gpu-tiny", load_format="random", device="cuda", dp_size=dp_size,
                             context_length=256, max_running_requests=4, chunked_prefill_size=64,
                             random_weight_std=0.05, disable_cuda_graph=True, mem_fraction_static=0.3,
                             max_total_tokens=4096))


def _pd_prompts():
    g = torch.Generator().manual_seed(9)
    return [torch.randint(0, 1000, (n,), generator=g).tolist() for n in (21, 40, 9)]


def _page_sums(pool, pages):
    """Per (buffer, page) byte sums of the given pages of every layer buffer (exact, order-free)."""
    from sglang_neuron_b200.disaggregation.pd import _pool_buffers
    idx = torch.tensor(pages, dtype=torch.long, device=_pool_buffers(pool)[0].device)
    return [b.index_select(0, idx).view(len(pages), -1).view(torch.uint8).long().sum(1).tolist()
            for b in _pool_buffers(pool)]


def _pd_worker(rank, world, port, q):
    """GPU 0 prefills (its own DP replica), GPU 1 decodes; KV pages move by the P2P copy kernel."""
    _init(rank, world, port)
    import time
    import torch.distributed as dist
    from sglang_neuron_b200.disaggregation.pd import DecodeSide, PDLink, PrefillSide
    from sglang_neuron_b200.managers.schedule_batch import SamplingParams
    eng = _pd_engine(2)
    store = dist.distributed_c10d._get_default_store()
    role = "prefill" if rank == 0 else "decode"
    link = PDLink(role, 1, store, timeout_s=60.0)
    assert link.p2p
    sums = {}
    P = eng.runner.page_size
    if role == "prefill":
        side = PrefillSide(eng, link)
        side.on_send = lambda rid, pages: sums.__setitem__(rid, _page_sums(eng.runner.kv_pool, pages))
        for i, p in enumerate(_pd_prompts()):
            side.submit(f"pd{i}", p, SamplingParams(max_new_tokens=7))
        t0 = time.time()
        while (eng.scheduler.has_work() or side.pending or side.sending) and time.time() - t0 < 120:
            side.step()
            time.sleep(0.001)
        result = {"sent": side.sent, "aborted": sorted(side.aborted), "sums": sums}
    else:
        side = DecodeSide(eng, link)
        side.on_admit = lambda h, pages: sums.__setitem__(h.rid, _page_sums(eng.runner.kv_pool, pages))
        t0 = time.time()
        want = {"pd0", "pd1", "pd2"}
        while time.time() - t0 < 120:
            side.step()
            if want.issubset(eng.scheduler.finished_by_rid):
                break
            time.sleep(0.001)
        eng.scheduler.drain()
        result = {"tokens": {rid: eng.scheduler.finished_by_rid[rid].output_ids for rid in sorted(want)
                             if rid in eng.scheduler.finished_by_rid}, "sums": sums, "P": P}
    torch.cuda.synchronize()
    q.put((rank, result))
    dist.barrier()
    dist.destroy_process_group()


def _pd_ref_worker(rank, world, port, q):
    _init(rank, world, port)
    eng = _pd_engine(1)
    out = eng.generate(_pd_prompts(), {"max_new_tokens": 7})
    q.put((rank, [o["output_ids"] for o in out]))


@needs2
def test_pd_p2p_pages_land_exactly_and_tokens_match_aggregated():
    """Prefill on GPU 0, decode on GPU 1: the P2P copy kernel writes every page of every layer into the decode
    pool (byte sums equal page for page), and the decoded tokens equal a one-GPU aggregated engine's."""
    res = _spawn(_pd_worker, 2)
    pre, dec = res[0][0], res[1][0]
    assert pre["sent"] == 3 and pre["aborted"] == []
    for rid, s in pre["sums"].items():
        assert dec["sums"][rid] == s, f"{rid}: pages differ after the P2P copy"
    ref = _spawn(_pd_ref_worker, 1)[0][0]
    assert [dec["tokens"][f"pd{i}"] for i in range(3)] == ref


def _sp_worker(rank, world, port, q):
    os.environ["SGLANG_B200_SP_NVLINK"] = "1"
    _init(rank, world, port)
    import torch.distributed as dist
    from sglang_neuron_b200.parallel.state import initialize_parallel
    from sglang_neuron_b200.parallel.symm_mem import IpcAllReduce
    initialize_parallel(world, device=torch.device("cuda", rank))
    ar = IpcAllReduce(capacity_bytes=8 << 20)
    errs = []
    for rows, H in [(136, 2880), (1, 2880), (512, 4096), (37, 1024)]:
        g = torch.Generator(device="cuda").manual_seed(rows + rank)
        blk = torch.randn(rows, H, generator=g, device="cuda").to(torch.bfloat16)
        ref = torch.empty(rows * world, H, dtype=torch.bfloat16, device="cuda")
        dist.all_gather_into_tensor(ref, blk)
        out = torch.empty_like(ref)
        for _ in range(2):
            ar.all_gather(blk, out)
        torch.cuda.synchronize()
        errs.append(float((out.float() - ref.float()).abs().max()))  # exact copy: 0
        part = torch.randn(rows * world, H, generator=g, device="cuda").to(torch.bfloat16)
        ref_rs = torch.empty(rows, H, dtype=torch.float32, device="cuda")
        dist.reduce_scatter_tensor(ref_rs, part.float())
        got = torch.empty(rows, H, dtype=torch.bfloat16, device="cuda")
        for _ in range(2):
            ar.reduce_scatter(part, got)
        torch.cuda.synchronize()
        errs.append(((got.float() - ref_rs).abs().max() / ref_rs.abs().max()).item())
    q.put((rank, errs, int(ar.status[0])))
    ar.close()
    dist.barrier()
    dist.destroy_process_group()


@needs2
def test_sp_allgather_reducescatter_match_nccl():
    """The sequence-parallel NVLink all-gather (exact) and reduce-scatter (bf16 sum) against NCCL."""
    res = _spawn(_sp_worker, 2)
    for rank, (errs, status) in res.items():
        assert status == 0, f"rank {rank}: bounded wait expired"
        assert all(e == 0.0 for e in errs[0::2]), f"rank {rank}: all-gather {errs[0::2]}"
        assert max(errs[1::2]) < 1e-2, f"rank {rank}: reduce-scatter {errs[1::2]}"
