"""Disaggregated prefill/decode on CPU ranks (gloo): rank 0 is the prefill group, rank 1 the decode group;
KV pages move rank to rank, and the decoded tokens equal the aggregated engine's. A second case drops the
decode side's acknowledgement (host-injected failure) and checks the prefill side aborts and frees pages."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

TINY = dict(num_hidden_layers=2, vocab_size=1000, hidden_size=256, intermediate_size=512,
            num_attention_heads=4, num_key_value_heads=2, head_dim=64)


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _prompts():
    g = torch.Generator().manual_seed(9)
    return [torch.randint(0, 1000, (n,), generator=g).tolist() for n in (21, 40, 9)]


def _engine(dp_size, tp_size=1, replica_tp=None):
    from sglang_neuron_b200.configs import model_config as mc
    from sglang_neuron_b200.engine import Engine
    from sglang_neuron_b200.parallel.state import destroy_parallel
    from sglang_neuron_b200.server_args import ServerArgs
    destroy_parallel()
    mc.PRESETS["pd-tiny"] = dict(mc.PRESETS["qwen3-0.6b"], **TINY)
    return Engine(ServerArgs(model="pd-tiny", device="cpu", dtype="float32", tp_size=tp_size, dp_size=dp_size,
                             context_length=256, max_running_requests=4, chunked_prefill_size=32,
                             random_weight_std=0.05, replica_tp_sizes=replica_tp))


def _worker(rank, port, drop_ack, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), WORLD_SIZE="2", RANK=str(rank), LOCAL_RANK="0")
    import time
    import torch.distributed as dist
    from sglang_neuron_b200.disaggregation.pd import DecodeSide, PDLink, PrefillSide
    from sglang_neuron_b200.managers.schedule_batch import SamplingParams
    eng = _engine(2)
    store = dist.distributed_c10d._get_default_store()
    role = "prefill" if rank == 0 else "decode"
    link = PDLink(role, 1, store, timeout_s=3.0 if drop_ack else 60.0)
    prompts = _prompts()
    result = None
    if role == "prefill":
        side = PrefillSide(eng, link)
        for i, p in enumerate(prompts):
            side.submit(f"pd{i}", p, SamplingParams(max_new_tokens=7))
        t0 = time.time()
        while (eng.scheduler.has_work() or side.pending or side.sending) and time.time() - t0 < 120:
            side.step()
            time.sleep(0.001)
        result = {"sent": side.sent, "aborted": sorted(side.aborted), "free": eng.scheduler.alloc.available()
                  + eng.scheduler.alloc.staged()}
    elif drop_ack:
        # injected failure: the decode group never answers (it stays up but never polls the store)
        time.sleep(6)
        result = {}
    else:
        side = DecodeSide(eng, link)
        t0 = time.time()
        want = {"pd0", "pd1", "pd2"}
        while time.time() - t0 < (8 if drop_ack else 120):
            side.step()
            if want.issubset(eng.scheduler.finished_by_rid):
                break
            time.sleep(0.001)
        eng.scheduler.drain()
        result = {rid: eng.scheduler.finished_by_rid[rid].output_ids for rid in sorted(want)
                  if rid in eng.scheduler.finished_by_rid}
    q.put((rank, result))
    dist.barrier()
    dist.destroy_process_group()


def _run(drop_ack):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_worker, args=(r, port, drop_ack, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = dict(q.get(timeout=300) for _ in ps)
    for p in ps:
        p.join(timeout=60)
    return res


def test_pd_matches_aggregated():
    res = _run(drop_ack=False)
    eng = _engine(1)
    ref = eng.generate(_prompts(), {"max_new_tokens": 7})
    assert res[0]["sent"] == 3 and res[0]["aborted"] == []
    assert [res[1][f"pd{i}"] for i in range(3)] == [o["output_ids"] for o in ref]


def test_pd_prefill_aborts_when_decode_never_answers():
    res = _run(drop_ack=True)
    assert res[0]["sent"] == 0 and res[0]["aborted"] == ["pd0", "pd1", "pd2"]
    assert res[1] == {}


def _worker_tp2(rank, port, q):
    """World 4: prefill group = ranks 0-1 (TP2), decode group = ranks 2-3 (TP2); every rank of a group makes
    the same calls (the group's rank 0 owns intake and the store protocol)."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), WORLD_SIZE="4", RANK=str(rank),
                      LOCAL_RANK="0")
    import time
    import torch.distributed as dist
    from sglang_neuron_b200.disaggregation.pd import DecodeSide, PDLink, PrefillSide
    from sglang_neuron_b200.managers.schedule_batch import SamplingParams
    eng = _engine(2, tp_size=2)
    store = dist.distributed_c10d._get_default_store()
    role = "prefill" if rank < 2 else "decode"
    link = PDLink(role, 2, store, timeout_s=60.0)
    result = None
    if role == "prefill":
        side = PrefillSide(eng, link)
        for i, p in enumerate(_prompts()):
            side.submit(f"pd{i}", p, SamplingParams(max_new_tokens=7))
        from sglang_neuron_b200.parallel.state import get_state
        t0 = time.time()
        while time.time() - t0 < 120:
            side.step()
            # the group's ranks stop together (step() is a lockstep call): MIN of their "done" flags
            done = torch.tensor([int(side.sent == 3 and not side.pending and not side.sending)])
            dist.all_reduce(done, op=dist.ReduceOp.MIN, group=get_state().cpu_group)
            if int(done):
                break
            time.sleep(0.001)
        result = {"sent": side.sent, "aborted": sorted(side.aborted)}
    else:
        side = DecodeSide(eng, link)
        t0 = time.time()
        want = {"pd0", "pd1", "pd2"}
        from sglang_neuron_b200.parallel.state import get_state
        while time.time() - t0 < 120:
            side.step()
            done = torch.tensor([int(want.issubset(eng.scheduler.finished_by_rid))])
            dist.all_reduce(done, op=dist.ReduceOp.MIN, group=get_state().cpu_group)
            if int(done):
                break
            time.sleep(0.001)
        eng.scheduler.drain()
        result = {rid: eng.scheduler.finished_by_rid[rid].output_ids for rid in sorted(want)
                  if rid in eng.scheduler.finished_by_rid}
    q.put((rank, result))
    dist.barrier()
    dist.destroy_process_group()


def test_pd_tp2_groups_match_aggregated():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_worker_tp2, args=(r, port, q)) for r in range(4)]
    for p in ps:
        p.start()
    res = dict(q.get(timeout=300) for _ in ps)
    for p in ps:
        p.join(timeout=60)
    ref = _engine(1).generate(_prompts(), {"max_new_tokens": 7})
    assert res[0]["sent"] == 3 and res[1]["sent"] == 3
    for r in (2, 3):
        assert [res[r][f"pd{i}"] for i in range(3)] == [o["output_ids"] for o in ref]


def _worker_mixed_tp(rank, port, tp_p, tp_d, q):
    """Prefill group of TP tp_p (ranks 0 .. tp_p - 1) and decode group of TP tp_d after it: the KV moves as
    head slices of each page (every decode rank gets its heads from the prefill ranks that hold them)."""
    world = tp_p + tp_d
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), WORLD_SIZE=str(world), RANK=str(rank),
                      LOCAL_RANK="0")
    import time
    import torch.distributed as dist
    from sglang_neuron_b200.disaggregation.pd import DecodeSide, PDLink, PrefillSide
    from sglang_neuron_b200.managers.schedule_batch import SamplingParams
    from sglang_neuron_b200.parallel.state import get_state
    role = "prefill" if rank < tp_p else "decode"
    own, other = (tp_p, tp_d) if role == "prefill" else (tp_d, tp_p)
    eng = _engine(2, tp_size=own, replica_tp=[tp_p, tp_d])
    store = dist.distributed_c10d._get_default_store()
    link = PDLink(role, own, store, timeout_s=60.0, peer_tp=other)
    group = get_state().cpu_group
    result = None
    t0 = time.time()
    if role == "prefill":
        side = PrefillSide(eng, link)
        for i, p in enumerate(_prompts()):
            side.submit(f"pd{i}", p, SamplingParams(max_new_tokens=7))
        while time.time() - t0 < 120:
            side.step()
            done = torch.tensor([int(side.sent == 3 and not side.pending and not side.sending)])
            if group is not None:
                dist.all_reduce(done, op=dist.ReduceOp.MIN, group=group)
            if int(done):
                break
            time.sleep(0.001)
        result = {"sent": side.sent, "aborted": sorted(side.aborted)}
    else:
        side = DecodeSide(eng, link)
        want = {"pd0", "pd1", "pd2"}
        while time.time() - t0 < 120:
            side.step()
            done = torch.tensor([int(want.issubset(eng.scheduler.finished_by_rid))])
            if group is not None:
                dist.all_reduce(done, op=dist.ReduceOp.MIN, group=group)
            if int(done):
                break
            time.sleep(0.001)
        eng.scheduler.drain()
        result = {rid: eng.scheduler.finished_by_rid[rid].output_ids for rid in sorted(want)
                  if rid in eng.scheduler.finished_by_rid}
    q.put((rank, result))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("tp_p,tp_d", [(1, 2), (2, 1)])
def test_pd_groups_of_different_tp_sizes_match_aggregated(tp_p, tp_d):
    """Prefill TP1 -> decode TP2 and prefill TP2 -> decode TP1 (two KV heads): every decode rank decodes the
    same tokens as the aggregated engine."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_worker_mixed_tp, args=(r, port, tp_p, tp_d, q)) for r in range(tp_p + tp_d)]
    for p in ps:
        p.start()
    res = dict(q.get(timeout=300) for _ in ps)
    for p in ps:
        p.join(timeout=60)
    ref = _engine(1).generate(_prompts(), {"max_new_tokens": 7})
    for r in range(tp_p):
        assert res[r]["sent"] == 3 and res[r]["aborted"] == []
    for r in range(tp_p, tp_p + tp_d):
        assert [res[r][f"pd{i}"] for i in range(3)] == [o["output_ids"] for o in ref]


def test_head_major_slice_plan_across_tp_sizes():
    """Prefill TP8 (1 KV head each) -> decode TP4 (2 heads each): decode rank j takes head 2j from prefill rank 2j
    and head 2j+1 from rank 2j+1, each a contiguous slice of the page; replicated heads come from the lowest
    holder; a decode head nobody holds is refused."""
    from sglang_neuron_b200.disaggregation.pd import slice_plan
    hb = 16 * 64  # page_size x head_dim bytes (fp8)
    pre = [{"head_start": i, "heads": 1, "head_bytes": hb} for i in range(8)]
    dec = [{"head_start": 2 * j, "heads": 2, "head_bytes": hb} for j in range(4)]
    plan = slice_plan(pre, dec)
    assert sorted(plan) == sorted([(2 * j + h, j, 0, h * hb, hb) for j in range(4) for h in range(2)])
    # decode TP8 from prefill TP4: each decode rank takes the half of one prefill rank's page
    plan = slice_plan(dec, pre)
    assert sorted(plan) == sorted([(i // 2, i, (i % 2) * hb, 0, hb) for i in range(8)])
    # equal TP: whole pages rank to rank
    assert slice_plan(dec, dec) == [(j, j, 0, 0, 2 * hb) for j in range(4)]
    # TP16 over 8 heads (replicated: ranks 2h and 2h+1 both hold head h) -> decode TP8: the lower holder sends
    rep = [{"head_start": r // 2, "heads": 1, "head_bytes": hb} for r in range(16)]
    assert sorted(slice_plan(rep, pre)) == sorted([(2 * i, i, 0, 0, hb) for i in range(8)])
    with pytest.raises(ValueError):
        slice_plan(pre[:4], dec)
