"""Tensor/expert parallelism on CPU ranks (gloo, world size 2): every TP rank runs the scheduler on the
broadcast request stream, shards QKV/MLP/experts/vocabulary, and the greedy tokens equal the TP=1 run."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

TINY_QWEN = dict(num_hidden_layers=2, vocab_size=1000, hidden_size=256, intermediate_size=512,
                 num_attention_heads=4, num_key_value_heads=2, head_dim=64)
TINY_MOE = dict(num_hidden_layers=2, vocab_size=1000, hidden_size=256, moe_intermediate_size=64, num_experts=8,
                num_experts_per_tok=2, num_attention_heads=4, num_key_value_heads=2, head_dim=64)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _run(rank, world, port, base, over, q, sp=None, args_over=None):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), WORLD_SIZE=str(world), RANK=str(rank),
                      LOCAL_RANK=str(rank))
    from sglang_neuron_b200.configs import model_config as mc
    from sglang_neuron_b200.engine import Engine
    from sglang_neuron_b200.parallel.state import destroy_parallel
    from sglang_neuron_b200.server_args import ServerArgs
    destroy_parallel()
    mc.PRESETS["tp-tiny"] = dict(mc.PRESETS[base], **over)
    from sglang_neuron_b200.models import common
    calls = [0]
    rs = common.sp_reduce_scatter

    def counted(*a, **k):
        calls[0] += 1
        return rs(*a, **k)

    common.sp_reduce_scatter = counted
    dp_calls = [0]
    fdp = common.MoEBlock.forward_dp

    def counted_dp(self, *a, **k):
        dp_calls[0] += 1
        return fdp(self, *a, **k)

    common.MoEBlock.forward_dp = counted_dp
    args_over = dict(args_over or {})
    want_lp = args_over.pop("want_logprobs", False)
    os.environ.update(args_over.pop("env", {}))
    eng = Engine(ServerArgs(model="tp-tiny", device="cpu", dtype="float32", tp_size=world, context_length=256,
                            max_running_requests=4, chunked_prefill_size=32, random_weight_std=0.05,
                            **(args_over or {})))
    g = torch.Generator().manual_seed(5)
    prompts = [torch.randint(0, 1000, (n,), generator=g).tolist() for n in (23, 7, 40)]
    # SPMD: every rank makes the same call; rank 0 owns intake and broadcasts, followers step in lockstep
    outs = eng.generate(prompts, sp or {"max_new_tokens": 6})
    if want_lp:
        q.put((rank, [o["output_ids"] for o in outs], [[lp for lp, _ in o["output_token_logprobs"]] for o in outs]))
    elif (args_over or {}).get("enable_dp_attention"):
        q.put((rank, [o["output_ids"] for o in outs], dp_calls[0], eng.scheduler.stats["output_tokens"]))
    else:
        q.put((rank, [o["output_ids"] for o in outs] + ([calls[0]] if (args_over or {}).get("sp_min_tokens") else [])))
    import torch.distributed as dist
    dist.barrier()
    dist.destroy_process_group()


def _tp(base, over, world, sp=None, args_over=None):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_run, args=(r, world, port, base, over, q, sp, args_over)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in procs:
        item = q.get(timeout=300)
        res[item[0]] = item[1] if len(item) == 2 else item[1:]
    for p in procs:
        p.join(timeout=60)
    return res


@pytest.mark.parametrize("base,over", [("qwen3-0.6b", TINY_QWEN), ("qwen3-30b-a3b", TINY_MOE)])
def test_tp2_equals_tp1(base, over):
    one = _tp(base, over, 1)[0]
    two = _tp(base, over, 2)
    assert two[0] == one, "TP=2 rank 0 tokens differ from TP=1"
    assert two[1] == one, "follower rank saw different tokens"


@pytest.mark.parametrize("base,over", [("qwen3-0.6b", TINY_QWEN), ("qwen3-30b-a3b", TINY_MOE)])
def test_tp2_sequence_parallel_prefill_equals_tp1(base, over):
    """Every prefill step sequence-parallel (sp_min_tokens=1; odd token counts pad the last rank's block):
    the reduce-scatter / all-gather forward gives the TP=1 tokens."""
    one = _tp(base, over, 1, args_over={"sp_min_tokens": 0})[0]
    two = _tp(base, over, 2, args_over={"sp_min_tokens": 1})
    assert two[0][-1] > 0, "no step ran sequence-parallel"
    assert two[0][:-1] == one and two[1][:-1] == one


@pytest.mark.parametrize("base,over", [("qwen3-30b-a3b", TINY_MOE), ("qwen3-0.6b", TINY_QWEN)])
def test_dp_attention_two_groups_equals_tp1(base, over):
    """Two attention groups of one rank (requests split between them, experts split over both ranks, tokens
    all-gathered / reduce-scattered around each MoE block, idle forwards once a group runs dry): the tokens
    of every request equal the single-rank run, on both ranks."""
    one = _tp(base, over, 1)[0]
    two = _tp(base, over, 2, args_over={"dp_size": 2, "enable_dp_attention": True})
    assert two[0][0] == one and two[1][0] == one
    # each group generated only its own requests' tokens (requests 0 and 2 on group 0, request 1 on group 1)
    assert two[0][2] == len(one[0]) + len(one[2]) and two[1][2] == len(one[1])
    if base == "qwen3-30b-a3b":
        assert two[0][1] > 0 and two[0][1] == two[1][1]  # same number of MoE exchanges (lockstep + idle)


def test_tp2_with_step_fence_equals_tp1():
    """SGLANG_B200_STEP_FENCE=1: every step the ranks compare the program they launch through shared memory;
    matching ranks run on unchanged."""
    one = _tp("qwen3-0.6b", TINY_QWEN, 1)[0]
    two = _tp("qwen3-0.6b", TINY_QWEN, 2, args_over={"env": {"SGLANG_B200_STEP_FENCE": "1"}})
    assert two[0] == one and two[1] == one


def test_dp_attention_publishes_logprobs_across_groups():
    """Logprobs of requests served by the other attention group reach every rank with their tokens."""
    sp = {"max_new_tokens": 4, "return_logprob": True, "top_logprobs_num": 2}
    two = _tp("qwen3-30b-a3b", TINY_MOE, 2, sp=sp, args_over={"dp_size": 2, "enable_dp_attention": True,
                                                              "want_logprobs": True})
    one = _tp("qwen3-30b-a3b", TINY_MOE, 1, sp=sp, args_over={"want_logprobs": True})
    ids1, lp1 = one[0]
    for r in (0, 1):
        ids, lp = two[r]
        assert ids == ids1
        assert len(lp) == 3 and all(len(x) == 4 for x in lp)
        for a, b in zip(lp, lp1):
            assert all(abs(u - v) < 1e-3 for u, v in zip(a, b))


@pytest.mark.slow
def test_dp_attention_groups_of_two_ranks_equals_tp1():
    """World 4: two attention groups of two TP ranks each; experts over all four ranks."""
    one = _tp("qwen3-30b-a3b", TINY_MOE, 1)[0]
    four = _tp("qwen3-30b-a3b", TINY_MOE, 4, args_over={"dp_size": 2, "enable_dp_attention": True})
    for r in range(4):
        assert four[r][0] == one, f"rank {r}"


def _contract_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), WORLD_SIZE=str(world), RANK=str(rank),
                      LOCAL_RANK=str(rank))
    import torch.distributed as dist
    from sglang_neuron_b200.parallel.contract import assert_fleet_consistent
    from sglang_neuron_b200.parallel.state import destroy_parallel, init_process_group_from_env, initialize_parallel
    destroy_parallel()
    init_process_group_from_env(backend="gloo", timeout_s=60)
    initialize_parallel(world, device=torch.device("cpu"))
    same = assert_fleet_consistent({"model": "x"})
    try:
        assert_fleet_consistent({"model": "x", "layers": 2 + rank})
        q.put((rank, same, "accepted"))
    except RuntimeError:
        q.put((rank, same, "refused"))
    dist.barrier()
    dist.destroy_process_group()


def test_fleet_contract_refuses_mismatched_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_contract_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = dict((r, (d, v)) for r, d, v in (q.get(timeout=120) for _ in ps))
    for p in ps:
        p.join(timeout=30)
    assert res[0][0] == res[1][0]
    assert res[0][1] == res[1][1] == "refused"


def test_tp2_filtered_sampling_equals_tp1():
    """Top-k/top-p sampling with a seed: the vocabulary-sharded candidate-pool merge gives the TP=1 tokens."""
    sp = {"max_new_tokens": 6, "temperature": 0.9, "top_k": 20, "top_p": 0.8, "seed": 7}
    one = _tp("qwen3-0.6b", TINY_QWEN, 1, sp)[0]
    two = _tp("qwen3-0.6b", TINY_QWEN, 2, sp)
    assert two[0] == one and two[1] == one
