"""Pipeline parallelism on CPU ranks (gloo): layers split into contiguous stages, (hidden, residual) sent
stage to stage, the last stage's sampled ids broadcast to every rank. Greedy tokens of PP=2 and PP=2 x TP=2
equal the single-rank run, on every rank; decode steps run pipelined in micro-batches."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

TINY_QWEN = dict(num_hidden_layers=3, vocab_size=1000, hidden_size=256, intermediate_size=512,
                 num_attention_heads=4, num_key_value_heads=2, head_dim=64)
TINY_MOE = dict(num_hidden_layers=3, vocab_size=1000, hidden_size=256, moe_intermediate_size=64, num_experts=8,
                num_experts_per_tok=2, num_attention_heads=4, num_key_value_heads=2, head_dim=64)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _run(rank, world, port, base, over, tp, pp, q, sp_min_tokens=0):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), WORLD_SIZE=str(world), RANK=str(rank),
                      LOCAL_RANK=str(rank))
    from sglang_neuron_b200.configs import model_config as mc
    from sglang_neuron_b200.engine import Engine
    from sglang_neuron_b200.parallel.state import destroy_parallel
    from sglang_neuron_b200.server_args import ServerArgs
    from sglang_neuron_b200.models import common
    destroy_parallel()
    calls = [0]
    orig = common.CausalLM._forward_pp_microbatched

    def spy(self, fb):
        calls[0] += 1
        return orig(self, fb)

    common.CausalLM._forward_pp_microbatched = spy  # counts the micro-batched (overlapped) decode steps
    mc.PRESETS["pp-tiny"] = dict(mc.PRESETS[base], **over)
    eng = Engine(ServerArgs(model="pp-tiny", device="cpu", dtype="float32", tp_size=tp, pp_size=pp,
                            context_length=256, max_running_requests=4, chunked_prefill_size=32,
                            random_weight_std=0.05, sp_min_tokens=sp_min_tokens))
    g = torch.Generator().manual_seed(5)
    prompts = [torch.randint(0, 1000, (n,), generator=g).tolist() for n in (23, 7, 40)]
    outs = eng.generate(prompts, {"max_new_tokens": 6})
    q.put((rank, ([o["output_ids"] for o in outs], calls[0])))
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()


def _launch(base, over, tp, pp, sp_min_tokens=0):
    world = tp * pp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_run, args=(r, world, port, base, over, tp, pp, q, sp_min_tokens))
             for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    return res


@pytest.mark.parametrize("base,over", [("qwen3-0.6b", TINY_QWEN), ("qwen3-30b-a3b", TINY_MOE)])
def test_pp2_equals_pp1(base, over):
    """Decode steps of more than one request run as micro-batches pipelined over the two stages."""
    one, n1 = _launch(base, over, 1, 1)[0]
    two = _launch(base, over, 1, 2)
    assert n1 == 0
    for r in (0, 1):
        assert two[r][0] == one and two[r][1] > 0, f"rank {r}"


@pytest.mark.slow
@pytest.mark.parametrize("sp_min_tokens", [0, 1])
def test_pp2_tp2_equals_pp1(sp_min_tokens):
    """sp_min_tokens=1: every prefill step sequence-parallel inside each stage; the stage boundary carries
    each TP rank's block of rows."""
    one = _launch("qwen3-0.6b", TINY_QWEN, 1, 1)[0][0]
    four = _launch("qwen3-0.6b", TINY_QWEN, 2, 2, sp_min_tokens)
    for r in range(4):
        assert four[r][0] == one and four[r][1] > 0, f"rank {r}"


def test_stage_layer_ranges():
    from sglang_neuron_b200.parallel.state import pp_layer_range
    assert [pp_layer_range(36, 4, r) for r in range(4)] == [(0, 9), (9, 18), (18, 27), (27, 36)]
    assert [pp_layer_range(7, 3, r) for r in range(3)] == [(0, 3), (3, 5), (5, 7)]
    with pytest.raises(ValueError):
        pp_layer_range(2, 3, 0)


def test_slice_decode_rebases_rows():
    """A decode step's requests [b0, b1) as a step of their own: per-request tensors sliced, the sampled-row
    index rebased, the split count kept, per-step caches dropped."""
    from sglang_neuron_b200.model_executor.forward_batch import ForwardBatch, ForwardMode
    B = 5
    fb = ForwardBatch(mode=ForwardMode.DECODE, batch_size=B, num_tokens=B, input_ids=torch.arange(B) + 100,
                      positions=torch.arange(B) + 7, out_cache_loc=torch.arange(B) * 16,
                      seq_lens=torch.arange(B, dtype=torch.int32) + 8,
                      block_table=torch.arange(B * 3, dtype=torch.int32).view(B, 3), logits_idx=torch.arange(B),
                      temperature=torch.rand(B), seeds=torch.arange(B), top_k=torch.zeros(B, dtype=torch.int64),
                      top_p=torch.ones(B), decode_splits=3)
    fb.extra.update(num_decode=B, logprob_k=-1, swa_fb="cached")
    sub = fb.slice_decode(2, 5)
    assert sub.batch_size == sub.num_tokens == 3 and sub.decode_splits == 3
    assert torch.equal(sub.input_ids, fb.input_ids[2:]) and torch.equal(sub.block_table, fb.block_table[2:])
    assert torch.equal(sub.logits_idx, torch.arange(3)) and torch.equal(sub.seq_lens, fb.seq_lens[2:])
    assert sub.extra == {"num_decode": 3, "logprob_k": -1}


def test_replica_sizes_must_cover_the_world():
    """Replicas of different TP sizes: on one rank a single TP1 replica is the plain layout; sizes that do not
    add up to the world are refused."""
    from sglang_neuron_b200.parallel.state import destroy_parallel, initialize_parallel, initialize_replicas
    st = initialize_replicas([1])
    assert (st.tp_size, st.tp_rank, st.dp_rank, st.replica_base, st.replica_tp) == (1, 0, 0, 0, (1,))
    with pytest.raises(ValueError):
        initialize_replicas([1, 2])
    with pytest.raises(ValueError):
        initialize_parallel(2, dp_size=1, replica_tp=[2])
    destroy_parallel()
