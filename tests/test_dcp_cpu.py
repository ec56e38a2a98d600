"""Decode context parallelism for the latent (MLA) pool: page ownership by logical index, the per-rank
partial attention over interleaved pages merged by log-sum-exp equals attention over the whole context, and
a TP=2 x DCP=2 DeepSeek-V2 engine (each rank stores half of every context) gives the single-rank tokens."""
import torch

from sglang_neuron_b200.parallel.dcp import DcpPageAllocator, merge_partials, partial_ref

TINY_DS = dict(num_hidden_layers=2, vocab_size=1000, hidden_size=256, intermediate_size=512, moe_intermediate_size=64,
               n_routed_experts=8, num_experts_per_tok=2, n_shared_experts=1, num_attention_heads=4,
               num_key_value_heads=4, kv_lora_rank=64, qk_nope_head_dim=32, qk_rope_head_dim=16, v_head_dim=32)


def test_allocator_owner_follows_logical_index():
    a = DcpPageAllocator(10, 16, 2)
    pages = a.alloc_at(3, 5)  # logical pages 3..7 -> owners 1, 0, 1, 0, 1
    assert [g % 2 for g in pages] == [1, 0, 1, 0, 1]
    assert all(g // 2 >= 1 for g in pages)  # local page 0 is reserved on every owner
    before = a.available()
    a.free(pages)
    assert a.available() >= before
    assert a.alloc_at(0, 40) == []  # more than one owner holds


def test_interleaved_partials_merge_to_full_attention():
    from sglang_neuron_b200.ops.mla import _one
    torch.manual_seed(0)
    P, D, r, rope = 4, 2, 64, 16
    chunks = [(0, 9), (13, 4), (6, 1)]          # (prefix, new tokens) per request
    lens = [p + n for p, n in chunks]
    n_log = max((L + P - 1) // P for L in lens)
    # global page ids: logical page j of request b -> owner j % D, local id per owner
    loc_next = [1] * D
    gbt = torch.zeros(len(chunks), n_log + 1, dtype=torch.int32)
    for b in range(len(chunks)):
        for j in range(n_log):
            o = j % D
            gbt[b, j] = loc_next[o] * D + o
            loc_next[o] += 1
    n_local = max(loc_next) + 1
    full = torch.randn(len(chunks), n_log * P, r + rope)           # every request's latent rows
    caches = [torch.zeros(n_local, 1, P, r + rope) for _ in range(D)]
    for b in range(len(chunks)):
        for t in range(lens[b]):
            g = int(gbt[b, t // P])
            caches[g % D][g // D, 0, t % P] = full[b, t]
    H = 3
    T = sum(n for _, n in chunks)
    q = torch.randn(T, H, r + rope)
    qo = torch.tensor([0] + list(torch.tensor([n for _, n in chunks]).cumsum(0)), dtype=torch.int32)
    seq = torch.tensor(lens, dtype=torch.int32)
    o_parts, l_parts = [], []
    for d in range(D):
        lbt = torch.div(gbt[:, d::D], D, rounding_mode="floor")
        o, l = partial_ref(q, caches[d], lbt, seq, qo, P, 0.2, D, d, r)
        o_parts.append(o)
        l_parts.append(l)
    got = merge_partials(torch.stack(o_parts), torch.stack(l_parts))
    # reference: one cache holding every page in logical order
    ref_cache = full.view(len(chunks), n_log, 1, P, r + rope)
    for b, (p, n) in enumerate(chunks):
        s0 = int(qo[b])
        bt = torch.arange(n_log, dtype=torch.int32)
        want = _one(q[s0:s0 + n], ref_cache[b], bt, lens[b], torch.arange(p, p + n), r, 0.2, P)
        assert torch.allclose(got[s0:s0 + n], want, atol=1e-4, rtol=1e-4)


def test_tp2_dcp2_deepseek_equals_tp1():
    from test_tp_cpu import _tp
    one = _tp("deepseek-v2-lite", TINY_DS, 1)[0]
    two = _tp("deepseek-v2-lite", TINY_DS, 2, args_over={"dcp_size": 2})
    assert two[0] == one and two[1] == one


def _prefix_worker(rank, world, port, q, dcp):
    import os
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), WORLD_SIZE=str(world), RANK=str(rank),
                      LOCAL_RANK=str(rank))
    from sglang_neuron_b200.configs import model_config as mc
    from sglang_neuron_b200.engine import Engine
    from sglang_neuron_b200.parallel.state import destroy_parallel
    from sglang_neuron_b200.server_args import ServerArgs
    destroy_parallel()
    mc.PRESETS["dcp-tiny"] = dict(mc.PRESETS["deepseek-v2-lite"], **TINY_DS)
    eng = Engine(ServerArgs(model="dcp-tiny", device="cpu", dtype="float32", tp_size=world, dcp_size=dcp,
                            page_size=4, context_length=256, max_running_requests=4, chunked_prefill_size=16,
                            random_weight_std=0.05))
    g = torch.Generator().manual_seed(9)
    shared = torch.randint(0, 1000, (37,), generator=g).tolist()
    outs = []
    for tail in (5, 9, 2):  # one after the other: later prompts hit the first one's cached pages
        p = shared + torch.randint(0, 1000, (tail,), generator=g).tolist()
        outs.append(eng.generate([p], {"max_new_tokens": 5})[0])
    q.put((rank, [o["output_ids"] for o in outs], [o["cached_tokens"] for o in outs]))
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()


def _spawn(world, dcp):
    import socket
    import torch.multiprocessing as mp
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_prefix_worker, args=(r, world, port, q, dcp)) for r in range(world)]
    for p in ps:
        p.start()
    res = {}
    for _ in ps:
        item = q.get(timeout=300)
        res[item[0]] = item[1:]
    for p in ps:
        p.join(timeout=60)
    return res


def test_dcp_prefix_cache_hits_keep_page_owners():
    """Prefix-cache hits under DCP reuse cached pages at the same logical indices (same owner rank): the
    tokens equal the single-rank run and the later prompts do hit."""
    one = _spawn(1, 1)[0]
    two = _spawn(2, 2)
    assert two[0][0] == one[0] and two[1][0] == one[0]
    assert two[0][1][1] > 0 and two[0][1][2] > 0


def test_dcp_view_local_tables_and_slots(monkeypatch):
    """Global page g = local * D + owner: rank d's table keeps logical pages d, d + D, ... as local ids, and a
    write slot survives only on the owner of its page (others get -1)."""
    from sglang_neuron_b200.model_executor.forward_batch import ForwardBatch, ForwardMode
    from sglang_neuron_b200.parallel import dcp as dcp_mod
    from sglang_neuron_b200.parallel.state import ParallelState

    P, D = 4, 2
    gbt = torch.tensor([[2 * 1 + 0, 2 * 1 + 1, 2 * 2 + 0, 2 * 2 + 1, 0]], dtype=torch.int32)  # logical 0..3 + pad
    loc = torch.tensor([gbt[0, 2].item() * P + 1, gbt[0, 3].item() * P + 3, -1], dtype=torch.int64)
    fb = ForwardBatch(mode=ForwardMode.EXTEND, batch_size=1, num_tokens=3, input_ids=torch.zeros(3, dtype=torch.int64),
                      positions=torch.zeros(3, dtype=torch.int64), out_cache_loc=loc,
                      seq_lens=torch.tensor([16], dtype=torch.int32), block_table=gbt,
                      logits_idx=torch.zeros(1, dtype=torch.int64))
    for d, want_bt, want_loc in [(0, [1, 2, 0], [2 * P + 1, -1, -1]), (1, [1, 2], [-1, 2 * P + 3, -1])]:
        monkeypatch.setattr(dcp_mod, "get_state", lambda d=d: ParallelState(dcp_size=D, dcp_rank=d))
        fb.extra.clear()
        bt, lloc = dcp_mod.DcpView(P).local(fb)
        assert bt[0].tolist() == want_bt and lloc.tolist() == want_loc
