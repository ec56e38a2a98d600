"""Prefix-cache reuse end to end on the CPU tier: a prompt that shares full pages with a finished request
reuses them (cache hit) and produces the same greedy tokens as without the cache; the same with the host
tier (HiCache) after the device tree has evicted the prefix."""
import torch

from sglang_neuron_b200.configs import model_config as mc
from sglang_neuron_b200.engine import Engine
from sglang_neuron_b200.parallel.state import destroy_parallel
from sglang_neuron_b200.server_args import ServerArgs

TINY = dict(num_hidden_layers=2, vocab_size=1000, hidden_size=128, intermediate_size=256,
            num_attention_heads=4, num_key_value_heads=2, head_dim=32)


def _engine(**kw):
    destroy_parallel()
    mc.PRESETS["pc-tiny"] = dict(mc.PRESETS["qwen3-0.6b"], **TINY)
    base = dict(model="pc-tiny", device="cpu", dtype="float32", context_length=512, max_running_requests=4,
                chunked_prefill_size=64, page_size=16, random_weight_std=0.05)
    base.update(kw)
    return Engine(ServerArgs(**base))


def _prompts():
    g = torch.Generator().manual_seed(9)
    shared = torch.randint(1, 1000, (70,), generator=g).tolist()
    return shared, [shared + torch.randint(1, 1000, (n,), generator=g).tolist() for n in (5, 19)]


def test_prefix_hit_matches_no_cache():
    shared, (a, b) = _prompts()
    ref = _engine(disable_radix_cache=True)
    want = [o["output_ids"] for o in ref.generate([a, b], {"max_new_tokens": 8})]
    eng = _engine()
    first = eng.generate([a], {"max_new_tokens": 8})[0]["output_ids"]
    second = eng.generate([b], {"max_new_tokens": 8})[0]["output_ids"]
    assert eng.scheduler.stats["cache_hit_tokens"] >= 64
    assert [first, second] == want


def test_prefix_hit_in_a_different_slot():
    """The request that reuses the prefix runs in a slot whose block-table row held another request's
    pages: the reused pages must be written into that row."""
    shared, (a, b) = _prompts()
    g = torch.Generator().manual_seed(11)
    c = torch.randint(1, 1000, (40,), generator=g).tolist()
    ref = _engine(disable_radix_cache=True)
    want = ref.generate([b], {"max_new_tokens": 8})[0]["output_ids"]
    for order in ([a, c], [c, a]):
        eng = _engine()
        eng.generate(order, {"max_new_tokens": 8})
        got = eng.generate([b], {"max_new_tokens": 8})[0]["output_ids"]
        assert eng.scheduler.stats["cache_hit_tokens"] >= 64
        assert got == want, f"order {order is a}"


def test_host_tier_reload_after_device_eviction():
    """A small device pool evicts the shared prefix from the device tree; the host tier (write-through at
    insert) reloads its pages for the next request and the tokens equal the no-cache run."""
    shared, (a, b) = _prompts()
    ref = _engine(disable_radix_cache=True)
    want = ref.generate([b], {"max_new_tokens": 8})[0]["output_ids"]
    eng = _engine(enable_hierarchical_cache=True, max_total_tokens=16 * 24, max_running_requests=2)
    eng.generate([a], {"max_new_tokens": 8})
    g = torch.Generator().manual_seed(13)
    for _ in range(3):  # unrelated prompts push the shared prefix out of the device tree
        eng.generate([torch.randint(1, 1000, (150,), generator=g).tolist()], {"max_new_tokens": 4})
    got = eng.generate([b], {"max_new_tokens": 8})[0]["output_ids"]
    st = eng.scheduler.stats
    assert st.get("host_hit_tokens", 0) >= 64, st
    assert eng.scheduler.hicache.stats["written_pages"] > 0 and eng.scheduler.hicache.stats["loaded_pages"] >= 4
    assert got == want


def test_chain_hashes_prefix_property():
    from sglang_neuron_b200.mem_cache.hicache import chain_hashes
    x = list(range(100))
    h1 = chain_hashes(x, 16, 6)
    h2 = chain_hashes(x[:64] + [7] * 36, 16, 6)
    assert h1[:4] == h2[:4] and h1[4] != h2[4] and h1[5] != h2[5]


def test_chunk_grid_prefix_hits_replay_uncached_chunks():
    """prefill_chunk_grid: chunks end on multiples of the grid and prefix hits are rounded down to it, so a
    request that hits the cache computes exactly the chunks it would have computed uncached: the greedy
    tokens equal a cache-less run."""
    import torch
    from sglang_neuron_b200.engine import Engine
    from sglang_neuron_b200.parallel.state import destroy_parallel
    from sglang_neuron_b200.server_args import ServerArgs
    mc.PRESETS["pc-tiny"] = dict(mc.PRESETS["qwen3-0.6b"], **TINY)
    outs = {}
    for cache in (False, True):
        destroy_parallel()
        eng = Engine(ServerArgs(model="pc-tiny", device="cpu", dtype="float32", page_size=4, context_length=256,
                                max_running_requests=4, chunked_prefill_size=32, prefill_chunk_grid=8,
                                disable_radix_cache=not cache, random_weight_std=0.05))
        g = torch.Generator().manual_seed(2)
        shared = torch.randint(0, 1000, (29,), generator=g).tolist()
        res, hits = [], []
        for tail in (3, 11):
            o = eng.generate([shared + torch.randint(0, 1000, (tail,), generator=g).tolist()], {"max_new_tokens": 4})[0]
            res.append(o["output_ids"])
            hits.append(o["cached_tokens"])
        outs[cache] = (res, hits)
    assert outs[True][0] == outs[False][0]
    assert outs[True][1][1] > 0 and outs[True][1][1] % 8 == 0
