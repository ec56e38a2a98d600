"""Native host runtime (C++ page allocator, radix prefix cache) against its Python twins, plus the platform
surface: env registry, serving policy, catalog refusals, hook registry."""
import random

import pytest

from sglang_neuron_b200.mem_cache.allocator import PyPageAllocator, PyRadixCache, RadixCacheHandle, make_page_allocator


def test_allocator_retire_aware_frees():
    for native in (True, False):
        a = make_page_allocator(10, 16, reserved=1, native=native)
        assert a.available() == 9
        p = list(a.alloc(4))
        assert len(p) == 4 and 0 not in p
        assert list(a.alloc(6)) == []  # all-or-nothing
        a.free_after(p[:2], epoch=5)
        assert a.available() == 5 and a.staged() == 2
        assert a.retire(4) == 0 and a.available() == 5
        assert a.retire(5) == 2 and a.available() == 7
        with pytest.raises((IndexError, Exception)):
            a.free([0])


def test_radix_native_matches_python_twin():
    rng = random.Random(0)
    P = 4
    nat, py = RadixCacheHandle(P, native=True), RadixCacheHandle(P, native=False)
    assert nat.native
    next_page = [1]
    seqs = []
    for i in range(60):
        if seqs and rng.random() < 0.6:
            base = rng.choice(seqs)
            cut = rng.randrange(0, len(base) + 1)
            s = base[:cut] + [rng.randrange(50) for _ in range(rng.randrange(0, 20))]
        else:
            s = [rng.randrange(50) for _ in range(rng.randrange(1, 30))]
        seqs.append(s)
        m1 = nat.match_prefix(s)
        m2 = py.match_prefix(s)
        assert m1[0] == m2[0] and list(m1[1]) == list(m2[1])
        n_pages = len(s) // P
        pages = list(m1[1]) + list(range(next_page[0], next_page[0] + n_pages - len(m1[1])))
        next_page[0] += n_pages
        d1 = nat.insert(s, pages)
        d2 = py.insert(s, pages)
        assert sorted(d1) == sorted(d2)
        assert nat.cached_pages() == py.cached_pages()
    for k in (3, 7, 100):
        assert sorted(nat.evict(k)) == sorted(py.evict(k))
        assert nat.cached_pages() == py.cached_pages()


def test_radix_lock_blocks_eviction():
    r = RadixCacheHandle(2, native=True)
    r.insert([1, 2, 3, 4], [10, 11])
    _, pages, node = r.match_prefix([1, 2, 3, 4, 9])
    assert list(pages) == [10, 11]
    r.inc_lock(node)
    assert r.evict(5) == [] or list(r.evict(5)) == []
    r.dec_lock(node)
    assert sorted(r.evict(5)) == [10, 11]


def test_env_registry_and_policy(monkeypatch):
    from sglang_neuron_b200 import env_registry, serving_policy
    from sglang_neuron_b200.server_args import ServerArgs
    env = {"SGLANG_B200_HOST_TRACE": "/tmp/x"}
    env_registry.refuse_unknown(env)
    with pytest.raises(env_registry.UnknownEnvError):
        env_registry.refuse_unknown({"SGLANG_B200_HOST_TRAC": "1"})
    pol = serving_policy.resolve(ServerArgs(tp_size=2, disable_radix_cache=True))
    e = {}
    serving_policy.export(pol, e)
    back = serving_policy.current(e)
    assert back == pol and back.prefix_cache == "none" and back.tp_size == 2


def test_catalog_and_platform_refusals():
    from sglang_neuron_b200.models.catalog import model_spec
    from sglang_neuron_b200.platform import B200SRTPlatform, check_kv_cache, refuse_unserved
    from sglang_neuron_b200.server_args import ServerArgs
    spec = model_spec("GptOssForCausalLM")
    assert spec.expert_format == "mxfp4" and spec.sinks
    with pytest.raises(ValueError):
        model_spec("KimiK3ForCausalLM")
    with pytest.raises(ValueError):
        refuse_unserved(ServerArgs(speculative_algorithm="MTP"), spec)
    with pytest.raises(ValueError):
        check_kv_cache(ServerArgs(page_size=12), spec)
    p = B200SRTPlatform()
    args = p.apply_server_args_defaults(ServerArgs(model="qwen3-0.6b", device="cpu"))
    assert args.model == "qwen3-0.6b"
    assert p.get_kv_pool_cls(kind="mla").__name__ == "MLATokenToKVPool"


def test_hook_registry_resolves_and_refuses_double_replace():
    from sglang_neuron_b200 import general_plugin as gp
    reg = gp.ResolvingHookRegistry()
    target = "sglang_neuron_b200.sglang_tree:rank_label"
    pin = gp.source_md5(gp.resolve_target(target)[2])
    reg.register(target, "AROUND", lambda orig: "wrapped-" + orig(), pin_md5=pin)
    from sglang_neuron_b200 import sglang_tree
    assert sglang_tree.rank_label().startswith("wrapped-")
    with pytest.raises(gp.HookError):
        reg.register("sglang_neuron_b200.sglang_tree:dp_widths", "REPLACE", lambda: (1, 1), pin_md5="0" * 32)
    reg.undo_all()
    assert not sglang_tree.rank_label().startswith("wrapped-")
    assert gp.register() == "sglang_neuron_b200.platform.B200SRTPlatform"


def test_contract_digests_and_clean_exit():
    import os
    import signal
    from sglang_neuron_b200.parallel.contract import assert_fleet_consistent, digest
    from sglang_neuron_b200.process_init import install_clean_exit
    assert digest({"a": 1, "b": [2, 3]}) == digest({"b": [2, 3], "a": 1})
    assert digest({"a": 1}) != digest({"a": 2})
    assert assert_fleet_consistent({"x": 1}) == digest({"x": 1})  # single process: no gather
    prev = signal.getsignal(signal.SIGTERM)
    try:
        install_clean_exit()
        import pytest
        with pytest.raises(SystemExit):
            os.kill(os.getpid(), signal.SIGTERM)
            import time
            time.sleep(1)
    finally:
        signal.signal(signal.SIGTERM, prev)


def _shm_worker(r, name, q):
    import time
    from sglang_neuron_b200._ext import _runtime as rt
    time.sleep(0.2)
    s = rt.ShmReduce(name, 3, r, 2, False)
    outs = [s.max([r, -r]) for _ in range(300)]
    q.put((r, outs[-1], s.min([r * 7, 5])))


def test_shm_reduce_min_max_over_processes():
    """Node shared-memory MIN / MAX over three processes, 300 calls in a row (double-buffered epochs), and a
    clear error when a rank never arrives."""
    import multiprocessing as mp
    import os
    import pytest
    from sglang_neuron_b200._ext import _runtime as rt
    if rt is None or not hasattr(rt, "ShmReduce"):
        pytest.skip("native runtime not built")
    name = f"/snb_test_{os.getpid()}"
    s0 = rt.ShmReduce(name, 3, 0, 2, True)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_shm_worker, args=(r, name, q)) for r in (1, 2)]
    for p in ps:
        p.start()
    outs = [s0.max([0, 0]) for _ in range(300)]
    last_min = s0.min([0, 5])
    got = dict((r, (a, b)) for r, a, b in (q.get(timeout=60) for _ in ps))
    for p in ps:
        p.join(timeout=30)
    assert outs[-1] == [2, 0] and last_min == [0, 5]
    assert got[1] == ([2, 0], [0, 5]) and got[2] == ([2, 0], [0, 5])
    lonely = rt.ShmReduce(name + "_b", 2, 0, 1, True)
    with pytest.raises(RuntimeError, match="did not arrive"):
        lonely.max([1], timeout_s=0.2)


def test_invalid_sampled_token_id_ends_only_that_request():
    """A sampled id outside the vocabulary (what a corrupted logits row gives) ends its request with an error
    reason; the other requests of the batch finish normally."""
    import torch
    from sglang_neuron_b200.configs import model_config as mc
    from sglang_neuron_b200.engine import Engine
    from sglang_neuron_b200.parallel.state import destroy_parallel
    from sglang_neuron_b200.server_args import ServerArgs
    destroy_parallel()
    mc.PRESETS["inv-tiny"] = dict(mc.PRESETS["qwen3-0.6b"], num_hidden_layers=1, vocab_size=500, hidden_size=128,
                                  intermediate_size=256, num_attention_heads=2, num_key_value_heads=1, head_dim=64)
    eng = Engine(ServerArgs(model="inv-tiny", device="cpu", dtype="float32", context_length=128,
                            max_running_requests=4, random_weight_std=0.05, disable_overlap_schedule=True))
    calls = [0]
    sample = eng.runner.sample

    def bad_third_step(*a, **k):
        ids = sample(*a, **k)
        calls[0] += 1
        if calls[0] == 3:
            ids[0] = 10_000  # the first request of this step gets an impossible id
        return ids

    eng.runner.sample = bad_third_step
    outs = eng.generate([[1, 2, 3], [4, 5, 6, 7]], {"max_new_tokens": 6})
    reasons = sorted(o["finish_reason"] for o in outs)
    assert reasons == ["error: invalid token id", "length"]
    assert all(0 <= t < 500 for o in outs for t in o["output_ids"])
    assert eng.scheduler.stats["invalid_token_ids"] == 1
