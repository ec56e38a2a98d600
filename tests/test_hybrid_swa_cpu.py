"""Hybrid sliding-window KV pool: GPT-OSS's sliding layers keep K/V in a window pool that holds only the
pages inside the window; greedy tokens equal the single-pool run, pages are released as requests move past
them, and the pool sizing bound refuses a pool that could run out."""
import pytest
import torch

from sglang_neuron_b200.configs import model_config as mc
from sglang_neuron_b200.engine import Engine
from sglang_neuron_b200.mem_cache.hybrid_swa import (SwaPageTracker, check_window_pool, window_blocks,
                                                     window_pool_pages)
from sglang_neuron_b200.mem_cache.allocator import make_page_allocator
from sglang_neuron_b200.parallel.state import destroy_parallel
from sglang_neuron_b200.server_args import ServerArgs

TINY = dict(num_hidden_layers=2, vocab_size=1000, hidden_size=256, intermediate_size=128, num_local_experts=8,
            num_attention_heads=4, num_key_value_heads=2, head_dim=64, sliding_window=8)


def _run(hybrid: bool, chunk: int = 16):
    destroy_parallel()
    mc.PRESETS["gpt-oss-swa-tiny"] = dict(mc.PRESETS["gpt-oss-120b"], **TINY)
    args = ServerArgs(model="gpt-oss-swa-tiny", device="cpu", dtype="float32", page_size=4, context_length=256,
                      max_running_requests=4, chunked_prefill_size=chunk, disable_cuda_graph=True,
                      random_weight_std=0.05, enable_hybrid_swa=hybrid)
    eng = Engine(args)
    g = torch.Generator().manual_seed(3)
    prompts = [torch.randint(0, 1000, (n,), generator=g).tolist() for n in (45, 11, 30)]
    outs = eng.generate(prompts, {"max_new_tokens": 24})
    return eng, [o["output_ids"] for o in outs]


def test_hybrid_swa_tokens_equal_single_pool():
    _, ref = _run(False)
    eng, got = _run(True)
    assert got == ref
    sched = eng.scheduler
    assert sched.swa is not None and sched.radix is None
    # every window page came back after the requests finished
    sched.drain()
    assert sched.swa.available() == eng.runner.swa_num_pages - 1
    pool = eng.runner.kv_pool
    sliding = [l for l in pool.layer_ids if eng.cfg.layer_window(l) > 0]
    assert sliding and all(pool.kv(l)[0].shape[0] == eng.runner.swa_num_pages for l in sliding)
    assert all(pool.kv(l)[0].shape[0] == eng.runner.num_pages for l in pool.layer_ids if l not in sliding)


def test_tracker_releases_pages_behind_the_window():
    class R:
        swa_pages, swa_freed, last_step = [], 0, 0
    alloc = make_page_allocator(64, 4, reserved=1, native=False)
    tr = SwaPageTracker(alloc, window=8, page_size=4)
    r = R()
    r.swa_pages = []
    upd = []
    pages = tr.alloc_for(10)
    tr.bind(r, list(range(100, 110)), pages, upd)
    assert upd[:3] == [-1, 100, pages[0]] and len(upd) == 30
    tr.trim(r, 20)  # queries at >= 20 read keys >= 13 (page 3 on); page 2 is kept as slack
    assert r.swa_freed == 2 and r.swa_pages[:2] == [0, 0] and r.swa_pages[2] != 0
    tr.trim(r, 40)
    assert r.swa_freed == 7 and all(p == 0 for p in r.swa_pages[:7])
    before = alloc.available()
    tr.retire(0)
    assert alloc.available() == before + 7
    tr.release(r)
    tr.retire(0)
    assert alloc.available() == 63


def test_window_pool_bound():
    assert window_blocks(128, 16) == 10
    need = window_pool_pages(64, 128, 16, 8192)
    assert need == 64 * 10 + 2 * (512 + 64) + 1
    check_window_pool(need, 64, 128, 16, 8192)
    with pytest.raises(ValueError):
        check_window_pool(need - 1, 64, 128, 16, 8192)


def test_hybrid_swa_refuses_prefix_reuse_features():
    from sglang_neuron_b200 import platform
    from sglang_neuron_b200.models.catalog import model_spec
    args = ServerArgs(model="gpt-oss-120b", enable_hybrid_swa=True, enable_hierarchical_cache=True)
    with pytest.raises(ValueError):
        platform.refuse_unserved(args, model_spec("GptOssForCausalLM"))


def test_kv_layout_declaration():
    """The stage's KV layout is declared before pools: sliding layers go to the window pool only with the
    hybrid layout, latent layers are one 576-wide row, and the digest tells layouts apart."""
    from sglang_neuron_b200.mem_cache.kv_spec import declare, phase

    class A:
        def __init__(self, i, w):
            self.layer_id, self.window, self.num_kv_heads = i, w, 2

    cfg = mc.resolve_model_config("gpt-oss-120b")
    attn = [A(0, 128), A(1, 0)]
    plain = declare(cfg, attn, 16, torch.float8_e4m3fn, hybrid_swa=False)
    hyb = declare(cfg, attn, 16, torch.float8_e4m3fn, hybrid_swa=True)
    assert plain.pool_layers("window") == [] and hyb.pool_layers("window") == [0] and hyb.max_window == 128
    assert [l.kind for l in hyb.layers] == ["sliding", "full"]
    assert plain.digest() != hyb.digest()
    ds = declare(mc.resolve_model_config("deepseek-v2-lite"), [A(0, 0)], 16, torch.bfloat16, False, dcp_size=2)
    assert ds.is_latent and ds.layers[0].head_dim == 576 and ds.dcp_size == 2
    assert phase("aggregated") == "all" and phase("decode") == "decode"
