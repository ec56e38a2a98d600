"""Plugin surface on the CPU tier: SGLang entry points, runtime hooks installed from the exported serving
policy (host sampler, serve profile window) with md5-pinned targets, the policy's overlap depth, the topology
reader, the host trace, and the rule that every registered SGLANG_B200_* name has a reader."""
import ast
import importlib
import os
import re

import pytest
import torch

from sglang_neuron_b200.configs import model_config as mc
from sglang_neuron_b200.parallel.state import destroy_parallel
from sglang_neuron_b200.server_args import ServerArgs

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
TINY = dict(num_hidden_layers=2, vocab_size=1000, hidden_size=128, intermediate_size=256,
            num_attention_heads=4, num_key_value_heads=2, head_dim=32)


def _engine(**kw):
    from sglang_neuron_b200.engine import Engine
    destroy_parallel()
    mc.PRESETS["plug-tiny"] = dict(mc.PRESETS["qwen3-0.6b"], **TINY)
    base = dict(model="plug-tiny", device="cpu", dtype="float32", context_length=256, max_running_requests=4,
                chunked_prefill_size=64, page_size=16, random_weight_std=0.05)
    base.update(kw)
    return Engine(ServerArgs(**base))


def test_entry_points_resolve():
    tree = ast.parse(open(os.path.join(ROOT, "setup.py")).read())
    eps = None
    for node in tree.body:
        if isinstance(node, ast.Assign) and getattr(node.targets[0], "id", "") == "ENTRY_POINTS":
            eps = ast.literal_eval(node.value)
    assert eps is not None and set(eps) == {"sglang.srt.platforms", "sglang.srt.plugins"}
    for group, items in eps.items():
        for item in items:
            name, target = [x.strip() for x in item.split("=")]
            mod, fn = target.split(":")
            assert callable(getattr(importlib.import_module(mod), fn)), (group, name)
    from sglang_neuron_b200 import activate
    assert activate() is None  # no sm_100 GPU here: another platform may claim the process


def test_hook_pins_are_current():
    from sglang_neuron_b200 import general_plugin as gp
    pins = gp.load_pins()
    assert set(pins) == set(gp.TARGETS.values())
    for target, md5 in pins.items():
        assert gp.source_md5(gp.resolve_target(target)[2]) == md5, f"{target} changed: re-pin its hook"


def test_every_registered_env_name_has_a_reader():
    from sglang_neuron_b200 import env_registry
    srcs = []
    for base, _, files in os.walk(os.path.join(ROOT, "sglang_neuron_b200")):
        for f in files:
            if f.endswith(".py") and f != "env_registry.py":
                srcs.append(open(os.path.join(base, f)).read())
    for base, _, files in os.walk(os.path.join(ROOT, "csrc")):
        for f in files:
            srcs.append(open(os.path.join(base, f)).read())
    blob = "\n".join(srcs)
    missing = [n for n in env_registry.REGISTRY if not re.search(re.escape(n) + r"\b", blob)]
    assert not missing, f"registered but never read: {missing}"


def test_policy_overlap_depth_and_host_sampler_resolution():
    from sglang_neuron_b200 import serving_policy
    pol = serving_policy.resolve(ServerArgs(), {"SGLANG_B200_MAX_INFLIGHT_LAUNCHES": "1"})
    assert not pol.async_execution and pol.max_inflight_launches == 1
    pol = serving_policy.resolve(ServerArgs(), {"SGLANG_B200_SAMPLER": "host"})
    assert pol.sampler == "host" and not pol.cuda_graph and "cuda_graph" in pol.launch_settings
    with pytest.raises(ValueError):
        serving_policy.resolve(ServerArgs(), {"SGLANG_B200_SAMPLER": "gpu"})


def test_host_sampler_hook_matches_device_rule(monkeypatch):
    from sglang_neuron_b200 import general_plugin as gp
    from sglang_neuron_b200.model_executor.model_runner import ModelRunner
    eng = _engine()
    ref = [list(o) for o in _run(eng, 0.7)]
    eng.shutdown()
    assert not gp.registry().applied
    monkeypatch.setenv("SGLANG_B200_SAMPLER", "host")
    calls = []
    orig = gp.host_sample

    def spy(*a, **k):
        calls.append(1)
        return orig(*a, **k)

    monkeypatch.setattr(gp, "host_sample", spy)
    eng = _engine()
    try:
        assert gp.TARGETS["sample"] in gp.registry().applied
        assert getattr(ModelRunner.sample, "__wrapped__", None) is not None
        got = [list(o) for o in _run(eng, 0.7)]
    finally:
        eng.shutdown()
        monkeypatch.delenv("SGLANG_B200_SAMPLER")
    assert calls and got == ref
    eng = _engine()  # the next launch without the switch undoes the hook
    eng.shutdown()
    assert getattr(ModelRunner.sample, "__wrapped__", None) is None


def test_serve_profile_window_hook_writes_a_trace(tmp_path, monkeypatch):
    from sglang_neuron_b200 import general_plugin as gp
    monkeypatch.setenv("SGLANG_B200_PROFILE_SERVE_START", "1")
    monkeypatch.setenv("SGLANG_B200_PROFILE_SERVE_STEPS", "2")
    monkeypatch.setenv("SGLANG_B200_PROFILE_DIR", str(tmp_path))
    eng = _engine()
    try:
        assert gp.TARGETS["step"] in gp.registry().applied
        _run(eng, 0.0)
    finally:
        eng.shutdown()
        for k in ("SGLANG_B200_PROFILE_SERVE_START", "SGLANG_B200_PROFILE_SERVE_STEPS", "SGLANG_B200_PROFILE_DIR"):
            monkeypatch.delenv(k)
    assert any(p.name.startswith("trace-") for p in tmp_path.iterdir())
    _engine().shutdown()
    assert not gp.registry().applied


def test_inflight_depth_one_matches_overlapped(monkeypatch):
    eng = _engine()
    ref = [list(o) for o in _run(eng, 0.0)]
    assert eng.scheduler.overlap and eng.scheduler.inflight_depth == 2
    eng.shutdown()
    monkeypatch.setenv("SGLANG_B200_MAX_INFLIGHT_LAUNCHES", "1")
    eng = _engine()
    try:
        assert not eng.scheduler.overlap
        got = [list(o) for o in _run(eng, 0.0)]
    finally:
        eng.shutdown()
    assert got == ref


def test_topology_reader_and_host_trace(tmp_path):
    from sglang_neuron_b200 import sglang_tree
    eng = _engine(host_trace_dir=str(tmp_path))
    try:
        par = sglang_tree.parallel_of()
        assert par["pp"] == 1 and par["tp"] == 1 and par["world"] == 1
        assert sglang_tree.rank_label() == "dp0-tp0"
        _run(eng, 0.0)
        eng.scheduler.trace.close()
    finally:
        eng.shutdown()
    rows = open(tmp_path / "host_trace_rankdp0-tp0.tsv").read().splitlines()
    phases = {r.split("\t")[0] for r in rows[1:]}
    assert {"select", "launch", "result"} <= phases


def test_dcp_with_host_tier_is_refused():
    from sglang_neuron_b200.platform import check_hybrid_swa
    with pytest.raises(ValueError):
        check_hybrid_swa(ServerArgs(tp_size=2, dcp_size=2, enable_hierarchical_cache=True))


def _run(eng, temperature):
    from sglang_neuron_b200.managers.schedule_batch import SamplingParams
    g = torch.Generator().manual_seed(3)
    prompts = [torch.randint(1, 1000, (n,), generator=g).tolist() for n in (9, 23)]
    reqs = [eng.submit(p, SamplingParams(max_new_tokens=6, temperature=temperature, ignore_eos=True, seed=11 + i))
            for i, p in enumerate(prompts)]
    for _ in range(200):
        if all(r.finished for r in reqs):
            break
        eng.scheduler.step()
    eng.scheduler.drain()
    assert all(r.finished for r in reqs)
    return [r.output_ids for r in reqs]
