"""Plugin entry and hook registry.

Parity: sglang_neuron/general_plugin.py — `register()` (:318) installs launch hooks in every process and
runtime hooks in spawned processes through `ResolvingHookRegistry` (:20), which resolves every hook target
eagerly and refuses a second REPLACE of the same target; each target's source is pinned by md5 against the
SGLang revision the plugin was written for (sglang_patches/source_guard.py). This build is a standalone
engine, so its hooks attach to its own seams (or to SGLang when it is installed), with the same rules.
"""
from __future__ import annotations

import hashlib
import importlib
import inspect
import json
import logging
import os
from typing import Callable, Dict, List, Optional, Tuple

logger = logging.getLogger(__name__)


class HookError(RuntimeError):
    pass


def source_md5(obj) -> str:
    return hashlib.md5(inspect.getsource(obj).encode()).hexdigest()


def resolve_target(path: str):
    """'pkg.module:Class.attr' -> (owner object, attribute name, current value)."""
    mod_name, _, attr_path = path.partition(":")
    owner = importlib.import_module(mod_name)
    parts = attr_path.split(".")
    for p in parts[:-1]:
        owner = getattr(owner, p)
    return owner, parts[-1], getattr(owner, parts[-1])


class ResolvingHookRegistry:
    """Hooks are (target, kind, fn). Kinds: REPLACE (swap the callable), AROUND (wrap it, receives the
    original as first argument). Targets are resolved when registered; a pinned md5 mismatch refuses the
    hook instead of patching code it was not written for."""

    def __init__(self):
        self.applied: Dict[str, Tuple[str, Callable, Callable]] = {}

    def register(self, target: str, kind: str, fn: Callable, pin_md5: Optional[str] = None) -> None:
        owner, attr, cur = resolve_target(target)
        if pin_md5 is not None:
            got = source_md5(cur)
            if got != pin_md5:
                raise HookError(f"{target}: source md5 {got} != pinned {pin_md5}; refusing to hook")
        if kind == "REPLACE":
            if target in self.applied and self.applied[target][0] == "REPLACE":
                raise HookError(f"{target} already replaced")
            setattr(owner, attr, fn)
        elif kind == "AROUND":
            orig = cur

            def wrapped(*a, __orig=orig, **k):
                return fn(__orig, *a, **k)

            wrapped.__wrapped__ = orig
            setattr(owner, attr, wrapped)
        else:
            raise HookError(f"unknown hook kind {kind!r}")
        self.applied[target] = (kind, fn, cur)

    def undo_all(self) -> None:
        for target, (_kind, _fn, orig) in reversed(list(self.applied.items())):
            owner, attr, _ = resolve_target(target)
            setattr(owner, attr, orig)
        self.applied.clear()


_REGISTRY = ResolvingHookRegistry()
_REGISTERED = [False]

# Runtime hook targets: this engine's own seams (SGLang is not a dependency). Each target's source is pinned
# by md5 in hook_pins.json; a target whose source changed refuses its hook until it is re-pinned with
# `python -m sglang_neuron_b200.general_plugin --pin` (the hook was written against the pinned source).
TARGETS = {
    "sample": "sglang_neuron_b200.model_executor.model_runner:ModelRunner.sample",
    "step": "sglang_neuron_b200.managers.scheduler:Scheduler.step",
}
PINS_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "hook_pins.json")


def load_pins() -> Dict[str, str]:
    with open(PINS_PATH) as f:
        return json.load(f)


def write_pins() -> Dict[str, str]:
    pins = {t: source_md5(resolve_target(t)[2]) for t in TARGETS.values()}
    with open(PINS_PATH, "w") as f:
        json.dump(pins, f, indent=1, sort_keys=True)
        f.write("\n")
    return pins


def host_sample(orig, runner, h_last, fb, req_idx, out=None):
    """SGLANG_B200_SAMPLER=host: the step's logits come back to the host and are sampled there with the
    device sampler's rule (greedy ties to the smallest id, Gumbel-max with the same hashed noise), so the
    host path is a token-for-token check of the device sampler. Vocabulary shards are merged like the device
    path (one all-gather of per-shard winners). Filtered (top-k/top-p) and logprob steps keep the device
    path. Parity: the reference's host sampling mode (SGLANG_NEURON_SAMPLER=host, sglang_neuron/sampling.py)."""
    import torch

    from .ops.sampling import sample_ref
    from .parallel.state import get_state
    if fb.needs_topk_topp or (fb.extra and fb.extra.get("logprob_k", -1) >= 0):
        return orig(runner, h_last, fb, req_idx, out)
    st = get_state()
    logits = runner.model.compute_logits(h_last)
    positions = fb.positions.index_select(0, fb.logits_idx) + 1
    ids, vals = sample_ref(logits.float().cpu(), fb.temperature.cpu(), fb.seeds.cpu(), positions.cpu(),
                           runner.vocab_start, runner.vocab_valid, return_vals=True)
    ids = ids.to(runner.device)
    if st.tp_size > 1:
        from .parallel.collectives import tp_all_gather_into
        B = ids.numel()
        pair = torch.stack([vals.to(runner.device), ids.float()], dim=1).contiguous()
        g = torch.empty(st.tp_size * B, 2, dtype=torch.float32, device=runner.device)
        tp_all_gather_into(g, pair)
        g = g.view(st.tp_size, B, 2)
        best = g[:, :, 0].argmax(dim=0)
        ids = g[:, :, 1].gather(0, best[None, :])[0].long()
    if out is not None:
        out.copy_(ids)
        ids = out
    runner.relay.index_copy_(0, req_idx.view(-1), ids.view(-1))
    return ids


class ServeProfileWindow:
    """SGLANG_B200_PROFILE_SERVE_START / _STEPS / _DIR / _RANKS: a bounded device-profile window over
    scheduler steps [start, start + steps) of a serving process, on the listed ranks (default: all),
    written as a Chrome trace. Parity: the reference's serving capture window
    (sglang_neuron/model_executor/profiling.py:211 `ServingCapture`)."""

    def __init__(self, start: int, steps: int, out_dir: str, ranks: Optional[List[int]] = None):
        self.start, self.steps, self.out_dir, self.ranks = start, steps, out_dir, ranks
        self.count = 0
        self.window = None
        self.paths: List[str] = []

    def __call__(self, orig, sched, *a, **k):
        from .parallel.state import get_state
        from .utils.profiling import ProfileWindow
        if self.count == self.start and (self.ranks is None or get_state().rank in self.ranks):
            self.window = ProfileWindow(self.out_dir, self.steps)
            self.window.start()
        self.count += 1
        r = orig(sched, *a, **k)
        if self.window is not None and self.window.step():
            self.paths.extend(p for p in [self.window.last_path] if p)
            self.window = None
        return r

    @classmethod
    def from_env(cls, environ=os.environ) -> Optional["ServeProfileWindow"]:
        from . import env_registry
        steps = env_registry.get("SGLANG_B200_PROFILE_SERVE_STEPS", None, environ)
        if not steps or int(steps) <= 0:
            return None
        start = int(env_registry.get("SGLANG_B200_PROFILE_SERVE_START", "0", environ))
        out_dir = env_registry.get("SGLANG_B200_PROFILE_DIR", "profile_out", environ)
        ranks = env_registry.get("SGLANG_B200_PROFILE_RANKS", None, environ)
        rl = [int(x) for x in ranks.split(",") if x.strip()] if ranks else None
        return cls(start, int(steps), out_dir, rl)


def runtime_hook_specs(policy, environ=os.environ) -> List[Tuple[str, str, Callable]]:
    """The runtime hooks a rank with this serving policy installs: (target, kind, fn)."""
    specs = []
    if policy is not None and policy.sampler == "host":
        specs.append((TARGETS["sample"], "AROUND", host_sample))
    window = ServeProfileWindow.from_env(environ)
    if window is not None:
        specs.append((TARGETS["step"], "AROUND", window))
    return specs


def _register_runtime(policy, environ=os.environ) -> List[str]:
    """(Re)install this launch's runtime hooks: hooks of an earlier launch in the process are undone first,
    every target is checked against its pinned source, and a failure undoes the partial set and raises."""
    _REGISTRY.undo_all()
    pins = load_pins()
    try:
        for target, kind, fn in runtime_hook_specs(policy, environ):
            _REGISTRY.register(target, kind, fn, pin_md5=pins.get(target))
    except Exception:
        _REGISTRY.undo_all()
        raise
    if _REGISTRY.applied:
        logger.info("runtime hooks: %s", ", ".join(_REGISTRY.applied))
    return list(_REGISTRY.applied)


def register() -> Optional[str]:
    """Plugin entry point (`sglang.srt.plugins`): selects this platform when SGLANG_PLATFORM names it (or
    is unset), refuses unknown SGLANG_B200_* names, and in a process whose serving policy is exported installs
    the runtime hooks that policy asks for. Returns the platform class path (None for another platform).
    Parity: sglang_neuron/general_plugin.py:444 `register` (launch process first, runtime hooks once the
    policy exists)."""
    from . import serving_policy
    want = os.environ.get("SGLANG_PLATFORM", "")
    if want and want not in ("b200", "sglang_neuron_b200"):
        return None
    from . import env_registry
    env_registry.refuse_unknown()
    _REGISTERED[0] = True
    policy = serving_policy.current()
    if policy is not None:
        _register_runtime(policy)
    return "sglang_neuron_b200.platform.B200SRTPlatform"


def registry() -> ResolvingHookRegistry:
    return _REGISTRY


if __name__ == "__main__":
    import sys
    if "--pin" in sys.argv:
        print(json.dumps(write_pins(), indent=1))
