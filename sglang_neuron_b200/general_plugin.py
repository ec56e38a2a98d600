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


def register() -> Optional[str]:
    """Plugin entry point: selects this platform when SGLANG_PLATFORM names it and installs the hooks.
    Returns the platform class path (or None when another platform was requested)."""
    want = os.environ.get("SGLANG_PLATFORM", "")
    if want and want not in ("b200", "sglang_neuron_b200"):
        return None
    if not _REGISTERED[0]:
        from . import env_registry
        env_registry.refuse_unknown()
        _REGISTERED[0] = True
    return "sglang_neuron_b200.platform.B200SRTPlatform"


def registry() -> ResolvingHookRegistry:
    return _REGISTRY
