"""The in-tree sm_100a extension, when built, must import on a CPU-only host too (an unresolved symbol
would otherwise only show on the GPU box)."""
import glob
import os

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_built_extension_imports():
    if not glob.glob(os.path.join(ROOT, "sglang_neuron_b200", "_C*.so")):
        pytest.skip("extension not built")
    import torch  # noqa: F401  (loads libc10 before the extension)
    from sglang_neuron_b200 import _ext
    assert _ext.available(), f"_C failed to import: {_ext._err}"
    if glob.glob(os.path.join(ROOT, "sglang_neuron_b200", "_runtime*.so")):
        assert _ext._runtime is not None, f"_runtime failed to import: {_ext._rt_err}"


def test_extension_imports_in_a_fresh_interpreter_without_torch_first():
    """The driver's build check imports the package before anything else has loaded torch."""
    if not glob.glob(os.path.join(ROOT, "sglang_neuron_b200", "_C*.so")):
        pytest.skip("extension not built")
    import subprocess
    import sys
    code = "import sglang_neuron_b200._ext as e; assert e._C is not None, e._err; print('ok')"
    out = subprocess.run([sys.executable, "-c", code], cwd=ROOT, capture_output=True, text=True, timeout=300)
    assert out.returncode == 0 and "ok" in out.stdout, out.stderr[-2000:]
