"""Build the sm_100a CUDA extension and the native runtime in-tree.

    python setup.py build_ext --inplace

produces ``sglang_neuron_b200/_C*.so`` (kernels) and ``sglang_neuron_b200/_runtime*.so`` (C++ host
runtime: paged allocator, radix tree, batch metadata). Every CUDA source is compiled for sm_100a only.
"""
import glob
import os

from pybind11.setup_helpers import Pybind11Extension
from setuptools import setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

ROOT = os.path.dirname(os.path.abspath(__file__))
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + [
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "--expt-relaxed-constexpr",
    "-DNDEBUG",
    "-U__CUDA_NO_HALF_OPERATORS__",
    "-U__CUDA_NO_HALF_CONVERSIONS__",
    "-U__CUDA_NO_BFLOAT16_OPERATORS__",
    "-U__CUDA_NO_BFLOAT16_CONVERSIONS__",
    "-U__CUDA_NO_BFLOAT162_OPERATORS__",
    "-U__CUDA_NO_BFLOAT162_CONVERSIONS__",
]
if os.environ.get("SNB_PTXAS_VERBOSE"):
    NVCC_FLAGS.append("-Xptxas=-v")

kernel_sources = sorted(glob.glob(os.path.join("csrc", "kernels", "*.cu"))) + ["csrc/bindings.cpp"]
runtime_sources = sorted(glob.glob(os.path.join("csrc", "runtime", "*.cpp")))

ext_modules = [
    CUDAExtension(
        name="sglang_neuron_b200._C",
        sources=kernel_sources,
        include_dirs=[os.path.join(ROOT, "csrc")],
        extra_compile_args={"cxx": ["-O3", "-std=c++17"], "nvcc": NVCC_FLAGS},
    ),
]
if runtime_sources:
    ext_modules.append(
        Pybind11Extension(
            "sglang_neuron_b200._runtime",
            sources=runtime_sources,
            include_dirs=[os.path.join(ROOT, "csrc")],
            extra_compile_args=["-O3", "-std=c++17"],
            libraries=["rt"],  # shm_open on older glibc
        )
    )

# SGLang selects a platform and loads plugins through these entry-point groups: `activate()` claims the process
# on an sm_100 GPU, `register()` refuses unknown SGLANG_B200_* names and installs the runtime hooks of the
# exported serving policy. Parity: the reference's pyproject.toml [project.entry-points] (same two groups).
ENTRY_POINTS = {
    "sglang.srt.platforms": ["b200 = sglang_neuron_b200:activate"],
    "sglang.srt.plugins": ["b200_hooks = sglang_neuron_b200.general_plugin:register"],
}

setup(
    name="sglang_neuron_b200",
    version="0.1.0",
    packages=["sglang_neuron_b200"] + ["sglang_neuron_b200." + p for p in (
        "attention", "benchmarks", "configs", "disaggregation", "entrypoints", "layers", "managers", "mem_cache",
        "model_executor", "models", "ops", "parallel", "speculative", "utils")],
    package_data={"sglang_neuron_b200": ["hook_pins.json"]},
    entry_points=ENTRY_POINTS,
    ext_modules=ext_modules,
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
