"""Builds the in-tree extensions of quail_b200.

    python setup.py build_ext --inplace

- quail_b200/_C: the sm_100a CUDA kernels (tcgen05 GEMMs, attention, fused
  layer kernels), compiled only for `-gencode arch=compute_100a,code=sm_100a`.
- quail_b200/_native: the C++ host runtime (SQL front end, planner cost
  model, tokenizer, worker IPC frames, shared tables), no CUDA.
"""

import os

from setuptools import setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join("quail_b200", "csrc")
NATIVE = os.path.join("quail_b200", "native")

cuda_sources = [os.path.join(CSRC, f) for f in sorted(os.listdir(os.path.join(HERE, CSRC)))
                if f.endswith((".cu", ".cpp"))]
native_sources = [os.path.join(NATIVE, f) for f in sorted(os.listdir(os.path.join(HERE, NATIVE)))
                  if f.endswith(".cpp")] if os.path.isdir(os.path.join(HERE, NATIVE)) else []

nvcc_flags = [
    "-O3",
    "-std=c++17",
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo",
    "--expt-relaxed-constexpr",
    "-U__CUDA_NO_HALF_OPERATORS__",
    "-U__CUDA_NO_HALF_CONVERSIONS__",
    "-U__CUDA_NO_BFLOAT16_CONVERSIONS__",
    "-U__CUDA_NO_HALF2_OPERATORS__",
]
if os.environ.get("QB_PTXAS_VERBOSE"):
    nvcc_flags.append("-Xptxas=-v")

ext_modules = [
    CUDAExtension(
        name="quail_b200._C",
        sources=cuda_sources,
        extra_compile_args={"cxx": ["-O3", "-std=c++17"], "nvcc": nvcc_flags},
    ),
]
if native_sources:
    from pybind11.setup_helpers import Pybind11Extension
    ext_modules.append(Pybind11Extension(
        "quail_b200._native",
        sources=native_sources,
        cxx_std=20,
        extra_compile_args=["-O3", "-fvisibility=hidden"],
        extra_link_args=["-lpthread"],
    ))

# torch's own arch list must not add targets: the -gencode above is the only one
os.environ.setdefault("TORCH_CUDA_ARCH_LIST", "10.0a")

setup(
    name="quail_b200",
    version="0.1.0",
    packages=["quail_b200"],
    ext_modules=ext_modules,
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
