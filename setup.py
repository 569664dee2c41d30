"""Build script for swarmllm_b200.

Two in-tree extensions are built (``python setup.py build_ext --inplace``):

* ``swarmllm_b200._C``      CUDA kernels for sm_100a (B200) and their PyTorch bindings.
* ``swarmllm_b200._native`` C++ runtime: paged-KV block manager, continuous-batching
                            scheduler, GGUF mmap reader, layer-range planner, draft-tree
                            planner.  Pure C++17 + pybind11; no torch dependency.

Only sm_100a machine code is generated (``-gencode arch=compute_100a,code=sm_100a``);
the ``-gencode`` flag in ``extra_compile_args`` stops torch from adding its own arch list.
"""
import glob
import os

from setuptools import setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension
import pybind11

ROOT = os.path.dirname(os.path.abspath(__file__))

# Use the system toolchain (dynamic libstdc++ shared with torch).  A compiler
# that links libstdc++ statically gives the extension private iostream/locale
# state, and formatting a number into a torch error message then crashes.
if not os.environ.get("SWARMLLM_KEEP_CXX"):
    for _var, _exe in (("CC", "/usr/bin/gcc"), ("CXX", "/usr/bin/g++")):
        if os.path.exists(_exe):
            os.environ[_var] = _exe
    if os.path.exists("/usr/bin/g++"):
        os.environ["LDSHARED"] = "/usr/bin/g++ -shared"
CSRC = os.path.join("swarmllm_b200", "csrc")

NVCC_FLAGS = [
    "-O3",
    "-std=c++17",
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo",
    "--expt-relaxed-constexpr",
    "-Xptxas", "-warn-spills",
    "-DNDEBUG",
]
if os.environ.get("SWARMLLM_PTXAS_VERBOSE"):
    NVCC_FLAGS += ["-Xptxas", "-v"]
if os.environ.get("SWARMLLM_KERNEL_TRACE"):
    # Per-unit %globaltimer timelines of the GEMM / attention kernels (profiling only).
    NVCC_FLAGS += ["-DSWARMLLM_KERNEL_TRACE=1"]
if os.environ.get("SWARMLLM_NVCC_DEFINES"):
    # Extra -D flags selecting kernel variants (A/B experiments, e.g.
    # -DSWARMLLM_QGEMM_HALVES=2).
    NVCC_FLAGS += os.environ["SWARMLLM_NVCC_DEFINES"].split()
if os.environ.get("SWARMLLM_DEVICE_CHECKS"):
    # Device-side bounds checks (record the bad index, skip the access).
    NVCC_FLAGS += ["-DSWARMLLM_DEVICE_CHECKS=1"]

CXX_FLAGS = ["-O3", "-std=c++17"]

kernel_sources = sorted(glob.glob(os.path.join(CSRC, "kernels", "*.cu")))
binding_sources = sorted(glob.glob(os.path.join(CSRC, "bindings", "*.cpp")))
native_sources = sorted(glob.glob(os.path.join(CSRC, "native", "*.cpp")))

ext_modules = [
    CUDAExtension(
        name="swarmllm_b200._C",
        sources=kernel_sources + binding_sources,
        include_dirs=[os.path.join(ROOT, CSRC, "kernels")],
        extra_compile_args={"cxx": CXX_FLAGS, "nvcc": NVCC_FLAGS},
    ),
]

from setuptools import Extension  # noqa: E402

ext_modules.append(
    Extension(
        name="swarmllm_b200._native",
        sources=native_sources,
        include_dirs=[pybind11.get_include(), os.path.join(ROOT, CSRC, "native")],
        extra_compile_args=CXX_FLAGS + ["-fvisibility=hidden", "-Wall", "-fopenmp"],
        extra_link_args=["-fopenmp"],
        language="c++",
    )
)

setup(
    name="swarmllm_b200",
    version="0.1.0",
    description="B200-native LLM inference engine (GGUF, paged KV, PP/TP/EP, tree speculation)",
    packages=["swarmllm_b200"],
    ext_modules=ext_modules,
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
