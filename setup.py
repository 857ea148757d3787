"""Build the in-tree extensions of multi_gpu_flashattention_b200.

    python setup.py build_ext --inplace

builds
  multi_gpu_flashattention_b200/_sched*.so  C++ workload model, schedulers, shard plans
  multi_gpu_flashattention_b200/_C*.so      sm_100a CUDA kernels + native ring engine
Set MGFA_BUILD=sched or MGFA_BUILD=cuda to build only one of them.
"""
import os

import pybind11
from setuptools import Extension, setup

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = "multi_gpu_flashattention_b200"
which = os.environ.get("MGFA_BUILD", "all")

SM100 = ["-gencode", "arch=compute_100a,code=sm_100a"]
CXX_FLAGS = ["-O3", "-std=c++17", "-Wall", "-Wno-unused-function"]
# MGFA_DEBUG=1: device-side bounds checks on the peer stores of the ring
# transports (a violation is reported in the status word and skipped)
DEBUG = ["-DMGFA_DEBUG"] if os.environ.get("MGFA_DEBUG", "0") == "1" else []

ext_modules = []
cmdclass = {}

if which in ("all", "sched"):
    ext_modules.append(
        Extension(
            f"{PKG}._sched",
            sources=[
                "csrc/sched/workload.cpp",
                "csrc/sched/scheduler.cpp",
                "csrc/sched/shard_plan.cpp",
                "csrc/sched/bindings.cpp",
                "csrc/host/cpu_attention.cpp",
            ],
            include_dirs=[pybind11.get_include()],
            language="c++",
            extra_compile_args=CXX_FLAGS + ["-fvisibility=hidden", "-pthread"],
            extra_link_args=["-pthread"],
        )
    )

if which in ("all", "cuda"):
    from torch.utils.cpp_extension import BuildExtension, CUDAExtension

    ext_modules.append(
        CUDAExtension(
            f"{PKG}._C",
            sources=[
                "csrc/ops/bindings.cpp",
                "csrc/ops/attn_api.cpp",
                "csrc/kernels/umma_probe.cu",
                "csrc/kernels/flash_fwd_sm100.cu",
                "csrc/kernels/attn_fwd_persistent.cu",
                "csrc/kernels/flash_bwd_sm100.cu",
                "csrc/kernels/attn_bwd_noalloc.cu",
                "csrc/kernels/legacy_fp32.cu",
                "csrc/comm/symmetric.cpp",
                "csrc/comm/ring_engine.cpp",
                "csrc/comm/ring_engine_p.cpp",
                "csrc/comm/ring_exchange.cpp",
                "csrc/comm/ring_bwd_engine.cpp",
                "csrc/kernels/ring_exchange.cu",
            ],
            include_dirs=[os.path.join(ROOT, "csrc")],
            extra_compile_args={
                "cxx": ["-O3", "-std=c++17"] + DEBUG,
                "nvcc": ["-O3", "-std=c++17", "-lineinfo", "--expt-relaxed-constexpr",
                         "-Xptxas=-v"] + SM100 + DEBUG,
            },
            libraries=["cuda"] if os.path.exists("/usr/lib/x86_64-linux-gnu/libcuda.so") else [],
        )
    )
    cmdclass["build_ext"] = BuildExtension.with_options(use_ninja=True)

setup(
    name="multi_gpu_flashattention_b200",
    version="0.1.0",
    packages=[PKG],
    ext_modules=ext_modules,
    cmdclass=cmdclass,
)
