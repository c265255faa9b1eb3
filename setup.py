"""Build the native runtime in-tree: ``python setup.py build_ext --inplace``.

Kernels are compiled for sm_100a only (B200).  The extension links the CUDA
runtime that torch loads and resolves driver-API symbols at run time, so it
imports on machines without a GPU driver.
"""

import os

from setuptools import setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")

NVCC_FLAGS = [
    "-gencode",
    "arch=compute_100a,code=sm_100a",
    "-lineinfo",
    "-O3",
    "-std=c++17",
    "--expt-relaxed-constexpr",
    "-Xptxas=-v" if os.environ.get("ENGRAM_PTXAS_VERBOSE") == "1" else "-Xptxas=-O3",
]
CXX_FLAGS = ["-O3", "-std=c++17", "-Wno-deprecated-declarations", "-Wno-interference-size"]

sources = [os.path.join("csrc", f) for f in ("runtime.cpp", "memory.cpp", "fdpass.cpp", "owner_service.cpp", "harness.cpp", "ops.cpp")]
sources += [os.path.join("csrc", "kernels", f) for f in ("gather.cu", "exchange.cu", "dedup.cu", "noalloc.cu", "litmus.cu", "peer_probe.cu", "barrier.cu")]

setup(
    name="engram_rdma_lab_b200",
    version="0.1.0",
    packages=[
        "engram_rdma_lab_b200",
        "engram_rdma_lab_b200.models",
        "engram_rdma_lab_b200.ops",
        "engram_rdma_lab_b200.parallel",
        "engram_rdma_lab_b200.utils",
    ],
    ext_modules=[
        CUDAExtension(
            name="engram_rdma_lab_b200._C",
            sources=sources,
            include_dirs=[CSRC],
            extra_compile_args={"cxx": CXX_FLAGS, "nvcc": NVCC_FLAGS},
        )
    ],
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
