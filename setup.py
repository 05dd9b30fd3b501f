"""Builds the sm_100a extension ``pan2_b200._C`` in-tree: ``python setup.py build_ext --inplace``."""
import glob
import os

from setuptools import setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

ROOT = os.path.dirname(os.path.abspath(__file__))
os.environ.setdefault("TORCH_CUDA_ARCH_LIST", "10.0a")

NVCC_FLAGS = [
    "-O3", "-std=c++17", "-lineinfo", "--expt-relaxed-constexpr",
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-Xptxas", "-v",
]

if os.environ.get("PAN_DEBUG_BOUNDS", "0") == "1":
    # bounds-checked debug build: data-driven indices are checked and recorded in error_flag()
    NVCC_FLAGS.append("-DPAN_DEBUG_BOUNDS")

sources = ["csrc/bindings.cpp"] + sorted(glob.glob("csrc/*.cu"))

setup(
    name="pan2_b200",
    version="0.1.0",
    packages=["pan2_b200"],
    ext_modules=[
        CUDAExtension(
            name="pan2_b200._C",
            sources=sources,
            include_dirs=[os.path.join(ROOT, "csrc")],
            extra_compile_args={"cxx": ["-O3", "-std=c++17"], "nvcc": NVCC_FLAGS},
        )
    ],
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
