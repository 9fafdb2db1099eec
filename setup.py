"""Build the bwn native extension in-tree for sm_100a (B200).

    python setup.py build_ext --inplace

produces ``bwn/_C*.so``.  Kernels in ``csrc/kernels`` and ``csrc/comm`` are
plain CUDA (no torch headers, so nvcc stays fast); ``csrc/ops.cpp`` binds them
to ``torch.ops.bwn.*``.  The arch list is passed explicitly, bypassing torch's
own ``TORCH_CUDA_ARCH_LIST``.
"""
import glob
import os

from setuptools import setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

ROOT = os.path.dirname(os.path.abspath(__file__))
DEBUG = os.environ.get("BWN_DEBUG", "0") == "1"

cu = sorted(glob.glob(os.path.join("csrc", "kernels", "*.cu")) + glob.glob(os.path.join("csrc", "comm", "*.cu")))
cpp = sorted(glob.glob(os.path.join("csrc", "*.cpp")) + glob.glob(os.path.join("csrc", "common", "*.cpp")) + glob.glob(os.path.join("csrc", "comm", "*.cpp")))

nvcc_flags = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "--expt-relaxed-constexpr", "-Xptxas=-warn-spills",
    "-I" + os.path.join(ROOT, "csrc"),
]
cxx_flags = ["-O3", "-std=c++17", "-I" + os.path.join(ROOT, "csrc")]
if DEBUG:
    nvcc_flags.append("-DBWN_DEBUG=1")
    cxx_flags.append("-DBWN_DEBUG=1")

setup(
    name="bwn",
    version="0.1.0",
    packages=["bwn"],
    ext_modules=[
        CUDAExtension(
            name="bwn._C",
            sources=cpp + cu,
            extra_compile_args={"cxx": cxx_flags, "nvcc": nvcc_flags},
        )
    ],
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
