"""Builds the aether_b200 native code in-tree.

* ``aether_b200/_C*.so``  -- torch extension with every sm_100a kernel
  (``python setup.py build_ext --inplace``).
The C-ABI runtime ``libaether_rt.so`` is built by ``aether_b200/_build.py``.
"""
import glob
import os

from setuptools import setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

ROOT = os.path.dirname(os.path.abspath(__file__))
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]

sources = sorted(glob.glob(os.path.join("csrc", "*.cu"))) + sorted(glob.glob(os.path.join("csrc", "*.cpp")))

setup(
    name="aether_b200",
    version="0.1.0",
    packages=["aether_b200"],
    ext_modules=[
        CUDAExtension(
            name="aether_b200._C",
            sources=sources,
            include_dirs=[os.path.join(ROOT, "csrc")],
            extra_compile_args={
                "cxx": ["-O3", "-std=c++17"],
                "nvcc": ARCH + ["-O3", "-std=c++17", "-lineinfo", "--expt-relaxed-constexpr", "-Xptxas=-v"],
            },
        )
    ],
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
