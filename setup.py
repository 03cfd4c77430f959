"""Build the in-tree sm_100a CUDA extension: ``python setup.py build_ext --inplace``.

The shared object lands at ``kimi_k3_b200/_C*.so``; it is not installed into
site-packages so every process imports the copy that sits next to the sources.
"""
import glob
import os

from setuptools import find_packages, setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

ROOT = os.path.dirname(os.path.abspath(__file__))
NVCC_FLAGS = [
    "-O3", "-std=c++17", "-lineinfo",
    "-gencode", "arch=compute_100a,code=sm_100a",
    "--expt-relaxed-constexpr", "-Xptxas=-warn-spills",
]


def extension():
    sources = sorted(glob.glob(os.path.join("csrc", "*.cu"))) + [os.path.join("csrc", "bindings.cpp")]
    return CUDAExtension(
        name="kimi_k3_b200._C",
        sources=sources,
        include_dirs=[os.path.join(ROOT, "csrc")],
        extra_compile_args={"cxx": ["-O3", "-std=c++17"], "nvcc": NVCC_FLAGS},
        libraries=["cuda"],
    )


setup(
    name="kimi_k3_b200",
    version="0.1.0",
    packages=find_packages(include=["kimi_k3_b200", "kimi_k3_b200.*"]),
    ext_modules=[extension()],
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
