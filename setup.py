"""Build the omnicoder sm_100a extension in place: ``python setup.py build_ext --inplace``.

Every CUDA source is compiled for sm_100a only (tcgen05 / TMEM / TMA need the
arch-specific target); the resulting ``omnicoder/_C*.so`` stays in the tree.
"""
import glob
import os

from setuptools import setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join("omnicoder", "csrc")

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "--expt-relaxed-constexpr",
    "-Xptxas", "-v" if os.environ.get("OMNI_PTXAS_VERBOSE") else "-O3",
]

sources = sorted(glob.glob(os.path.join(CSRC, "*.cpp"))) + sorted(glob.glob(os.path.join(CSRC, "*.cu")))

setup(
    name="omnicoder-b200",
    version="0.1.0",
    packages=[],
    ext_modules=[
        CUDAExtension(
            name="omnicoder._C",
            sources=sources,
            include_dirs=[os.path.join(HERE, CSRC)],
            extra_compile_args={"cxx": ["-O3", "-std=c++17"], "nvcc": NVCC_FLAGS},
        )
    ],
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
