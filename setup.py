"""Build of the everserve_b200 native code.

`python setup.py build_ext --inplace` compiles the sm_100a kernels into `everserve_b200/_C*.so`
inside the source tree (the extension travels with the checkout). The C++ control-plane binaries
are built separately by `make -C cpp`.
"""

import glob
import os

from setuptools import setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join("everserve_b200", "csrc")

NVCC_FLAGS = [
    "-gencode",
    "arch=compute_100a,code=sm_100a",
    "-lineinfo",
    "-O3",
    "-std=c++17",
    "--expt-relaxed-constexpr",
    "-Xptxas=-v" if os.environ.get("ES_PTXAS_VERBOSE") else "-Xptxas=-O3",
]

sources = sorted(glob.glob(os.path.join(CSRC, "*.cu"))) + sorted(glob.glob(os.path.join(CSRC, "*.cpp")))

setup(
    name="everserve_b200",
    version="0.1.0",
    packages=[],
    ext_modules=[
        CUDAExtension(
            name="everserve_b200._C",
            sources=sources,
            include_dirs=[os.path.join(HERE, CSRC)],
            extra_compile_args={"cxx": ["-O3", "-std=c++17"], "nvcc": NVCC_FLAGS},
        )
    ],
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
