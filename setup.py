"""Build the sm_100a CUDA extension in-tree: ``python setup.py build_ext --inplace``.

Produces ``sigma0_b200/_C*.so`` next to the package sources so it travels with
the repository snapshot.  Every CUDA source is compiled for sm_100a only.
"""
import glob
import os

from setuptools import setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join("sigma0_b200", "csrc")
# attention_tc.cu (a tcgen05 flash-attention forward) is left out of the build: it failed
# with an unspecified launch failure on multi-wave grids and its cause is not found
PARKED = {"attention_tc.cu"}
sources = [s for s in sorted(glob.glob(os.path.join(CSRC, "*.cu"))) if os.path.basename(s) not in PARKED]
sources += sorted(glob.glob(os.path.join(CSRC, "*.cpp")))

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
nvcc_flags = ARCH + ["-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr",
                     "-Xptxas=-v" if os.environ.get("S0_PTXAS_VERBOSE") else "-Xptxas=-O3"]

setup(
    name="sigma0_b200",
    version="0.1.0",
    packages=["sigma0_b200"],
    ext_modules=[CUDAExtension(
        name="sigma0_b200._C",
        sources=sources,
        include_dirs=[os.path.join(HERE, CSRC)],
        extra_compile_args={"cxx": ["-O3", "-std=c++17"], "nvcc": nvcc_flags},
    )],
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
