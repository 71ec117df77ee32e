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
sources = sorted(glob.glob(os.path.join(CSRC, "*.cu"))) + sorted(glob.glob(os.path.join(CSRC, "*.cpp")))

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
nvcc_flags = ARCH + ["-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr",
                     "-Xptxas=-v" if os.environ.get("S0_PTXAS_VERBOSE") else "-Xptxas=-O3"]
if os.environ.get("S0_CHECK"):
    nvcc_flags.append("-DS0_CHECK=1")
if os.environ.get("S0_PHASE_PROBE"):      # per-phase clock counters in the chunk backward
    nvcc_flags.append("-DS0_PHASE_PROBE=1")

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
