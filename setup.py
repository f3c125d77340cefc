"""Build the sm_100a extension in-tree:  python setup.py build_ext --inplace

Produces ``rl_project_b200/_C*.so``.  Kernels are compiled only for sm_100a
(B200): ``-gencode arch=compute_100a,code=sm_100a``.
"""

import glob
import os

from setuptools import find_packages, setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

HERE = os.path.dirname(os.path.abspath(__file__))
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]

sources = sorted(glob.glob(os.path.join("csrc", "*.cu"))) + ["csrc/bindings.cpp"]
nvcc_flags = ARCH + ["-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr", "-Xptxas=-v" if os.environ.get("RLB_PTXAS_V") else "-DRLB_QUIET"]
if os.environ.get("RLB_DEBUG_BOUNDS"):
    nvcc_flags.append("-DRLB_DEBUG_BOUNDS=1")

setup(
    name="rl_project_b200",
    version="0.1.0",
    packages=find_packages(include=["rl_project_b200", "rl_project_b200.*"]),
    package_data={"rl_project_b200": ["dashboard/static/*"]},
    ext_modules=[
        CUDAExtension(
            name="rl_project_b200._C",
            sources=sources,
            include_dirs=[os.path.join(HERE, "csrc")],
            extra_compile_args={"cxx": ["-O3", "-std=c++17"], "nvcc": nvcc_flags},
            # no libcuda link: driver entry points are resolved at run time (cudaGetDriverEntryPoint), so
            # the extension imports on a build machine without a GPU driver
        )
    ],
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
    entry_points={"console_scripts": ["forgeline-b200=rl_project_b200.cli.main:main"]},
)
