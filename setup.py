"""Build the sm_100a extension in-tree: ``python setup.py build_ext --inplace``.

Kernels are compiled only for ``sm_100a`` (B200); passing ``-gencode`` explicitly keeps torch from
adding its own architecture list.
"""

import glob
import os

from setuptools import setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

ROOT = os.path.dirname(os.path.abspath(__file__))
SOURCES = sorted(glob.glob(os.path.join("csrc", "*.cu"))) + [os.path.join("csrc", "bindings.cpp")]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "--expt-relaxed-constexpr",
    "-Xptxas=-warn-spills",
    "-U__CUDA_NO_HALF_OPERATORS__", "-U__CUDA_NO_HALF_CONVERSIONS__",
    "-U__CUDA_NO_BFLOAT16_OPERATORS__", "-U__CUDA_NO_BFLOAT16_CONVERSIONS__",
]
if os.environ.get("ACCERL_DEBUG_CHECKS", "0") not in ("", "0"):
    # range checks on data-dependent indices; failures are recorded and read with ops.debug_status()
    NVCC_FLAGS.append("-DACCERL_DEBUG_CHECKS")

setup(
    name="accerl_agent_b200",
    version="0.1.0",
    packages=["accerl_agent_b200"],
    ext_modules=[
        CUDAExtension(
            name="accerl_agent_b200._C",
            sources=SOURCES,
            extra_compile_args={"cxx": ["-O3", "-std=c++17"], "nvcc": NVCC_FLAGS},
            libraries=["cuda"],
            library_dirs=["/usr/local/cuda/lib64/stubs"],
        )
    ],
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
