"""Builds the sm_100a CUDA extension in place: ``python setup.py build_ext --inplace``.

Every kernel is hand-written and compiled for ``-gencode arch=compute_100a,code=sm_100a`` only
(B200); no third-party kernel library is compiled in.
"""
import glob
import os

from setuptools import setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

ROOT = os.path.dirname(os.path.abspath(__file__))


NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-std=c++17", "-lineinfo", "--expt-relaxed-constexpr", "--expt-extended-lambda",
    "-DNDEBUG", "-U__CUDA_NO_HALF_OPERATORS__", "-U__CUDA_NO_HALF_CONVERSIONS__",
    "-U__CUDA_NO_BFLOAT16_OPERATORS__", "-U__CUDA_NO_BFLOAT16_CONVERSIONS__",
    "-U__CUDA_NO_BFLOAT162_OPERATORS__", "-U__CUDA_NO_BFLOAT162_CONVERSIONS__",
]


def extensions():
    inc = [os.path.join(ROOT, "csrc")]
    srcs = sorted(glob.glob(os.path.join(ROOT, "csrc", "*.cu"))) + [os.path.join(ROOT, "csrc", "bindings.cpp")]
    return [CUDAExtension(
        name="trida_stack_b200._C",
        sources=[os.path.relpath(s, ROOT) for s in srcs],
        include_dirs=inc,
        extra_compile_args={"cxx": ["-O3", "-std=c++17"], "nvcc": NVCC_FLAGS},
    )]


if __name__ == "__main__":
    os.environ.setdefault("MAX_JOBS", str(max(1, os.cpu_count() or 1)))
    setup(name="trida_stack_b200_ext", ext_modules=extensions(),
          cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)})
