"""Builds the sm_100a extension in-tree: `python setup.py build_ext --inplace`.

Every CUDA source under csrc/ goes into helexa_b200/_C*.so, compiled only for
sm_100a (B200); torch's own arch list is bypassed by the explicit -gencode.
"""
import glob
import os

from setuptools import setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

ROOT = os.path.dirname(os.path.abspath(__file__))
srcs = sorted(glob.glob(os.path.join("csrc", "*.cu")) + glob.glob(os.path.join("csrc", "*.cpp")))
os.environ.setdefault("MAX_JOBS", str(max(1, os.cpu_count() or 1)))
os.environ.setdefault("TORCH_CUDA_ARCH_LIST", "10.0a")

setup(
    name="helexa_b200_ext",
    ext_modules=[CUDAExtension(
        name="helexa_b200._C",
        sources=srcs,
        include_dirs=[os.path.join(ROOT, "csrc")],
        extra_compile_args={
            "cxx": ["-O3", "-std=c++17"],
            "nvcc": ["-O3", "-std=c++17", "-gencode", "arch=compute_100a,code=sm_100a", "-lineinfo",
                     "--expt-relaxed-constexpr", "-U__CUDA_NO_HALF_OPERATORS__",
                     "-U__CUDA_NO_BFLOAT16_CONVERSIONS__", "-U__CUDA_NO_HALF2_OPERATORS__"],
        },
        libraries=["cuda"],
    )],
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
