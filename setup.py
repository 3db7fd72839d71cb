"""Build the sm_100a extension in-tree: ``python setup.py build_ext --inplace``.

Every CUDA source is compiled for ``sm_100a`` only (``-gencode arch=compute_100a,
code=sm_100a``), bypassing torch's own architecture list.
"""

import os

from setuptools import setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join("neural_scaling_weather_b200", "ops", "csrc")

SOURCES = [
    os.path.join(CSRC, "bindings.cpp"),
    os.path.join(CSRC, "elementwise.cu"),
    os.path.join(CSRC, "attention.cu"),
    os.path.join(CSRC, "attention_tc.cu"),
    os.path.join(CSRC, "gemm_tcgen05.cu"),
    os.path.join(CSRC, "noalloc_rmsnorm.cu"),
    os.path.join(CSRC, "rmsnorm_tma.cu"),
    os.path.join(CSRC, "sht.cu"),
    os.path.join(CSRC, "dp_fused.cu"),
    os.path.join(CSRC, "halo_roll.cu"),
]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "--expt-relaxed-constexpr",
    "-U__CUDA_NO_HALF_OPERATORS__", "-U__CUDA_NO_HALF_CONVERSIONS__",
    "-U__CUDA_NO_BFLOAT16_CONVERSIONS__", "-U__CUDA_NO_HALF2_OPERATORS__",
]

os.environ.setdefault("TORCH_CUDA_ARCH_LIST", "10.0a")
os.environ.setdefault("MAX_JOBS", str(max(1, (os.cpu_count() or 2))))

setup(
    name="neural_scaling_weather_b200",
    version="0.1.0",
    packages=["neural_scaling_weather_b200"],
    ext_modules=[
        CUDAExtension(
            name="neural_scaling_weather_b200._C",
            sources=SOURCES,
            include_dirs=[os.path.join(HERE, CSRC)],
            extra_compile_args={"cxx": ["-O3", "-std=c++17"], "nvcc": NVCC_FLAGS},
        )
    ],
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
