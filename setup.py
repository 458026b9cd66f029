"""Build the native parts of openmini_v1_b200 in place.

    python setup.py build_ext --inplace

produces
  openmini_v1_b200/_C*.so   sm_100a CUDA kernels (tcgen05 / TMA / TMEM)
  openmini_v1_b200/_rt*.so  C++ runtime (paged-KV block manager, IPC framing,
                            GGUF index)
Only sm_100a is targeted: the arch flags below bypass torch's arch list.
"""
import glob
import os

from setuptools import setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension, CppExtension

ROOT = os.path.dirname(os.path.abspath(__file__))
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _srcs(*patterns):
    out = []
    for p in patterns:
        out += sorted(glob.glob(os.path.join(ROOT, p), recursive=True))
    return [os.path.relpath(s, ROOT) for s in out]


cuda_sources = ["csrc/bindings.cpp"] + _srcs(
    "csrc/gemm/*.cu", "csrc/norm/*.cu", "csrc/attn/*.cu", "csrc/sampler/*.cu",
    "csrc/quant/*.cu", "csrc/moe/*.cu", "csrc/dsa/*.cu", "csrc/comm/*.cu")

nvcc_flags = ARCH + [
    "-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr", "-DNDEBUG",
    "-U__CUDA_NO_HALF_OPERATORS__", "-U__CUDA_NO_HALF_CONVERSIONS__",
    "-U__CUDA_NO_BFLOAT16_CONVERSIONS__", "-U__CUDA_NO_BFLOAT162_OPERATORS__",
    "-U__CUDA_NO_HALF2_OPERATORS__", "-U__CUDA_NO_BFLOAT16_OPERATORS__",
]
if os.environ.get("OM_PTXAS_VERBOSE"):
    nvcc_flags.append("-Xptxas=-v")

ext_modules = [
    CUDAExtension(
        name="openmini_v1_b200._C",
        sources=cuda_sources,
        include_dirs=[os.path.join(ROOT, "csrc")],
        extra_compile_args={"cxx": ["-O3", "-std=c++17"], "nvcc": nvcc_flags},
    ),
    CppExtension(
        name="openmini_v1_b200._rt",
        sources=_srcs("csrc/runtime/*.cpp"),
        include_dirs=[os.path.join(ROOT, "csrc")],
        extra_compile_args={"cxx": ["-O3", "-std=c++17"]},
    ),
]

setup(
    name="openmini_v1_b200",
    version="0.1.0",
    packages=["openmini_v1_b200"],
    ext_modules=ext_modules,
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
