"""In-tree build of the bloom_b200 native extensions.

    python setup.py build_ext --inplace

Builds
  bloom_b200/_C        CUDA kernels, compiled for sm_100a only
  bloom_b200/_runtime  C++ host runtime (scheduler, KV block manager, GGUF,
                       CPU kernels); no CUDA dependency so it imports anywhere
  bloom_b200/_C_checked  (BLOOM_BUILD=checked, in its own build folder:
                       `--build-temp build/temp_checked`) the CUDA kernels with
                       -DBLOOM_KERNEL_CHECKS: table indices (KV block ids, cache
                       slots, token ids, expert rows) are checked, a bad one sets
                       a status bit and its access is skipped.  Loaded instead of
                       _C when BLOOM_KERNEL_CHECKS=1.
"""
import glob
import os

from setuptools import setup
from torch.utils.cpp_extension import BuildExtension, CppExtension, CUDAExtension

ROOT = os.path.dirname(os.path.abspath(__file__))
INC = [os.path.join(ROOT, "csrc", "include")]

SM100A = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = SM100A + [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "--use_fast_math",
    "--expt-relaxed-constexpr",
    "-U__CUDA_NO_HALF_OPERATORS__",
    "-U__CUDA_NO_HALF_CONVERSIONS__",
    "-U__CUDA_NO_BFLOAT16_OPERATORS__",
    "-U__CUDA_NO_BFLOAT16_CONVERSIONS__",
]
CXX_FLAGS = ["-O3", "-std=c++17"]


def cuda_sources():
    return sorted(glob.glob(os.path.join("csrc", "kernels", "*.cu"))) + [
        os.path.join("csrc", "bindings", "ops_bindings.cpp")
    ]


def runtime_sources():
    return sorted(glob.glob(os.path.join("csrc", "runtime", "*.cpp"))) + [
        os.path.join("csrc", "bindings", "runtime_bindings.cpp")
    ]


def extensions(which=("cuda", "runtime")):
    exts = []
    if "cuda" in which:
        exts.append(
            CUDAExtension(
                "bloom_b200._C",
                cuda_sources(),
                include_dirs=INC,
                extra_compile_args={"cxx": CXX_FLAGS, "nvcc": NVCC_FLAGS},
            )
        )
    if "checked" in which:
        exts.append(
            CUDAExtension(
                "bloom_b200._C_checked",
                cuda_sources(),
                include_dirs=INC,
                extra_compile_args={"cxx": CXX_FLAGS + ["-DBLOOM_KERNEL_CHECKS"],
                                    "nvcc": NVCC_FLAGS + ["-DBLOOM_KERNEL_CHECKS"]},
            )
        )
    if "runtime" in which:
        exts.append(
            CppExtension(
                "bloom_b200._runtime",
                runtime_sources(),
                include_dirs=INC,
                extra_compile_args={"cxx": CXX_FLAGS + ["-march=x86-64-v3"]},
            )
        )
    return exts


if __name__ == "__main__":
    which = os.environ.get("BLOOM_BUILD", "cuda,runtime").split(",")
    setup(
        name="bloom_b200",
        version="0.1.0",
        packages=["bloom_b200"],
        ext_modules=extensions(which),
        cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
    )
