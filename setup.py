"""Build the native extensions of rlx_models_b200 in-tree.

    python setup.py build_ext --inplace -j 8

* ``rlx_models_b200._C``       - sm_100a CUDA kernels (tcgen05 GEMM, attention,
                                 norms, sampling, MoE, comm, training kernels)
* ``rlx_models_b200._runtime`` - host C++ runtime (paged-KV block manager,
                                 continuous-batching scheduler, safetensors index,
                                 token-packing data loader)

Every CUDA source is compiled for ``sm_100a`` only; the explicit ``-gencode``
bypasses torch's own arch list.
"""
import glob
import os

from setuptools import setup
from torch.utils.cpp_extension import BuildExtension, CppExtension, CUDAExtension

ROOT = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join("rlx_models_b200", "csrc")

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "--expt-relaxed-constexpr",
    "-Xptxas", "-O3",
]
if os.environ.get("B200_PTXAS_VERBOSE"):
    NVCC_FLAGS += ["-Xptxas", "-v"]
if os.environ.get("B200_DEBUG_CHECKS"):
    NVCC_FLAGS += ["-DB200_DEBUG_CHECKS=1"]
CXX_FLAGS = ["-O3", "-std=c++17"]


def cuda_sources():
    srcs = sorted(glob.glob(os.path.join(CSRC, "**", "*.cu"), recursive=True))
    return [os.path.join(CSRC, "bindings.cpp")] + [s for s in srcs if "/runtime/" not in s]


def runtime_sources():
    return sorted(glob.glob(os.path.join(CSRC, "runtime", "*.cpp")))


ext_modules = [
    CUDAExtension(
        name="rlx_models_b200._C",
        sources=cuda_sources(),
        include_dirs=[os.path.join(ROOT, CSRC)],
        extra_compile_args={"cxx": CXX_FLAGS, "nvcc": NVCC_FLAGS},
    ),
]
if runtime_sources():
    ext_modules.append(
        CppExtension(
            name="rlx_models_b200._runtime",
            sources=runtime_sources(),
            include_dirs=[os.path.join(ROOT, CSRC)],
            extra_compile_args={"cxx": CXX_FLAGS},
        )
    )

setup(
    name="rlx_models_b200",
    version="0.1.0",
    packages=["rlx_models_b200"],
    ext_modules=ext_modules,
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
