"""Build the sm_100a CUDA extension lora_kernel_b200._C in-tree.

    python setup.py build_ext --inplace

Every .cu file under csrc/ is compiled for sm_100a only (tcgen05/TMEM/TMA
kernels do not exist on other architectures); csrc/bindings.cpp holds the
torch bindings.
"""
import glob
import os

from setuptools import setup
from torch.utils.cpp_extension import BuildExtension, CppExtension, CUDAExtension

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "--expt-relaxed-constexpr",
    "-Xptxas", "-v" if os.environ.get("LK_PTXAS_VERBOSE") else "-O3",
]

sources = sorted(glob.glob(os.path.join(CSRC, "*.cu"))) + [os.path.join(CSRC, "bindings.cpp")]
sources = [os.path.relpath(s, HERE) for s in sources]
rt_sources = sorted(os.path.relpath(s, HERE) for s in glob.glob(os.path.join(CSRC, "runtime", "*.cpp")))

setup(
    name="lora_kernel_b200",
    version="0.1.0",
    packages=["lora_kernel_b200"],
    ext_modules=[
        CUDAExtension(
            name="lora_kernel_b200._C",
            sources=sources,
            include_dirs=[CSRC],
            extra_compile_args={"cxx": ["-O3", "-std=c++17"], "nvcc": NVCC_FLAGS},
        ),
        # host runtime (no device code): work-stealing pool, host arena, token
        # loader, parallel CRC-32
        CppExtension(
            name="lora_kernel_b200._rt",
            sources=rt_sources,
            include_dirs=[os.path.join(CSRC, "runtime")],
            extra_compile_args={"cxx": ["-O3", "-std=c++17", "-pthread", "-fvisibility=hidden"]},
            extra_link_args=["-pthread"],
        ),
    ],
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
