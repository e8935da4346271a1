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



def _debug_sources():
    """One wrapper per source under build/dbgsrc/ that defines LK_BOUNDS_CHECK and
    includes the real file: the debug objects get paths of their own, so both
    modules keep incremental builds.  Wrappers are rewritten only on change."""
    out_dir = os.path.join(HERE, "build", "dbgsrc")
    os.makedirs(out_dir, exist_ok=True)
    out = []
    for src in sources:
        path = os.path.join(out_dir, os.path.basename(src))
        text = '#define LK_BOUNDS_CHECK 1\n#include "%s"\n' % os.path.join(HERE, src)
        if not os.path.exists(path) or open(path).read() != text:
            with open(path, "w") as f:
                f.write(text)
        out.append(os.path.relpath(path, HERE))
    return out


# The bounds-checked debug build (LK_DEBUG_BOUNDS=1 selects it at import): the
# same sources compiled with LK_BOUNDS_CHECK; LK_SKIP_DEBUG_BUILD=1 builds only _C.
debug_ext = [] if os.environ.get("LK_SKIP_DEBUG_BUILD") == "1" else [
    CUDAExtension(
        name="lora_kernel_b200._C_debug",
        sources=_debug_sources(),
        include_dirs=[CSRC],
        extra_compile_args={"cxx": ["-O3", "-std=c++17"], "nvcc": NVCC_FLAGS},
    )
]

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
    ] + debug_ext,
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
